"""Token sampling (Gumbel-max with exponential noise): host side of ``csrc/sampler.cu``.

* ``Sampler`` -- ``nanovllm/layers/sampler.py:6-12``: ``forward(logits, temperatures)``
  returns argmax(softmax(logits.float() / T) / max(E, 1e-10)), E ~ Exp(1).
* ``draft_sample_step`` -- the per-step sampling of the draft proposer,
  ``nanovllm/spec_decode/draft_proposer.py:505-510``: keeps the fp32 copy of the
  step's logits in ``out_logits[:, s]`` and the sampled tokens in ``cands[:, s]``,
  in the same launch that samples.
* ``sample`` -- the general form.

The noise is Philox4x32-10 stream 2 keyed by ``(seed, offset)`` (with neither given:
``torch.initial_seed()`` and an offset that advances by one per call), or a given
(B, V) tensor ``exponentials`` (parity with the reference given identical draws).
Unlike the reference, fp32 logits are not divided in place.
"""

from __future__ import annotations

import itertools
from typing import Optional

import torch
from torch import nn

from . import _lib

_offsets = itertools.count()


def workspace_bytes(B: int, V: int) -> int:
    return int(_lib.lib().sdb_sample_workspace_size(B, V))


def sample(logits: torch.Tensor, temperatures: Optional[torch.Tensor] = None, *,
           exponentials: Optional[torch.Tensor] = None, seed: Optional[int] = None,
           offset: Optional[int] = None, out: Optional[torch.Tensor] = None,
           logits_out: Optional[torch.Tensor] = None,
           offset_tensor: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Tokens (B,) int64 for logits (B, V) fp32 / bf16 / fp16 (rows may be strided).

    ``temperatures`` (B,) (or (B, 1)) float32, > 0 as in the reference; None = 1.
    ``out``: int64 destination with B elements, any stride (e.g. ``cands[:, s]``).
    ``logits_out``: (B, V) float32 destination of ``logits.float()`` (any row stride).
    ``offset_tensor``: a one-element int64 CUDA tensor holding the Philox offset, read when
    the kernels run and advanced by one after the call (graph-safe in-kernel noise).
    """
    _lib.require_cuda(logits)
    if logits.dim() != 2:
        raise ValueError(f"logits must be (B, V), got {tuple(logits.shape)}")
    if logits.dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"unsupported logits dtype {logits.dtype}")
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
    if out.dtype != torch.int64 or out.numel() != B or out.dim() != 1:
        raise ValueError("out must be a 1-D int64 tensor with one entry per row")
    temps = None
    if temperatures is not None:
        temps = temperatures.reshape(-1).to(device=logits.device, dtype=torch.float32).contiguous()
        if temps.numel() != B:
            raise ValueError(f"temperatures must have {B} entries")
    e = None
    if exponentials is not None:
        e = exponentials.to(device=logits.device, dtype=torch.float32).contiguous()
        if tuple(e.shape) != (B, V):
            raise ValueError(f"exponentials must be ({B}, {V})")
    if logits_out is not None:
        if logits_out.dtype != torch.float32 or tuple(logits_out.shape) != (B, V) or logits_out.stride(-1) != 1:
            raise ValueError("logits_out must be a (B, V) float32 tensor with contiguous rows")
    if seed is None:
        seed = torch.initial_seed()
    if offset is None:
        offset = next(_offsets)
    need = workspace_bytes(B, V)
    ws = _lib.WORKSPACES.get(logits.device, "sample", need)
    if offset_tensor is not None:
        if e is not None:
            raise ValueError("offset_tensor draws in-kernel: no exponentials")
        if offset_tensor.dtype != torch.int64 or offset_tensor.numel() != 1 or not offset_tensor.is_cuda:
            raise ValueError("offset_tensor must be a one-element int64 CUDA tensor")
        rc = _lib.lib().sdb_sample_dev_offset(
            logits.data_ptr(), logits.stride(0), _lib.DTYPE_CODE[logits.dtype], _lib.ptr(temps),
            int(seed) & (2**64 - 1), offset_tensor.data_ptr(), out.data_ptr(), out.stride(0),
            _lib.ptr(logits_out), logits_out.stride(0) if logits_out is not None else 0, B, V,
            ws.data_ptr(), ws.numel(), _lib.stream_of(logits))
        _lib.check(rc, "sdb_sample_dev_offset")
        return out
    rc = _lib.lib().sdb_sample(
        logits.data_ptr(), logits.stride(0), _lib.DTYPE_CODE[logits.dtype], _lib.ptr(temps), _lib.ptr(e),
        int(seed) & (2**64 - 1), int(offset) & (2**64 - 1), out.data_ptr(), out.stride(0),
        _lib.ptr(logits_out), logits_out.stride(0) if logits_out is not None else 0, B, V,
        ws.data_ptr(), ws.numel(), _lib.stream_of(logits))
    _lib.check(rc, "sdb_sample")
    return out


class Sampler(nn.Module):
    """Mirror of ``nanovllm/layers/sampler.py:6-12``."""

    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor):
        return sample(logits, temperatures)


def draft_sample_step(logits: torch.Tensor, temps: torch.Tensor, out_logits: torch.Tensor,
                      cands: torch.Tensor, s: int, *, seed: Optional[int] = None,
                      offset: Optional[int] = None,
                      exponentials: Optional[torch.Tensor] = None,
                      offset_tensor: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One step of ``draft_proposer.py:505-510`` in one launch pair: ``out_logits[:, s]``
    = logits.float(), ``cands[:, s]`` = the sampled tokens, which are also returned
    (a view, ready to feed the next step's forward)."""
    dst = cands[:, s]
    sample(logits, temps, exponentials=exponentials, seed=seed, offset=offset, out=dst,
           logits_out=out_logits[:, s], offset_tensor=offset_tensor)
    return dst
