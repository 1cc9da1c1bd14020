"""Speculative-decoding rejection sampling: host side of ``csrc/verify_sample.cu``.

Mirror of ``nanovllm/spec_decode/verify.py:32-175``: same arguments, same
``VerifyResult`` fields and dtypes (int64 accepted / bonus / n_proposed, bool
accept_mask), same alignment (candidate j against target row j, bonus from row
``accepted``), same residual fallback and clamps.  The two random draws of the
reference (``torch.rand`` at :120 and ``exponential_`` at :209) are either given
explicitly (``uniforms`` / ``exponentials``) or generated inside the kernel from
Philox4x32-10 keyed by ``(seed, offset)``; with neither given, the seed is
``torch.initial_seed()`` and the offset advances by one per call.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib


@dataclass
class VerifyResult:
    accepted: torch.Tensor      # (batch,) int64 accepted prefix length
    bonus: torch.Tensor         # (batch,) int64 token emitted after the prefix (always valid)
    n_proposed: torch.Tensor    # (batch,) int64
    accept_mask: torch.Tensor   # (batch, k) bool


_offsets = itertools.count()


def workspace_bytes(B: int, k: int, target_rows: int, V: int) -> int:
    return int(_lib.lib().sdb_verify_workspace_size(B, k, target_rows, V))


@torch.no_grad()
def verify_batch(draft_probs: torch.Tensor, target_logits: torch.Tensor, draft_tokens: torch.Tensor,
                 temperatures: Optional[torch.Tensor] = None, draft_is_point_mass: bool = False, *,
                 uniforms: Optional[torch.Tensor] = None, exponentials: Optional[torch.Tensor] = None,
                 seed: Optional[int] = None, offset: Optional[int] = None,
                 out: Optional[VerifyResult] = None) -> VerifyResult:
    """draft_probs (B, k, V): raw draft logits (probabilities if ``draft_is_point_mass``);
    target_logits (B, k+1, V) (or (B, k, V)); draft_tokens (B, k); temperatures (B,) or None."""
    _lib.require_cuda(draft_probs, target_logits, draft_tokens, temperatures, uniforms, exponentials)
    B, k, V = draft_probs.shape
    Tr = target_logits.shape[1]
    if target_logits.shape[0] != B or target_logits.shape[2] != V or Tr not in (k, k + 1):
        raise ValueError(f"target_logits {tuple(target_logits.shape)} vs draft {tuple(draft_probs.shape)}")
    if tuple(draft_tokens.shape) != (B, k):
        raise ValueError(f"draft_tokens must be ({B}, {k})")
    # float32 / bfloat16 / float16 logits are read as they are (converted exactly in the
    # kernels, as the reference's .float()); other types are converted here
    draft = (draft_probs if draft_probs.dtype in _lib.DTYPE_CODE else draft_probs.float()).contiguous()
    target = (target_logits if target_logits.dtype in _lib.DTYPE_CODE else target_logits.float()).contiguous()
    tokens = draft_tokens.to(torch.int64).contiguous()
    temps = None
    if temperatures is not None:
        t = temperatures.float()
        temps = (t.expand(B) if t.dim() == 0 else t.reshape(B)).contiguous()
    u = None if uniforms is None else uniforms.float().reshape(B, k).contiguous()
    e = None if exponentials is None else exponentials.float().reshape(B, V).contiguous()
    if seed is None:
        seed = torch.initial_seed()
    if offset is None:
        offset = next(_offsets)
    if out is None:
        dev = draft.device
        out = VerifyResult(accepted=torch.empty(B, dtype=torch.int64, device=dev),
                           bonus=torch.empty(B, dtype=torch.int64, device=dev),
                           n_proposed=torch.full((B,), k, dtype=torch.int64, device=dev),
                           accept_mask=torch.empty(B, k, dtype=torch.bool, device=dev))
    L = _lib.lib()
    need = int(L.sdb_verify_workspace_size(B, k, Tr, V))
    ws = _lib.WORKSPACES.get(draft.device, "verify", need)
    rc = L.sdb_verify_batch_ex(draft.data_ptr(), _lib.DTYPE_CODE[draft.dtype], target.data_ptr(),
                               _lib.DTYPE_CODE[target.dtype], tokens.data_ptr(), _lib.ptr(temps),
                               _lib.ptr(u), _lib.ptr(e), int(seed) & (2**64 - 1), int(offset) & (2**64 - 1),
                               1 if draft_is_point_mass else 0, out.accepted.data_ptr(),
                               out.bonus.data_ptr(), out.accept_mask.data_ptr(), B, k, Tr, V,
                               ws.data_ptr(), ws.numel(), _lib.stream_of(draft))
    _lib.check(rc, "sdb_verify_batch_ex")
    return out


def philox_draws(rows: int, cols: int, seed: int, offset: int, stream_id: int,
                 device="cuda") -> torch.Tensor:
    """The sampler's Philox stream written out: 0 = acceptance uniforms, 1 = exponentials."""
    outp = torch.empty(rows, cols, dtype=torch.float32, device=device)
    rc = _lib.lib().sdb_philox_fill(outp.data_ptr(), rows, cols, int(seed) & (2**64 - 1),
                                    int(offset) & (2**64 - 1), stream_id, _lib.stream_of(outp))
    _lib.check(rc, "sdb_philox_fill")
    return outp
