"""Decoder-layer elementwise steps on the sm_100a kernels (``csrc/layer_ops.cu``).

* ``rms_norm(x, weight, eps, residual=None)`` -- ``RMSNorm.forward``
  (``nanovllm/layers/layernorm.py:17-50``): returns ``y`` without a residual, else
  ``(y, x + residual)``; float32 statistics, the same model-dtype roundings.
* ``silu_and_mul(gate_up)`` -- ``SiluAndMul.forward`` (``nanovllm/layers/activation.py:8-13``).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _rows(t: torch.Tensor) -> torch.Tensor:
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1 or t2.data_ptr() % 16 or t2.stride(0) % 8:
        t2 = t2.contiguous()
    return t2


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
    _lib.require_cuda(x, weight, residual)
    if x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype:
        raise ValueError("x and weight must share a bf16 / fp16 dtype")
    x2 = _rows(x)
    T, H = x2.shape
    if weight.numel() != H:
        raise ValueError(f"weight has {weight.numel()} entries, rows have {H}")
    y = out if out is not None else torch.empty_like(x2)
    r_in = r_out = None
    if residual is not None:
        r_in = _rows(residual)
        if r_in.shape != x2.shape or r_in.dtype != x.dtype:
            raise ValueError("residual must match x")
        r_out = torch.empty_like(x2)
    rc = _lib.lib().sdb_rms_norm(
        x2.data_ptr(), x2.stride(0), _lib.ptr(r_in), r_in.stride(0) if r_in is not None else 0,
        y.data_ptr(), y.stride(0), _lib.ptr(r_out), r_out.stride(0) if r_out is not None else 0,
        weight.contiguous().data_ptr(), T, H, float(eps), _lib.DTYPE_CODE[x.dtype], _lib.stream_of(x2))
    _lib.check(rc, "sdb_rms_norm")
    y = y.view(x.shape)
    return y if residual is None else (y, r_out.view(x.shape))


def silu_and_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _lib.require_cuda(gate_up)
    if gate_up.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("gate_up must be bf16 or fp16")
    g2 = _rows(gate_up)
    T, F2 = g2.shape
    if F2 % 2:
        raise ValueError("gate_up rows must hold gate and up halves")
    F = F2 // 2
    y = out if out is not None else torch.empty(T, F, dtype=gate_up.dtype, device=gate_up.device)
    rc = _lib.lib().sdb_silu_mul(g2.data_ptr(), g2.stride(0), y.data_ptr(), y.stride(0), T, F,
                                 _lib.DTYPE_CODE[gate_up.dtype], _lib.stream_of(g2))
    _lib.check(rc, "sdb_silu_mul")
    return y.view(*gate_up.shape[:-1], F)
