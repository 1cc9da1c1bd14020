"""W8A16 int8-weight linear: host side of ``csrc/w8a16.cu``.

Mirrors ``nanovllm/layers/quant.py``:

* ``quantize_weight(w, granularity, group_size)`` (:123-148) -> (q int8, scale bf16),
  on the GPU, bit-identical to the reference (float32 scale = max(amax/127, 1e-8),
  round half to even, clamp +-127, scale rounded once to bf16).
* ``dequantize_weight(q, scale, granularity, group_size)`` (:151-159): the float32
  reference dequantisation (a test helper there as here).
* ``int8_linear(x, qweight, scale, bias, granularity, group_size, out_features, cfg_)``
  (:262-310): y = x @ dequant(q).T + bias with the dequantisation fused into the
  sm_100a kernel.  ``cfg_`` tuned Triton tiles there and is accepted and ignored.
"""

from __future__ import annotations

import torch

from . import _lib

QMAX = 127


def quantize_weight(w: torch.Tensor, granularity: str = "per_channel", group_size: int = 128,
                    scale_dtype: torch.dtype = torch.bfloat16):
    _lib.require_cuda(w)
    if w.dim() != 2:
        raise AssertionError(f"only 2-D weights are quantised, got {tuple(w.shape)}")
    N, K = w.shape
    if granularity == "per_channel":
        G = 0
        scale = torch.empty(N, dtype=scale_dtype, device=w.device)
    elif granularity == "per_group":
        if not (group_size > 0 and K % group_size == 0):
            raise AssertionError("group_size must divide K")
        G = group_size
        scale = torch.empty(N, K // group_size, dtype=scale_dtype, device=w.device)
    else:
        raise ValueError(granularity)
    wc = w.contiguous()
    q = torch.empty(N, K, dtype=torch.int8, device=w.device)
    rc = _lib.lib().sdb_quantize_weight(wc.data_ptr(), _lib.DTYPE_CODE[wc.dtype], q.data_ptr(),
                                        scale.data_ptr(), _lib.DTYPE_CODE[scale_dtype], N, K, G,
                                        _lib.stream_of(wc))
    _lib.check(rc, "sdb_quantize_weight")
    return q, scale


def dequantize_weight(q: torch.Tensor, scale: torch.Tensor, granularity: str = "per_channel",
                      group_size: int = 128) -> torch.Tensor:
    N, K = q.shape
    qf = q.to(torch.float32)
    if granularity == "per_channel":
        return qf * scale.to(torch.float32).unsqueeze(1)
    G = group_size
    return (qf.view(N, K // G, G) * scale.to(torch.float32).unsqueeze(-1)).view(N, K)


def workspace_bytes(M: int, N: int, K: int) -> int:
    return int(_lib.lib().sdb_w8a16_workspace_size(M, N, K))


def int8_linear(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor,
                bias: torch.Tensor | None = None, granularity: str = "per_channel",
                group_size: int = 128, out_features: int | None = None, cfg_: dict | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    _lib.require_cuda(x, qweight, scale, bias)
    if qweight.dtype != torch.int8:
        raise AssertionError("qweight must be int8")
    N, K = qweight.shape
    N = out_features or N
    x2 = x.reshape(-1, x.shape[-1])
    M = x2.shape[0]
    if x2.shape[1] != K:
        raise AssertionError(f"K mismatch: x {tuple(x2.shape)} vs w {tuple(qweight.shape)}")
    if x2.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("activations must be bf16 or fp16")
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    qw = qweight if qweight.is_contiguous() else qweight.contiguous()
    sc = scale.contiguous()
    G = 0 if granularity == "per_channel" else group_size
    if bias is not None:
        bias = bias.to(x2.dtype).contiguous()
    y = out if out is not None else torch.empty((M, N), device=x.device, dtype=x2.dtype)
    L = _lib.lib()
    need = int(L.sdb_w8a16_workspace_size(M, N, K))
    ws = _lib.WORKSPACES.get(x.device, "w8a16", need)
    rc = L.sdb_w8a16_linear(x2.data_ptr(), x2.stride(0), qw.data_ptr(), sc.data_ptr(),
                            _lib.DTYPE_CODE[sc.dtype], G, _lib.ptr(bias), y.data_ptr(), y.stride(0),
                            M, N, K, _lib.DTYPE_CODE[x2.dtype], ws.data_ptr(), ws.numel(),
                            _lib.stream_of(x2))
    _lib.check(rc, "sdb_w8a16_linear")
    return y.view(*x.shape[:-1], N)
