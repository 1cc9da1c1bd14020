"""W8A16 oracle (CPU, numpy).  Test infrastructure only.

Restates the reference's ``nanovllm/layers/quant.py``:

* ``quantize_weight`` (:123-148): symmetric, zero point 0.  Per output channel
  ``scale = max(amax(|w|) / 127, 1e-8)`` in float32, ``q = clamp(round(w / scale),
  -127, 127)`` with round-half-to-even (``torch.round``), and the *returned* scale
  is that float32 scale rounded to bfloat16 (:148) -- q is computed with the
  unrounded float32 scale.  Per group: the same over ``[N, K/G, G]`` (:137-143).
* ``dequantize_weight`` (:151-159): ``q.float() * scale.float()`` (float32).
* the reference product used by the reference's own GEMM check
  (``scripts/bench_int8_gemm.py:139-142``): ``x.float() @ dequantize_weight(q, s).T``.
"""

from __future__ import annotations

import numpy as np

from .numerics import round_bf16

QMAX = 127


def quantize_weight(w, granularity: str = "per_channel", group_size: int = 128,
                    scale_round=round_bf16):
    """Returns (q int8 [N,K], scale float32 values already rounded by ``scale_round``)."""
    wf = np.asarray(w, dtype=np.float32)
    assert wf.ndim == 2
    N, K = wf.shape
    if granularity == "per_channel":
        amax = np.abs(wf).max(axis=1, keepdims=True)
        scale = np.maximum(amax / np.float32(QMAX), np.float32(1e-8)).astype(np.float32)
        q = np.clip(np.rint(wf / scale), -QMAX, QMAX).astype(np.int8)
        scale = scale[:, 0]
    elif granularity == "per_group":
        assert group_size > 0 and K % group_size == 0
        wg = wf.reshape(N, K // group_size, group_size)
        amax = np.abs(wg).max(axis=2, keepdims=True)
        scale = np.maximum(amax / np.float32(QMAX), np.float32(1e-8)).astype(np.float32)
        q = np.clip(np.rint(wg / scale), -QMAX, QMAX).astype(np.int8).reshape(N, K)
        scale = scale[..., 0]
    else:
        raise ValueError(granularity)
    return q, scale_round(scale)


def dequantize_weight(q, scale, granularity: str = "per_channel", group_size: int = 128):
    qf = np.asarray(q).astype(np.float32)
    s = np.asarray(scale, dtype=np.float32)
    N, K = qf.shape
    if granularity == "per_channel":
        return qf * s[:, None]
    G = group_size
    return (qf.reshape(N, K // G, G) * s[:, :, None]).reshape(N, K)


def int8_linear(x, q, scale, bias=None, granularity: str = "per_channel",
                group_size: int = 128, dtype=np.float32):
    """y = x @ dequant(q, scale).T (+ bias), computed in ``dtype``."""
    xf = np.asarray(x, dtype=dtype)
    w = dequantize_weight(q, scale, granularity, group_size).astype(dtype)
    y = xf.reshape(-1, xf.shape[-1]) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=dtype)
    return y.reshape(*xf.shape[:-1], w.shape[0])


def algorithmic_bytes(M: int, N: int, K: int, act_elem: int = 2, scale_elem: int = 2,
                      n_scales: int | None = None) -> int:
    """int8 W once, scales once, x in, y out."""
    if n_scales is None:
        n_scales = N
    return N * K + n_scales * scale_elem + M * K * act_elem + M * N * act_elem
