"""Attention-prologue oracle (CPU, numpy).  Test infrastructure only.

Restates, for one Qwen3 layer, what ``Qwen3Attention.forward`` does between the QKV
projection and the attention call (``nanovllm/models/qwen3.py:77-86``):

* split of the fused projection into q (Hq heads), k and v (Hkv heads each) (:78-81);
* ``RMSNorm.rms_forward`` (``nanovllm/layers/layernorm.py:16-25``) on every q and k
  head: x in float32, var = mean(x^2), x * rsqrt(var + eps) rounded to the model
  dtype, then times the weight (a model-dtype multiply: float32 product rounded);
* ``apply_rotary_emb`` (``nanovllm/layers/rotary_embedding.py:6-14``) with the
  cos / sin rows of ``cos_sin_cache[positions]`` (:44-46): x in float32,
  y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin, rounded to the model dtype.
"""

from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, f32_to_bf16_bits


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def rms_norm(x, weight, eps: float, dtype: str) -> np.ndarray:
    """layernorm.py:16-25 on the last axis; x and weight hold model-dtype values as float32."""
    x = np.asarray(x, dtype=np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    xn = _round(x * inv, dtype)
    return _round(xn * np.asarray(weight, dtype=np.float32), dtype)


def apply_rotary(x, cos, sin, dtype: str) -> np.ndarray:
    """rotary_embedding.py:6-14; cos / sin broadcast over the head axis."""
    x = np.asarray(x, dtype=np.float32)
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    y1 = (x1 * cos).astype(np.float32) - (x2 * sin).astype(np.float32)
    y2 = (x2 * cos).astype(np.float32) + (x1 * sin).astype(np.float32)
    return _round(np.concatenate([y1, y2], axis=-1), dtype)


def qk_prologue(qkv, positions, Hq: int, Hkv: int, D: int, cos_sin_cache, q_norm_weight,
                k_norm_weight, eps: float, dtype: str):
    """(q, k, v) as (T, H, D) float32 arrays of model-dtype values."""
    qkv = np.asarray(qkv, dtype=np.float32)
    T = qkv.shape[0]
    q = qkv[:, :Hq * D].reshape(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
    if q_norm_weight is not None:
        q = rms_norm(q, q_norm_weight, eps, dtype)
        k = rms_norm(k, k_norm_weight, eps, dtype)
    cs = np.asarray(cos_sin_cache, dtype=np.float32).reshape(np.shape(cos_sin_cache)[0], D)[np.asarray(positions)]
    cos, sin = cs[:, None, :D // 2], cs[:, None, D // 2:]
    return apply_rotary(q, cos, sin, dtype), apply_rotary(k, cos, sin, dtype), v.copy()
