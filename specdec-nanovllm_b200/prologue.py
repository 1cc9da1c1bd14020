"""Attention prologue of a Qwen3 layer (split, q/k RMSNorm, rotary, KV store) in one launch.

Host side of ``csrc/qk_prologue.cu``.  ``qk_norm_rope_store`` replaces, for one
layer, the sequence of ``Qwen3Attention.forward`` (``nanovllm/models/qwen3.py:77-86``)
between the QKV projection and the attention call -- ``qkv.split``, ``q_norm`` /
``k_norm`` (``RMSNorm``, ``nanovllm/layers/layernorm.py:16-25``) and ``rotary_emb``
(``nanovllm/layers/rotary_embedding.py:38-50``) -- plus the ``store_kvcache`` that
``Attention.forward`` runs first (``attention.py:59-63``).  Attention then runs over
the cache without a store (``paged_attention``).

``rope_cos_sin_cache`` builds the same (max_position, D) table as
``RotaryEmbedding.__init__`` (``rotary_embedding.py:18-35``).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def rope_cos_sin_cache(head_dim: int, max_position: int, base: float,
                       device="cuda") -> torch.Tensor:
    """(max_position, head_dim) float32 rows [cos | sin] of the reference's formula."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(device)


def qk_norm_rope_store(qkv: torch.Tensor, positions: torch.Tensor, num_heads: int,
                       num_kv_heads: int, head_dim: int, cos_sin_cache: torch.Tensor,
                       q_norm_weight: Optional[torch.Tensor] = None,
                       k_norm_weight: Optional[torch.Tensor] = None, eps: float = 1e-6,
                       k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None,
                       slot_mapping: Optional[torch.Tensor] = None, return_kv: bool = False,
                       q_out: Optional[torch.Tensor] = None):
    """q (T, Hq, D) normalised and rotated; with ``return_kv`` also k (normalised,
    rotated) and v as (T, Hkv, D).  With ``k_cache`` / ``v_cache`` / ``slot_mapping``
    the k / v rows are stored into the paged cache (slot -1 skipped).

    ``cos_sin_cache`` is (max_position, D) or the module's (max_position, 1, D) buffer.
    """
    _lib.require_cuda(qkv, positions, cos_sin_cache)
    T = qkv.shape[0]
    qkv2 = qkv.reshape(T, -1)
    if qkv2.stride(-1) != 1:
        qkv2 = qkv2.contiguous()
    D, Hq, Hkv = head_dim, num_heads, num_kv_heads
    if qkv2.shape[1] != (Hq + 2 * Hkv) * D:
        raise ValueError(f"qkv rows have {qkv2.shape[1]} elements, expected {(Hq + 2 * Hkv) * D}")
    if qkv.dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"unsupported dtype {qkv.dtype}")
    cs = cos_sin_cache.reshape(cos_sin_cache.shape[0], -1)
    if cs.dtype != torch.float32 or cs.shape[1] != D or cs.stride(-1) != 1:
        raise ValueError("cos_sin_cache must be float32 (max_position, D) with contiguous rows")
    pos = positions.to(torch.int64).contiguous()
    for w in (q_norm_weight, k_norm_weight):
        if w is not None and (w.numel() != D or w.dtype != qkv.dtype):
            raise ValueError("norm weights must have head_dim entries of the model dtype")
    qw = None if q_norm_weight is None else q_norm_weight.contiguous()
    kw = None if k_norm_weight is None else k_norm_weight.contiguous()
    if q_out is None:
        q_out = torch.empty(T, Hq, D, dtype=qkv.dtype, device=qkv.device)
    k_out = v_out = None
    if return_kv:
        k_out = torch.empty(T, Hkv, D, dtype=qkv.dtype, device=qkv.device)
        v_out = torch.empty_like(k_out)
    store = slot_mapping is not None and k_cache is not None and v_cache is not None \
        and k_cache.numel() > 0
    nb = page = 0
    sb = sp = sh = 0
    slots = None
    if store:
        nb, page, hkv2, d2 = k_cache.shape
        if (hkv2, d2) != (Hkv, D) or v_cache.shape != k_cache.shape or v_cache.stride() != k_cache.stride():
            raise ValueError("cache shapes disagree with the heads")
        if k_cache.dtype != qkv.dtype:
            raise ValueError("cache dtype differs from qkv")
        sb, sp, sh = k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
        slots = slot_mapping.to(torch.int32).contiguous()
        if slots.numel() != T:
            raise ValueError("slot_mapping must have one entry per token")
    ws = _lib.WORKSPACES.get(qkv.device, "attention", 256)
    rc = _lib.lib().sdb_qk_norm_rope_store(
        qkv2.data_ptr(), qkv2.stride(0), _lib.ptr(qw), _lib.ptr(kw), float(eps), cs.data_ptr(), cs.stride(0),
        cs.shape[0], pos.data_ptr(), q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
        _lib.ptr(k_out), _lib.ptr(v_out), k_out.stride(0) if k_out is not None else 0,
        k_out.stride(1) if k_out is not None else 0,
        _lib.ptr(k_cache if store else None), _lib.ptr(v_cache if store else None), sb, sp, sh,
        _lib.ptr(slots), T, Hq, Hkv, D, page, nb, _lib.DTYPE_CODE[qkv.dtype], ws.data_ptr(),
        _lib.stream_of(qkv))
    _lib.check(rc, "sdb_qk_norm_rope_store")
    return (q_out, k_out, v_out) if return_kv else q_out
