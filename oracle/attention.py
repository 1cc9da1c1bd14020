"""Paged decode / verify attention oracle (CPU, numpy).  Test infrastructure only.

Restates ``paged_decode_attention_ref`` (reference
``nanovllm/kernels/paged_decode_attn.py:472-495``): gather the pages of each
sequence through its block table, upcast to float, softmax(q.K^T * scale).V per
query head with GQA head sharing (``repeat_interleave``, :484-485), and emit
zeros for a sequence whose cache length is 0 (:480-482).

The k+1-row verify form follows flash-attn's ``flash_attn_varlen_func(...,
causal=True, block_table=...)`` as called at ``nanovllm/layers/attention.py:67-70``
with ``cu_seqlens_k`` = the cache length of each sequence
(``nanovllm/engine/model_runner.py:531``): causal masking is aligned to the
bottom-right corner, so query row r of n (r = 0..n-1) sees keys
``j <= L - n + r``.  A row that sees no key (only possible when L < n) is zero,
which is what flash-attn writes for a fully masked row.  With n = 1 this is
exactly the decode oracle.
"""

from __future__ import annotations

import numpy as np


def visible_keys(L: int, n: int, r: int) -> int:
    """Number of keys query row ``r`` of ``n`` sees in a cache of length ``L``."""
    return max(0, min(L, L - n + r + 1))


def paged_attention(q, k_cache, v_cache, block_tables, cache_seqlens, scale,
                    n_q: int = 1, compute_dtype=np.float32):
    """Oracle for decode (n_q = 1) and speculative verify (n_q = k+1).

    q            : (B*n_q, Hq, D)   rows of sequence b are b*n_q .. b*n_q+n_q-1
    k_cache      : (NB, page, Hkv, D)
    v_cache      : (NB, page, Hkv, D)
    block_tables : (B, max_blocks) int32, -1 padded; only the first
                   ceil(L/page) entries are read
    cache_seqlens: (B,) int32, the cache length L of each sequence (it already
                   includes the n_q new tokens in the verify step)
    returns      : (B*n_q, Hq, D) in ``compute_dtype``
    """
    q = np.asarray(q)
    k_cache = np.asarray(k_cache)
    v_cache = np.asarray(v_cache)
    block_tables = np.asarray(block_tables)
    cache_seqlens = np.asarray(cache_seqlens)
    total, Hq, D = q.shape
    _, page, Hkv, _ = k_cache.shape
    B = cache_seqlens.shape[0]
    assert total == B * n_q, (total, B, n_q)
    assert Hq % Hkv == 0
    rep = Hq // Hkv
    out = np.zeros((total, Hq, D), dtype=compute_dtype)
    # row r of n sees keys [0, visible_keys(L, n, r)); the rest are masked to -inf
    for b in range(B):
        L = int(cache_seqlens[b])
        if L <= 0:
            continue                                   # zeros (paged_decode_attn.py:480-482)
        nblk = (L + page - 1) // page
        phys = block_tables[b, :nblk].astype(np.int64)
        k = k_cache[phys].reshape(-1, Hkv, D)[:L].astype(compute_dtype)   # (L, Hkv, D)
        v = v_cache[phys].reshape(-1, Hkv, D)[:L].astype(compute_dtype)
        nv = np.array([visible_keys(L, n_q, r) for r in range(n_q)])
        cols = np.arange(L)
        masked = cols[None, :] >= nv[:, None]                             # (n_q, L)
        qb = q[b * n_q:(b + 1) * n_q].astype(compute_dtype)               # (n_q, Hq, D)
        for h in range(Hkv):
            # the GQA group of kv head h (repeat_interleave order, :484-485): q heads h*rep ..
            qg = qb[:, h * rep:(h + 1) * rep].reshape(n_q * rep, D)
            logits = (qg @ k[:, h].T).reshape(n_q, rep, L) * compute_dtype(scale)
            logits = np.where(masked[:, None, :], -np.inf, logits)
            mx = logits.max(axis=-1, keepdims=True)
            mx = np.where(np.isfinite(mx), mx, 0.0)
            p = np.exp(logits - mx)
            den = p.sum(axis=-1, keepdims=True)
            p = p / np.where(den > 0, den, 1.0)                          # rows that see no key stay 0
            out[b * n_q:(b + 1) * n_q, h * rep:(h + 1) * rep] = (p.reshape(n_q * rep, L) @ v[:, h]).reshape(
                n_q, rep, D)
    return out


def algorithmic_bytes(cache_seqlens, n_q: int, Hq: int, Hkv: int, D: int,
                      kv_elem: int, q_elem: int) -> int:
    """Bytes a perfect kernel moves: every visible K/V row once plus q in and o out."""
    L = np.asarray(cache_seqlens, dtype=np.int64)
    kv = int(L.sum()) * 2 * Hkv * D * kv_elem
    qo = 2 * L.shape[0] * n_q * Hq * D * q_elem
    return kv + qo


def paged_attention_pairs(q, k_cache, v_cache, block_tables, cache_seqlens, scale, n_q, pairs):
    """The same computation restricted to a list of (sequence, kv head) pairs, in float32
    with batched matmuls (the timed CPU baseline: the reference's
    ``paged_decode_attention_ref`` math, one GQA group at a time).

    Returns {(b, kvh): (n_q, G, D) float32}.
    """
    total, Hq, D = q.shape
    _, page, Hkv, _ = k_cache.shape
    G = Hq // Hkv
    out = {}
    for b, h in pairs:
        L = int(cache_seqlens[b])
        res = np.zeros((n_q, G, D), dtype=np.float32)
        if L > 0:
            nblk = (L + page - 1) // page
            phys = block_tables[b, :nblk].astype(np.int64)
            k = k_cache[phys, :, h].reshape(-1, D)[:L].astype(np.float32)     # (L, D)
            v = v_cache[phys, :, h].reshape(-1, D)[:L].astype(np.float32)
            qg = q[b * n_q:(b + 1) * n_q, h * G:(h + 1) * G].astype(np.float32)  # (n_q, G, D)
            logits = (qg.reshape(n_q * G, D) @ k.T).reshape(n_q, G, L) * np.float32(scale)
            for r in range(n_q):
                nv = visible_keys(L, n_q, r)
                if nv == 0:
                    continue
                lg = logits[r, :, :nv]
                lg = lg - lg.max(axis=-1, keepdims=True)
                p = np.exp(lg)
                p /= p.sum(axis=-1, keepdims=True)
                res[r] = p @ v[:nv]
        out[(b, h)] = res
    return out
