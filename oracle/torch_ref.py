"""The reference's CPU torch path for attention, restated in torch.  Test and benchmark
infrastructure only: ``bench.py`` times it as the CPU baseline (``cpu_baseline`` and
``--impl reference``); nothing in the shipped package imports it.

``paged_attention_torch`` restates ``paged_decode_attention_ref``
(``nanovllm/kernels/paged_decode_attn.py:472-495``) operation for operation -- gather
the sequence's pages through its block table (:487-489), ``repeat_interleave`` the kv
heads to the query heads and upcast to float32 (:490-491), ``einsum`` logits times the
scale (:492), ``softmax`` (:493), ``einsum`` with V (:494), zeros for an empty
sequence (:480-482), cast back to the query dtype (:495) -- and extends it to the
k+1 verify rows of flash-attn's bottom-right causal alignment
(``nanovllm/layers/attention.py:64-70``): row r of n sees keys j <= L - n + r, as a
-inf mask before the softmax.  With n = 1 it is the reference function itself.  The
reference cannot be imported where the benchmark runs, so this restatement is what
runs there; ``tests/test_oracle_golden.py`` pins it to the reference's own outputs.
"""

from __future__ import annotations

import torch


def paged_attention_torch(q, k_cache, v_cache, block_table, context_lens, scale, n_q: int = 1,
                          seqs=None):
    """q (B*n_q, Hq, D); caches (NB, page, Hkv, D); returns (len(seqs)*n_q, Hq, D) in q.dtype.

    ``seqs``: the sequence indices to compute (all by default), so a benchmark can time a
    bounded sample of a large batch.
    """
    total, num_q_heads, head_dim = q.shape
    _, block_size, num_kv_heads, _ = k_cache.shape
    rep = num_q_heads // num_kv_heads
    seqs = range(context_lens.shape[0]) if seqs is None else seqs
    outs = []
    for s in seqs:
        L = int(context_lens[s])
        if L == 0:
            outs.append(torch.zeros(n_q, num_q_heads, head_dim, dtype=q.dtype))
            continue
        nblk = (L + block_size - 1) // block_size
        phys = block_table[s, :nblk].long()
        k = k_cache[phys].reshape(-1, num_kv_heads, head_dim)[:L]
        v = v_cache[phys].reshape(-1, num_kv_heads, head_dim)[:L]
        k = k.repeat_interleave(rep, dim=1).float()                    # (L, Hq, D)
        v = v.repeat_interleave(rep, dim=1).float()
        qs = q[s * n_q:(s + 1) * n_q].float()                          # (n_q, Hq, D)
        logits = torch.einsum("rhd,lhd->rhl", qs, k) * scale           # (n_q, Hq, L)
        if n_q > 1:
            r = torch.arange(n_q).view(n_q, 1, 1)
            j = torch.arange(L).view(1, 1, L)
            logits = logits.masked_fill(j > L - n_q + r, float("-inf"))
        p = torch.softmax(logits, dim=-1)
        p = torch.nan_to_num(p, nan=0.0)                               # rows that see no key
        outs.append(torch.einsum("rhl,lhd->rhd", p, v).to(q.dtype))
    return torch.cat(outs) if outs else q.new_zeros(0, num_q_heads, head_dim)
