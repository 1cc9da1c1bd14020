"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference measures this path on no public dataset; every input here is
random with the distributions the configurations name (N(0,1) q/k/v, N(0, 3^2)
target logits, uniform int8 weights, ...), drawn from fixed seeds.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

# Qwen3-4B target / Qwen3-0.6B draft attention shapes
QWEN3_4B = dict(Hq=32, Hkv=8, D=128)
QWEN3_06B = dict(Hq=16, Hkv=8, D=128)
PAGE = 256
VOCAB = 151936
W8A16_SHAPES = {  # name: (K, N) of the Qwen3-4B projections
    "qkv": (2560, 6144),
    "o": (4096, 2560),
    "gate_up": (2560, 19456),
    "down": (9728, 2560),
}


@dataclass
class PagedCase:
    q: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_tables: torch.Tensor
    cache_seqlens: torch.Tensor
    scale: float
    n_q: int

    @property
    def B(self) -> int:
        return self.cache_seqlens.shape[0]


def paged_case(lens, n_q: int, Hq: int, Hkv: int, D: int, page: int = PAGE,
               dtype=torch.bfloat16, device="cuda", seed: int = 0, extra_blocks: int = 1,
               max_blocks: int | None = None, generate_on_device: bool = False) -> PagedCase:
    """Paged KV cache with a seeded scattered block table (-1 padded).

    ``extra_blocks`` unused pool blocks are filled with NaN so a kernel that reads
    past a sequence's visible keys is caught by the parity checks.
    """
    lens = [int(x) for x in lens]
    B = len(lens)
    nblk = [(L + page - 1) // page for L in lens]
    if max_blocks is None:
        max_blocks = max(1, max(nblk))
    NB = sum(nblk) + extra_blocks
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(NB, generator=g)
    bt = torch.full((B, max_blocks), -1, dtype=torch.int32)
    used = 0
    for b in range(B):
        bt[b, :nblk[b]] = perm[used:used + nblk[b]].to(torch.int32)
        used += nblk[b]
    spare = perm[used:]
    if generate_on_device:
        gd = torch.Generator(device=device).manual_seed(seed)
        k = torch.randn(NB, page, Hkv, D, generator=gd, device=device, dtype=dtype)
        v = torch.randn(NB, page, Hkv, D, generator=gd, device=device, dtype=dtype)
        q = torch.randn(B * n_q, Hq, D, generator=gd, device=device, dtype=dtype)
    else:
        k = torch.randn(NB, page, Hkv, D, generator=g).to(dtype)
        v = torch.randn(NB, page, Hkv, D, generator=g).to(dtype)
        q = torch.randn(B * n_q, Hq, D, generator=g).to(dtype)
    if len(spare):
        k[spare.to(k.device)] = float("nan")
        v[spare.to(v.device)] = float("nan")
    # slots past each sequence's length inside its last page: garbage, NaN in V
    for b, L in enumerate(lens):
        if L % page and nblk[b]:
            last = int(bt[b, nblk[b] - 1])
            v[last, L % page:] = float("nan")
            k[last, L % page:] = float("nan")
    return PagedCase(q=q.to(device), k_cache=k.to(device), v_cache=v.to(device),
                     block_tables=bt.to(device), cache_seqlens=torch.tensor(lens, dtype=torch.int32, device=device),
                     scale=1.0 / math.sqrt(D), n_q=n_q)


def cfg1_lens(seed: int = 0, B: int = 4):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(1, 1025, (B,), generator=g).tolist()


def cfg1_case(device="cuda", seed: int = 0) -> PagedCase:
    """Decode, B=4, 16/8 heads, fp32, pool of 64 pages of 256, L ~ U[1, 1024]."""
    lens = cfg1_lens(seed)
    nblk = sum((L + PAGE - 1) // PAGE for L in lens)
    return paged_case(lens, 1, dtype=torch.float32, device=device, seed=seed,
                      extra_blocks=64 - nblk, max_blocks=4, **QWEN3_06B)


def cfg2_lens(B: int, ctx: int, seed: int = 0):
    """Lengths around ``ctx`` that include exact multiples of 256 and their neighbours."""
    if B == 1:
        return [ctx]
    g = torch.Generator().manual_seed(seed)
    specials = [ctx, ctx - 1, max(1, ctx - 255), (ctx // 2 // PAGE) * PAGE or PAGE,
                (ctx // 2 // PAGE) * PAGE + 1, 7, 1, PAGE]
    lens = []
    for b in range(B):
        lens.append(specials[b] if b < len(specials) else int(torch.randint(8, ctx + 1, (1,), generator=g)))
    return [min(ctx, max(7, L)) for L in lens]


def cfg4_inputs(B: int = 64, k: int = 6, V: int = VOCAB, device="cuda", seed: int = 0):
    """Target logits N(0, 3^2), draft = target + N(0,1), draft tokens ~ softmax(draft)."""
    g = torch.Generator(device=device).manual_seed(seed)
    target = torch.randn(B, k + 1, V, generator=g, device=device) * 3.0
    draft = target[:, :k] + torch.randn(B, k, V, generator=g, device=device)
    probs = torch.softmax(draft, dim=-1).reshape(B * k, V)
    tokens = torch.multinomial(probs, 1, generator=g).reshape(B, k)
    return draft.contiguous(), target.contiguous(), tokens


def cfg3_inputs(M: int, K: int, N: int, device="cuda", seed: int = 0, act_dtype=torch.float16,
                scale_dtype=torch.float16):
    """int8 U[-127, 127], scales |N(0,1)|*0.01, activations N(0,1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int32).to(torch.int8)
    s = (torch.randn(N, generator=g, device=device).abs() * 0.01).to(scale_dtype)
    x = torch.randn(M, K, generator=g, device=device).to(act_dtype)
    return x, q, s
