"""Attention prologue (split + q/k RMSNorm + rotary + KV store) on the GPU.

Bar: within the bf16 tolerance (rtol 1e-2 / atol 1e-3, i.e. one bf16 ulp) of the
reference's RMSNorm + RotaryEmbedding (golden fixture) and of the oracle, with at
least 98 % of the elements bit-identical (the sum of squares is reduced in another
order); v rows and the cache store bit-exact.
"""

import numpy as np
import pytest
import torch

from oracle import prologue as op
from oracle.numerics import allclose_report, bf16_bits_to_f32

pytestmark = pytest.mark.gpu


def _close(got, want, frac=0.98):
    got = got.float().cpu().numpy().reshape(want.shape)
    ok, err, _ = allclose_report(got, want, rtol=1e-2, atol=1e-3)
    assert ok, err
    assert np.mean(got == want) >= frac, np.mean(got == want)


def _bf16(bits):
    return torch.from_numpy(bf16_bits_to_f32(bits)).to(torch.bfloat16).cuda()


def test_golden_reference(pkg, golden):
    g = golden("prologue_qwen3")
    Hq, Hkv, D = int(g["Hq"]), int(g["Hkv"]), int(g["D"])
    cs = torch.full((int(g["max_position"]), D), float("nan"))
    cs[torch.from_numpy(g["positions"])] = torch.from_numpy(g["cos_sin_rows"])
    q, k, v = pkg.qk_norm_rope_store(_bf16(g["qkv"]), torch.from_numpy(g["positions"]).cuda(), Hq, Hkv, D,
                                     cs.cuda(), _bf16(g["q_norm_w"]), _bf16(g["k_norm_w"]), float(g["eps"]),
                                     return_kv=True)
    torch.cuda.synchronize()
    _close(q, bf16_bits_to_f32(g["q"]))
    _close(k, bf16_bits_to_f32(g["k"]))
    _close(v, bf16_bits_to_f32(g["v"]), frac=1.0)


@pytest.mark.parametrize("dtype,D,norm", [(torch.bfloat16, 128, True), (torch.float16, 128, True),
                                          (torch.bfloat16, 64, True), (torch.bfloat16, 256, False),
                                          (torch.float32, 128, True)])
def test_against_oracle_with_cache_store(pkg, dtype, D, norm):
    g = torch.Generator().manual_seed(D + (7 if norm else 0))
    T, Hq, Hkv, page, NB = 37, 16, 4, 256, 6
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, generator=g) * 3.0).to(dtype)
    qw = (torch.rand(D, generator=g) * 2.0).to(dtype) if norm else None
    kw = (torch.rand(D, generator=g) * 2.0).to(dtype) if norm else None
    pos = torch.randint(0, 4000, (T,), generator=g)
    cs = pkg.rope_cos_sin_cache(D, 4096, 1e6, device="cpu")
    kc = torch.full((NB, page, Hkv, D), float("nan"), dtype=dtype)
    vc = kc.clone()
    slots = torch.randperm(NB * page, generator=g)[:T].to(torch.int32)
    slots[5] = -1
    kcd, vcd = kc.cuda(), vc.cuda()
    q, k, v = pkg.qk_norm_rope_store(qkv.cuda(), pos.cuda(), Hq, Hkv, D, cs.cuda(),
                                     None if qw is None else qw.cuda(), None if kw is None else kw.cuda(), 1e-6,
                                     k_cache=kcd, v_cache=vcd, slot_mapping=slots.cuda(), return_kv=True)
    torch.cuda.synchronize()
    name = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    wq, wk, wv = op.qk_prologue(qkv.float().numpy(), pos.numpy(), Hq, Hkv, D, cs.numpy(),
                                None if qw is None else qw.float().numpy(),
                                None if kw is None else kw.float().numpy(), 1e-6, name)
    frac = 0.98 if dtype != torch.float32 else 0.9
    if dtype == torch.float32:  # no rounding to a 16-bit type: compare at fp32 precision
        ok, err, _ = allclose_report(q.cpu().numpy(), wq, rtol=1e-5, atol=1e-5)
        assert ok, err
        ok, err, _ = allclose_report(k.cpu().numpy(), wk, rtol=1e-5, atol=1e-5)
        assert ok, err
    else:
        _close(q, wq, frac)
        _close(k, wk, frac)
    assert torch.equal(v.cpu(), qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D))
    # the cache holds k / v of every stored token (bits of the kernel's own k / v)
    kc_h, vc_h = kcd.cpu().view(NB * page, Hkv, D), vcd.cpu().view(NB * page, Hkv, D)
    bits = torch.int32 if dtype == torch.float32 else torch.int16
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        assert torch.equal(kc_h[s].view(bits), k[t].cpu().view(bits))
        assert torch.equal(vc_h[s].view(bits), v[t].cpu().view(bits))
    n_written = int((~torch.isnan(kc_h[:, 0, 0].float())).sum())
    assert n_written == T - 1


def test_feeds_attention(pkg):
    """Prologue (store) then attention over the cache = prologue (no store) then the
    fused store + attention call."""
    from specdec_nanovllm_b200 import workloads
    B, n_q = 4, 7
    lens = [300, 1024, 77, 513]
    case = workloads.paged_case(lens, n_q, seed=5, max_blocks=4, **workloads.QWEN3_4B)
    Hq, Hkv, D = 32, 8, 128
    g = torch.Generator().manual_seed(9)
    qkv = (torch.randn(B * n_q, (Hq + 2 * Hkv) * D, generator=g) * 2).to(torch.bfloat16).cuda()
    qw = (torch.rand(D, generator=g) * 2).to(torch.bfloat16).cuda()
    kw = (torch.rand(D, generator=g) * 2).to(torch.bfloat16).cuda()
    bt = case.block_tables.cpu()
    pos, slots = [], []
    for b, L in enumerate(lens):
        for p_ in range(L - n_q, L):
            pos.append(p_)
            slots.append(int(bt[b, p_ // 256]) * 256 + p_ % 256)
    pos = torch.tensor(pos).cuda()
    sm = torch.tensor(slots, dtype=torch.int32).cuda()
    cs = pkg.rope_cos_sin_cache(D, 4096, 1e6)
    kc1, vc1 = case.k_cache.clone(), case.v_cache.clone()
    q1 = pkg.qk_norm_rope_store(qkv, pos, Hq, Hkv, D, cs, qw, kw, 1e-6, k_cache=kc1, v_cache=vc1, slot_mapping=sm)
    o1 = pkg.paged_attention(q1, kc1, vc1, case.block_tables, case.cache_seqlens, case.scale, n_q=n_q)
    kc2, vc2 = case.k_cache.clone(), case.v_cache.clone()
    q2, k2, v2 = pkg.qk_norm_rope_store(qkv, pos, Hq, Hkv, D, cs, qw, kw, 1e-6, return_kv=True)
    o2 = pkg.paged_attention(q2, kc2, vc2, case.block_tables, case.cache_seqlens, case.scale, n_q=n_q,
                             k_new=k2, v_new=v2, slot_mapping=sm)
    torch.cuda.synchronize()
    assert torch.equal(kc1.view(torch.int16), kc2.view(torch.int16))
    assert torch.equal(vc1.view(torch.int16), vc2.view(torch.int16))
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    assert pkg.attention.error_word() == 0
