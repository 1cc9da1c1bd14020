"""Paged decode / verify attention on the GPU against the CPU oracle and reference goldens.

Tolerances: bf16/fp16 rtol 2e-2 / atol 2e-3 (against the float64 oracle of the
same bf16 inputs); fp32 rtol 1e-5 / atol 1e-5.
"""

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.numerics import allclose_report, bf16_bits_to_f32

pytestmark = pytest.mark.gpu

BF16_TOL = dict(rtol=2e-2, atol=2e-3)
FP32_TOL = dict(rtol=1e-5, atol=1e-5)


def _oracle(case):
    return oatt.paged_attention(case.q.float().cpu().numpy(), case.k_cache.float().cpu().numpy(),
                                case.v_cache.float().cpu().numpy(), case.block_tables.cpu().numpy(),
                                case.cache_seqlens.cpu().numpy(), case.scale, n_q=case.n_q,
                                compute_dtype=np.float64)


def _check(got, want, tol):
    ok, err, viol = allclose_report(got.float().cpu().numpy(), want, **tol)
    assert ok, f"max abs err {err}, worst violation {viol}"


@pytest.fixture(autouse=True, params=["auto", "mma"])
def kernel_choice(request, monkeypatch):
    """Every test runs on the default kernel (tcgen05 where the shape allows) and on
    the mma.sync kernel (SDB_ATTN_KERNEL=mma)."""
    if request.param == "mma":
        monkeypatch.setenv("SDB_ATTN_KERNEL", "mma")
    else:
        monkeypatch.delenv("SDB_ATTN_KERNEL", raising=False)
    return request.param


@pytest.fixture(scope="module")
def W(pkg):
    from specdec_nanovllm_b200 import workloads
    return workloads


# ------------------------------------------------------------------ goldens
def test_golden_decode_fp32(pkg, golden):
    g = golden("attn_decode_fp32")
    dev = "cuda"
    out = pkg.paged_attention(torch.from_numpy(g["q"]).to(dev), torch.from_numpy(g["k_cache"]).to(dev),
                              torch.from_numpy(g["v_cache"]).to(dev),
                              torch.from_numpy(g["block_tables"]).to(dev),
                              torch.from_numpy(g["cache_seqlens"]).to(dev), float(g["scale"]), n_q=1)
    torch.cuda.synchronize()
    _check(out, g["out"], FP32_TOL)


@pytest.mark.parametrize("n_q", [1, 4])
def test_golden_bf16(pkg, golden, n_q):
    g = golden(f"attn_bf16_nq{n_q}")
    dev = "cuda"

    def t(bits):
        return torch.from_numpy(bf16_bits_to_f32(bits)).to(torch.bfloat16).to(dev)

    out = pkg.paged_attention(t(g["q"]), t(g["k_cache"]), t(g["v_cache"]),
                              torch.from_numpy(g["block_tables"]).to(dev),
                              torch.from_numpy(g["cache_seqlens"]).to(dev), float(g["scale"]), n_q=n_q)
    torch.cuda.synchronize()
    _check(out, g["out_f32"], BF16_TOL)


# ------------------------------------------------------------------ configs
def test_cfg1_decode_fp32(pkg, W):
    case = W.cfg1_case(seed=0)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=1)
    torch.cuda.synchronize()
    _check(out, _oracle(case), FP32_TOL)


_CFG2_CACHE = {}


def _cfg2_case_and_oracle(W, B, ctx, n_q):
    """Inputs and float64 oracle output of one cfg2 point, shared by both kernel choices."""
    key = (B, ctx, n_q)
    if key not in _CFG2_CACHE:  # all 24 points together hold about 6 GB of device memory
        lens = W.cfg2_lens(B, ctx, seed=B + ctx)
        case = W.paged_case(lens, n_q, seed=ctx + n_q, max_blocks=ctx // 256, generate_on_device=B >= 32,
                            **W.QWEN3_4B)
        _CFG2_CACHE[key] = (case, _oracle(case))
    return _CFG2_CACHE[key]


@pytest.mark.parametrize("ctx", [512, 2048, 4096])
@pytest.mark.parametrize("B", [1, 8, 32, 64])
@pytest.mark.parametrize("n_q", [7, 1])
def test_cfg2_verify_and_decode(pkg, W, B, ctx, n_q, kernel_choice):
    """The whole cfg2 grid (B x ctx, verify k=6 and decode), every sequence against the
    float64 oracle, on both kernels; the launch plan of each point is recorded."""
    case, want = _cfg2_case_and_oracle(W, B, ctx, n_q)
    kind, slots, _ = pkg.attention.plan(B, n_q, 32, 8, 128, 256, ctx // 256, torch.bfloat16)
    assert kind == ("mma" if kernel_choice == "mma" else kind)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=n_q)
    torch.cuda.synchronize()
    _check(out, want, BF16_TOL)


# one shape per decomposition of the tcgen05 plan (B200, 148 SMs): strided with 1, 2 and
# >= 3 key chunks per (sequence, kv head), and the balanced grouped partition
_PLAN_SHAPES = [
    ("tcgen05_strided", 1, 16, 4096),
    ("tcgen05_strided", 2, 8, 2048),
    ("tcgen05_strided", 3, 5, 2048),
    ("tcgen05_strided", 11, 1, 4096),
    ("tcgen05_grouped", 4, 1, 512),
    ("tcgen05_grouped", 5, 5, 4096),
    ("tcgen05_grouped", 3, 10, 2048),
    ("tcgen05_grouped", 2, 24, 4096),
]


@pytest.mark.parametrize("want_kind,want_slots,B,ctx", _PLAN_SHAPES)
@pytest.mark.parametrize("n_q", [7, 1])
def test_each_umma_plan_outcome(pkg, W, want_kind, want_slots, B, ctx, n_q, kernel_choice):
    if kernel_choice == "mma":
        pytest.skip("plan outcomes of the tcgen05 kernel")
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("the plan table is for 148 SMs")
    kind, slots, _ = pkg.attention.plan(B, n_q, 32, 8, 128, 256, ctx // 256, torch.bfloat16)
    assert (kind, slots) == (want_kind, want_slots)
    lens = W.cfg2_lens(B, ctx, seed=7 * B + ctx)
    lens[-1] = ctx  # the longest sequence spans every split / group boundary
    case = W.paged_case(lens, n_q, seed=B * ctx + n_q, max_blocks=ctx // 256, **W.QWEN3_4B)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=n_q)
    torch.cuda.synchronize()
    _check(out, _oracle(case), BF16_TOL)


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 16])
def test_any_split_count(pkg, W, splits):
    lens = [2048, 2047, 1, 256, 1025, 7]
    case = W.paged_case(lens, 7, seed=splits, max_blocks=8, **W.QWEN3_4B)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=7, splits=splits)
    torch.cuda.synchronize()
    _check(out, _oracle(case), BF16_TOL)


@pytest.mark.parametrize("Hq,Hkv,n_q", [(16, 8, 1), (16, 8, 7), (32, 8, 2), (8, 8, 5), (64, 8, 8),
                                        (4, 1, 7), (32, 4, 7)])
def test_gqa_groups_and_row_counts(pkg, W, Hq, Hkv, n_q):
    lens = [300, 256, 9, 1000]
    case = W.paged_case(lens, n_q, Hq=Hq, Hkv=Hkv, D=128, seed=Hq * 10 + n_q, max_blocks=4)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=n_q)
    torch.cuda.synchronize()
    _check(out, _oracle(case), BF16_TOL)


def test_fp16_and_page_512(pkg, W):
    lens = [700, 512, 33]
    case = W.paged_case(lens, 7, page=512, dtype=torch.float16, seed=5, max_blocks=2, **W.QWEN3_4B)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=7)
    torch.cuda.synchronize()
    _check(out, _oracle(case), BF16_TOL)


def test_edge_lengths_zero_and_shorter_than_window(pkg, W):
    # L = 0 (graph pad row), L < n_q (rows with no visible key), L = 1, exact pages
    lens = [0, 3, 1, 256, 512, 0, 6]
    case = W.paged_case(lens, 7, seed=11, max_blocks=2, **W.QWEN3_4B)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=7)
    torch.cuda.synchronize()
    want = _oracle(case)
    _check(out, want, BF16_TOL)
    o = out.float().cpu()
    assert torch.all(o[0:7] == 0) and torch.all(o[35:42] == 0)       # L = 0 sequences
    assert torch.all(o[7:7 + 4] == 0)                                 # L=3: rows 0..3 see nothing
    assert torch.isfinite(o).all()


def test_pad_rows_block_zero_ctx_zero(pkg, W):
    """Graph padding rule (graph_pad.py:33-69): block table row of zeros, ctx 0 -> zeros, no NaN."""
    case = W.paged_case([500, 1], 7, seed=2, max_blocks=2, **W.QWEN3_4B)
    bt = torch.cat([case.block_tables, torch.zeros(2, 2, dtype=torch.int32, device="cuda")])
    cl = torch.cat([case.cache_seqlens, torch.zeros(2, dtype=torch.int32, device="cuda")])
    q = torch.cat([case.q, torch.randn(14, 32, 128, device="cuda").to(torch.bfloat16)])
    out = pkg.paged_attention(q, case.k_cache, case.v_cache, bt, cl, case.scale, n_q=7)
    torch.cuda.synchronize()
    assert torch.all(out[14:] == 0)
    _check(out[:14], _oracle(case), BF16_TOL)


def test_head_major_layout(pkg, W):
    case = W.paged_case([400, 77], 1, seed=8, max_blocks=2, **W.QWEN3_4B)
    k_hm = case.k_cache.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    v_hm = case.v_cache.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    out = pkg.paged_attention(case.q, k_hm, v_hm, case.block_tables, case.cache_seqlens, case.scale)
    torch.cuda.synchronize()
    _check(out, _oracle(case), BF16_TOL)


# ------------------------------------------------------------------ properties at full size
def test_full_size_verify_rows_equal_truncated_decodes(pkg, W):
    """B=64, ctx=4096, k=6: verify row r equals a decode of length L-6+r (the causal rule)
    to within one bf16 ulp (decode and verify slice the keys of a tile differently, so
    their fp32 summation orders differ), and all 64 sequences match the oracle."""
    B, ctx, n_q = 64, 4096, 7
    case = W.paged_case([ctx] * B, n_q, seed=1, generate_on_device=True, extra_blocks=0, **W.QWEN3_4B)
    out = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                              case.scale, n_q=n_q)
    qv = case.q.view(B, n_q, 32, 128)
    splits = pkg.attention.default_splits(B, n_q, 32, 8, 128, 256, 16, torch.bfloat16)
    for r in range(n_q):
        lens_r = case.cache_seqlens - (n_q - 1) + r
        dec = pkg.paged_attention(qv[:, r].contiguous(), case.k_cache, case.v_cache, case.block_tables,
                                  lens_r, case.scale, n_q=1, splits=splits)
        ver = out.view(B, n_q, 32, 128)[:, r]
        assert torch.allclose(dec.float(), ver.float(), rtol=1e-2, atol=1e-4), f"row {r}"
    _check(out, _oracle(case), BF16_TOL)  # every sequence against the float64 oracle


def test_block_placement_invariance_and_determinism(pkg, W):
    case = W.paged_case([3000, 1234, 4096, 17], 7, seed=4, max_blocks=16, **W.QWEN3_4B)
    out1 = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                               case.scale, n_q=7)
    out2 = pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                               case.scale, n_q=7)
    # move every block to a new physical slot (reverse the pool) -> identical bits
    NB = case.k_cache.shape[0]
    perm = torch.arange(NB - 1, -1, -1, device="cuda")
    k2 = case.k_cache[perm]
    v2 = case.v_cache[perm]
    bt2 = torch.where(case.block_tables >= 0, NB - 1 - case.block_tables, case.block_tables)
    out3 = pkg.paged_attention(case.q, k2, v2, bt2.to(torch.int32), case.cache_seqlens, case.scale, n_q=7)
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)
    assert torch.equal(out1, out3)


def test_cuda_graph_capture_and_replay(pkg, W):
    case = W.paged_case([1500, 800], 7, seed=6, max_blocks=8, **W.QWEN3_4B)
    out = torch.empty_like(case.q)
    pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                        case.scale, n_q=7, out=out)  # sizes the workspace
    torch.cuda.synchronize()
    ref = out.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                                case.scale, n_q=7, out=out)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # new lengths through the same graph (device data only; shorter, so every key is written data)
    case.cache_seqlens.copy_(torch.tensor([700, 513], dtype=torch.int32))
    g.replay()
    torch.cuda.synchronize()
    _check(out, _oracle(case), BF16_TOL)
    del g


def test_invalid_block_ids_are_flagged_not_faulted(pkg, W):
    from specdec_nanovllm_b200 import _lib
    case = W.paged_case([600], 1, seed=3, max_blocks=3, **W.QWEN3_4B)
    bt = case.block_tables.clone()
    bt[0, 1] = 10_000_000            # outside the pool: the kernel clamps to block 0 and flags it
    pkg.attention.clear_error_word()
    pkg.paged_attention(case.q, case.k_cache, case.v_cache, bt, case.cache_seqlens, case.scale, splits=1)
    torch.cuda.synchronize()
    assert pkg.attention.error_word() & _lib.SDB_KERR_BLOCK_ID
    pkg.attention.clear_error_word()
    cl = torch.tensor([10_000], dtype=torch.int32, device="cuda")  # longer than the table holds
    pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, cl, case.scale, splits=1)
    torch.cuda.synchronize()
    assert pkg.attention.error_word() & _lib.SDB_KERR_SEQLEN
    pkg.attention.clear_error_word()


def test_host_rejects_bad_arguments(pkg, W):
    case = W.paged_case([100], 7, seed=3, max_blocks=1, **W.QWEN3_4B)
    with pytest.raises(ValueError):
        pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                            case.scale, n_q=6)            # 7 rows for B=1 is not B*n_q
    with pytest.raises(ValueError):
        pkg.paged_attention(case.q.float(), case.k_cache, case.v_cache, case.block_tables,
                            case.cache_seqlens, case.scale, n_q=7)


def test_readonly_twin_runs(pkg, W):
    case = W.paged_case([2048] * 4, 7, seed=9, max_blocks=8, **W.QWEN3_4B)
    pkg.paged_attention_readonly(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens, n_q=7)
    torch.cuda.synchronize()
    assert pkg.attention.error_word(kind="attention_ro") == 0


# ------------------------------------------------------------------ module mirrors
def test_store_kvcache_and_attention_module_verify_step(pkg, W):
    """One verify step through the Attention module: store k+1 new rows, attend with
    cu_seqlens metadata as prepare_verify builds it (model_runner.py:522-548)."""
    from specdec_nanovllm_b200 import context as ctx
    torch.manual_seed(0)
    B, n_q, Hq, Hkv, D, page = 3, 7, 32, 8, 128, 256
    lens_before = [300, 256 - 7, 1000]        # confirmed tokens already in cache
    lens = [L + n_q for L in lens_before]
    case = W.paged_case(lens, n_q, seed=21, max_blocks=5, **W.QWEN3_4B)
    k_new = torch.randn(B * n_q, Hkv, D, device="cuda").to(torch.bfloat16)
    v_new = torch.randn(B * n_q, Hkv, D, device="cuda").to(torch.bfloat16)
    slots = []
    bt = case.block_tables.cpu()
    for b in range(B):
        for pos in range(lens_before[b], lens[b]):
            slots.append(int(bt[b, pos // page]) * page + pos % page)
    slots[3] = -1                              # a skipped row keeps the old cache content
    slot_mapping = torch.tensor(slots, dtype=torch.int32, device="cuda")
    kc = case.k_cache.clone()
    vc = case.v_cache.clone()
    attn = pkg.Attention(Hq, D, case.scale, Hkv)
    attn.k_cache, attn.v_cache = kc, vc
    cu_q = torch.arange(0, (B + 1) * n_q, n_q, dtype=torch.int32, device="cuda")
    cu_k = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    ctx.set_context(True, cu_q, cu_k, n_q, max(lens), slot_mapping, None, case.block_tables,
                    is_spec_verify=True)
    try:
        out = attn(case.q, k_new, v_new)
    finally:
        ctx.reset_context()
    torch.cuda.synchronize()
    # expected cache: the stored rows land at their slots (except the skipped one)
    kexp = case.k_cache.clone().view(-1, Hkv, D)
    vexp = case.v_cache.clone().view(-1, Hkv, D)
    for i, s in enumerate(slots):
        if s >= 0:
            kexp[s] = k_new[i]
            vexp[s] = v_new[i]
    # bit comparison (the pool holds NaN in never-written slots)
    assert torch.equal(kc.view(-1, Hkv, D).view(torch.int16), kexp.view(torch.int16))
    assert torch.equal(vc.view(-1, Hkv, D).view(torch.int16), vexp.view(torch.int16))
    want = oatt.paged_attention(case.q.float().cpu().numpy(), kexp.view_as(kc).float().cpu().numpy(),
                                vexp.view_as(vc).float().cpu().numpy(), case.block_tables.cpu().numpy(),
                                np.array(lens, dtype=np.int32), case.scale, n_q=n_q, compute_dtype=np.float64)
    _check(out, want, BF16_TOL)


def test_attention_module_decode_and_reference_mirrors(pkg, W):
    from specdec_nanovllm_b200 import context as ctx
    case = W.paged_case([513, 64], 1, seed=31, max_blocks=3, **W.QWEN3_06B)
    want = _oracle(case)
    attn = pkg.Attention(16, 128, case.scale, 8)
    attn.k_cache, attn.v_cache = case.k_cache, case.v_cache
    kv = torch.zeros(2, 8, 128, dtype=torch.bfloat16, device="cuda")
    skip = torch.full((2,), -1, dtype=torch.int32, device="cuda")   # graph-pad slots: nothing written
    ctx.set_context(False, slot_mapping=skip, context_lens=case.cache_seqlens, block_tables=case.block_tables)
    try:
        o = attn(case.q, kv, kv)
        ctx.set_context(False, slot_mapping=skip[:1], context_lens=case.cache_seqlens[:1],
                        block_tables=case.block_tables[:1])
        o1 = attn(case.q[:1].reshape(16, 128), kv[:1], kv[:1])  # batch-1 (Hq, D) form
    finally:
        ctx.reset_context()
    torch.cuda.synchronize()
    assert o.shape == (2, 1, 16, 128)
    _check(o.view(2, 16, 128), want, BF16_TOL)
    o_ref_api = pkg.paged_decode_attention(case.q, case.k_cache, case.v_cache, case.block_tables,
                                           case.cache_seqlens, case.scale)
    o_cuda_api = pkg.paged_decode_attention_cuda(case.q, case.k_cache, case.v_cache, case.block_tables,
                                                 case.cache_seqlens, case.scale, splits=4)
    torch.cuda.synchronize()
    _check(o_ref_api, want, BF16_TOL)
    _check(o_cuda_api, want, BF16_TOL)
    assert o1.shape == (1, 1, 16, 128)
    _check(o1.view(1, 16, 128), want[:1], BF16_TOL)


# ------------------------------------------------------------------ fused store + attention
def _own_slots(case, n_q, page=256):
    """slot_mapping as prepare_decode / prepare_verify build it (model_runner.py:469-476,
    :537-548): token i of sequence b -> the slot of position L_b - n_q + i."""
    bt = case.block_tables.cpu()
    slots = []
    for b, L in enumerate(case.cache_seqlens.cpu().tolist()):
        for pos in range(L - n_q, L):
            slots.append(int(bt[b, pos // page]) * page + pos % page if pos >= 0 else -1)
    return slots


def _fused_vs_separate(pkg, case, slots, splits=0, seed=5):
    """The fused call must leave the same cache bits and return the same output bits as
    store_kvcache followed by paged_attention with the same split count."""
    n_q, (total, Hq, D) = case.n_q, case.q.shape
    Hkv = case.k_cache.shape[2]
    g = torch.Generator(device="cpu").manual_seed(seed)
    k_new = torch.randn(total, Hkv, D, generator=g).to(case.q.dtype).cuda()
    v_new = torch.randn(total, Hkv, D, generator=g).to(case.q.dtype).cuda()
    sm = torch.tensor(slots, dtype=torch.int32, device="cuda")
    kc1, vc1 = case.k_cache.clone(), case.v_cache.clone()
    kc2, vc2 = case.k_cache.clone(), case.v_cache.clone()
    pkg.store_kvcache(k_new, v_new, kc1, vc1, sm)
    want = pkg.paged_attention(case.q, kc1, vc1, case.block_tables, case.cache_seqlens, case.scale,
                               n_q=n_q, splits=splits)
    got = pkg.paged_attention(case.q, kc2, vc2, case.block_tables, case.cache_seqlens, case.scale,
                              n_q=n_q, splits=splits, k_new=k_new, v_new=v_new, slot_mapping=sm)
    torch.cuda.synchronize()
    bits = torch.int32 if case.q.dtype == torch.float32 else torch.int16
    assert torch.equal(kc1.view(bits), kc2.view(bits)), "K cache differs"
    assert torch.equal(vc1.view(bits), vc2.view(bits)), "V cache differs"
    assert torch.equal(want.view(bits), got.view(bits)), "attention output differs"
    return got, kc2, vc2


@pytest.mark.parametrize("splits", [0, 1, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_store_verify(pkg, W, splits, dtype):
    # new positions inside one tile, across a 128-key tile edge, across a page edge,
    # fewer keys than new tokens (L < n_q), L == n_q, and a long sequence
    lens = [300, 131, 260, 3, 7, 1500]
    case = W.paged_case(lens, 7, seed=41, max_blocks=6, dtype=dtype, **W.QWEN3_4B)
    slots = _own_slots(case, 7)
    slots[2] = -1  # a skipped row keeps the old cache content
    used = set(case.block_tables.flatten().tolist())
    spare = [b for b in range(case.k_cache.shape[0]) if b not in used][0]
    for i in range(4):  # the L = 3 sequence's tokens at negative positions are still stored
        slots[3 * 7 + i] = spare * 256 + 9 * i
    _fused_vs_separate(pkg, case, slots, splits=splits)
    assert pkg.attention.error_word() == 0


def test_fused_store_decode(pkg, W):
    case = W.paged_case([513, 64, 1, 256, 257], 1, seed=43, max_blocks=3, **W.QWEN3_06B)
    slots = _own_slots(case, 1)
    slots[3] = -1
    _fused_vs_separate(pkg, case, slots)
    assert pkg.attention.error_word() == 0


def test_fused_store_empty_sequence_and_fp32(pkg, W):
    """L = 0: the row has no position (nothing reads it) but is still stored, as
    store_kvcache would; fp32 runs the store kernel + CUDA-core path."""
    for dtype in (torch.bfloat16, torch.float32):
        case = W.paged_case([0, 40, 0], 1, seed=44, max_blocks=2, extra_blocks=2, dtype=dtype,
                            **W.QWEN3_06B)
        used = set(case.block_tables.flatten().tolist())
        spare = [b for b in range(case.k_cache.shape[0]) if b not in used]
        slots = _own_slots(case, 1)
        slots[0] = spare[0] * 256 + 5
        slots[2] = spare[1] * 256 + 255
        got, _, _ = _fused_vs_separate(pkg, case, slots)
        assert torch.count_nonzero(got[0].float()) == 0 and torch.count_nonzero(got[2].float()) == 0
        assert pkg.attention.error_word() == 0


def test_fused_store_foreign_slot_flags(pkg, W, kernel_choice):
    """A slot that is not the position's own is written (store semantics) and, on the
    tcgen05 path, reported with SDB_KERR_SLOT; the attention reads the position's own
    slot, exactly as a separate store followed by attention does."""
    case = W.paged_case([200, 90], 4, seed=45, max_blocks=1, extra_blocks=1, **W.QWEN3_4B)
    used = set(case.block_tables.flatten().tolist())
    spare = [b for b in range(case.k_cache.shape[0]) if b not in used][0]
    slots = _own_slots(case, 4)
    slots[1] = spare * 256 + 17
    try:
        _fused_vs_separate(pkg, case, slots)
        err = pkg.attention.error_word()
        assert err == (0x10 if kernel_choice == "auto" else 0)
    finally:
        pkg.attention.clear_error_word()
