"""verify_batch rejection sampling on the GPU.

Bar: accept/reject decisions, accepted lengths and emitted tokens bit-exact
against the reference (golden fixtures, identical injected draws) and against the
oracle at full configuration size (identical Philox draws).
"""

import numpy as np
import pytest
import torch

from oracle import philox
from oracle import verify as ov

pytestmark = pytest.mark.gpu

CASES = ["random", "temps", "all_accept", "point_mass", "k_rows_target", "align_all", "align_reject0"]


def _t(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("name", CASES)
def test_golden_injected_draws_bit_exact(pkg, golden, name):
    g = golden("verify_" + name)
    temps = _t(g["temps"]) if bool(g["has_temps"]) else None
    r = pkg.verify_batch(_t(g["draft"]), _t(g["target"]), _t(g["tokens"]), temps, bool(g["point"]),
                         uniforms=_t(g["u"]), exponentials=_t(g["e"]))
    torch.cuda.synchronize()
    assert np.array_equal(r.accepted.cpu().numpy(), g["accepted"])
    assert np.array_equal(r.accept_mask.cpu().numpy(), g["accept_mask"])
    assert np.array_equal(r.bonus.cpu().numpy(), g["bonus"])
    assert r.accepted.dtype == torch.int64 and r.bonus.dtype == torch.int64
    assert r.accept_mask.dtype == torch.bool


@pytest.mark.parametrize("name", ["random", "temps", "point_mass"])
def test_golden_inputs_with_in_kernel_philox_match_oracle(pkg, golden, name):
    """Same inputs, draws generated inside the kernel: equals the oracle fed the Philox streams."""
    g = golden("verify_" + name)
    B, k, V = g["draft"].shape
    temps = g["temps"] if bool(g["has_temps"]) else None
    seed, off = 1234567 + B, 42
    r = pkg.verify_batch(_t(g["draft"]), _t(g["target"]), _t(g["tokens"]),
                         _t(temps) if temps is not None else None, bool(g["point"]), seed=seed, offset=off)
    want = ov.verify_batch(g["draft"], g["target"], g["tokens"], temps, bool(g["point"]),
                           uniforms=philox.uniforms(seed, off, B, k),
                           exponentials=philox.exponentials(seed, off, B, V))
    torch.cuda.synchronize()
    assert np.array_equal(r.accepted.cpu().numpy(), want.accepted)
    assert np.array_equal(r.accept_mask.cpu().numpy(), want.accept_mask)
    assert np.array_equal(r.bonus.cpu().numpy(), want.bonus)


@pytest.mark.parametrize("stream_id,rows,cols", [(0, 64, 6), (1, 3, 151936), (1, 7, 1001)])
def test_philox_streams_bit_exact(pkg, stream_id, rows, cols):
    from specdec_nanovllm_b200.verify import philox_draws
    got = philox_draws(rows, cols, seed=0xDEADBEEF12345, offset=9, stream_id=stream_id).cpu().numpy()
    if stream_id == 0:
        want = philox.uniforms(0xDEADBEEF12345, 9, rows, cols)
    else:
        want = philox.exponentials(0xDEADBEEF12345, 9, rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_cfg4_full_size_bit_exact_against_oracle(pkg):
    """B=64, k=6, V=151936, target N(0,9), draft = target + N(0,1), T = 1, Philox draws."""
    from specdec_nanovllm_b200.workloads import cfg4_inputs
    draft, target, tokens = cfg4_inputs(seed=0)
    seed, off = 2024, 7
    r = pkg.verify_batch(draft, target, tokens, torch.ones(64, device="cuda"), seed=seed, offset=off)
    torch.cuda.synchronize()
    d, t, tk = draft.cpu().numpy(), target.cpu().numpy(), tokens.cpu().numpy()
    want = ov.verify_batch(d, t, tk, np.ones(64, np.float32), uniforms=philox.uniforms(seed, off, 64, 6),
                           exponentials=philox.exponentials(seed, off, 64, 151936))
    assert np.array_equal(r.accepted.cpu().numpy(), want.accepted)
    assert np.array_equal(r.accept_mask.cpu().numpy(), want.accept_mask)
    assert np.array_equal(r.bonus.cpu().numpy(), want.bonus)
    # sanity on the statistics: this draft is close to the target
    assert 1.0 < float(want.accepted.mean()) < 6.0


# ------------------------------------------------------------ the reference's known-answer tests
def test_ref_2A_q_equals_p_accepts_all(pkg):
    """tests/test_spec_decode.py:85-99."""
    torch.manual_seed(0)
    B, K, V = 1, 3, 20
    dl = torch.randn(B, K, V)
    probs = torch.softmax(dl[0], -1)
    tok = torch.stack([torch.multinomial(probs[j], 1).squeeze(0) for j in range(K)]).unsqueeze(0)
    r = pkg.verify_batch(dl.cuda(), dl.clone().cuda(), tok.cuda())   # k target rows, as the reference test
    assert int(r.accepted[0]) == K


def test_ref_2B_sharp_target_rejects_early(pkg):
    """tests/test_spec_decode.py:101-111."""
    B, K, V = 1, 3, 20
    dl = torch.zeros(B, K, V)
    tok = torch.zeros(B, K, dtype=torch.long)
    tl = torch.full((B, K + 1, V), -50.0)
    tl[:, :, 7] = 50.0
    dl[:, 0, 7] = 50.0
    r = pkg.verify_batch(dl.cuda(), tl.cuda(), tok.cuda())
    assert int(r.accepted[0]) <= 1


def test_ref_2C_bonus_in_residual_support(pkg):
    """tests/test_spec_decode.py:113-130: point-mass draft of 3, target peaked on 5."""
    N, K, V = 4000, 1, 20
    p = torch.full((V,), 1e-6)
    p[5] = 1.0
    logits = p.log().view(1, 1, V).expand(N, 2, V).contiguous()
    draft_tok = torch.full((N, K), 3, dtype=torch.long)
    dq = torch.zeros(N, K, V)
    dq.scatter_(2, draft_tok.unsqueeze(-1), 1.0)
    r = pkg.verify_batch(dq.cuda(), logits.cuda(), draft_tok.cuda(), draft_is_point_mass=True)
    counts = torch.bincount(r.bonus.cpu(), minlength=V)
    assert int(counts.argmax()) == 5
    assert bool((r.accepted == 0).all())


def _tv_at(pkg, probs, n, seed):
    V = probs.numel()
    g = torch.Generator().manual_seed(seed)
    tok = torch.multinomial(probs.expand(n, V), 1, replacement=True, generator=g)
    dq = torch.zeros(n, 1, V)
    dq.scatter_(2, tok.unsqueeze(-1), 1.0)
    tgt = probs.log().view(1, 1, V).expand(n, 2, V).contiguous()
    r = pkg.verify_batch(dq.cuda(), tgt.cuda(), tok.cuda(), draft_is_point_mass=True, seed=seed)
    final = torch.where(r.accepted.cpu() == 1, tok.squeeze(1), r.bonus.cpu())
    c = torch.bincount(final, minlength=V).float()
    c /= c.sum()
    return 0.5 * float((c - probs).abs().sum())


def test_ref_3_lossless_tv_shrinks_with_n(pkg):
    """tests/test_spec_decode.py:132-185: the output distribution equals p (TV ~ 1/sqrt(N))."""
    probs = torch.tensor([0.5, 0.2, 0.15, 0.05, 0.05, 0.05])
    small = np.mean([_tv_at(pkg, probs, 40_000, s) for s in range(5)])
    large = np.mean([_tv_at(pkg, probs, 400_000, 100 + s) for s in range(3)])
    assert small / large > 2.0 and large < 0.004, (small, large)


def test_ref_5_draft_logits_not_probs(pkg):
    """tests/test_spec_decode.py:239-277: q == p given logits -> accept everything, lossless."""
    V, N = 6, 200_000
    p5 = torch.tensor([0.5, 0.2, 0.15, 0.05, 0.05, 0.05])
    g = torch.Generator().manual_seed(0)
    cand = torch.multinomial(p5.expand(N, V), 1, replacement=True, generator=g)
    tgt = p5.log().view(1, 1, V).expand(N, 2, V).contiguous().cuda()

    def acc_tv(draft_side):
        r = pkg.verify_batch(draft_side.cuda(), tgt, cand.cuda(), seed=5)
        final = torch.where(r.accepted.cpu() == 1, cand.squeeze(1), r.bonus.cpu())
        h = torch.bincount(final, minlength=V).float()
        h /= h.sum()
        return float((r.accepted.cpu() == 1).float().mean()), 0.5 * float((h - p5).abs().sum())

    acc_lg, tv_lg = acc_tv(p5.log().view(1, 1, V).expand(N, 1, V).contiguous())
    acc_pr, tv_pr = acc_tv(p5.view(1, 1, V).expand(N, 1, V).contiguous())
    assert acc_lg > 0.999
    assert tv_lg < 0.01
    assert tv_pr > 5 * tv_lg


def test_ref_6_candidate_row_alignment(pkg):
    """tests/test_spec_decode.py:279-322."""
    K6, V6 = 3, 20
    tl6 = torch.full((1, K6 + 1, V6), -30.0)
    for j in range(K6 + 1):
        tl6[0, j, 10 + j] = 30.0
    dl6 = tl6[:, :K6].clone()
    r6 = pkg.verify_batch(dl6.cuda(), tl6.cuda(), torch.tensor([[10, 11, 12]]).cuda())
    assert int(r6.accepted[0]) == K6 and int(r6.bonus[0]) == 10 + K6
    dl7 = dl6.clone()
    dl7[0, 0, 10] = -30.0
    dl7[0, 0, 3] = 30.0
    r7 = pkg.verify_batch(dl7.cuda(), tl6.cuda(), torch.tensor([[3, 11, 12]]).cuda())
    assert int(r7.accepted[0]) == 0 and int(r7.bonus[0]) == 10


def test_ref_temp_broadcast_per_request(pkg):
    """tests/test_temp_broadcast.py section 2: per-request temperatures along the batch dim."""
    V, B, N = 5, 3, 30000
    p_base = torch.tensor([0.5, 0.2, 0.15, 0.1, 0.05])
    logits = p_base.log()
    temps = torch.tensor([0.25, 1.0, 0.5])
    cand = torch.full((N, 1), 1, dtype=torch.long)
    draft = torch.zeros(N, 1, V)
    draft.scatter_(2, cand.unsqueeze(-1), 1.0)
    target = logits.view(1, 1, V).expand(N, 2, V).contiguous()
    r = pkg.verify_batch(draft.cuda(), target.cuda(), cand.cuda(), temps.repeat(N // B).cuda(),
                         draft_is_point_mass=True, seed=7)
    acc = r.accept_mask.float().cpu().reshape(N // B, B).mean(dim=0)
    for i in range(B):
        want = float(torch.softmax(logits / temps[i], dim=-1)[1])
        assert abs(float(acc[i]) - want) < 0.02, (i, float(acc[i]), want)


def test_graph_capture_with_fixed_draws(pkg):
    from specdec_nanovllm_b200.workloads import cfg4_inputs
    draft, target, tokens = cfg4_inputs(B=8, V=32000, seed=3)
    out = pkg.verify_batch(draft, target, tokens, seed=1, offset=0)
    torch.cuda.synchronize()
    ref = (out.accepted.clone(), out.bonus.clone(), out.accept_mask.clone())
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            pkg.verify_batch(draft, target, tokens, seed=1, offset=0, out=out)
    torch.cuda.current_stream().wait_stream(s)
    out.accepted.zero_()
    out.bonus.zero_()
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.accepted, ref[0]) and torch.equal(out.bonus, ref[1])
    assert torch.equal(out.accept_mask, ref[2])
    del g


# ------------------------------------------------------------ 16-bit logits (no float32 copy)
@pytest.mark.parametrize("ddt,tdt", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                     (torch.float16, torch.float16), (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("V", [151936, 997, 4100])
def test_16bit_logits_equal_float32_path(pkg, ddt, tdt, V):
    """The engine passes the LM head's bf16 logits (model_runner.py:1101-1103) and the
    reference converts with .float(): decisions and tokens must equal the float32 path on
    the converted values bit for bit (V 997: scalar rows; 4100: V % 8 != 0, no bulk copy
    for 16-bit rows)."""
    g = torch.Generator().manual_seed(V + 3)
    B, k = 12, 5
    target = (torch.randn(B, k + 1, V, generator=g) * 3.0).to(tdt).cuda()
    draft = (target[:, :k].float() + torch.randn(B, k, V, generator=g).cuda()).to(ddt)
    tokens = torch.randint(0, V, (B, k), generator=g).cuda()
    temps = torch.linspace(0.6, 1.4, B).cuda()
    temps[0] = 1.0
    r16 = pkg.verify_batch(draft, target, tokens, temps, seed=77, offset=5)
    r32 = pkg.verify_batch(draft.float(), target.float(), tokens, temps, seed=77, offset=5)
    torch.cuda.synchronize()
    assert torch.equal(r16.accepted, r32.accepted)
    assert torch.equal(r16.accept_mask, r32.accept_mask)
    assert torch.equal(r16.bonus, r32.bonus)


def test_cfg4_bf16_target_full_size_against_oracle(pkg):
    """cfg4 with the target logits in bf16 as the LM head emits them."""
    from specdec_nanovllm_b200.workloads import cfg4_inputs
    draft, target, tokens = cfg4_inputs(seed=1)
    target = target.to(torch.bfloat16)
    seed, off = 99, 3
    r = pkg.verify_batch(draft, target, tokens, None, seed=seed, offset=off)
    torch.cuda.synchronize()
    want = ov.verify_batch(draft.cpu().numpy(), target.float().cpu().numpy(), tokens.cpu().numpy(), None,
                           uniforms=philox.uniforms(seed, off, 64, 6),
                           exponentials=philox.exponentials(seed, off, 64, 151936))
    assert np.array_equal(r.accepted.cpu().numpy(), want.accepted)
    assert np.array_equal(r.accept_mask.cpu().numpy(), want.accept_mask)
    assert np.array_equal(r.bonus.cpu().numpy(), want.bonus)


# ------------------------------------------------------------ vocabulary-parallel form
def _shards(V, tp):
    base, extra = divmod(V, tp)
    out, s = [], 0
    for r in range(tp):
        n = base + (1 if r < extra else 0)
        out.append((s, s + n))
        s += n
    return out


def _run_vp_emulated(pkg, draft, target, tokens, temps, point, tp, **kw):
    """All tp ranks' phases on one GPU, the all-gathers emulated by concatenation."""
    V = draft.shape[2]
    ranks = [pkg.VocabParallelVerify(draft[:, :, s:e], target[:, :, s:e], tokens, temps, point,
                                     vocab_start=s, vocab_size=V, tp=tp, **kw) for s, e in _shards(V, tp)]
    gathered = None
    for n in (1, 2, 3, 4):
        sends = [r.phase(n, gathered) for r in ranks]
        gathered = torch.cat(sends) if sends[0] is not None else None
    return [r.result for r in ranks]


@pytest.mark.parametrize("tp", [2, 3, 8])
@pytest.mark.parametrize("V,tdt,point", [(151936, torch.float32, False), (151936, torch.bfloat16, False),
                                         (997, torch.float32, False), (4100, torch.float32, True)])
def test_vocab_parallel_equals_single_device(pkg, tp, V, tdt, point):
    g = torch.Generator().manual_seed(V * 7 + tp)
    B, k = 16, 6
    target = (torch.randn(B, k + 1, V, generator=g) * 3.0).to(tdt).cuda()
    tokens = torch.randint(0, V, (B, k), generator=g).cuda()
    if point:
        draft = torch.zeros(B, k, V).scatter_(2, tokens.cpu().unsqueeze(-1), 1.0).cuda()
    else:
        draft = target[:, :k].float() + torch.randn(B, k, V, generator=g).cuda()
    temps = torch.linspace(0.7, 1.3, B).cuda()
    temps[3] = 1.0
    want = pkg.verify_batch(draft, target, tokens, temps, point, seed=5, offset=9)
    results = _run_vp_emulated(pkg, draft, target, tokens, temps, point, tp, seed=5, offset=9)
    torch.cuda.synchronize()
    for r in results:  # every rank holds the same result, equal to the single-device call
        assert torch.equal(r.accepted, want.accepted)
        assert torch.equal(r.accept_mask, want.accept_mask)
        assert torch.equal(r.bonus, want.bonus)
    assert 0 < int(want.accepted.sum()) < B * k or point


def test_vocab_parallel_injected_draws_match_oracle(pkg, golden):
    g = golden("verify_temps")
    B, k, V = g["draft"].shape
    res = _run_vp_emulated(pkg, _t(g["draft"]), _t(g["target"]), _t(g["tokens"]), _t(g["temps"]), False, 3,
                           seed=0, offset=0, uniforms=_t(g["u"]), exponentials=_t(g["e"]))
    torch.cuda.synchronize()
    for r in res:
        assert np.array_equal(r.accepted.cpu().numpy(), g["accepted"])
        assert np.array_equal(r.accept_mask.cpu().numpy(), g["accept_mask"])
        assert np.array_equal(r.bonus.cpu().numpy(), g["bonus"])


def test_device_offset_draws_equal_host_offset_and_advance_in_graphs(pkg):
    """sdb_verify_batch_dev_offset: the offset is read on the device and advanced after the
    call, so a captured call draws new values on every replay, each replay equal to the
    host-offset call at that offset."""
    from specdec_nanovllm_b200 import workloads
    draft, target, tokens = workloads.cfg4_inputs(B=8, k=6, V=4096, seed=21)
    off = torch.tensor([5], dtype=torch.int64, device="cuda")
    r = pkg.verify_batch(draft, target, tokens, None, seed=3, offset_tensor=off)
    w = pkg.verify_batch(draft, target, tokens, None, seed=3, offset=5)
    torch.cuda.synchronize()
    assert torch.equal(r.accepted, w.accepted) and torch.equal(r.bonus, w.bonus)
    assert torch.equal(r.accept_mask, w.accept_mask)
    assert int(off.item()) == 6
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            pkg.verify_batch(draft, target, tokens, None, seed=3, offset_tensor=off, out=r)
    torch.cuda.current_stream().wait_stream(st)
    for v in (6, 7, 8):
        g.replay()
        torch.cuda.synchronize()
        w = pkg.verify_batch(draft, target, tokens, None, seed=3, offset=v)
        torch.cuda.synchronize()
        assert torch.equal(r.accepted, w.accepted) and torch.equal(r.bonus, w.bonus), v
    assert int(off.item()) == 9
    del g
