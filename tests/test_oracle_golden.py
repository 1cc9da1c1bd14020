"""Pin the CPU oracle to outputs of the reference's own code (fixtures in tests/golden/)."""

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import philox
from oracle import quant as oq
from oracle import verify as ov
from oracle.numerics import allclose_report, bf16_bits_to_f32, f32_to_bf16_bits


def test_attention_decode_fp32_matches_reference(golden):
    g = golden("attn_decode_fp32")
    out = oatt.paged_attention(g["q"], g["k_cache"], g["v_cache"], g["block_tables"],
                               g["cache_seqlens"], float(g["scale"]), n_q=1,
                               compute_dtype=np.float64)
    ok, err, _ = allclose_report(out, g["out"], rtol=1e-5, atol=1e-5)
    assert ok, err
    assert np.all(out[0] == 0)                       # L = 0 row is exactly zero


@pytest.mark.parametrize("n_q", [1, 4])
def test_attention_bf16_decode_and_verify_match_reference(golden, n_q):
    g = golden(f"attn_bf16_nq{n_q}")
    q = bf16_bits_to_f32(g["q"])
    k = bf16_bits_to_f32(g["k_cache"])
    v = bf16_bits_to_f32(g["v_cache"])
    out = oatt.paged_attention(q, k, v, g["block_tables"], g["cache_seqlens"],
                               float(g["scale"]), n_q=n_q, compute_dtype=np.float64)
    ok, err, _ = allclose_report(out, g["out_f32"], rtol=1e-5, atol=1e-5)
    assert ok, err
    # The reference's bf16 output is its fp32 result rounded once to bf16.
    ok, err, _ = allclose_report(bf16_bits_to_f32(f32_to_bf16_bits(out.astype(np.float32))),
                                 bf16_bits_to_f32(g["out_bf16"]), rtol=1e-2, atol=1e-3)
    assert ok, err


@pytest.mark.parametrize("name,n_q", [("attn_decode_fp32", 1), ("attn_bf16_nq1", 1), ("attn_bf16_nq4", 4)])
def test_torch_restatement_matches_reference(golden, name, n_q):
    """The torch restatement bench.py times as the CPU baseline reproduces the reference."""
    import torch
    from oracle.torch_ref import paged_attention_torch
    g = golden(name)
    conv = (lambda a: torch.from_numpy(bf16_bits_to_f32(a))) if "bf16" in name else torch.from_numpy
    out = paged_attention_torch(conv(g["q"]), conv(g["k_cache"]), conv(g["v_cache"]),
                                torch.from_numpy(g["block_tables"]), torch.from_numpy(g["cache_seqlens"]),
                                float(g["scale"]), n_q=n_q)
    want = g["out"] if "out" in g else g["out_f32"]
    ok, err, _ = allclose_report(out.numpy(), want, rtol=1e-5, atol=1e-5)
    assert ok, err


def test_visible_keys_rule():
    # bottom-right causal: last row sees everything, row r sees L-n+r+1 keys
    assert [oatt.visible_keys(10, 4, r) for r in range(4)] == [7, 8, 9, 10]
    assert [oatt.visible_keys(2, 4, r) for r in range(4)] == [0, 0, 1, 2]
    assert oatt.visible_keys(0, 1, 0) == 0


@pytest.mark.parametrize("gran,gs", [("per_channel", 128), ("per_group", 64)])
def test_quantize_matches_reference(golden, gran, gs):
    g = golden("quant")
    q, s = oq.quantize_weight(g["w"], gran, gs)
    assert np.array_equal(q, g[f"{gran}_q"])                       # bit-exact int8
    assert np.array_equal(f32_to_bf16_bits(s), g[f"{gran}_scale"])  # bit-exact bf16 scale
    deq = oq.dequantize_weight(q, s, gran, gs)
    assert np.array_equal(deq, g[f"{gran}_deq"])
    x = bf16_bits_to_f32(g["x"])
    y = oq.int8_linear(x, q, s, granularity=gran, group_size=gs, dtype=np.float64)
    ok, err, _ = allclose_report(y, g[f"{gran}_y"], rtol=1e-5, atol=1e-4)
    assert ok, err


VERIFY_CASES = ["random", "temps", "all_accept", "point_mass", "k_rows_target",
                "align_all", "align_reject0"]


@pytest.mark.parametrize("name", VERIFY_CASES)
def test_verify_batch_matches_reference(golden, name):
    g = golden("verify_" + name)
    temps = g["temps"] if bool(g["has_temps"]) else None
    r = ov.verify_batch(g["draft"], g["target"], g["tokens"], temps, bool(g["point"]),
                        uniforms=g["u"], exponentials=g["e"])
    assert np.array_equal(r.accepted, g["accepted"])
    assert np.array_equal(r.accept_mask, g["accept_mask"])
    assert np.array_equal(r.bonus, g["bonus"])


def test_fixture_draws_are_the_philox_streams(golden):
    g = golden("verify_random")
    B, k = g["u"].shape
    V = g["e"].shape[1]
    seed = int(g["seed"])
    assert np.array_equal(philox.uniforms(seed, 0, B, k), g["u"])
    assert np.array_equal(philox.exponentials(seed, 0, B, V), g["e"])


@pytest.mark.parametrize("name", ["random", "bf16_chunks", "ragged_vocab", "peaked", "ties"])
def test_sampler_matches_reference(golden, name):
    """oracle.sampler against the reference's Sampler.forward with the same injected noise."""
    from oracle import sampler as osm
    g = golden(f"sampler_{name}")
    logits = bf16_bits_to_f32(g["logits"]) if bool(g["is_bf16"]) else g["logits"]
    tok = osm.sample(logits, g["temps"], exponentials=g["e"])
    assert np.array_equal(tok, g["tokens"])
    if name != "ties":  # the stored noise is the sampler's Philox stream
        e = philox.exponentials(int(g["seed"]), 0, *logits.shape, stream=philox.STREAM_SAMPLE)
        assert np.array_equal(e.view(np.uint32), g["e"].view(np.uint32))


def test_prologue_matches_reference(golden):
    """oracle.prologue against the reference's RMSNorm + RotaryEmbedding (qwen3.py:82-85)."""
    from oracle import prologue as op
    g = golden("prologue_qwen3")
    Hq, Hkv, D = int(g["Hq"]), int(g["Hkv"]), int(g["D"])
    qkv = bf16_bits_to_f32(g["qkv"])
    T = qkv.shape[0]
    # a table holding only the rows the positions use (anything else would be NaN)
    cs = np.full((int(g["max_position"]), D), np.nan, dtype=np.float32)
    cs[g["positions"]] = g["cos_sin_rows"]
    q, k, v = op.qk_prologue(qkv, g["positions"], Hq, Hkv, D, cs, bf16_bits_to_f32(g["q_norm_w"]),
                             bf16_bits_to_f32(g["k_norm_w"]), float(g["eps"]), "bf16")
    for got, key in ((q, "q"), (k, "k"), (v, "v")):
        want = bf16_bits_to_f32(g[key]).reshape(got.shape)
        # the mean of squares is summed in another order than torch's: at most one
        # bf16 ulp apart, on a small fraction of the elements
        ok, err, _ = allclose_report(got, want, rtol=1e-2, atol=1e-3)
        assert ok, (key, err)
        assert np.mean(got == want) > 0.98, key


def test_rope_table_matches_reference(golden, pkg):
    g = golden("prologue_qwen3")
    cs = pkg.rope_cos_sin_cache(int(g["D"]), int(g["max_position"]), float(g["rope_base"]), device="cpu")
    assert np.array_equal(cs.numpy()[g["positions"]].view(np.uint32), g["cos_sin_rows"].view(np.uint32))
