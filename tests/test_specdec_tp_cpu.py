"""The tensor-parallel slices of the end-to-end step's random Qwen3 models (CPU).

Rank r of `tp` holds q heads [r Hq/tp, (r+1) Hq/tp) and the matching k and v heads of the
fused qkv weight, the same columns of o_proj, gate rows [r F/tp, ...) and up rows
[F + r F/tp, ...) of gate_up, the same columns of down_proj, and kv heads
[r Hkv/tp, ...) of each KV cache -- the Megatron split of the reference's
ColumnParallelLinear / QKVParallelLinear / MergedColumnParallelLinear /
RowParallelLinear (nanovllm/layers/linear.py:68-170).  The slices of all ranks put
back together are the single-device model with the same seed.
"""

import pytest
import torch


def _shape():
    from specdec_nanovllm_b200.specdec import Qwen3Shape
    return Qwen3Shape(layers=2, hidden=64, heads=8, kv_heads=4, ffn=96, vocab=50, head_dim=16)


@pytest.mark.parametrize("tp", [2, 4])
def test_slices_reassemble_the_single_device_weights(pkg, tp):
    from specdec_nanovllm_b200.specdec import RandomQwen3
    s = _shape()
    full = RandomQwen3(s, "cpu", seed=3, max_position=64)
    ranks = [RandomQwen3(s, "cpu", seed=3, max_position=64, tp_rank=r, tp_size=tp) for r in range(tp)]
    D, hq, hk, fl = s.head_dim, s.heads // tp * s.head_dim, s.kv_heads // tp * s.head_dim, s.ffn // tp
    for i, lw in enumerate(full.layers):
        parts = [m.layers[i] for m in ranks]
        q = torch.cat([p["qkv"][:hq] for p in parts])
        k = torch.cat([p["qkv"][hq:hq + hk] for p in parts])
        v = torch.cat([p["qkv"][hq + hk:] for p in parts])
        assert torch.equal(torch.cat([q, k, v]), lw["qkv"])
        assert torch.equal(torch.cat([p["o"] for p in parts], dim=1), lw["o"])
        gate = torch.cat([p["gate_up"][:fl] for p in parts])
        up = torch.cat([p["gate_up"][fl:] for p in parts])
        assert torch.equal(torch.cat([gate, up]), lw["gate_up"])
        assert torch.equal(torch.cat([p["down"] for p in parts], dim=1), lw["down"])
    for m in ranks:                       # replicated: embedding / tied LM head
        assert torch.equal(m.embed, full.embed)
        assert (m.heads, m.kv_heads) == (s.heads // tp, s.kv_heads // tp)


def test_caches_hold_the_rank_heads_and_bad_tp_is_rejected(pkg):
    from specdec_nanovllm_b200.specdec import RandomQwen3
    s = _shape()
    full = RandomQwen3(s, "cpu", seed=1, max_position=64)
    want = full.new_cache(3, 16, "cpu", seed=9)
    for r in range(2):
        m = RandomQwen3(s, "cpu", seed=1, max_position=64, tp_rank=r, tp_size=2)
        got = m.new_cache(3, 16, "cpu", seed=9)
        for (kc, vc), (kf, vf) in zip(got, want):
            assert torch.equal(kc, kf[:, :, 2 * r:2 * r + 2]) and torch.equal(vc, vf[:, :, 2 * r:2 * r + 2])
    with pytest.raises(ValueError):
        RandomQwen3(s, "cpu", seed=1, max_position=64, tp_rank=0, tp_size=3)


def test_forward_steps_yield_two_partial_sums_per_layer(pkg, monkeypatch):
    """The generator form of the forward yields the o_proj and down_proj partial sums of
    every layer, in order, and returns the final hidden states (the GPU kernels replaced
    by shape-preserving stand-ins, so only the control flow runs here)."""
    import specdec_nanovllm_b200.specdec as sd
    s = _shape()
    m = sd.RandomQwen3(s, "cpu", seed=2, max_position=64)
    T = 3
    monkeypatch.setattr(sd, "qk_norm_rope_store",
                        lambda qkv, pos, h, hk, d, *a, **k: qkv[:, :h * d].reshape(qkv.shape[0], h, d))
    monkeypatch.setattr(sd, "paged_attention", lambda q, *a, **k: q)
    monkeypatch.setattr(sd, "layer_rms_norm",
                        lambda x, w, eps, residual=None: x if residual is None else (x + residual, x + residual))
    monkeypatch.setattr(sd, "silu_and_mul", lambda gu: gu[:, :gu.shape[1] // 2])
    steps = m.forward_steps(torch.zeros(T, dtype=torch.long), None, None, None, None, 1, [(None, None)] * s.layers)
    shapes = []
    part = next(steps)
    try:
        while True:
            shapes.append(tuple(part.shape))
            part = steps.send(part)
    except StopIteration as done:
        out = done.value
    assert shapes == [(T, s.hidden)] * (2 * s.layers)
    assert out.shape == (T, s.hidden)
