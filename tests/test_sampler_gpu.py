"""Token sampling (Sampler / draft step) on the GPU.

Bar: sampled tokens bit-exact against the reference's ``Sampler.forward`` (golden
fixtures, identical injected noise) and against the oracle with identical Philox
noise (stream 2) up to the full draft size (B=64, V=151936); the fp32 logits copy
bit-exact.
"""

import numpy as np
import pytest
import torch

from oracle import philox
from oracle import sampler as osm
from oracle.numerics import bf16_bits_to_f32

pytestmark = pytest.mark.gpu

GOLDEN = ["random", "bf16_chunks", "ragged_vocab", "peaked", "ties"]


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("name", GOLDEN)
def test_golden_injected_noise(pkg, golden, name):
    g = golden("sampler_" + name)
    if bool(g["is_bf16"]):
        logits = _t(bf16_bits_to_f32(g["logits"])).to(torch.bfloat16)
    else:
        logits = _t(g["logits"])
    tok = pkg.sample(logits, _t(g["temps"]), exponentials=_t(g["e"]))
    torch.cuda.synchronize()
    assert tok.dtype == torch.int64
    assert np.array_equal(tok.cpu().numpy(), g["tokens"])


def _oracle_philox(logits, temps, seed, offset):
    x = logits.float().cpu().numpy()
    e = philox.exponentials(seed, offset, *x.shape, stream=philox.STREAM_SAMPLE)
    return osm.sample(x, None if temps is None else temps.cpu().numpy(), exponentials=e)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,V", [(3, 997), (5, 8192 * 3), (4, 16389), (7, 151936)])
def test_philox_noise_matches_oracle(pkg, dtype, B, V):
    g = torch.Generator().manual_seed(B * 131 + V)
    logits = (torch.randn(B, V, generator=g) * 3.0).to(dtype).cuda()
    temps = torch.linspace(0.5, 1.5, B).cuda()
    temps[0] = 1.0
    for seed, off in ((5, 0), (2**40 + 3, 17)):
        tok = pkg.sample(logits, temps, seed=seed, offset=off)
        torch.cuda.synchronize()
        assert np.array_equal(tok.cpu().numpy(), _oracle_philox(logits, temps, seed, off))


def test_full_draft_size_and_logits_copy(pkg):
    """B=64 rows of the Qwen3 vocabulary, bf16 logits as the LM head emits them, written
    into strided (B, k, V) / (B, k) buffers like the draft proposer's."""
    B, V, k, s = 64, 151936, 6, 2
    gd = torch.Generator(device="cuda").manual_seed(7)
    logits = (torch.randn(B, V, generator=gd, device="cuda") * 3.0).to(torch.bfloat16)
    temps = torch.ones(B, 1, device="cuda")
    out_logits = torch.full((B, k, V), float("nan"), device="cuda")
    cands = torch.full((B, k), -1, dtype=torch.int64, device="cuda")
    nxt = pkg.draft_sample_step(logits, temps, out_logits, cands, s, seed=11, offset=3)
    torch.cuda.synchronize()
    assert torch.equal(out_logits[:, s], logits.float())
    assert torch.isnan(out_logits[:, :s]).all() and torch.isnan(out_logits[:, s + 1:]).all()
    assert (cands[:, :s] == -1).all() and (cands[:, s + 1:] == -1).all()
    assert nxt.data_ptr() == cands[:, s].data_ptr()
    assert np.array_equal(cands[:, s].cpu().numpy(), _oracle_philox(logits, None, 11, 3))


def test_strided_rows_and_module(pkg):
    g = torch.Generator().manual_seed(3)
    big = (torch.randn(6, 5000, generator=g) * 2).cuda()
    logits = big[:, 1001:1001 + 4096]  # rows 5000 apart, not 16-byte aligned: the scalar path
    temps = torch.full((6,), 0.9, device="cuda")
    tok = pkg.sample(logits, temps, seed=1, offset=2)
    torch.cuda.synchronize()
    assert np.array_equal(tok.cpu().numpy(), _oracle_philox(logits, temps, 1, 2))
    m = pkg.Sampler()
    a = m(logits.contiguous(), temps)
    torch.cuda.synchronize()
    assert a.shape == (6,) and a.dtype == torch.int64 and bool(((a >= 0) & (a < 4096)).all())


def test_tie_in_a_later_chunk_takes_first_index(pkg):
    """Exact ties over a whole chunk (more candidates than a chunk keeps): the warp
    evaluates the chunk in full and the first index wins, as torch.argmax."""
    V = 8192 * 3
    logits = torch.zeros(2, V, device="cuda")
    logits[:, :8192] = -50.0
    e = torch.ones(2, V, device="cuda")
    tok = pkg.sample(logits, None, exponentials=e)
    torch.cuda.synchronize()
    assert tok.tolist() == [8192, 8192]


def test_philox_fill_stream2_matches_oracle(pkg):
    out = pkg.verify.philox_draws(3, 1001, seed=9, offset=4, stream_id=2)
    torch.cuda.synchronize()
    want = philox.exponentials(9, 4, 3, 1001, stream=philox.STREAM_SAMPLE)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_frequencies_follow_softmax(pkg):
    """Gumbel-max property: over many independent rows the sampled tokens follow
    softmax(logits / T)."""
    V, B = 6, 1 << 16
    base = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, 3.0])
    T = 1.5
    logits = base.repeat(B, 1).cuda()
    tok = pkg.sample(logits, torch.full((B,), T, device="cuda"), seed=123, offset=0)
    freq = torch.bincount(tok, minlength=V).float().cpu() / B
    p = torch.softmax(base / T, -1)
    assert torch.allclose(freq, p, atol=5.0 * float(p.max()) ** 0.5 / B ** 0.5)


def test_device_offset_noise_equals_host_offset_and_advances_in_graphs(pkg):
    """sdb_sample_dev_offset: the noise offset lives on the device and advances after each
    call, so a captured draft sampling step samples new noise on every replay."""
    g0 = torch.Generator(device="cuda").manual_seed(4)
    logits = (torch.randn(16, 30000, generator=g0, device="cuda") * 2.0).to(torch.bfloat16)
    off = torch.tensor([11], dtype=torch.int64, device="cuda")
    tok = pkg.sample(logits, None, seed=9, offset_tensor=off)
    want = pkg.sample(logits, None, seed=9, offset=11)
    torch.cuda.synchronize()
    assert torch.equal(tok, want) and int(off.item()) == 12
    out = torch.empty(16, dtype=torch.int64, device="cuda")
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            pkg.sample(logits, None, seed=9, offset_tensor=off, out=out)
    torch.cuda.current_stream().wait_stream(st)
    seen = []
    for v in (12, 13, 14):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, pkg.sample(logits, None, seed=9, offset=v)), v
        seen.append(out.clone())
    assert not torch.equal(seen[0], seen[1])  # new noise on every replay
    assert int(off.item()) == 15
    del g
