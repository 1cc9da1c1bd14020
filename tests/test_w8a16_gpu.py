"""W8A16 linear and quantize_weight on the GPU.

quantize_weight: bit-exact against the reference (golden q and bf16 scales).
int8_linear: rtol 2e-2 / atol 2e-3 against the float32 product x.float() @ dequant(q, s).T
(the reference's own check, scripts/bench_int8_gemm.py:139-142), computed in float64.
"""

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle.numerics import allclose_report, bf16_bits_to_f32

pytestmark = pytest.mark.gpu

TOL = dict(rtol=2e-2, atol=2e-3)


@pytest.fixture(autouse=True, params=["auto", "cluster", "umma", "mma", "gemv"])
def kernel_choice(request, monkeypatch):
    """Every test runs on the default kernel (where the shape allows: the weight-stream kernel
    up to 16 tokens, else the register kernel, for 17 to 128 the cluster split-K tcgen05
    kernel unless its plan is unbalanced, else and above 128 the stream-K tcgen05 kernel),
    on the cluster kernel
    wherever it has a plan (SDB_W8A16_KERNEL=cluster), on the stream-K kernel alone above 16
    tokens (SDB_W8A16_KERNEL=umma), on the register kernel (SDB_W8A16_KERNEL=mma) and on the
    weight-stream kernel wherever it has a plan (SDB_W8A16_KERNEL=gemv: 1-16 tokens,
    per-channel scales, K % 128 == 0, the tokens within its shared memory)."""
    if request.param == "auto":
        monkeypatch.delenv("SDB_W8A16_KERNEL", raising=False)
    else:
        monkeypatch.setenv("SDB_W8A16_KERNEL", request.param)
    return request.param


def _ref(x, q, s, bias=None, granularity="per_channel", group_size=128):
    w = (q.double() * s.double().unsqueeze(1) if granularity == "per_channel" else
         (q.double().view(q.shape[0], -1, group_size) * s.double().unsqueeze(-1)).view(q.shape))
    y = x.double() @ w.T
    if bias is not None:
        y = y + bias.double()
    return y


def _check(got, want):
    ok, err, viol = allclose_report(got.float().cpu().numpy(), want.cpu().numpy(), **TOL)
    assert ok, f"max abs err {err}, worst violation {viol}"


@pytest.mark.parametrize("gran,gs", [("per_channel", 128), ("per_group", 64)])
def test_quantize_weight_bit_exact_vs_reference(pkg, golden, gran, gs):
    g = golden("quant")
    w = torch.from_numpy(g["w"]).cuda()
    q, s = pkg.quantize_weight(w, gran, gs)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), g[f"{gran}_q"])
    assert np.array_equal(s.cpu().view(torch.int16).numpy().view(np.uint16), g[f"{gran}_scale"])


@pytest.mark.parametrize("gran,gs", [("per_channel", 128), ("per_group", 64)])
def test_int8_linear_golden(pkg, golden, gran, gs):
    g = golden("quant")
    x = torch.from_numpy(bf16_bits_to_f32(g["x"])).to(torch.bfloat16).cuda()
    q = torch.from_numpy(g[f"{gran}_q"]).cuda()
    s = torch.from_numpy(bf16_bits_to_f32(g[f"{gran}_scale"])).to(torch.bfloat16).cuda()
    y = pkg.int8_linear(x, q, s, granularity=gran, group_size=gs)
    torch.cuda.synchronize()
    ok, err, _ = allclose_report(y.float().cpu().numpy(), g[f"{gran}_y"], **TOL)
    assert ok, err


@pytest.mark.parametrize("name", ["qkv", "o", "gate_up", "down"])
@pytest.mark.parametrize("M", [1, 7, 64, 448])
def test_cfg3_shapes(pkg, name, M):
    from specdec_nanovllm_b200.workloads import W8A16_SHAPES, cfg3_inputs
    K, N = W8A16_SHAPES[name]
    x, q, s = cfg3_inputs(M, K, N, seed=M)
    y = pkg.int8_linear(x, q, s)
    torch.cuda.synchronize()
    assert y.dtype == torch.float16 and y.shape == (M, N)
    _check(y, _ref(x, q, s))


@pytest.mark.parametrize("M", [17, 33, 64, 100, 128])
@pytest.mark.parametrize("N,K", [(6144, 2560), (19456, 2560), (2560, 9728), (203, 384), (1030, 1280)])
def test_cluster_split_shapes(pkg, M, N, K):
    """Shapes that give the cluster plan one tile per cluster (6144 x 2560, 2560 x 9728),
    several tiles per cluster with CTAs spanning tile boundaries (19456 x 2560), a single
    small cluster (203 x 384) and ragged feature counts (203, 1030: the scalar y tail)."""
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    q = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int32).to(torch.int8)
    s = (torch.rand(N, generator=g, device="cuda") * 0.01).to(torch.float16)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.float16)
    bias = torch.randn(N, generator=g, device="cuda").to(torch.float16)
    y = pkg.int8_linear(x, q, s, bias)
    torch.cuda.synchronize()
    _check(y, _ref(x, q, s, bias))


@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("N,K", [(7, 128), (203, 384), (1030, 1280), (2560, 9728), (19456, 2560)])
def test_small_token_counts(pkg, M, N, K):
    """1-16 tokens: fewer features than CTAs (7, 203), ragged tiles (1030 rows over the CTAs),
    the down projection (9728-wide token rows: 16 tokens do not fit the weight-stream kernel's
    shared memory and take the register kernel) and gate_up; one and two 8-token fragments,
    f16 and bf16 activations, bias on odd token counts."""
    g = torch.Generator(device="cuda").manual_seed(M * 31 + N + K)
    dt = torch.bfloat16 if M in (3, 9) else torch.float16     # bf16 with one and two fragments
    q = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int32).to(torch.int8)
    s = torch.rand(N, generator=g, device="cuda") * 0.01
    s = s if dt == torch.bfloat16 else s.to(torch.float16)    # float32 scales with bf16
    x = torch.randn(M, K, generator=g, device="cuda").to(dt)
    bias = torch.randn(N, generator=g, device="cuda").to(dt) if M % 2 else None
    y = pkg.int8_linear(x, q, s, bias)
    torch.cuda.synchronize()
    _check(y, _ref(x, q, s, bias))


@pytest.mark.parametrize("M", [17, 64, 128])
@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.bfloat16])
def test_cluster_bf16_activations_scale_dtypes_and_error_word(pkg, M, scale_dtype):
    """bf16 activations with float32 / bf16 scales and a bias on a shape whose clusters hold
    several tiles (3 x 2560 -> 6144 is the qkv projection); the kernels' device error word
    (bounded waits report there) stays clear."""
    from specdec_nanovllm_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(100 + M)
    N, K = 6144, 2560
    q = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int32).to(torch.int8)
    s = (torch.rand(N, generator=g, device="cuda") * 0.01).to(scale_dtype)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    bias = torch.randn(N, generator=g, device="cuda").to(torch.bfloat16)
    y = pkg.int8_linear(x, q, s, bias)
    torch.cuda.synchronize()
    _check(y, _ref(x, q, s, bias))
    ws = _lib.WORKSPACES.get(x.device, "w8a16", 1)
    err_word = ws[256 * 1024:256 * 1024 + 4].view(torch.int32).item()  # error word of the tcgen05 kernels
    assert err_word == 0


@pytest.mark.parametrize("width", [2600, 2562])
def test_strided_output_rows(pkg, width):
    """y written into a wider buffer: row stride a multiple of 4 (packed 8-byte stores) and not."""
    from specdec_nanovllm_b200.workloads import cfg3_inputs
    x, q, s = cfg3_inputs(40, 4096, 2560, seed=11)
    buf = torch.full((40, width), 7.0, device="cuda", dtype=torch.float16)
    out = buf[:, :2560]
    pkg.int8_linear(x, q, s, out=out)
    torch.cuda.synchronize()
    _check(out, _ref(x, q, s))
    assert torch.all(buf[:, 2560:] == 7.0)


@pytest.mark.parametrize("M", [3, 40])
def test_bf16_bias_and_odd_shapes(pkg, M):
    g = torch.Generator(device="cuda").manual_seed(5)
    N, K = 200, 320                              # N not a multiple of the 64-feature tile
    q = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int32).to(torch.int8)
    s = (torch.rand(N, generator=g, device="cuda") * 0.01).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    bias = torch.randn(N, generator=g, device="cuda").to(torch.bfloat16)
    y = pkg.int8_linear(x.view(M, K), q, s, bias)
    torch.cuda.synchronize()
    _check(y, _ref(x, q, s, bias))


@pytest.mark.parametrize("M", [1, 64])
def test_per_group_fp32_scales(pkg, M):
    g = torch.Generator(device="cuda").manual_seed(9)
    N, K, G = 512, 1024, 128
    q = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int32).to(torch.int8)
    s = torch.rand(N, K // G, generator=g, device="cuda") * 0.01
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.float16)
    y = pkg.int8_linear(x, q, s, granularity="per_group", group_size=G)
    torch.cuda.synchronize()
    _check(y, _ref(x, q, s, granularity="per_group", group_size=G))


def test_quantize_then_linear_matches_dequantized_product(pkg):
    g = torch.Generator(device="cuda").manual_seed(1)
    w = torch.randn(6144, 2560, generator=g, device="cuda") * 0.02
    q, s = pkg.quantize_weight(w)
    x = torch.randn(7, 2560, generator=g, device="cuda").to(torch.bfloat16)
    y = pkg.int8_linear(x, q, s)
    torch.cuda.synchronize()
    _check(y, x.double() @ pkg.dequantize_weight(q, s).double().T)
    qo, so = oq.quantize_weight(w.cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), qo)


def test_deterministic_and_graph_capturable(pkg):
    from specdec_nanovllm_b200.workloads import cfg3_inputs
    x, q, s = cfg3_inputs(1, 9728, 2560, seed=2)
    y1 = pkg.int8_linear(x, q, s)
    y = torch.empty_like(y1)
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            pkg.int8_linear(x, q, s, out=y)
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y1)
    del g
