"""Decoder-layer elementwise kernels against the reference's torch code restated
(nanovllm/layers/layernorm.py:17-43, nanovllm/layers/activation.py:8-13) on the same bf16 /
fp16 inputs: within one ulp of the model dtype (the reductions run in another order and
rsqrt is the hardware one) and the reference rounds twice (after the normalisation and
after the weight product), so a one-ulp difference at the first rounding can reach two at
the output: the bar is two ulps of the model dtype, with almost every element
bit-identical."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ref_rms(x, w, eps, residual=None):
    orig = x.dtype
    if residual is not None:
        xf = x.float() + residual.float()
        res = xf.to(orig)
    else:
        xf = x.float()
        res = None
    y = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return y.to(orig) * w, res


def _close(got, want, min_identical=0.97):
    ulp = 2 * want.float().abs().clamp_min(1e-30) * (2.0 ** -7 if want.dtype == torch.bfloat16 else 2.0 ** -10)
    diff = (got.float() - want.float()).abs()
    assert bool((diff <= ulp + 1e-6).all()), float((diff - ulp).max())
    assert (got == want).float().mean().item() >= min_identical


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,H", [(1, 1024), (64, 1024), (448, 2560), (7, 8192)])
def test_rms_norm_with_and_without_residual(pkg, dtype, T, H):
    from specdec_nanovllm_b200.layers import rms_norm
    g = torch.Generator(device="cuda").manual_seed(T + H)
    x = torch.randn(T, H, generator=g, device="cuda").to(dtype)
    r = torch.randn(T, H, generator=g, device="cuda").to(dtype)
    w = (torch.rand(H, generator=g, device="cuda") + 0.5).to(dtype)
    y = rms_norm(x, w, 1e-6)
    want, _ = _ref_rms(x, w, 1e-6)
    _close(y, want)
    y2, res = rms_norm(x, w, 1e-6, residual=r)
    want2, wres = _ref_rms(x, w, 1e-6, residual=r)
    assert torch.equal(res, wres)
    _close(y2, want2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,Fd", [(1, 3072), (64, 9728), (448, 9728)])
def test_silu_and_mul(pkg, dtype, T, Fd):
    from specdec_nanovllm_b200.layers import silu_and_mul
    g = torch.Generator(device="cuda").manual_seed(T + Fd)
    gu = (torch.randn(T, 2 * Fd, generator=g, device="cuda") * 3).to(dtype)
    y = silu_and_mul(gu)
    a, b = gu.chunk(2, -1)
    _close(y, F.silu(a) * b, min_identical=0.98)
