"""Generate the golden fixtures in this directory by running the REFERENCE's own Python code.

Run once in a container that holds the reference checkout:

    python tests/golden/make_golden.py --reference /path/to/specdec-nanovllm

It loads three reference modules by file path (the same way the reference's
own tests do, ``tests/test_spec_decode.py:14-26``), bypassing the package
``__init__`` and its GPU-only imports:

* ``nanovllm/kernels/paged_decode_attn.py`` -> ``paged_decode_attention_ref`` (:472)
* ``nanovllm/layers/quant.py``              -> ``quantize_weight`` / ``dequantize_weight`` (:123, :151)
* ``nanovllm/spec_decode/verify.py``        -> ``verify_batch`` (:42)
* ``nanovllm/layers/sampler.py``            -> ``Sampler`` (:6-12)
* ``nanovllm/layers/layernorm.py``          -> ``RMSNorm`` (:6-44)
* ``nanovllm/layers/rotary_embedding.py``   -> ``RotaryEmbedding`` (:17-50)

(the last three with their ``torch.compile`` decorators replaced by the identity while
the module loads, so the eager ops run on CPU)

``paged_decode_attn.py`` and ``quant.py`` import triton at module level; the
Triton kernels are only defined there (``@triton.jit`` does not need a GPU), never
launched.  ``verify_batch`` draws ``torch.rand`` (:120) and
``Tensor.exponential_`` (:209) internally; both draws are replaced for the
duration of each call by fixed tensors (Philox streams of ``oracle/philox.py``)
that are saved with the case, so any implementation given the same draws must
reproduce the same decisions and tokens.

The fixtures are small ``.npz`` files; bf16 tensors are stored as uint16 bits.
"""

from __future__ import annotations

import argparse
import contextlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import philox  # noqa: E402


def _load(root, name, rel):
    spec = importlib.util.spec_from_file_location(name, os.path.join(root, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@contextlib.contextmanager
def injected_draws(u: torch.Tensor, e: torch.Tensor):
    """Replace the two random draws inside the reference's verify_batch."""
    real_rand = torch.rand
    real_exp = torch.Tensor.exponential_

    def fake_rand(*size, **kw):
        shape = size[0] if len(size) == 1 and isinstance(size[0], (tuple, list)) else size
        assert tuple(shape) == tuple(u.shape), (shape, u.shape)
        return u.clone().to(kw.get("dtype", torch.float32))

    def fake_exp(self, lambd=1.0, **kw):
        assert tuple(self.shape) == tuple(e.shape), (self.shape, e.shape)
        self.copy_(e)
        return self

    torch.rand = fake_rand
    torch.Tensor.exponential_ = fake_exp
    try:
        yield
    finally:
        torch.rand = real_rand
        torch.Tensor.exponential_ = real_exp


# ---------------------------------------------------------------------------
def make_paged_inputs(g, B, Hq, Hkv, D, page, NB, max_blocks, lens, dtype):
    lens = torch.tensor(lens, dtype=torch.int32)
    bt = torch.full((B, max_blocks), -1, dtype=torch.int32)
    perm = torch.randperm(NB, generator=g)
    used = 0
    for b in range(B):
        nblk = (int(lens[b]) + page - 1) // page
        bt[b, :nblk] = perm[used:used + nblk].to(torch.int32)
        used += nblk
    assert used <= NB
    k = torch.randn(NB, page, Hkv, D, generator=g).to(dtype)
    v = torch.randn(NB, page, Hkv, D, generator=g).to(dtype)
    return k, v, bt, lens


def attention_cases(ref, out_dir):
    pda = ref["attn"]
    g = torch.Generator().manual_seed(1234)
    # --- decode, fp32, GQA 2 (the cfg1 path at a fixture-sized shape) -------------
    B, Hq, Hkv, D, page, NB, mb = 5, 4, 2, 32, 16, 12, 4
    lens = [0, 5, 16, 37, 64]
    k, v, bt, cl = make_paged_inputs(g, B, Hq, Hkv, D, page, NB, mb, lens, torch.float32)
    q = torch.randn(B, Hq, D, generator=g)
    scale = D ** -0.5
    o = pda.paged_decode_attention_ref(q, k, v, bt, cl, scale)
    np.savez_compressed(os.path.join(out_dir, "attn_decode_fp32.npz"),
                        q=q.numpy(), k_cache=k.numpy(), v_cache=v.numpy(),
                        block_tables=bt.numpy(), cache_seqlens=cl.numpy(),
                        scale=np.float32(scale), n_q=np.int32(1), out=o.numpy())

    # --- decode + verify, bf16, GQA 4, head_dim 128 -------------------------------
    B, Hq, Hkv, D, page, NB, mb = 5, 8, 2, 128, 64, 12, 4
    lens = [0, 3, 64, 129, 250]
    k, v, bt, cl = make_paged_inputs(g, B, Hq, Hkv, D, page, NB, mb, lens, torch.bfloat16)
    scale = D ** -0.5
    for n_q in (1, 4):
        q = torch.randn(B * n_q, Hq, D, generator=g).to(torch.bfloat16)
        # Verify rows are pinned through the reference's decode oracle: under
        # flash-attn's bottom-right causal alignment, row r of n sees exactly the
        # first L - n + r + 1 keys, i.e. it IS a decode with that cache length.
        out_bf16 = torch.zeros(B * n_q, Hq, D, dtype=torch.bfloat16)
        out_f32 = torch.zeros(B * n_q, Hq, D, dtype=torch.float32)
        for r in range(n_q):
            vis = torch.clamp(cl - n_q + r + 1, min=0).to(torch.int32)
            vis = torch.minimum(vis, cl)
            rows = torch.arange(B) * n_q + r
            out_bf16[rows] = pda.paged_decode_attention_ref(q[rows], k, v, bt, vis, scale)
            out_f32[rows] = pda.paged_decode_attention_ref(q[rows].float(), k.float(), v.float(),
                                                           bt, vis, scale)
        np.savez_compressed(os.path.join(out_dir, f"attn_bf16_nq{n_q}.npz"),
                            q=bf16_bits(q), k_cache=bf16_bits(k), v_cache=bf16_bits(v),
                            block_tables=bt.numpy(), cache_seqlens=cl.numpy(),
                            scale=np.float32(scale), n_q=np.int32(n_q),
                            out_bf16=bf16_bits(out_bf16), out_f32=out_f32.numpy())


def quant_cases(ref, out_dir):
    qm = ref["quant"]
    g = torch.Generator().manual_seed(99)
    N, K, M = 48, 256, 5
    w = torch.randn(N, K, generator=g) * 0.05
    w[3, 7] = 0.0
    w[5] = 0.0                               # all-zero row: scale clamps to 1e-8
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    res = {"w": w.numpy(), "x": bf16_bits(x)}
    for gran, gs in (("per_channel", 128), ("per_group", 64)):
        q, s = qm.quantize_weight(w, gran, gs)
        deq = qm.dequantize_weight(q, s, gran, gs)
        y = x.float() @ deq.T
        res[f"{gran}_q"] = q.numpy()
        res[f"{gran}_scale"] = bf16_bits(s)
        res[f"{gran}_deq"] = deq.numpy()
        res[f"{gran}_y"] = y.numpy()
    np.savez_compressed(os.path.join(out_dir, "quant.npz"), **res)


def verify_cases(ref, out_dir):
    vb = ref["verify"].verify_batch
    g = torch.Generator().manual_seed(7)
    cases = {}

    def run(name, draft, target, tokens, temps=None, point=False, seed=0):
        B, k, V = draft.shape
        u = torch.from_numpy(philox.uniforms(seed, 0, B, k))
        e = torch.from_numpy(philox.exponentials(seed, 0, B, V))
        with injected_draws(u, e):
            r = vb(draft, target, tokens, temps, draft_is_point_mass=point)
        cases[name] = dict(draft=draft.numpy(), target=target.numpy(), tokens=tokens.numpy(),
                           temps=(temps.numpy() if temps is not None else np.zeros(0, np.float32)),
                           has_temps=np.bool_(temps is not None), point=np.bool_(point),
                           seed=np.int64(seed), u=u.numpy(), e=e.numpy(),
                           accepted=r.accepted.numpy(), bonus=r.bonus.numpy(),
                           accept_mask=r.accept_mask.numpy())

    def sample_tokens(logits):
        B, k, V = logits.shape
        pr = torch.softmax(logits, -1).reshape(B * k, V)
        return torch.multinomial(pr, 1, generator=g).reshape(B, k)

    # cfg4-like statistics at a small vocabulary
    B, k, V = 8, 6, 997
    target = torch.randn(B, k + 1, V, generator=g) * 3.0
    draft = target[:, :k] + torch.randn(B, k, V, generator=g)
    run("random", draft, target, sample_tokens(draft), seed=11)
    temps = torch.tensor([0.5, 1.0, 2.0, 0.7, 1.3, 1.0, 3.0, 0.25])
    run("temps", draft, target, sample_tokens(draft / temps[:, None, None]), temps=temps, seed=12)
    # draft == target: everything accepted, bonus drawn from row k
    t2 = torch.randn(4, 4, 300, generator=g) * 2.0
    run("all_accept", t2[:, :3].clone(), t2, sample_tokens(t2[:, :3]), seed=13)
    # point-mass draft (n-gram route)
    B, k, V = 6, 3, 50
    tgt = torch.randn(B, k + 1, V, generator=g) * 2.0
    tok = torch.randint(0, V, (B, k), generator=g)
    pm = torch.zeros(B, k, V)
    pm.scatter_(2, tok.unsqueeze(-1), 1.0)
    run("point_mass", pm, tgt, tok, point=True, seed=14)
    # degenerate target with only k rows (no bonus row): p index clamps to k-1
    tk = torch.randn(5, 3, 64, generator=g) * 2.0
    dk = tk + torch.randn(5, 3, 64, generator=g)
    run("k_rows_target", dk, tk, sample_tokens(dk), seed=15)
    # the alignment case of the reference's test 6 (row j peaks at token 10+j)
    K6, V6 = 3, 20
    tl6 = torch.full((1, K6 + 1, V6), -30.0)
    for j in range(K6 + 1):
        tl6[0, j, 10 + j] = 30.0
    run("align_all", tl6[:, :K6].clone(), tl6, torch.tensor([[10, 11, 12]]), seed=16)
    dl7 = tl6[:, :K6].clone()
    dl7[0, 0, 10] = -30.0
    dl7[0, 0, 3] = 30.0
    run("align_reject0", dl7, tl6.clone(), torch.tensor([[3, 11, 12]]), seed=17)
    for name, c in cases.items():
        np.savez_compressed(os.path.join(out_dir, f"verify_{name}.npz"), **c)


def sampler_cases(ref, out_dir):
    """Sampler.forward (nanovllm/layers/sampler.py:8-12) with its exponential draw injected."""
    sampler = ref["sampler"].Sampler()
    g = torch.Generator().manual_seed(23)
    cases = {}

    def run(name, logits, temps, seed, e=None):
        B, V = logits.shape
        if e is None:
            e = torch.from_numpy(philox.exponentials(seed, 0, B, V, stream=philox.STREAM_SAMPLE))
        with injected_draws(torch.zeros(0), e):
            # on fp32 logits the reference divides its argument in place (.float() is a
            # no-op there, then div_), so it gets a copy
            tok = sampler.forward(logits.clone(), temps)
        is_bf16 = logits.dtype == torch.bfloat16
        cases[name] = dict(logits=bf16_bits(logits) if is_bf16 else logits.numpy(), is_bf16=np.bool_(is_bf16),
                           temps=temps.numpy(), seed=np.int64(seed), e=e.numpy(), tokens=tok.numpy())

    run("random", torch.randn(6, 997, generator=g) * 3.0,
        torch.tensor([1.0, 0.5, 2.0, 0.7, 1.0, 1.3]), seed=31)
    # bf16 logits as the LM head emits them (logits.float() in the reference), 3 chunks of 8192
    run("bf16_chunks", (torch.randn(2, 24576, generator=g) * 4.0).to(torch.bfloat16),
        torch.tensor([0.8, 1.0]), seed=32)
    # a vocabulary that is not a multiple of 8 (the kernel's scalar path)
    run("ragged_vocab", torch.randn(2, 16389, generator=g) * 2.0, torch.ones(2), seed=33)
    # one dominant logit per row
    pk = torch.randn(4, 512, generator=g)
    pk[torch.arange(4), torch.tensor([3, 100, 511, 0])] += 25.0
    run("peaked", pk, torch.ones(4), seed=34)
    # exact ties everywhere: constant logits and constant noise -> first index
    run("ties", torch.zeros(2, 9000), torch.ones(2), seed=35, e=torch.ones(2, 9000))
    for name, c in cases.items():
        np.savez_compressed(os.path.join(out_dir, f"sampler_{name}.npz"), **c)


def prologue_cases(ref, out_dir):
    """q_norm / k_norm (RMSNorm.rms_forward, layernorm.py:16-25) and rotary_emb
    (RotaryEmbedding.forward, rotary_embedding.py:38-50) as qwen3.py:77-85 applies them,
    bf16 on CPU."""
    g = torch.Generator().manual_seed(29)
    T, Hq, Hkv, D = 12, 8, 2, 128
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, generator=g) * 2.0).to(torch.bfloat16)
    positions = torch.tensor([0, 1, 7, 300, 4095, 4096, 17, 1000, 2047, 5, 63, 64])
    q_norm = ref["layernorm"].RMSNorm(D, eps=1e-6)
    k_norm = ref["layernorm"].RMSNorm(D, eps=1e-6)
    with torch.no_grad():
        q_norm.weight.copy_(torch.rand(D, generator=g) * 2.0)
        k_norm.weight.copy_(torch.rand(D, generator=g) * 2.0)
    q_norm = q_norm.to(torch.bfloat16)
    k_norm = k_norm.to(torch.bfloat16)
    rope = ref["rope"].RotaryEmbedding(D, D, 8192, 1000000.0)
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    q = q.reshape(-1, Hq, D)
    k = k.reshape(-1, Hkv, D)
    v = v.reshape(-1, Hkv, D)
    with torch.no_grad():
        qn = q_norm(q)
        kn = k_norm(k)
        qr, kr = rope(positions, qn, kn)
    np.savez_compressed(os.path.join(out_dir, "prologue_qwen3.npz"),
                        qkv=bf16_bits(qkv), positions=positions.numpy(),
                        q_norm_w=bf16_bits(q_norm.weight.data), k_norm_w=bf16_bits(k_norm.weight.data),
                        eps=np.float32(1e-6), rope_base=np.float64(1000000.0), max_position=np.int64(8192),
                        cos_sin_rows=rope.cos_sin_cache.squeeze(1)[positions].numpy(),
                        q=bf16_bits(qr), k=bf16_bits(kr), v=bf16_bits(v), Hq=np.int64(Hq),
                        Hkv=np.int64(Hkv), D=np.int64(D))


def _load_compiled(root, name, rel):
    """Load a reference module whose methods carry torch.compile, with the decorator as
    the identity so the plain eager ops run on CPU."""
    real = torch.compile
    torch.compile = lambda fn=None, **kw: fn if fn is not None else (lambda f: f)
    try:
        return _load(root, name, rel)
    finally:
        torch.compile = real


def _load_sampler(root):
    """layers/sampler.py decorates forward with torch.compile; load it with the decorator
    as the identity so the plain eager ops run on CPU."""
    real = torch.compile
    torch.compile = lambda fn=None, **kw: fn if fn is not None else (lambda f: f)
    try:
        return _load(root, "ref_sampler", "nanovllm/layers/sampler.py")
    finally:
        torch.compile = real


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPECDEC_REFERENCE"),
                    help="checkout of the reference (or set SPECDEC_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference or set SPECDEC_REFERENCE to the reference checkout")
    ref = {
        "attn": _load(a.reference, "ref_paged_decode_attn", "nanovllm/kernels/paged_decode_attn.py"),
        "quant": _load(a.reference, "ref_quant", "nanovllm/layers/quant.py"),
        "verify": _load(a.reference, "ref_verify", "nanovllm/spec_decode/verify.py"),
        "sampler": _load_sampler(a.reference),
        "layernorm": _load_compiled(a.reference, "ref_layernorm", "nanovllm/layers/layernorm.py"),
        "rope": _load_compiled(a.reference, "ref_rope", "nanovllm/layers/rotary_embedding.py"),
    }
    torch.manual_seed(0)
    attention_cases(ref, a.out)
    quant_cases(ref, a.out)
    verify_cases(ref, a.out)
    sampler_cases(ref, a.out)
    prologue_cases(ref, a.out)
    print("golden fixtures written to", a.out)


if __name__ == "__main__":
    main()
