"""End-to-end speculative decode step on the sm_100a kernels, with random-init Qwen3 models.

The reference's step (``nanovllm/engine/model_runner.py:945-1120`` with the batched draft
of ``nanovllm/spec_decode/draft_proposer.py:414-518``):

1. propose: k batched draft decode steps.  Step s feeds the last confirmed token (s = 0)
   or draft token s-1 at position len-1+s, writes its K/V into the draft's paged cache,
   and samples draft token s from softmax(logits / T) with exponential noise, keeping
   the raw logits (:495-510);
2. verify: one target forward over the k+1 tokens of every sequence (positions
   len-1 .. len+k-1, causal inside the window; ``prepare_verify``, :492-584), its K/V
   written into the target cache, then the LM head;
3. ``verify_batch`` on the raw draft logits and the target logits: accepted prefix
   length and the bonus token of every sequence (:1051-1119, batched here).

Every layer runs the sm_100a kernels of this package -- the fused split / q-k RMSNorm /
rotary / KV store (``qk_norm_rope_store``), the paged decode or verify attention, the
draft sampler and ``verify_batch`` -- and the residual RMSNorm and SiLU * up of ``layers.py``
(``layers/layernorm.py``, ``layers/activation.py``) -- around bf16 cuBLAS GEMMs for the
projections and the LM head (``torch.nn.functional.linear``, the reference's
``F.linear``) and torch's embedding lookup.  The draft's k steps are one captured CUDA
graph, and the target's verify forward with ``verify_batch`` is another (the reference
captures both forwards, ``model_runner.py:1218-1347``).  The draws inside the graphs
(the draft noise, the acceptance uniforms and the bonus noise) come from Philox offsets
kept on the device, which each call reads and advances, so every replay draws anew.

Models are random-init (there are no checkpoints): weights N(0, 0.02) in bf16, norm
weights 1, tied embeddings.  The KV caches start filled with N(0, 1) values standing for
a ``context``-token prefix, so a step runs at that context without a prefill.

Tensor parallel (``tp_size`` > 1, one rank per GPU): the Megatron split of the reference's
``linear.py:68-170`` -- q/k/v heads and the gate/up rows column-parallel, o_proj and
down_proj row-parallel followed by an NCCL all-reduce of their (tokens, hidden) partial
sums (``RowParallelLinear.forward``, :165-170), the KV cache holding the rank's kv heads.
The embedding and the tied LM head are replicated rather than vocab-parallel, so every
rank holds the same logits and runs the same sampler and ``verify_batch`` draws: no
collective besides the two all-reduces per layer.  Each rank's slices are cut from the
same full weights a single-device model with the same seed holds.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .attention import paged_attention
from .layers import rms_norm as layer_rms_norm
from .layers import silu_and_mul
from .prologue import qk_norm_rope_store, rope_cos_sin_cache
from .sampler import draft_sample_step
from .verify import VerifyResult, verify_batch


@dataclass(frozen=True)
class Qwen3Shape:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int = 151936
    head_dim: int = 128
    eps: float = 1e-6
    rope_theta: float = 1e6


QWEN3_4B = Qwen3Shape(layers=36, hidden=2560, heads=32, kv_heads=8, ffn=9728)
QWEN3_06B = Qwen3Shape(layers=28, hidden=1024, heads=16, kv_heads=8, ffn=3072)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """``RMSNorm`` with the residual convention of ``Qwen3DecoderLayer.forward``
    (qwen3.py:145-159): without a residual the input itself becomes the residual."""
    if residual is None:
        return layer_rms_norm(x, w, eps), x
    return layer_rms_norm(x, w, eps, residual=residual)


class RandomQwen3:
    """A Qwen3 decoder with random bf16 weights, run on the package's kernels; with
    ``tp_size`` > 1 the rank's tensor-parallel slice of it (all-reduce over ``group``)."""

    def __init__(self, shape: Qwen3Shape, device, seed: int, max_position: int = 8192,
                 dtype=torch.bfloat16, tp_rank: int = 0, tp_size: int = 1, group=None):
        if shape.heads % tp_size or shape.kv_heads % tp_size or shape.ffn % tp_size:
            raise ValueError(f"tp_size {tp_size} must divide heads {shape.heads}, kv heads "
                             f"{shape.kv_heads} and ffn {shape.ffn}")
        self.s = shape
        self.dtype = dtype
        self.tp_rank, self.tp_size, self.group = tp_rank, tp_size, group
        self.heads, self.kv_heads = shape.heads // tp_size, shape.kv_heads // tp_size
        g = torch.Generator(device=device).manual_seed(seed)
        H, D, F_ = shape.hidden, shape.head_dim, shape.ffn
        r, hq, hk, fl = tp_rank, self.heads * D, self.kv_heads * D, F_ // tp_size

        def w(out_f, in_f):
            return (torch.randn(out_f, in_f, generator=g, device=device, dtype=torch.float32) * 0.02).to(dtype)

        def rows(t, *ranges):          # the rank's row ranges of a full weight, concatenated
            return torch.cat([t[a:b] for a, b in ranges]).contiguous()

        self.embed = w(shape.vocab, H)          # tied with the LM head
        self.layers = []
        for _ in range(shape.layers):
            qkv, o, gate_up, down = (w((shape.heads + 2 * shape.kv_heads) * D, H), w(H, shape.heads * D),
                                     w(2 * F_, H), w(H, F_))
            q0, k0, v0 = 0, shape.heads * D, (shape.heads + shape.kv_heads) * D
            self.layers.append(dict(
                ln1=torch.ones(H, device=device, dtype=dtype),
                ln2=torch.ones(H, device=device, dtype=dtype),
                qkv=rows(qkv, (q0 + r * hq, q0 + (r + 1) * hq), (k0 + r * hk, k0 + (r + 1) * hk),
                         (v0 + r * hk, v0 + (r + 1) * hk)),
                q_norm=torch.ones(D, device=device, dtype=dtype),
                k_norm=torch.ones(D, device=device, dtype=dtype),
                o=o[:, r * hq:(r + 1) * hq].contiguous(),
                gate_up=rows(gate_up, (r * fl, (r + 1) * fl), (F_ + r * fl, F_ + (r + 1) * fl)),
                down=down[:, r * fl:(r + 1) * fl].contiguous()))
            del qkv, o, gate_up, down
        self.norm = torch.ones(H, device=device, dtype=dtype)
        self.cos_sin = rope_cos_sin_cache(D, max_position, shape.rope_theta, device=device)
        self.scale = 1.0 / math.sqrt(D)

    def new_cache(self, num_blocks: int, page: int, device, seed: int):
        """Per layer (num_blocks, page, Hkv / tp, D) K and V caches: the rank's kv heads of
        full caches filled with N(0, 1)."""
        g = torch.Generator(device=device).manual_seed(seed)
        shp = (num_blocks, page, self.s.kv_heads, self.s.head_dim)
        h0, h1 = self.tp_rank * self.kv_heads, (self.tp_rank + 1) * self.kv_heads
        out = []
        for _ in range(self.s.layers):
            kv = []
            for _ in range(2):
                full = torch.randn(shp, generator=g, device=device, dtype=self.dtype)
                kv.append(full if self.tp_size == 1 else full[:, :, h0:h1].contiguous())
                del full
            out.append(tuple(kv))
        return out

    def forward_steps(self, ids, positions, slots, block_tables, seqlens, n_q: int, cache):
        """The forward as a generator: it yields the (T, H) partial sums of o_proj and of
        down_proj and resumes with their sums over the tensor-parallel ranks; it returns the
        final hidden states.  ``forward`` drives it with an NCCL all-reduce."""
        s = self.s
        h = F.embedding(ids, self.embed)
        residual = None
        for lw, (kc, vc) in zip(self.layers, cache):
            x, residual = rms_norm(h, lw["ln1"], s.eps, residual)
            qkv = F.linear(x, lw["qkv"])
            q = qk_norm_rope_store(qkv, positions, self.heads, self.kv_heads, s.head_dim, self.cos_sin,
                                   lw["q_norm"], lw["k_norm"], s.eps, k_cache=kc, v_cache=vc,
                                   slot_mapping=slots)
            o = paged_attention(q, kc, vc, block_tables, seqlens, self.scale, n_q=n_q)
            h = yield F.linear(o.view(o.shape[0], -1), lw["o"])
            x, residual = rms_norm(h, lw["ln2"], s.eps, residual)
            gu = F.linear(x, lw["gate_up"])
            h = yield F.linear(silu_and_mul(gu), lw["down"])
        h, _ = rms_norm(h, self.norm, s.eps, residual)
        return h

    def forward(self, ids, positions, slots, block_tables, seqlens, n_q: int, cache) -> torch.Tensor:
        """Hidden states (T, H) of T = B * n_q tokens, rows b * n_q .. b * n_q + n_q - 1 of
        sequence b at consecutive positions ending at seqlens[b] - 1 (decode: n_q = 1)."""
        steps = self.forward_steps(ids, positions, slots, block_tables, seqlens, n_q, cache)
        part = next(steps)
        while True:
            if self.tp_size > 1:
                dist.all_reduce(part, group=self.group)
            try:
                part = steps.send(part)
            except StopIteration as done:
                return done.value

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return F.linear(h, self.embed)


class SpecDecodeStep:
    """B sequences at a fixed ``context`` (tokens already in both caches), k drafts per
    step.  ``step()`` runs propose -> verify -> verify_batch and returns the accepted
    counts and bonus tokens (device tensors); the caches keep the context fixed, so every
    step measures the same work.  Sequences own disjoint blocks (one pool per model,
    scattered block ids)."""

    def __init__(self, target: RandomQwen3, draft: RandomQwen3, B: int, context: int, k: int, device,
                 page: int = 256, seed: int = 0, use_graphs: bool = True):
        self.t, self.d, self.B, self.L, self.k = target, draft, B, context, k
        self.dev = device
        self.page = page
        max_len = context + k + 1
        nblk = (max_len + page - 1) // page
        gen = torch.Generator().manual_seed(seed)
        perm = torch.randperm(B * nblk, generator=gen).to(torch.int32)
        self.block_tables = perm.view(B, nblk).to(device)
        self.t_cache = target.new_cache(B * nblk, page, device, seed + 1)
        self.d_cache = draft.new_cache(B * nblk, page, device, seed + 2)
        self.last_tokens = torch.randint(0, target.s.vocab, (B,), generator=gen).to(device)
        self.temps = torch.ones(B, 1, device=device)
        bt = self.block_tables.long()
        base = torch.full((B,), context - 1, dtype=torch.int64, device=device)  # last confirmed token

        def slots_at(pos):                                                  # (B, n) positions -> slots
            return (bt.gather(1, pos // page) * page + pos % page).to(torch.int32)

        # draft step s: one token per sequence at position L-1+s, cache length L+s
        self.d_pos = [(base + s).view(B) for s in range(k)]
        self.d_slots = [slots_at((base + s).view(B, 1)).view(B) for s in range(k)]
        self.d_lens = [torch.full((B,), context + s, dtype=torch.int32, device=device) for s in range(k)]
        # verify: k+1 tokens per sequence at L-1 .. L+k-1, cache length L+k
        vpos = base.view(B, 1) + torch.arange(k + 1, device=device).view(1, k + 1)
        self.v_pos = vpos.reshape(-1)
        self.v_slots = slots_at(vpos).reshape(-1)
        self.v_lens = torch.full((B,), context + k, dtype=torch.int32, device=device)
        V = target.s.vocab
        self.draft_logits = torch.empty(B, k, V, device=device)
        self.cands = torch.empty(B, k, dtype=torch.int64, device=device)
        self.v_ids = torch.empty(B, k + 1, dtype=torch.int64, device=device)
        self.target_logits = None
        # Philox offsets of the draft sampler and of verify_batch, on the device: each call
        # reads its offset and advances it, so every graph replay draws new values
        self.sample_offset = torch.zeros(1, dtype=torch.int64, device=device)
        self.verify_offset = torch.zeros(1, dtype=torch.int64, device=device)
        self.result = VerifyResult(accepted=torch.empty(B, dtype=torch.int64, device=device),
                                   bonus=torch.empty(B, dtype=torch.int64, device=device),
                                   n_proposed=torch.full((B,), k, dtype=torch.int64, device=device),
                                   accept_mask=torch.empty(B, k, dtype=torch.bool, device=device))
        self.seed = 1234 + seed
        self.n_steps = 0
        self.use_graphs = use_graphs
        self.g_draft = self.g_target = None

    # ---- the two phases (captured as graphs after one eager run)
    def _propose(self):
        tok = self.last_tokens
        for s in range(self.k):
            h = self.d.forward(tok, self.d_pos[s], self.d_slots[s], self.block_tables, self.d_lens[s], 1,
                               self.d_cache)
            lg = self.d.logits(h)
            tok = draft_sample_step(lg, self.temps, self.draft_logits, self.cands, s, seed=self.seed,
                                    offset_tensor=self.sample_offset)

    def _verify_forward(self):
        self.v_ids[:, 0] = self.last_tokens
        self.v_ids[:, 1:] = self.cands
        h = self.t.forward(self.v_ids.view(-1), self.v_pos, self.v_slots, self.block_tables, self.v_lens,
                           self.k + 1, self.t_cache)
        self.target_logits = self.t.logits(h).view(self.B, self.k + 1, -1)
        verify_batch(self.draft_logits, self.target_logits, self.cands, self.temps.view(-1), seed=self.seed,
                     offset_tensor=self.verify_offset, out=self.result)

    def _capture(self, fn):
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream(self.dev)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                fn()
        torch.cuda.current_stream().wait_stream(st)
        return g

    def prepare(self):
        """One eager step (sizes every workspace), then the graph captures."""
        self._propose()
        self._verify_forward()
        torch.cuda.synchronize()
        if self.use_graphs:
            self.g_draft = self._capture(self._propose)
            self.g_target = self._capture(self._verify_forward)
            self.graph_target_logits = self.target_logits  # the graph's output buffer

    def step(self) -> VerifyResult:
        """One step; the result (accepted counts, bonus tokens) is the step's device buffer."""
        if self.use_graphs:
            self.g_draft.replay()
            self.g_target.replay()
            self.target_logits = self.graph_target_logits
        else:
            self._propose()
            self._verify_forward()
        self.n_steps += 1
        return self.result

    def close(self):
        self.g_draft = self.g_target = None
