"""Speculative-decoding rejection sampling: host side of ``csrc/verify_sample.cu``.

Mirror of ``nanovllm/spec_decode/verify.py:32-175``: same arguments, same
``VerifyResult`` fields and dtypes (int64 accepted / bonus / n_proposed, bool
accept_mask), same alignment (candidate j against target row j, bonus from row
``accepted``), same residual fallback and clamps.  The two random draws of the
reference (``torch.rand`` at :120 and ``exponential_`` at :209) are either given
explicitly (``uniforms`` / ``exponentials``) or generated inside the kernel from
Philox4x32-10 keyed by ``(seed, offset)``; with neither given, the seed is
``torch.initial_seed()`` and the offset advances by one per call.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib


@dataclass
class VerifyResult:
    accepted: torch.Tensor      # (batch,) int64 accepted prefix length
    bonus: torch.Tensor         # (batch,) int64 token emitted after the prefix (always valid)
    n_proposed: torch.Tensor    # (batch,) int64
    accept_mask: torch.Tensor   # (batch, k) bool


_offsets = itertools.count()


def workspace_bytes(B: int, k: int, target_rows: int, V: int) -> int:
    return int(_lib.lib().sdb_verify_workspace_size(B, k, target_rows, V))


@torch.no_grad()
def verify_batch(draft_probs: torch.Tensor, target_logits: torch.Tensor, draft_tokens: torch.Tensor,
                 temperatures: Optional[torch.Tensor] = None, draft_is_point_mass: bool = False, *,
                 uniforms: Optional[torch.Tensor] = None, exponentials: Optional[torch.Tensor] = None,
                 seed: Optional[int] = None, offset: Optional[int] = None,
                 out: Optional[VerifyResult] = None,
                 offset_tensor: Optional[torch.Tensor] = None) -> VerifyResult:
    """draft_probs (B, k, V): raw draft logits (probabilities if ``draft_is_point_mass``);
    target_logits (B, k+1, V) (or (B, k, V)); draft_tokens (B, k); temperatures (B,) or None.

    ``offset_tensor``: a one-element int64 CUDA tensor holding the Philox offset, read when
    the kernels run and advanced by one after the call, so a call captured in a CUDA graph
    draws new values on every replay (in-kernel draws only: no ``uniforms`` /
    ``exponentials``, no ``offset``)."""
    _lib.require_cuda(draft_probs, target_logits, draft_tokens, temperatures, uniforms, exponentials)
    B, k, V = draft_probs.shape
    Tr = target_logits.shape[1]
    if target_logits.shape[0] != B or target_logits.shape[2] != V or Tr not in (k, k + 1):
        raise ValueError(f"target_logits {tuple(target_logits.shape)} vs draft {tuple(draft_probs.shape)}")
    if tuple(draft_tokens.shape) != (B, k):
        raise ValueError(f"draft_tokens must be ({B}, {k})")
    # float32 / bfloat16 / float16 logits are read as they are (converted exactly in the
    # kernels, as the reference's .float()); other types are converted here
    draft = (draft_probs if draft_probs.dtype in _lib.DTYPE_CODE else draft_probs.float()).contiguous()
    target = (target_logits if target_logits.dtype in _lib.DTYPE_CODE else target_logits.float()).contiguous()
    tokens = draft_tokens.to(torch.int64).contiguous()
    temps = None
    if temperatures is not None:
        t = temperatures.float()
        temps = (t.expand(B) if t.dim() == 0 else t.reshape(B)).contiguous()
    u = None if uniforms is None else uniforms.float().reshape(B, k).contiguous()
    e = None if exponentials is None else exponentials.float().reshape(B, V).contiguous()
    if seed is None:
        seed = torch.initial_seed()
    if offset is None:
        offset = next(_offsets)
    if out is None:
        dev = draft.device
        out = VerifyResult(accepted=torch.empty(B, dtype=torch.int64, device=dev),
                           bonus=torch.empty(B, dtype=torch.int64, device=dev),
                           n_proposed=torch.full((B,), k, dtype=torch.int64, device=dev),
                           accept_mask=torch.empty(B, k, dtype=torch.bool, device=dev))
    L = _lib.lib()
    need = int(L.sdb_verify_workspace_size(B, k, Tr, V))
    ws = _lib.WORKSPACES.get(draft.device, "verify", need)
    if offset_tensor is not None:
        if u is not None or e is not None:
            raise ValueError("offset_tensor draws in-kernel: no uniforms / exponentials")
        if offset_tensor.dtype != torch.int64 or offset_tensor.numel() != 1 or not offset_tensor.is_cuda:
            raise ValueError("offset_tensor must be a one-element int64 CUDA tensor")
        rc = L.sdb_verify_batch_dev_offset(
            draft.data_ptr(), _lib.DTYPE_CODE[draft.dtype], target.data_ptr(), _lib.DTYPE_CODE[target.dtype],
            tokens.data_ptr(), _lib.ptr(temps), int(seed) & (2**64 - 1), offset_tensor.data_ptr(),
            1 if draft_is_point_mass else 0, out.accepted.data_ptr(), out.bonus.data_ptr(),
            out.accept_mask.data_ptr(), B, k, Tr, V, ws.data_ptr(), ws.numel(), _lib.stream_of(draft))
        _lib.check(rc, "sdb_verify_batch_dev_offset")
        return out
    rc = L.sdb_verify_batch_ex(draft.data_ptr(), _lib.DTYPE_CODE[draft.dtype], target.data_ptr(),
                               _lib.DTYPE_CODE[target.dtype], tokens.data_ptr(), _lib.ptr(temps),
                               _lib.ptr(u), _lib.ptr(e), int(seed) & (2**64 - 1), int(offset) & (2**64 - 1),
                               1 if draft_is_point_mass else 0, out.accepted.data_ptr(),
                               out.bonus.data_ptr(), out.accept_mask.data_ptr(), B, k, Tr, V,
                               ws.data_ptr(), ws.numel(), _lib.stream_of(draft))
    _lib.check(rc, "sdb_verify_batch_ex")
    return out


def philox_draws(rows: int, cols: int, seed: int, offset: int, stream_id: int,
                 device="cuda") -> torch.Tensor:
    """The sampler's Philox stream written out: 0 = acceptance uniforms, 1 = exponentials."""
    outp = torch.empty(rows, cols, dtype=torch.float32, device=device)
    rc = _lib.lib().sdb_philox_fill(outp.data_ptr(), rows, cols, int(seed) & (2**64 - 1),
                                    int(offset) & (2**64 - 1), stream_id, _lib.stream_of(outp))
    _lib.check(rc, "sdb_philox_fill")
    return outp


# ------------------------------------------------------------------ vocabulary-parallel form
class VocabParallelVerify:
    """One rank's part of ``verify_batch`` when the LM head is split by vocabulary
    columns across ``tp`` ranks (``ParallelLMHead``, ``nanovllm/layers/embed_head.py:56-75``).

    The reference gathers every rank's (rows, V/tp) logits on rank 0 (``dist.gather``,
    :71-74) and samples there.  Here each rank keeps its shard, and the ranks exchange
    only per-sequence statistics, in three all-gathers:

    1. each row's local (max, sum of exp) and the candidates' logits on the rank that
       owns their columns;
    2. the residual and p sums of row ``accepted``;
    3. each rank's best (value, global column) of the bonus argmax.

    Every rank ends with identical ``accepted`` / ``accept_mask`` / ``bonus``.  Draws are
    keyed by global columns, so the results equal the single-device call on the full
    logits, except where two values tie within float32 rounding: the shards' sums are
    added in another order.

    Drive it with ``verify_batch_vocab_parallel`` (torch.distributed), or call
    ``phase(1..4, gathered)`` yourself with any all-gather that concatenates the ranks'
    ``send`` tensors in rank order.
    """

    def __init__(self, draft_shard, target_shard, draft_tokens, temperatures=None,
                 draft_is_point_mass=False, *, vocab_start: int, vocab_size: int, tp: int,
                 seed: int, offset: int, uniforms=None, exponentials=None):
        _lib.require_cuda(draft_shard, target_shard, draft_tokens, temperatures, uniforms, exponentials)
        B, k, Vl = draft_shard.shape
        Tr = target_shard.shape[1]
        if target_shard.shape[0] != B or target_shard.shape[2] != Vl or Tr not in (k, k + 1):
            raise ValueError(f"target shard {tuple(target_shard.shape)} vs draft {tuple(draft_shard.shape)}")
        if not 0 <= vocab_start <= vocab_size - Vl:
            raise ValueError(f"columns [{vocab_start}, {vocab_start + Vl}) outside the vocabulary {vocab_size}")
        self.draft = (draft_shard if draft_shard.dtype in _lib.DTYPE_CODE else draft_shard.float()).contiguous()
        self.target = (target_shard if target_shard.dtype in _lib.DTYPE_CODE else target_shard.float()).contiguous()
        self.tokens = draft_tokens.to(torch.int64).reshape(B, k).contiguous()
        self.temps = None
        if temperatures is not None:
            t = temperatures.float()
            self.temps = (t.expand(B) if t.dim() == 0 else t.reshape(B)).contiguous()
        self.u = None if uniforms is None else uniforms.float().reshape(B, k).contiguous()
        self.e = None if exponentials is None else exponentials.float().reshape(B, vocab_size).contiguous()
        self.B, self.k, self.Tr, self.Vl = B, k, Tr, Vl
        self.col0, self.V, self.tp = vocab_start, vocab_size, tp
        self.seed, self.offset, self.point = int(seed), int(offset), bool(draft_is_point_mass)
        dev = self.draft.device
        self.result = VerifyResult(accepted=torch.empty(B, dtype=torch.int64, device=dev),
                                   bonus=torch.empty(B, dtype=torch.int64, device=dev),
                                   n_proposed=torch.full((B,), k, dtype=torch.int64, device=dev),
                                   accept_mask=torch.empty(B, k, dtype=torch.bool, device=dev))
        L = _lib.lib()
        need = int(L.sdb_verify_workspace_size(B, k, Tr, Vl))
        # a workspace of its own: the decisions live there between the phases
        self.ws = torch.zeros(need, dtype=torch.uint8, device=dev)

    def send_size(self, phase: int) -> int:
        return int(_lib.lib().sdb_verify_shard_send_floats(self.B, self.k, self.Tr, phase))

    def phase(self, n: int, gathered: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """Run phase ``n`` (1-4) with the previous exchange ``gathered`` (tp x send floats,
        rank-major; none for phase 1).  Returns this rank's next ``send`` (none after 4)."""
        send = None
        if n < 4:
            send = torch.empty(self.send_size(n), dtype=torch.float32, device=self.draft.device)
        if gathered is not None:
            gathered = gathered.float().contiguous()
        r = self.result
        rc = _lib.lib().sdb_verify_batch_shard(
            n, self.draft.data_ptr(), _lib.DTYPE_CODE[self.draft.dtype], self.target.data_ptr(),
            _lib.DTYPE_CODE[self.target.dtype], self.tokens.data_ptr(), _lib.ptr(self.temps), _lib.ptr(self.u),
            _lib.ptr(self.e), self.seed & (2**64 - 1), self.offset & (2**64 - 1), 1 if self.point else 0,
            r.accepted.data_ptr(), r.bonus.data_ptr(), r.accept_mask.data_ptr(), self.B, self.k, self.Tr,
            self.Vl, self.col0, self.V, self.tp, _lib.ptr(gathered), _lib.ptr(send), self.ws.data_ptr(),
            self.ws.numel(), _lib.stream_of(self.draft))
        _lib.check(rc, "sdb_verify_batch_shard")
        return send


@torch.no_grad()
def verify_batch_vocab_parallel(draft_shard: torch.Tensor, target_shard: torch.Tensor,
                                draft_tokens: torch.Tensor, temperatures: Optional[torch.Tensor] = None,
                                draft_is_point_mass: bool = False, *, vocab_start: int, vocab_size: int,
                                group=None, seed: Optional[int] = None, offset: Optional[int] = None,
                                uniforms: Optional[torch.Tensor] = None,
                                exponentials: Optional[torch.Tensor] = None) -> VerifyResult:
    """``verify_batch`` over vocabulary shards, one process per GPU (torch.distributed,
    NCCL).  Each rank passes its columns ``[vocab_start, vocab_start + V/tp)`` of the
    draft and target logits; every rank returns the same result.  With ``seed`` /
    ``offset`` not given, rank 0's ``torch.initial_seed()`` and offset counter are
    broadcast (the draws must agree across ranks)."""
    import torch.distributed as dist
    tp = dist.get_world_size(group)
    if seed is None or offset is None:
        so = torch.tensor([torch.initial_seed() & (2**63 - 1), next(_offsets)], dtype=torch.int64,
                          device=draft_shard.device)
        dist.broadcast(so, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        seed = int(so[0]) if seed is None else seed
        offset = int(so[1]) if offset is None else offset
    vp = VocabParallelVerify(draft_shard, target_shard, draft_tokens, temperatures, draft_is_point_mass,
                             vocab_start=vocab_start, vocab_size=vocab_size, tp=tp, seed=seed, offset=offset,
                             uniforms=uniforms, exponentials=exponentials)
    gathered = None
    for n in (1, 2, 3, 4):
        send = vp.phase(n, gathered)
        if send is not None:
            gathered = torch.empty(tp * send.numel(), dtype=torch.float32, device=send.device)
            dist.all_gather_into_tensor(gathered, send, group=group)
    return vp.result
