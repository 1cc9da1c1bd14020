"""Multi-GPU partition layer: one process per GPU, torch.distributed for the plumbing.

Two modes, as in the reference's parallel layout:

* **Sequence sharding** (the primary mode; independent sequences): every rank
  holds the full weights and its own KV pool and runs the decode / verify path on
  a contiguous shard of the batch.  No collective runs on the data path; the only
  exchange is the tiny per-step result (accepted length and bonus token per
  sequence), gathered after the step.
* **Tensor parallel** (head sharding, ``nanovllm/layers/linear.py:51-170`` and
  ``nanovllm/models/qwen3.py:29-35``): q and kv heads split evenly across ranks,
  so the attention kernel runs unchanged with Hq/tp and Hkv/tp heads; the
  row-parallel projections (o_proj, down_proj) all-reduce their partial sums
  (``linear.py:165-170``) over NCCL, with the bias added on rank 0 only (:166).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Balanced contiguous [start, end) of n items for ``rank`` of ``world``."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class SequenceShard:
    start: int
    end: int

    @property
    def size(self) -> int:
        return self.end - self.start

    def take(self, t: torch.Tensor, rows_per_seq: int = 1) -> torch.Tensor:
        """Rows of this shard from a per-sequence (or per-query-row) tensor."""
        return t[self.start * rows_per_seq:self.end * rows_per_seq]


def sequence_shard(num_seqs: int, world: int, rank: int) -> SequenceShard:
    return SequenceShard(*shard_range(num_seqs, world, rank))


def gather_step_results(accepted: torch.Tensor, bonus: torch.Tensor, num_seqs: int,
                        group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather the per-sequence (accepted, bonus) of every rank's shard, in sequence order.

    The only cross-rank traffic of sequence sharding: 2 x int64 per sequence.
    """
    world = dist.get_world_size(group)
    if world == 1:
        return accepted, bonus
    pack = torch.stack([accepted.to(torch.int64), bonus.to(torch.int64)], dim=1)
    width = max(shard_range(num_seqs, world, r)[1] - shard_range(num_seqs, world, r)[0]
                for r in range(world))
    padded = torch.zeros(width, 2, dtype=torch.int64, device=pack.device)
    padded[:pack.shape[0]] = pack
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    rows = []
    for r in range(world):
        s, e = shard_range(num_seqs, world, r)
        rows.append(bufs[r][:e - s])
    allr = torch.cat(rows, dim=0)
    return allr[:, 0], allr[:, 1]


# ------------------------------------------------------------------ tensor parallel
@dataclass
class HeadShard:
    q_start: int
    q_end: int
    kv_start: int
    kv_end: int

    @property
    def num_q_heads(self) -> int:
        return self.q_end - self.q_start

    @property
    def num_kv_heads(self) -> int:
        return self.kv_end - self.kv_start


def tp_head_shard(num_q_heads: int, num_kv_heads: int, tp: int, rank: int) -> HeadShard:
    """Heads of ``rank`` under tensor parallelism (qwen3.py:29-35 divides both by tp)."""
    if num_q_heads % tp or num_kv_heads % tp:
        raise ValueError(f"heads ({num_q_heads}, {num_kv_heads}) must divide by tp={tp}")
    hq, hk = num_q_heads // tp, num_kv_heads // tp
    return HeadShard(rank * hq, (rank + 1) * hq, rank * hk, (rank + 1) * hk)


def row_parallel_shard(weight_cols: int, tp: int, rank: int) -> tuple[int, int]:
    """Input-dim slice of a row-parallel weight (linear.py:151-160 narrows dim 1)."""
    if weight_cols % tp:
        raise ValueError(f"input size {weight_cols} must divide by tp={tp}")
    per = weight_cols // tp
    return rank * per, (rank + 1) * per


class RowParallelInt8Linear(torch.nn.Module):
    """Row-parallel W8A16 projection: local int8_linear on this rank's input slice, then
    an all-reduce of the partial sums (``RowParallelLinear.forward``, linear.py:165-170).

    ``matmul`` defaults to the sm_100a ``int8_linear``; CPU tests pass a reference
    product to exercise the sharding and the collective on gloo ranks.
    """

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor],
                 tp_rank: int, tp_size: int, group=None, matmul: Optional[Callable] = None):
        super().__init__()
        s, e = row_parallel_shard(qweight.shape[1], tp_size, tp_rank)
        self.qweight = qweight[:, s:e].contiguous()
        self.scale = scale
        self.bias = bias if tp_rank == 0 else None
        self.tp_rank, self.tp_size, self.group = tp_rank, tp_size, group
        if matmul is None:
            from .quant import int8_linear
            matmul = int8_linear
        self.matmul = matmul

    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        y = self.matmul(x_local, self.qweight, self.scale, self.bias)
        if self.tp_size > 1:
            dist.all_reduce(y, group=self.group)
        return y


# ------------------------------------------------------- vocabulary-parallel embedding
def vocab_shard(num_embeddings: int, tp: int, rank: int) -> tuple[int, int]:
    """Rows [start, end) of the embedding / LM-head table held by ``rank``
    (``VocabParallelEmbedding.__init__``, embed_head.py:19-23: equal shards, no remainder)."""
    if num_embeddings % tp:
        raise ValueError(f"vocabulary {num_embeddings} must divide by tp={tp}")
    per = num_embeddings // tp
    return rank * per, (rank + 1) * per


class VocabParallelEmbedding(torch.nn.Module):
    """Token embedding with the table split by rows across tp ranks
    (``VocabParallelEmbedding``, embed_head.py:9-43).

    Each rank looks up the ids that fall in its shard, zeroes the rows of the others
    (:36-40) and the ranks sum their outputs with one all-reduce (:41).  ``weight`` is
    the full table or this rank's shard (``weight_loader``, :27-32, narrows dim 0).
    """

    def __init__(self, weight: torch.Tensor, tp_rank: int = 0, tp_size: int = 1, group=None,
                 num_embeddings: Optional[int] = None):
        super().__init__()
        n = num_embeddings if num_embeddings is not None else weight.shape[0]
        self.vocab_start, self.vocab_end = vocab_shard(n, tp_size, tp_rank)
        per = self.vocab_end - self.vocab_start
        if weight.shape[0] == n and tp_size > 1:
            weight = weight[self.vocab_start:self.vocab_end]
        if weight.shape[0] != per:
            raise ValueError(f"weight has {weight.shape[0]} rows, shard wants {per}")
        self.weight = weight.contiguous()
        self.num_embeddings = n
        self.tp_rank, self.tp_size, self.group = tp_rank, tp_size, group

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        if self.tp_size == 1:
            return torch.nn.functional.embedding(ids, self.weight)
        mask = (ids >= self.vocab_start) & (ids < self.vocab_end)
        y = torch.nn.functional.embedding(mask * (ids - self.vocab_start), self.weight)
        y = mask.unsqueeze(-1) * y
        dist.all_reduce(y, group=self.group)
        return y


class ParallelLMHead(VocabParallelEmbedding):
    """LM head over the same row split (``ParallelLMHead``, embed_head.py:44-75).

    ``forward(x)`` keeps the reference's contract: every rank computes its logit
    columns and rank 0 gathers them into the full (tokens, V) row (:70-74; the other
    ranks get None).  ``forward_shard(x)`` returns this rank's columns only, the
    input of ``VocabParallelVerify`` / ``verify_batch_vocab_parallel``, which decide
    the verify step from the shards and never assemble the 151936-wide row.
    Trimming to the last row of each sequence at prefill (:66-68) is the caller's.
    """

    def forward_shard(self, x: torch.Tensor) -> torch.Tensor:
        return torch.nn.functional.linear(x, self.weight)

    def forward(self, x: torch.Tensor) -> Optional[torch.Tensor]:
        logits = self.forward_shard(x)
        if self.tp_size == 1:
            return logits
        parts = [torch.empty_like(logits) for _ in range(self.tp_size)] if self.tp_rank == 0 else None
        dist.gather(logits, parts, dst=0, group=self.group)
        return torch.cat(parts, dim=-1) if self.tp_rank == 0 else None
