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
