"""Partition layer on CPU: shard arithmetic and two gloo ranks for the collectives."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package


def test_shard_range_covers_everything_once():
    pkg = load_package()
    from specdec_nanovllm_b200.partition import shard_range
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            seen = []
            sizes = []
            for r in range(world):
                s, e = shard_range(n, world, r)
                seen.extend(range(s, e))
                sizes.append(e - s)
            assert seen == list(range(n))
            assert max(sizes) - min(sizes) <= 1
    assert pkg is not None


def test_tp_head_shard():
    load_package()
    from specdec_nanovllm_b200.partition import tp_head_shard
    hs = [tp_head_shard(32, 8, 8, r) for r in range(8)]
    assert all(h.num_q_heads == 4 and h.num_kv_heads == 1 for h in hs)
    assert hs[3].q_start == 12 and hs[3].kv_start == 3
    with pytest.raises(ValueError):
        tp_head_shard(32, 8, 3, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        load_package()
        from specdec_nanovllm_b200.partition import (ParallelLMHead, RowParallelInt8Linear,
                                                     VocabParallelEmbedding, gather_step_results,
                                                     sequence_shard)
        # --- sequence sharding: each rank produces results for its own sequences
        B = 7
        sh = sequence_shard(B, world, rank)
        acc = torch.arange(sh.start, sh.end) * 10
        bonus = torch.arange(sh.start, sh.end) + 1000
        ga, gb = gather_step_results(acc, bonus, B)
        results[f"seq{rank}"] = (ga.tolist(), gb.tolist())
        # --- tensor parallel row-parallel projection: all-reduce of partial sums
        g = torch.Generator().manual_seed(3)
        N, K, M = 16, 64, 3
        q = torch.randint(-127, 128, (N, K), generator=g).to(torch.int8)
        s = torch.rand(N, generator=g) * 0.01
        bias = torch.randn(N, generator=g)
        x = torch.randn(M, K, generator=g)

        def ref_matmul(xl, ql, sl, bl):
            y = xl.float() @ (ql.float() * sl[:, None]).T
            return y + bl if bl is not None else y

        layer = RowParallelInt8Linear(q, s, bias, rank, world, matmul=ref_matmul)
        ks = K // world
        y = layer(x[:, rank * ks:(rank + 1) * ks])
        full = ref_matmul(x, q, s, bias)
        results[f"tp{rank}"] = float((y - full).abs().max())
        # --- vocabulary-parallel embedding and LM head (embed_head.py:33-75)
        V, H = 10, 6
        table = torch.randn(V, H, generator=g)
        ids = torch.tensor([[0, 4, 5, 9], [7, 2, 3, 1]])
        emb = VocabParallelEmbedding(table, rank, world)
        results[f"emb{rank}"] = bool(torch.equal(emb(ids), table[ids]))
        head = ParallelLMHead(table, rank, world)
        h = torch.randn(3, H, generator=g)
        full_logits = h @ table.T
        shard = head.forward_shard(h)
        lo, hi = rank * V // world, (rank + 1) * V // world
        results[f"head_shard{rank}"] = bool(torch.allclose(shard, full_logits[:, lo:hi], atol=1e-6))
        gathered = head(h)
        results[f"head{rank}"] = (None if gathered is None
                                  else bool(torch.allclose(gathered, full_logits, atol=1e-6)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_sequence_gather_and_row_parallel_allreduce():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, port, results), nprocs=world, join=True)
        res = dict(results)
    for r in range(world):
        acc, bonus = res[f"seq{r}"]
        assert acc == [i * 10 for i in range(7)]
        assert bonus == [i + 1000 for i in range(7)]
        assert res[f"tp{r}"] < 1e-4
        assert res[f"emb{r}"] and res[f"head_shard{r}"]
    assert res["head0"] is True and res["head1"] is None


def test_vocab_shard_and_single_rank_embedding():
    load_package()
    from specdec_nanovllm_b200.partition import ParallelLMHead, VocabParallelEmbedding, vocab_shard
    assert [vocab_shard(151936, 8, r) for r in (0, 7)] == [(0, 18992), (132944, 151936)]
    with pytest.raises(ValueError):
        vocab_shard(10, 3, 0)
    t = torch.randn(12, 4)
    ids = torch.tensor([3, 11, 0])
    assert torch.equal(VocabParallelEmbedding(t)(ids), t[ids])
    x = torch.randn(2, 4)
    assert torch.allclose(ParallelLMHead(t)(x), x @ t.T)
