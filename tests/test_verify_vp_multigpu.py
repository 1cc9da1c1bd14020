"""The multi-GPU forms on 2 GPUs (one process per GPU, NCCL): verify_batch over
vocabulary shards (every rank must return the single-device result on the full
logits) and the row-parallel W8A16 projection (all-reduced partial sums against the
single-device product, bf16 bar).  Skipped when fewer than two GPUs are visible.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    from conftest import load_package
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        pkg = load_package()
        B, k, V = 32, 6, 151936
        g = torch.Generator().manual_seed(11)
        target = (torch.randn(B, k + 1, V, generator=g) * 3.0).to(torch.bfloat16).cuda()
        draft = target[:, :k].float() + torch.randn(B, k, V, generator=g).cuda()
        tokens = torch.randint(0, V, (B, k), generator=g).cuda()
        per = V // world
        s, e = rank * per, (rank + 1) * per
        r = pkg.verify_batch_vocab_parallel(draft[:, :, s:e], target[:, :, s:e], tokens, None,
                                            vocab_start=s, vocab_size=V, seed=3, offset=1)
        want = pkg.verify_batch(draft, target, tokens, None, seed=3, offset=1)
        torch.cuda.synchronize()
        results[rank] = (torch.equal(r.accepted, want.accepted), torch.equal(r.accept_mask, want.accept_mask),
                         torch.equal(r.bonus, want.bonus), int(want.accepted.sum()))
        # row-parallel o_proj (linear.py:165-170): each rank multiplies its input slice
        from specdec_nanovllm_b200.partition import RowParallelInt8Linear
        from specdec_nanovllm_b200.workloads import cfg3_inputs
        x, q, sc = cfg3_inputs(64, 4096, 2560, seed=4)
        layer = RowParallelInt8Linear(q, sc, None, rank, world)
        ks = 4096 // world
        y = layer(x[:, rank * ks:(rank + 1) * ks].contiguous())
        # the same partial products made on one device and added in fp16, as NCCL adds them
        parts = [pkg.int8_linear(x[:, r * ks:(r + 1) * ks].contiguous(), q[:, r * ks:(r + 1) * ks].contiguous(), sc)
                 for r in range(world)]
        emulated = parts[0]
        for pr in parts[1:]:
            emulated = emulated + pr
        full = pkg.int8_linear(x, q, sc)
        torch.cuda.synchronize()
        # against the one-device product: the fp16 rounding of each partial (|partial| up to
        # ~200, half an ulp 0.06) on top of the bf16 bar
        bound = 2e-2 * full.float().abs() + 2e-3 + sum(pr.float().abs() for pr in parts) * 2.0 ** -11
        results[f"tp{rank}"] = (torch.equal(y, emulated), float(((y.float() - full.float()).abs() - bound).max()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_nccl():
    world = 2
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    for rank in range(world):
        acc, mask, bonus, n = res[rank]
        assert acc and mask and bonus, res
        assert 0 < n < 32 * 6
        same, excess = res[f"tp{rank}"]
        assert same and excess <= 0.0, res
