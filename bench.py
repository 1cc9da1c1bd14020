"""Benchmark of the speculative-verify attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one process per GPU)

Workload (BASELINE configuration 2 at its target point): paged verify attention,
Qwen3-4B shapes (32 q / 8 kv heads, head_dim 128), k = 6 (7 causal query rows per
sequence), 64 sequences of 4096 cached tokens, page 256, scattered block tables,
bf16, synthetic N(0,1) data.  A step is one kernel pass over the batch.  Multi-GPU
runs shard the 64 sequences over the ranks (strong scaling: 8 per GPU at N = 8),
each rank with its own KV pool; no collective on the data path.

Metric: HBM GB/s of algorithmic bytes (every visible K/V row once + q in + o out)
per second for the whole batch, timed with CUDA events around captured graphs of
steps (max over ranks).  One JSON line on rank 0.  ``--impl reference`` times the
reference's CPU torch path (``paged_decode_attention_ref`` restated with the k+1
causal rows, oracle/torch_ref.py) on this host's cores.
"""

from __future__ import annotations

import argparse
import datetime
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CTX, K_SPEC, PAGE = 4096, 6, 256
HQ, HKV, D = 32, 8, 128
N_Q = K_SPEC + 1
METRIC = "verify-attn HBM GB/s (% of 8 TB/s)"
FALLBACK_HBM_GBS = 6650.0


def load_package():
    name = "specdec_nanovllm_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = os.path.join(ROOT, "specdec-nanovllm_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(workload: str):
    """dram bytes per launch from the committed ncu summary (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(workload)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", "100"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- CPU legs
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_case(n_seqs: int, seed: int = 0):
    """A host copy of ``n_seqs`` sequences of the workload, bf16 like the GPU run."""
    import torch
    g = torch.Generator().manual_seed(seed)
    nblk = CTX // PAGE
    nb = n_seqs * nblk
    k = torch.randn(nb, PAGE, HKV, D, generator=g).to(torch.bfloat16)
    v = torch.randn(nb, PAGE, HKV, D, generator=g).to(torch.bfloat16)
    q = torch.randn(n_seqs * N_Q, HQ, D, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g).to(torch.int32).reshape(n_seqs, nblk)
    cl = torch.full((n_seqs,), CTX, dtype=torch.int32)
    return q, k, v, bt, cl


def seq_bytes() -> int:
    """Algorithmic bytes of one sequence of the workload (bf16 K/V rows + q + o)."""
    return CTX * 2 * HKV * D * 2 + 2 * N_Q * HQ * D * 2


class CpuReference:
    """The reference's CPU torch path (``paged_decode_attention_ref``, restated in
    oracle/torch_ref.py with the k+1 causal rows) on this host's cores, one bounded
    sample of sequences per step."""

    def __init__(self, per_step_s: float):
        import torch
        from oracle.torch_ref import paged_attention_torch
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.fn = paged_attention_torch
        self.data = cpu_case(4)
        q, k, v, bt, cl = self.data
        self.run([0])                                   # warm-up
        t0 = time.perf_counter()
        self.run([1])
        per_seq = max(time.perf_counter() - t0, 1e-3)
        self.n = max(1, min(64, int(per_step_s / per_seq)))
        self.seqs = [i % 4 for i in range(self.n)]

    def run(self, seqs=None):
        q, k, v, bt, cl = self.data
        return self.fn(q, k, v, bt, cl, D ** -0.5, n_q=N_Q, seqs=self.seqs if seqs is None else seqs)

    def describe(self) -> str:
        return (f"{self.n} sequence(s) of the workload per step (ctx {CTX}, k={K_SPEC}, Qwen3-4B heads, bf16 "
                f"inputs); torch restatement of paged_decode_attention_ref with the k+1 causal rows, "
                f"{self.threads} threads, {cpu_model()}")


def time_cpu_reference(per_step_s: float, steps: int):
    """(GB/s, threads, description) of the CPU baseline: median over ``steps`` samples."""
    ref = CpuReference(per_step_s)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        ref.run()
        times.append(time.perf_counter() - t0)
    gbs = ref.n * seq_bytes() / statistics.median(times) / 1e9
    return gbs, ref.threads, ref.describe() + f", median of {steps}"


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    total_steps = args.steps + args.warmup
    ref = CpuReference(per_step_s=max(0.05, 150.0 / max(total_steps, 1)))
    for _ in range(args.warmup):
        ref.run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref.run()
    dt = time.perf_counter() - t0
    gbs = ref.n * seq_bytes() * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / max(args.steps, 1) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args.global_batch), "global_batch": args.global_batch,
                   "seq_len": CTX, "k": K_SPEC, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": ref.threads, "kind": "port",
                         "sample": ref.describe()},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- our arm
def workload_name(global_batch: int) -> str:
    return (f"verify-attn B={global_batch} ctx={CTX} k={K_SPEC} (Qwen3-4B heads 32/8, head_dim 128, page {PAGE}), "
            f"sequences sharded over the GPUs")


def graph_len(steps: int, cap: int = 20) -> int:
    """Steps per captured graph: the largest divisor of ``steps`` up to ``cap``."""
    for g in range(min(cap, steps), 0, -1):
        if steps % g == 0:
            return g
    return 1


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    pkg = load_package()
    from specdec_nanovllm_b200 import workloads
    from specdec_nanovllm_b200.partition import shard_range
    from oracle.attention import algorithmic_bytes

    lo, hi = shard_range(args.global_batch, world, rank)
    B = hi - lo
    case = workloads.paged_case([CTX] * B, N_Q, Hq=HQ, Hkv=HKV, D=D, page=PAGE,
                                dtype=torch.bfloat16, device=dev, seed=1000 + lo,
                                extra_blocks=0, generate_on_device=True)
    bytes_rank = algorithmic_bytes([CTX] * B, N_Q, HQ, HKV, D, 2, 2)
    bytes_total = algorithmic_bytes([CTX] * args.global_batch, N_Q, HQ, HKV, D, 2, 2)
    out = torch.empty_like(case.q)
    G = graph_len(args.steps)

    def step():
        pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                            case.scale, n_q=N_Q, out=out)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Host cost of one eager call (launches queue behind the GPU, so the wall time of
    # issuing them is the host's own work per call).
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    n_host = 200
    t0 = time.perf_counter()
    for _ in range(n_host):
        step()
    host_us = (time.perf_counter() - t0) / n_host * 1e6
    torch.cuda.synchronize()

    # ---- device timing: G steps per CUDA graph (the reference runs its verify step as a
    # captured graph, model_runner.py:1257-1310), EXACTLY args.steps steps timed
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cap):
        for _ in range(G):
            step()
    torch.cuda.current_stream().wait_stream(cap)
    for _ in range(max(1, args.warmup // G)):
        g.replay()
    barrier()
    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)  # the sampler's first reading lands inside the timed region
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record()
    for _ in range(args.steps // G):
        g.replay()
    ev1.record()
    barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_step = ms / args.steps
    value = bytes_total / (ms_step * 1e-3) / 1e9
    del g

    # ---- e2e: the public call with pinned host buffers and copies inside the timed region.
    # Every step copies its query rows, block table and lengths host->device and reads its
    # output back device->host.  Copies run on their own streams, double-buffered, so step
    # i's copies overlap step i-1's attention; G such steps are one captured graph.
    q_h = case.q.cpu().pin_memory()
    bt_h = case.block_tables.cpu().pin_memory()
    cl_h = case.cache_seqlens.cpu().pin_memory()
    out_h = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    q_d = [torch.empty_like(case.q) for _ in range(2)]
    bt_d = [torch.empty_like(case.block_tables) for _ in range(2)]
    cl_d = [torch.empty_like(case.cache_seqlens) for _ in range(2)]
    o_d = [torch.empty_like(out) for _ in range(2)]
    comp = torch.cuda.Stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        j = i & 1
        s_in.wait_event(ev_comp[j])              # step i-2 finished reading q_d[j]
        with torch.cuda.stream(s_in):
            q_d[j].copy_(q_h, non_blocking=True)
            bt_d[j].copy_(bt_h, non_blocking=True)
            cl_d[j].copy_(cl_h, non_blocking=True)
            ev_in[j].record(s_in)
        comp.wait_event(ev_in[j])
        comp.wait_event(ev_out[j])               # step i-2's output has been read back
        pkg.paged_attention(q_d[j], case.k_cache, case.v_cache, bt_d[j], cl_d[j], case.scale,
                            n_q=N_Q, out=o_d[j])
        ev_comp[j].record(comp)
        s_out.wait_event(ev_comp[j])
        with torch.cuda.stream(s_out):
            out_h[j].copy_(o_d[j], non_blocking=True)
            ev_out[j].record(s_out)

    def e2e_block():
        for e in ev_comp + ev_out:
            e.record(comp)
        for i in range(G):
            e2e_step(i)
        comp.wait_event(ev_out[0])
        comp.wait_event(ev_out[1])

    comp.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(comp):
        e2e_block()                              # eager once (sizes nothing new; checks the flow)
    ge = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ge, stream=comp):
        e2e_block()
    torch.cuda.current_stream().wait_stream(comp)
    ge.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps // G):
        ge.replay()
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    e2e_val = bytes_total / (e2e_ms * 1e-3) / 1e9
    last = (G - 1) & 1
    assert torch.equal(out_h[last].to(dev), o_d[last])
    h2d = q_h.numel() * q_h.element_size() + bt_h.numel() * 4 + cl_h.numel() * 4
    d2h = out_h[0].numel() * out_h[0].element_size()
    del ge

    # ---- memory-floor twin (same TMA stream, no math), outside the timed region
    ro_ws = pkg.paged_attention_readonly(case.q, case.k_cache, case.v_cache, case.block_tables,
                                         case.cache_seqlens, n_q=N_Q)
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_ro = 50
    r0.record()
    for _ in range(n_ro):
        pkg.paged_attention_readonly(case.q, case.k_cache, case.v_cache, case.block_tables,
                                     case.cache_seqlens, n_q=N_Q, workspace=ro_ws)
    r1.record()
    torch.cuda.synchronize()
    kv_bytes = CTX * B * 2 * HKV * D * 2
    ro_gbs = kv_bytes / (r0.elapsed_time(r1) / n_ro * 1e-3) / 1e9

    peak, peak_kind = measured_peak()
    per_gpu_gbs = bytes_rank / (ms_step * 1e-3) / 1e9
    traffic = committed_traffic(f"verify-attn B={B} ctx={CTX} k={K_SPEC}")
    kind, slots, _ = pkg.attention.plan(B, N_Q, HQ, HKV, D, PAGE, CTX // PAGE, torch.bfloat16)
    merge = slots > 1
    launches_per_step = 2 if merge else 1  # attention (+ the split merge)

    cpu = None
    if world == 1 and rank == 0 and not args.skip_cpu:
        gbs, threads, desc = time_cpu_reference(per_step_s=4.0, steps=3)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": workload_name(args.global_batch), "global_batch": args.global_batch,
                       "seqs_per_gpu": B, "seq_len": CTX, "k": K_SPEC,
                       "parallelism": f"seq-shard{world}", "plan": f"{kind} x{slots}",
                       "graph_steps": G,
                       "l2": f"no flush: {kv_bytes / 1e9:.2f} GB of KV per GPU per step exceeds the 126 MB L2"
                             if kv_bytes > 126e6 else "KV per GPU fits L2: steps re-read it from L2",
                       "bytes_per_step": bytes_total, "bytes_per_step_per_gpu": bytes_rank},
            "pct_of_8tbs": round(100.0 * per_gpu_gbs / 8000.0, 2),
            "roofline": {"bound": "hbm", "achieved": round(per_gpu_gbs, 2), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(per_gpu_gbs / peak, 4),
                         "traffic": traffic, "kernel": "pa_umma_kernel",
                         "achieved_over": "whole step per GPU (pa_umma_kernel + pa_umma_merge_kernel)"
                                          if merge else "whole step per GPU (pa_umma_kernel)",
                         "readonly_floor_gbs": round(ro_gbs, 2)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 5),
                    "copies": f"pinned host, own streams, double-buffered; {G} steps per captured graph"},
            "host_us_per_call": round(host_us, 1),
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------- tensor-parallel step
def run_tp_step(args):
    """One tensor-parallel verify step of the target's attention block on N GPUs: every
    rank holds 32/N q and 8/N kv heads of the B=64 x 4096 k=6 verify batch, runs the paged
    verify attention over its heads, then its slice of the W8A16 o_proj (row-parallel,
    4096/N input columns -> 2560) and the NCCL all-reduce of the (448, 2560) bf16 partial
    sums (RowParallelLinear, linear.py:165-170).  Times G steps per captured graph, max
    over ranks, plus each part alone."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    pkg = load_package()
    from specdec_nanovllm_b200 import workloads
    from specdec_nanovllm_b200.partition import RowParallelInt8Linear, tp_head_shard
    B = args.global_batch
    hs = tp_head_shard(HQ, HKV, world, rank)
    case = workloads.paged_case([CTX] * B, N_Q, Hq=hs.num_q_heads, Hkv=hs.num_kv_heads, D=D, page=PAGE,
                                dtype=torch.bfloat16, device=dev, seed=2000 + rank, extra_blocks=0,
                                generate_on_device=True)
    T = B * N_Q
    K_o, N_o = workloads.W8A16_SHAPES["o"]
    g = torch.Generator(device=dev).manual_seed(7)
    qw = torch.randint(-127, 128, (N_o, K_o), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
    sc = (torch.randn(N_o, generator=g, device=dev).abs() * 0.01).to(torch.bfloat16)
    oproj = RowParallelInt8Linear(qw, sc, None, rank, world)
    attn_out = torch.empty_like(case.q)

    def attention():
        pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cache_seqlens,
                            case.scale, n_q=N_Q, out=attn_out)

    y = torch.empty(T, N_o, dtype=torch.bfloat16, device=dev)

    def matmul():
        pkg.int8_linear(attn_out.view(T, -1), oproj.qweight, oproj.scale, out=y)

    def allreduce():
        if world > 1:
            dist.all_reduce(y)

    def step():
        attention()
        matmul()
        allreduce()

    def time_graph(fn, G=20, reps=50):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(gr, stream=st):
                for _ in range(G):
                    fn()
        torch.cuda.current_stream().wait_stream(st)
        gr.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (G * reps)
        del gr
        if world > 1:
            t = torch.tensor([us], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        return us

    step()
    parts = {"attention": time_graph(attention), "o_proj_int8": time_graph(matmul)}
    parts["all_reduce"] = time_graph(allreduce) if world > 1 else 0.0
    total = time_graph(step)
    ar_bytes = T * N_o * 2
    if rank == 0:
        line = {"metric": "tensor-parallel verify attention block us/step", "value": round(total, 2), "unit": "us",
                "n_gpus": world, "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"verify attention B={B} ctx={CTX} k={K_SPEC}, heads {hs.num_q_heads}/"
                                       f"{hs.num_kv_heads} per rank, o_proj int8 {K_o // world}->{N_o} per rank, "
                                       f"all-reduce of ({T}, {N_o}) bf16", "parallelism": f"tp{world}"},
                "parts_us": {k: round(v, 2) for k, v in parts.items()},
                "all_reduce_bytes": ar_bytes,
                "all_reduce_busbw_gbs": round(2 * (world - 1) / world * ar_bytes / (parts["all_reduce"] * 1e-6) / 1e9, 1)
                if world > 1 else None}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------- end-to-end step
def run_specdec_e2e(args):
    """a speculative decode step with a random-init Qwen3-4B
    target and Qwen3-0.6B draft (bf16), k = 6, 64 sequences at 2048 tokens of context in
    paged KV caches, CUDA graphs; sequences sharded over the ranks under torchrun.
    Tokens per step = accepted drafts + the bonus token of every sequence."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    load_package()
    from specdec_nanovllm_b200.partition import shard_range
    from specdec_nanovllm_b200.specdec import QWEN3_06B, QWEN3_4B, RandomQwen3, SpecDecodeStep
    Bg, ctx, k = args.global_batch, 2048, K_SPEC
    tp = world if args.tp else 1
    # sequence sharding: each rank its share of the batch; tensor parallel: every rank all
    # of it, with the rank's slice of both models
    lo, hi = shard_range(Bg, world, rank) if tp == 1 else (0, Bg)
    group = dist.group.WORLD if tp > 1 else None
    target = RandomQwen3(QWEN3_4B, dev, seed=1, tp_rank=rank if tp > 1 else 0, tp_size=tp, group=group)
    draft = RandomQwen3(QWEN3_06B, dev, seed=2, tp_rank=rank if tp > 1 else 0, tp_size=tp, group=group)
    st = SpecDecodeStep(target, draft, hi - lo, ctx, k, dev, seed=100 + lo)
    st.prepare()
    steps = max(1, min(args.steps, 50))
    acc_h = torch.empty(steps, hi - lo, dtype=torch.int64, pin_memory=True)
    for _ in range(args.warmup):
        st.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        r = st.step()
        acc_h[i].copy_(r.accepted, non_blocking=True)   # the engine reads the counts back every step
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / steps
    tokens = float((acc_h + 1).sum()) / steps                # accepted drafts + bonus, this rank
    # phases, timed apart (same graphs)
    def phase(fn, n=10):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n
    t_draft = phase(st.g_draft.replay)
    t_target = phase(st.g_target.replay)           # verify forward + verify_batch (one graph)
    from specdec_nanovllm_b200 import verify_batch
    t_verify = phase(lambda: verify_batch(st.draft_logits, st.target_logits, st.cands, st.temps.view(-1),
                                          seed=7, offset=0))
    stats = torch.tensor([ms, tokens, t_draft, t_target, t_verify], device=dev, dtype=torch.float64)
    if world > 1:
        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms, t_draft, t_target, t_verify = float(mx[0]), float(mx[2]), float(mx[3]), float(mx[4])
        tokens = float(sm[1]) if tp == 1 else float(stats[1])   # TP: every rank commits the same tokens
    tok_s = tokens / (ms * 1e-3)
    if rank == 0:
        line = {"metric": "spec-decode tok/s, Qwen3-4B target + Qwen3-0.6B draft, k=6", "value": round(tok_s, 1),
                "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (random-init weights, N(0,1) KV context)",
                "config": {"workload": f"spec decode step, {Bg} sequences x {ctx} context, k={k}, CUDA graphs",
                           "global_batch": Bg, "seq_len": ctx, "k": k,
                           "parallelism": f"tp{world}" if tp > 1 else f"seq-shard{world}"},
                "tokens_per_step": round(tokens, 2),
                "mean_accepted_per_seq": round(tokens / Bg - 1.0, 3),
                "phases_ms": {"draft_k_steps": round(t_draft, 3),
                              "target_verify_forward_and_verify_batch": round(t_target, 3),
                              "verify_batch_alone": round(t_verify, 3)},
                "clocks": clocks}
        print(json.dumps(line), flush=True)
    st.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------- side modes
def _time_events(fn, steps, warmup, per_graph=20):
    """Device ms per call: ``per_graph`` calls captured in one CUDA graph, replayed so that
    short kernels are timed back to back instead of at the host's launch rate."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for _ in range(per_graph):
                fn()
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    torch.cuda.synchronize()
    reps = max(1, steps // per_graph)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / (reps * per_graph)


def run_side(args):
    """Secondary kernels of the path, one JSON line each (single GPU)."""
    import numpy as np
    import torch
    torch.cuda.set_device(0)
    pkg = load_package()
    from specdec_nanovllm_b200 import workloads
    peak, peak_kind = measured_peak()
    steps = min(args.steps, 500)
    if args.mode == "verify_batch":
        from oracle.verify import algorithmic_bytes
        B, k, V = 64, 6, workloads.VOCAB
        draft, target, tokens = workloads.cfg4_inputs(B=B, k=k, V=V, seed=0)
        temps = torch.ones(B, device="cuda")
        res = pkg.verify_batch(draft, target, tokens, temps, seed=1, offset=0)
        ms = _time_events(lambda: pkg.verify_batch(draft, target, tokens, temps, seed=1, offset=0, out=res),
                          steps, args.warmup)
        nbytes = algorithmic_bytes(B, k, V)
        gbs = nbytes / (ms * 1e-3) / 1e9
        line = {"metric": "verify_batch HBM GB/s", "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1,
                "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
                "dtype": "f32", "data": "synthetic",
                "config": {"workload": f"verify_batch B={B} k={k} V={V} (target N(0,9), draft = target + N(0,1), "
                                       "T=1, in-kernel Philox draws)", "bytes_per_step": nbytes},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": round(gbs / peak, 4),
                             "note": "whole call (4 launches) against one read of every logit"},
                "gpu_launches": 4 * steps}
    elif args.mode == "w8a16":
        from oracle.quant import algorithmic_bytes
        M = args.m
        shapes = workloads.W8A16_SHAPES
        # The four projections hold 101 MB of int8 weights, less than the 126 MB L2: every
        # step uses the next of NSET weight copies (404 MB together), so no call finds its
        # weights in L2 from the previous step.
        NSET = 4
        sets = [{n: workloads.cfg3_inputs(M, K, N, seed=16 * j + i) for i, (n, (K, N)) in enumerate(shapes.items())}
                for j in range(NSET)]
        outs = {n: pkg.int8_linear(*sets[0][n]) for n in shapes}
        ctr = [0]

        def step():
            ins = sets[ctr[0] % NSET]
            ctr[0] += 1
            for n in ins:
                pkg.int8_linear(*ins[n], out=outs[n])
        ms = _time_events(step, steps, args.warmup, per_graph=4 * NSET)
        per = {}
        for n in shapes:
            def one(n=n):
                x, q, sc = sets[ctr[0] % NSET][n]
                ctr[0] += 1
                pkg.int8_linear(x, q, sc, out=outs[n])
            ms_n = _time_events(one, steps, args.warmup, per_graph=4 * NSET)
            K, N = shapes[n]
            b = algorithmic_bytes(M, N, K)
            per[n] = {"us": round(ms_n * 1e3, 2), "GB/s": round(b / (ms_n * 1e-3) / 1e9, 1),
                      "TFLOP/s": round(2 * M * N * K / (ms_n * 1e-3) / 1e12, 2)}
        nbytes = sum(algorithmic_bytes(M, N, K) for K, N in shapes.values())
        flops = sum(2 * M * N * K for K, N in shapes.values())
        gbs = nbytes / (ms * 1e-3) / 1e9
        line = {"metric": "w8a16 HBM GB/s (4 Qwen3-4B projections)", "value": round(gbs, 2), "unit": "GB/s",
                "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
                "higher_is_better": True, "dtype": "fp16 x int8", "data": "synthetic",
                "config": {"workload": f"int8_linear M={M} over qkv/o/gate_up/down", "per_projection": per,
                           "bytes_per_step": nbytes, "flops_per_step": flops,
                           "l2": f"{NSET} weight copies rotated per step (404 MB > 126 MB L2)"},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": round(gbs / peak, 4),
                             "tflops": round(flops / (ms * 1e-3) / 1e12, 2)},
                "gpu_launches": 4 * steps}
    elif args.mode == "sample":
        # one draft-proposer sampling step (draft_proposer.py:505-510): B rows of bf16 LM-head
        # logits -> fp32 copy into out_logits[:, s] + Gumbel-max token into cands[:, s]
        B, V, k = 64, workloads.VOCAB, 6
        NSET = 8  # 8 x 19.4 MB of logits rotated per step (155 MB > 126 MB L2)
        gd = torch.Generator(device="cuda").manual_seed(0)
        lg = [(torch.randn(B, V, generator=gd, device="cuda") * 3.0).to(torch.bfloat16) for _ in range(NSET)]
        temps = torch.ones(B, 1, device="cuda")
        out_logits = torch.empty(B, k, V, device="cuda")
        cands = torch.empty(B, k, dtype=torch.int64, device="cuda")
        ctr = [0]

        def step():
            i = ctr[0]
            ctr[0] += 1
            pkg.draft_sample_step(lg[i % NSET], temps, out_logits, cands, i % k, seed=1, offset=i)
        ms = _time_events(step, steps, args.warmup, per_graph=2 * NSET)
        nbytes = B * V * (2 + 4)
        gbs = nbytes / (ms * 1e-3) / 1e9
        line = {"metric": "draft sample step HBM GB/s", "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1,
                "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
                "dtype": "bf16 in, f32 copy", "data": "synthetic",
                "config": {"workload": f"draft_sample_step B={B} V={V} (logits N(0,9) bf16, T=1, in-kernel Philox "
                                       "noise)", "bytes_per_step": nbytes,
                           "l2": f"{NSET} logit tensors rotated per step (155 MB > 126 MB L2)"},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": round(gbs / peak, 4),
                             "note": "issue-bound: the Philox noise of every column is most of the instructions"},
                "gpu_launches": 2 * steps}
    elif args.mode == "attn_sweep":
        # the cfg2 grid: verify (k=6) and decode over B x ctx, one line with a row per point
        from oracle.attention import algorithmic_bytes
        rows = []
        for n_q in (N_Q, 1):
            for B in (1, 8, 32, 64):
                for L in (512, 2048, 4096):
                    # cases that fit L2 rotate over copies (>= 256 MB together), so every call reads HBM
                    kv = B * L * 2 * HKV * D * 2
                    n_cp = min(128, -(-256_000_000 // kv))
                    cases = [workloads.paged_case([L] * B, n_q, device="cuda", seed=B + L + 97 * c, extra_blocks=0,
                                                  generate_on_device=True, **workloads.QWEN3_4B)
                             for c in range(n_cp)]
                    out = torch.empty_like(cases[0].q)
                    ctr = [0]

                    def fn(cases=cases, out=out, n_q=n_q):
                        c = cases[ctr[0] % len(cases)]
                        ctr[0] += 1
                        pkg.paged_attention(c.q, c.k_cache, c.v_cache, c.block_tables, c.cache_seqlens, c.scale,
                                            n_q=n_q, out=out)
                    ms = _time_events(fn, steps, args.warmup, per_graph=max(20, n_cp))
                    nbytes = algorithmic_bytes([L] * B, n_q, HQ, HKV, D, 2, 2)
                    kind, slots, _ = pkg.attention.plan(B, n_q, HQ, HKV, D, PAGE, L // PAGE, torch.bfloat16)
                    gbs = nbytes / (ms * 1e-3) / 1e9
                    rows.append({"n_q": n_q, "B": B, "ctx": L, "us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                                 "frac": round(gbs / peak, 3), "plan": f"{kind} x{slots}",
                                 "copies": n_cp})
                    del cases, out
        line = {"metric": "attention cfg2 sweep", "unit": "GB/s", "n_gpus": 1, "steps": steps,
                "warmup": args.warmup, "dtype": "bf16", "data": "synthetic", "peak": peak, "peak_kind": peak_kind,
                "rows": rows}
    else:  # decode attention
        from oracle.attention import algorithmic_bytes
        B, L = 64, CTX
        case = workloads.paged_case([L] * B, 1, device="cuda", seed=3, extra_blocks=0, generate_on_device=True,
                                    **workloads.QWEN3_4B)
        out = torch.empty_like(case.q)
        fn = lambda: pkg.paged_attention(case.q, case.k_cache, case.v_cache, case.block_tables,
                                         case.cache_seqlens, case.scale, n_q=1, out=out)
        ms = _time_events(fn, steps, args.warmup)
        nbytes = algorithmic_bytes([L] * B, 1, HQ, HKV, D, 2, 2)
        gbs = nbytes / (ms * 1e-3) / 1e9
        line = {"metric": "decode-attn HBM GB/s", "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1,
                "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"decode-attn B={B} ctx={L} (Qwen3-4B heads)", "bytes_per_step": nbytes},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": round(gbs / peak, 4)},
                "gpu_launches": steps}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--global-batch", type=int, default=64,
                    help="sequences of the whole job, sharded over the GPUs (strong scaling)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline leg")
    ap.add_argument("--mode", choices=["verify_attn", "decode_attn", "attn_sweep", "verify_batch", "w8a16", "sample", "tp_step",
                             "specdec_e2e"],
                    default="verify_attn", help="verify_attn is the headline; the others measure the "
                    "secondary kernels of the path on one GPU")
    ap.add_argument("--m", type=int, default=1, help="tokens (M) for --mode w8a16")
    ap.add_argument("--tp", action="store_true",
                    help="--mode specdec_e2e under torchrun: tensor-parallel models over the ranks "
                         "(all-reduce after o_proj / down_proj) instead of sharded sequences")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.mode == "tp_step":
        return run_tp_step(args)
    if args.mode == "specdec_e2e":
        return run_specdec_e2e(args)
    if args.mode != "verify_attn":
        return run_side(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
