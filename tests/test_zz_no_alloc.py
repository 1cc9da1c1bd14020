"""The no-allocation attention entry point, checked against the workspace entry point.

Some callers cannot allocate device memory when they run attention: a plugin
inside another runtime's enqueue callback whose memory pool forbids raw
allocations, a steady-state serving loop that cannot take cudaMalloc's implicit
device-wide synchronisation, a deployment with a fixed memory budget.
``sdb_paged_attention_noalloc`` serves them from a static 16 MiB device array
instead of a caller workspace.  These tests call it through the C ABI, twice in
a row, and compare with ``sdb_paged_attention`` on the same inputs within the
bf16 tolerance of the other attention tests.  This file is collected last so a
run that stops at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle.numerics import allclose_report

pytestmark = pytest.mark.gpu

BF16_TOL = dict(rtol=2e-2, atol=2e-3)


def _args(case, out):
    nb, page, hkv, d = case.k_cache.shape
    return [case.q.data_ptr(), case.q.stride(0), case.q.stride(1), case.k_cache.data_ptr(),
            case.v_cache.data_ptr(), case.k_cache.stride(0), case.k_cache.stride(1), case.k_cache.stride(2),
            case.block_tables.data_ptr(), case.block_tables.stride(0), case.cache_seqlens.data_ptr(),
            out.data_ptr(), out.stride(0), out.stride(1), case.B, case.n_q, case.q.shape[1], hkv, d, page,
            case.block_tables.shape[1], nb, ctypes.c_float(case.scale), 1, 0]


def _with_workspace(lib, case):
    out = torch.empty_like(case.q)
    nb, page, hkv, d = case.k_cache.shape
    splits = lib.sdb_paged_attention_default_splits(case.B, case.n_q, case.q.shape[1], hkv, d, page,
                                                    case.block_tables.shape[1], 1)
    ws = torch.zeros(lib.sdb_paged_attention_workspace_size(case.B, case.n_q, case.q.shape[1], hkv, d, splits),
                     dtype=torch.uint8, device="cuda")
    args = _args(case, out)
    args[-1] = splits
    rc = lib.sdb_paged_attention(*args, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sdb_last_error()
    return out


def _no_alloc(lib, case):
    out = torch.empty_like(case.q)
    rc = lib.sdb_paged_attention_noalloc(*_args(case, out), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sdb_last_error()
    return out


def test_no_alloc_matches_workspace_entry_point_on_two_calls_in_a_row(pkg):
    from specdec_nanovllm_b200 import workloads as W
    lib = pkg.load_library()
    # split partials are needed here (several splits per sequence), so the static array is used
    case = W.paged_case(W.cfg2_lens(8, 2048, seed=3), 7, seed=77, max_blocks=8, **W.QWEN3_4B)
    want = _with_workspace(lib, case)
    torch.cuda.synchronize()
    for _ in range(2):
        got = _no_alloc(lib, case)
        torch.cuda.synchronize()
        ok, err, _ = allclose_report(got.float().cpu().numpy(), want.float().cpu().numpy(), **BF16_TOL)
        assert ok, f"max abs err {err}"
    # a different shape right after: the array keeps the previous call's contents
    case2 = W.paged_case([4096, 300, 1], 1, seed=5, max_blocks=16, **W.QWEN3_4B)
    want2 = _with_workspace(lib, case2)
    for _ in range(2):
        got2 = _no_alloc(lib, case2)
        torch.cuda.synchronize()
        ok, err, _ = allclose_report(got2.float().cpu().numpy(), want2.float().cpu().numpy(), **BF16_TOL)
        assert ok, f"max abs err {err}"
    assert np.isfinite(got2.float().cpu().numpy()).all()


def test_no_alloc_rejects_shapes_beyond_its_array(pkg):
    from specdec_nanovllm_b200 import _lib
    lib = pkg.load_library()
    small = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = small.data_ptr()
    # 4096 sequences x 8 kv heads x 4 splits of partials: far beyond 16 MiB; nothing is launched
    rc = lib.sdb_paged_attention_noalloc(p, 32 * 128, 128, p, p, 256 * 8 * 128, 8 * 128, 128, p, 16, p, p,
                                         32 * 128, 128, 4096, 7, 32, 8, 128, 256, 16, 1024,
                                         ctypes.c_float(0.088), 1, 4, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SDB_ERR_WORKSPACE
    assert "static array" in lib.sdb_last_error().decode()
