"""The no-allocation attention entry point, checked against the workspace entry point.

Some callers cannot allocate device memory when they run attention: a plugin
inside another runtime's enqueue callback whose memory pool forbids raw
allocations, a steady-state serving loop that cannot take cudaMalloc's implicit
device-wide synchronisation, a deployment with a fixed memory budget.
``sdb_paged_attention_noalloc`` serves them from a static 16 MiB device array
instead of a caller workspace.  These tests call it through the C ABI, twice in
a row, and compare with ``sdb_paged_attention`` on the same inputs and the same
split count: it is the same kernel with the same decomposition, so the outputs
must be identical bit for bit.  They also read the array's error word through
``sdb_paged_attention_noalloc_error_word``, the only way these callers can see
what the kernels flag.  This file is collected last so a run that stops at the
first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _args(case, out, splits, bt=None):
    nb, page, hkv, d = case.k_cache.shape
    bt = case.block_tables if bt is None else bt
    return [case.q.data_ptr(), case.q.stride(0), case.q.stride(1), case.k_cache.data_ptr(),
            case.v_cache.data_ptr(), case.k_cache.stride(0), case.k_cache.stride(1), case.k_cache.stride(2),
            bt.data_ptr(), bt.stride(0), case.cache_seqlens.data_ptr(),
            out.data_ptr(), out.stride(0), out.stride(1), case.B, case.n_q, case.q.shape[1], hkv, d, page,
            bt.shape[1], nb, ctypes.c_float(case.scale), 1, splits]


def _splits(lib, case):
    nb, page, hkv, d = case.k_cache.shape
    return lib.sdb_paged_attention_default_splits(case.B, case.n_q, case.q.shape[1], hkv, d, page,
                                                  case.block_tables.shape[1], 1)


def _with_workspace(lib, case, splits):
    out = torch.empty_like(case.q)
    nb, page, hkv, d = case.k_cache.shape
    ws = torch.zeros(lib.sdb_paged_attention_workspace_size(case.B, case.n_q, case.q.shape[1], hkv, d, splits),
                     dtype=torch.uint8, device="cuda")
    rc = lib.sdb_paged_attention(*_args(case, out, splits), ws.data_ptr(), ws.numel(),
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sdb_last_error()
    return out


def _no_alloc(lib, case, splits, bt=None):
    out = torch.empty_like(case.q)
    rc = lib.sdb_paged_attention_noalloc(*_args(case, out, splits, bt), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sdb_last_error()
    return out


def _error_word(lib, clear):
    word = ctypes.c_int32(-1)
    rc = lib.sdb_paged_attention_noalloc_error_word(ctypes.byref(word), int(clear),
                                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sdb_last_error()
    torch.cuda.current_stream().synchronize()
    return word.value


def test_no_alloc_matches_workspace_entry_point_on_two_calls_in_a_row(pkg):
    from specdec_nanovllm_b200 import workloads as W
    lib = pkg.load_library()
    # split partials are needed here (several splits per sequence), so the static array is used
    case = W.paged_case(W.cfg2_lens(8, 2048, seed=3), 7, seed=77, max_blocks=8, **W.QWEN3_4B)
    splits = _splits(lib, case)
    want = _with_workspace(lib, case, splits)
    torch.cuda.synchronize()
    for _ in range(2):
        got = _no_alloc(lib, case, splits)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    # a different shape right after: the array keeps the previous call's contents
    case2 = W.paged_case([4096, 300, 1], 1, seed=5, max_blocks=16, **W.QWEN3_4B)
    splits2 = _splits(lib, case2)
    want2 = _with_workspace(lib, case2, splits2)
    for _ in range(2):
        got2 = _no_alloc(lib, case2, splits2)
        torch.cuda.synchronize()
        assert torch.equal(got2, want2)
    assert np.isfinite(got2.float().cpu().numpy()).all()
    assert _error_word(lib, clear=True) == 0


def test_no_alloc_flags_a_bad_block_id_in_its_error_word(pkg):
    from specdec_nanovllm_b200 import _lib
    from specdec_nanovllm_b200 import workloads as W
    lib = pkg.load_library()
    case = W.paged_case([600], 1, seed=3, max_blocks=3, **W.QWEN3_4B)
    _error_word(lib, clear=True)
    bt = case.block_tables.clone()
    bt[0, 1] = 10_000_000            # outside the pool: the kernel clamps it to block 0 and flags it
    _no_alloc(lib, case, 1, bt)
    assert _error_word(lib, clear=False) & _lib.SDB_KERR_BLOCK_ID
    assert _error_word(lib, clear=True) & _lib.SDB_KERR_BLOCK_ID   # still set until cleared
    assert _error_word(lib, clear=False) == 0
    _no_alloc(lib, case, 1)          # a valid call leaves the word clear
    assert _error_word(lib, clear=True) == 0


def test_no_alloc_sizes_explicit_splits_as_launched(pkg):
    """An explicit split count above what the kernel launches is clamped before the size check."""
    from specdec_nanovllm_b200 import workloads as W
    lib = pkg.load_library()
    case = W.paged_case([4096, 4096], 7, seed=12, max_blocks=16, **W.QWEN3_4B)
    kind, slots, need = pkg.attention.plan(2, 7, 32, 8, 128, 256, 16, torch.bfloat16, splits=1000)
    assert need <= (16 << 20)
    want = _with_workspace(lib, case, slots)
    got = _no_alloc(lib, case, 1000)
    torch.cuda.synchronize()
    assert torch.equal(got, want), kind


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
