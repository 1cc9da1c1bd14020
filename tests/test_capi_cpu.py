"""The C-ABI library loads without a GPU, exports every symbol the header declares,
and rejects bad arguments on the host before any CUDA call."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "specdec_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sdb_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("sdb_paged_attention", "sdb_verify_batch", "sdb_w8a16_linear", "sdb_quantize_weight",
                 "sdb_store_kvcache", "sdb_paged_attention_workspace_size"):
        assert must in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # every declared function also has a ctypes signature in the binding
    from specdec_nanovllm_b200 import _lib
    assert set(declared_functions()) <= set(_lib.SIGNATURES), set(declared_functions()) - set(_lib.SIGNATURES)


def test_build_info_names_sm100a(pkg):
    info = pkg.load_library().sdb_build_info().decode()
    assert "sm_100a" in info


def test_null_pointers_rejected_on_host(pkg):
    from specdec_nanovllm_b200 import _lib
    L = _lib.lib()
    rc = L.sdb_paged_attention(None, 0, 0, None, None, 0, 0, 0, None, 0, None, None, 0, 0,
                               1, 1, 1, 1, 128, 256, 1, 1, 1.0, 1, 0, None, 0, None)
    assert rc == _lib.SDB_ERR_INVALID_ARG
    assert "null" in L.sdb_last_error().decode()
    rc = L.sdb_verify_batch(None, None, None, None, None, None, 0, 0, 0, None, None, None,
                            1, 1, 2, 10, None, 0, None)
    assert rc == _lib.SDB_ERR_INVALID_ARG
    rc = L.sdb_w8a16_linear(None, 0, None, None, 1, 0, None, None, 0, 1, 1, 64, 1, None, 0, None)
    assert rc == _lib.SDB_ERR_INVALID_ARG


def test_bad_sizes_rejected_on_host(pkg):
    from specdec_nanovllm_b200 import _lib
    L = _lib.lib()
    fake = ctypes.c_void_p(4096)  # never dereferenced: validation fails first
    # Hq not a multiple of Hkv
    rc = L.sdb_paged_attention(fake, 384, 128, fake, fake, 1, 1, 1, fake, 1, fake, fake, 384, 128,
                               1, 1, 3, 2, 128, 256, 1, 1, 1.0, 1, 0, fake, 1 << 20, None)
    assert rc == _lib.SDB_ERR_INVALID_ARG
    # k out of range for the sampler
    rc = L.sdb_verify_batch(fake, fake, fake, None, None, None, 0, 0, 0, fake, fake, fake,
                            2, 40, 41, 100, fake, 1 << 20, None)
    assert rc == _lib.SDB_ERR_INVALID_ARG
    # K not a multiple of 64
    rc = L.sdb_w8a16_linear(fake, 100, fake, fake, 1, 0, None, fake, 8, 1, 8, 100, 1, fake, 1 << 20, None)
    assert rc == _lib.SDB_ERR_UNSUPPORTED


def test_workspace_sizes_are_host_only_and_monotone(pkg):
    from specdec_nanovllm_b200 import _lib
    L = _lib.lib()
    a = L.sdb_paged_attention_workspace_size(64, 7, 32, 8, 128, 1)
    b = L.sdb_paged_attention_workspace_size(64, 7, 32, 8, 128, 4)
    assert 0 < a < b
    # 4 splits x 512 (seq, kv head) pairs x 28 rows x (128 + 2) floats of partials
    assert b >= 4 * 512 * 28 * 130 * 4
    v = L.sdb_verify_workspace_size(64, 6, 7, 151936)
    assert v > 64 * 13 * 8
    assert L.sdb_w8a16_workspace_size(1, 6144, 2560) >= 256


def test_python_api_refuses_cpu_tensors(pkg):
    import torch
    q = torch.zeros(4, 8, 128, dtype=torch.bfloat16)
    k = torch.zeros(2, 256, 2, 128, dtype=torch.bfloat16)
    bt = torch.zeros(4, 1, dtype=torch.int32)
    cl = torch.ones(4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.paged_attention(q, k, k, bt, cl, 0.1)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.verify_batch(torch.zeros(1, 2, 5), torch.zeros(1, 3, 5), torch.zeros(1, 2, dtype=torch.long))
