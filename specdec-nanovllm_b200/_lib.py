"""ctypes binding of ``libspecdec_b200.so`` (the C ABI declared in include/specdec_b200.h).

The library is the only compute path: if it is missing or a tensor is not on a
CUDA device, calls raise instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libspecdec_b200.so")

SDB_OK = 0
SDB_ERR_INVALID_ARG = 1
SDB_ERR_UNSUPPORTED = 2
SDB_ERR_WORKSPACE = 3
SDB_ERR_CUDA = 4

SDB_KERR_SEQLEN = 0x1
SDB_KERR_BLOCK_ID = 0x2
SDB_KERR_TIMEOUT = 0x4
SDB_KERR_TOKEN = 0x8

# decomposition of an attention launch (sdb_paged_attention_plan)
ATTN_PLAN_NAMES = {0: "cuda_core", 1: "mma", 2: "tcgen05_strided", 3: "tcgen05_grouped"}

SDB_F32, SDB_BF16, SDB_F16 = 0, 1, 2
DTYPE_CODE = {torch.float32: SDB_F32, torch.bfloat16: SDB_BF16, torch.float16: SDB_F16}


class SdbError(RuntimeError):
    """A library call returned an error status (the reference raises RuntimeError
    through TORCH_CHECK for the same conditions, paged_decode_attn_cuda.cu:1406-1407)."""

    def __init__(self, code: int, where: str, msg: str):
        super().__init__(f"{where}: status {code}: {msg}")
        self.code = code


_c_i32 = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_u64 = ctypes.c_uint64
_c_f32 = ctypes.c_float
_c_sz = ctypes.c_size_t
_c_p = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/specdec_b200.h
SIGNATURES = {
    "sdb_last_error": (ctypes.c_char_p, []),
    "sdb_build_info": (ctypes.c_char_p, []),
    "sdb_paged_attention_workspace_size": (_c_sz, [_c_i32] * 6),
    "sdb_paged_attention_default_splits": (_c_i32, [_c_i32] * 8),
    "sdb_paged_attention_plan": (_c_sz, [_c_i32] * 9 + [_c_p, _c_p]),
    "sdb_paged_attention": (_c_i32, [
        _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p,
        _c_p, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_f32, _c_i32, _c_i32, _c_p, _c_sz, _c_p]),
    "sdb_paged_attention_store": (_c_i32, [
        _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p,
        _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p,
        _c_p, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_f32, _c_i32, _c_i32, _c_p, _c_sz, _c_p]),
    "sdb_paged_attention_noalloc": (_c_i32, [
        _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p,
        _c_p, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_f32, _c_i32, _c_i32, _c_p]),
    "sdb_paged_attention_noalloc_error_word": (_c_i32, [_c_p, _c_i32, _c_p]),
    "sdb_paged_attention_readonly": (_c_i32, [
        _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_p, _c_sz, _c_p]),
    "sdb_paged_attention_error_word": (_c_p, [_c_p] + [_c_i32] * 6),
    "sdb_store_kvcache": (_c_i32, [
        _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p]),
    "sdb_verify_workspace_size": (_c_sz, [_c_i32] * 4),
    "sdb_verify_batch": (_c_i32, [
        _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_u64, _c_u64, _c_i32, _c_p, _c_p, _c_p,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_sz, _c_p]),
    "sdb_verify_batch_ex": (_c_i32, [
        _c_p, _c_i32, _c_p, _c_i32, _c_p, _c_p, _c_p, _c_p, _c_u64, _c_u64, _c_i32, _c_p, _c_p, _c_p,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_sz, _c_p]),
    "sdb_verify_batch_dev_offset": (_c_i32, [
        _c_p, _c_i32, _c_p, _c_i32, _c_p, _c_p, _c_u64, _c_p, _c_i32, _c_p, _c_p, _c_p,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_sz, _c_p]),
    "sdb_verify_shard_send_floats": (_c_sz, [_c_i32] * 4),
    "sdb_verify_batch_shard": (_c_i32, [
        _c_i32, _c_p, _c_i32, _c_p, _c_i32, _c_p, _c_p, _c_p, _c_p, _c_u64, _c_u64, _c_i32, _c_p, _c_p, _c_p,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p, _c_p, _c_sz, _c_p]),
    "sdb_philox_fill": (_c_i32, [_c_p, _c_i32, _c_i32, _c_u64, _c_u64, _c_i32, _c_p]),
    "sdb_qk_norm_rope_store": (_c_i32, [
        _c_p, _c_i64, _c_p, _c_p, _c_f32, _c_p, _c_i64, _c_i32, _c_p,
        _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p,
        _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p]),
    "sdb_sample_workspace_size": (_c_sz, [_c_i32, _c_i32]),
    "sdb_sample_dev_offset": (_c_i32, [
        _c_p, _c_i64, _c_i32, _c_p, _c_u64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i32, _c_i32,
        _c_p, _c_sz, _c_p]),
    "sdb_sample": (_c_i32, [
        _c_p, _c_i64, _c_i32, _c_p, _c_p, _c_u64, _c_u64, _c_p, _c_i64, _c_p, _c_i64, _c_i32, _c_i32,
        _c_p, _c_sz, _c_p]),
    "sdb_w8a16_workspace_size": (_c_sz, [_c_i32] * 3),
    "sdb_w8a16_linear": (_c_i32, [
        _c_p, _c_i64, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_i64, _c_i32, _c_i32, _c_i32,
        _c_i32, _c_p, _c_sz, _c_p]),
    "sdb_quantize_weight": (_c_i32, [_c_p, _c_i32, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_p]),
    "sdb_rms_norm": (_c_i32, [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p,
                              _c_i32, _c_i32, _c_f32, _c_i32, _c_p]),
    "sdb_silu_mul": (_c_i32, [_c_p, _c_i64, _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_p]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load the library once (torch is imported first so its CUDA runtime is shared)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python specdec-nanovllm_b200/build.py` "
                        "(there is no fallback path)")
                h = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def check(rc: int, where: str) -> None:
    if rc != SDB_OK:
        msg = lib().sdb_last_error().decode(errors="replace")
        raise SdbError(rc, where, msg)


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("specdec_b200 kernels run on CUDA tensors only (no CPU fallback)")


class WorkspacePool:
    """Caller-owned workspaces, zero-filled once and grown only outside graph capture.

    The kernels return their atomic counters to zero after every call, so a
    workspace can be reused by consecutive launches on one stream (and by CUDA
    graph replays).  Concurrent launches on different streams need different
    ``kind`` keys.
    """

    def __init__(self):
        self._bufs: dict = {}

    def get(self, device: torch.device, kind: str, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), kind)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(f"workspace '{kind}' must be sized before CUDA graph capture "
                                   f"(need {nbytes} bytes); call the op once eagerly first")
            size = max(nbytes, 1 << 16)
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


WORKSPACES = WorkspacePool()
