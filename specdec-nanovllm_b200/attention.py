"""Paged decode / speculative-verify attention: host side of the sm_100a kernels.

Drop-in mirrors of the reference's attention entry points, all running the one
kernel family of ``csrc/attention.cu`` through the C ABI:

* ``Attention`` -- ``nanovllm/layers/attention.py:43-82``: writes this step's K/V
  rows into the paged cache (``store_kvcache``, :33-40) and attends, reading the
  global ``Context``.  Decode (1 query row per sequence) and speculative verify
  (k+1 rows per sequence, ``is_spec_verify``) are supported; dense prefill is
  outside this library.
* ``flash_attn_with_kvcache`` / ``flash_attn_varlen_func`` -- the subsets of the
  flash-attn 2 calls the reference makes at ``attention.py:78-81`` and :67-70
  (paged, causal, uniform k+1 query rows per sequence).
* ``paged_decode_attention`` -- ``nanovllm/kernels/paged_decode_attn.py:352``.
* ``paged_decode_attention_cuda`` -- ``nanovllm/kernels/paged_decode_attn_cuda.py:52``.
* ``paged_attention`` -- the general form: q (B*n_q, Hq, D), bottom-right causal.

Every call launches on the current stream, allocates only its output (pass
``out=`` to avoid even that), and never reads device data on the host, so it can
be captured in a CUDA graph after one eager call has sized the workspace.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib
from .context import get_context


def _kv_geometry(k_cache: torch.Tensor, layout: str = "interleaved"):
    """(num_blocks, page, Hkv, D, stride_block, stride_page, stride_head) in elements."""
    if k_cache.dim() != 4:
        raise ValueError(f"k_cache must be 4-D, got {tuple(k_cache.shape)}")
    if layout == "head_major":  # (num_blocks, Hkv, page, D)
        nb, hkv, page, d = k_cache.shape
        return nb, page, hkv, d, k_cache.stride(0), k_cache.stride(2), k_cache.stride(1)
    nb, page, hkv, d = k_cache.shape
    return nb, page, hkv, d, k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)


def workspace_bytes(B: int, n_q: int, Hq: int, Hkv: int, D: int, splits: int) -> int:
    return int(_lib.lib().sdb_paged_attention_workspace_size(B, n_q, Hq, Hkv, D, max(splits, 1)))


def default_splits(B, n_q, Hq, Hkv, D, page, max_blocks, dtype: torch.dtype) -> int:
    return int(_lib.lib().sdb_paged_attention_default_splits(
        B, n_q, Hq, Hkv, D, page, max_blocks, _lib.DTYPE_CODE[dtype]))


def plan(B, n_q, Hq, Hkv, D, page, max_blocks, dtype: torch.dtype, splits: int = 0):
    """(kernel, partial slots per pair, workspace bytes) of the launch ``paged_attention``
    makes for this static shape: kernel is one of "tcgen05_strided", "tcgen05_grouped",
    "mma" or "cuda_core" (host-side query, no launch)."""
    import ctypes
    k, s = ctypes.c_int(-1), ctypes.c_int(0)
    need = _lib.lib().sdb_paged_attention_plan(B, n_q, Hq, Hkv, D, page, max_blocks, _lib.DTYPE_CODE[dtype],
                                               splits, ctypes.byref(k), ctypes.byref(s))
    if k.value < 0:
        raise ValueError("invalid attention shape")
    return _lib.ATTN_PLAN_NAMES[k.value], int(s.value), int(need)


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_tables: torch.Tensor, cache_seqlens: torch.Tensor, softmax_scale: float,
                    n_q: int = 1, splits: int = 0, out: torch.Tensor | None = None,
                    workspace: torch.Tensor | None = None, layout: str = "interleaved",
                    k_new: torch.Tensor | None = None, v_new: torch.Tensor | None = None,
                    slot_mapping: torch.Tensor | None = None) -> torch.Tensor:
    """Decode (n_q = 1) or verify (n_q = k+1) attention over a paged KV cache.

    q (B*n_q, Hq, D); k_cache / v_cache (num_blocks, page, Hkv, D); block_tables
    (B, max_blocks) int32 (-1 padded); cache_seqlens (B,) int32, the cache length
    including the n_q new tokens.  Row r of sequence b sees keys j <= L_b - n_q + r.

    With ``k_new`` / ``v_new`` (B*n_q, Hkv, D) and ``slot_mapping`` (B*n_q,) the
    call first stores the new rows like ``store_kvcache`` -- row b*n_q + i is the
    token at position L_b - n_q + i, its slot -1 or that position's slot -- fused
    into the attention kernel where the tcgen05 path runs (one launch).
    """
    _lib.require_cuda(q, k_cache, v_cache, block_tables, cache_seqlens)
    if q.dim() != 3:
        raise ValueError(f"q must be (B*n_q, Hq, D), got {tuple(q.shape)}")
    total, Hq, D = q.shape
    nb, page, Hkv, Dk, sb, sp, sh = _kv_geometry(k_cache, layout)
    if Dk != D or v_cache.shape != k_cache.shape or v_cache.stride() != k_cache.stride():
        raise ValueError("k_cache / v_cache / q head_dim or layout mismatch")
    if q.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
        raise ValueError(f"q / cache dtypes differ: {q.dtype} vs {k_cache.dtype}")
    if q.dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"unsupported dtype {q.dtype}")
    if block_tables.dtype != torch.int32 or cache_seqlens.dtype != torch.int32:
        raise ValueError("block_tables and cache_seqlens must be int32")
    B = cache_seqlens.shape[0]
    if total != B * n_q:
        raise ValueError(f"q has {total} rows, expected B*n_q = {B}*{n_q}")
    if q.stride(-1) != 1 or k_cache.stride(-1) != 1:
        raise ValueError("the head_dim axis must be contiguous")
    if block_tables.stride(-1) != 1:
        block_tables = block_tables.contiguous()
    cache_seqlens = cache_seqlens.contiguous()
    if out is None:
        out = torch.empty_like(q)
    max_blocks = block_tables.shape[1]
    dt = _lib.DTYPE_CODE[q.dtype]
    L = _lib.lib()
    if splits <= 0:
        splits = int(L.sdb_paged_attention_default_splits(B, n_q, Hq, Hkv, D, page, max_blocks, dt))
    need = int(L.sdb_paged_attention_workspace_size(B, n_q, Hq, Hkv, D, splits))
    if workspace is None:
        workspace = _lib.WORKSPACES.get(q.device, "attention", need)
    if k_new is None and v_new is None and slot_mapping is None:
        rc = L.sdb_paged_attention(
            q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), sb, sp,
            sh, block_tables.data_ptr(), block_tables.stride(0), cache_seqlens.data_ptr(),
            out.data_ptr(), out.stride(0), out.stride(1), B, n_q, Hq, Hkv, D, page, max_blocks, nb,
            float(softmax_scale), dt, splits, workspace.data_ptr(), workspace.numel(),
            _lib.stream_of(q))
        _lib.check(rc, "sdb_paged_attention")
        return out
    if k_new is None or v_new is None or slot_mapping is None:
        raise ValueError("k_new, v_new and slot_mapping go together")
    _lib.require_cuda(k_new, v_new, slot_mapping)
    if k_new.shape != (B * n_q, Hkv, D) or v_new.shape != k_new.shape:
        raise ValueError(f"k_new / v_new must be ({B * n_q}, {Hkv}, {D}), got "
                         f"{tuple(k_new.shape)} / {tuple(v_new.shape)}")
    if k_new.dtype != q.dtype or v_new.dtype != q.dtype:
        raise ValueError("k_new / v_new dtype differs from q")
    if k_new.stride(-1) != 1 or v_new.stride(-1) != 1:
        raise ValueError("k_new / v_new rows must be contiguous")
    if slot_mapping.numel() != B * n_q:
        raise ValueError(f"slot_mapping must have {B * n_q} entries, got {slot_mapping.numel()}")
    slots = slot_mapping.to(torch.int32).contiguous()
    rc = L.sdb_paged_attention_store(
        q.data_ptr(), q.stride(0), q.stride(1), k_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        v_new.data_ptr(), v_new.stride(0), v_new.stride(1), slots.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), sb, sp, sh,
        block_tables.data_ptr(), block_tables.stride(0), cache_seqlens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), B, n_q, Hq, Hkv, D, page, max_blocks, nb,
        float(softmax_scale), dt, splits, workspace.data_ptr(), workspace.numel(),
        _lib.stream_of(q))
    _lib.check(rc, "sdb_paged_attention_store")
    return out


def paged_attention_readonly(q, k_cache, v_cache, block_tables, cache_seqlens, n_q: int = 1,
                             splits: int = 0, workspace=None):
    """Memory-floor twin: the same grid and TMA traffic with no math (roofline evidence)."""
    _lib.require_cuda(q, k_cache, v_cache, block_tables, cache_seqlens)
    total, Hq, D = q.shape
    nb, page, Hkv, _, sb, sp, sh = _kv_geometry(k_cache)
    B = cache_seqlens.shape[0]
    dt = _lib.DTYPE_CODE[q.dtype]
    L = _lib.lib()
    max_blocks = block_tables.shape[1]
    if splits <= 0:
        splits = int(L.sdb_paged_attention_default_splits(B, n_q, Hq, Hkv, D, page, max_blocks, dt))
    need = int(L.sdb_paged_attention_workspace_size(B, n_q, Hq, Hkv, D, splits))
    if workspace is None:
        workspace = _lib.WORKSPACES.get(q.device, "attention_ro", need)
    rc = L.sdb_paged_attention_readonly(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), sb, sp, sh,
        block_tables.data_ptr(), block_tables.stride(0), cache_seqlens.data_ptr(), B, n_q, Hq, Hkv,
        D, page, max_blocks, nb, dt, splits, workspace.data_ptr(), workspace.numel(),
        _lib.stream_of(q))
    _lib.check(rc, "sdb_paged_attention_readonly")
    return workspace


def error_word(device=None, kind: str = "attention") -> int:
    """Read the kernels' SDB_KERR_* bits (synchronises; debugging aid)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    buf = _lib.WORKSPACES.get(dev, kind, 256)
    return int(buf[:4].view(torch.int32).item())


def clear_error_word(device=None, kind: str = "attention") -> None:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _lib.WORKSPACES.get(dev, kind, 256)[:4].zero_()


# ----------------------------------------------------------------------- mirrors
def paged_decode_attention(q, k_cache, v_cache, block_table, context_lens, scale, version=2,
                           block_n=128, splits=8, num_warps=None, num_stages=None,
                           layout="interleaved"):
    """Mirror of ``nanovllm/kernels/paged_decode_attn.py:352``.

    ``version`` / ``block_n`` / ``num_warps`` / ``num_stages`` selected Triton
    variants there; here one kernel serves every case and they are accepted and
    ignored.  ``splits`` is honoured (0 = automatic).  GQA requires Hq % Hkv == 0
    (the reference asserts the same, :384).
    """
    if q.shape[1] % (k_cache.shape[2] if layout != "head_major" else k_cache.shape[1]) != 0:
        raise AssertionError("GQA requires num_q_heads to be a multiple of num_kv_heads")
    return paged_attention(q, k_cache, v_cache, block_table.to(torch.int32),
                           context_lens.to(torch.int32), scale, n_q=1,
                           splits=splits if version == 3 else 0, layout=layout)


def paged_decode_attention_cuda(q, k_cache, v_cache, block_table, context_lens, scale, splits=8,
                                block_n=64, warps=4, stages=3, fused=True):
    """Mirror of ``nanovllm/kernels/paged_decode_attn_cuda.py:52`` (split count honoured,
    tile knobs fixed by the sm_100a kernel; the split merge is always fused)."""
    return paged_attention(q, k_cache, v_cache, block_table, context_lens, scale, n_q=1, splits=splits)


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, cache_seqlens=None,
                            block_table=None, softmax_scale=None, causal=True, **unused):
    """The subset of flash-attn's ``flash_attn_with_kvcache`` used at ``attention.py:78-81``.

    q (B, s, Hq, D) with s query rows per sequence (s = 1: decode; s > 1: verify,
    bottom-right causal); returns (B, s, Hq, D).  Appending k/v through this call is
    not supported (the reference writes the cache with store_kvcache first).
    """
    if k is not None or v is not None:
        raise NotImplementedError("append K/V with store_kvcache before attention")
    if block_table is None or cache_seqlens is None:
        raise NotImplementedError("only the paged form (block_table, cache_seqlens) is supported")
    if q.dim() != 4:
        raise ValueError(f"q must be (B, s, Hq, D), got {tuple(q.shape)}")
    B, s, Hq, D = q.shape
    if s > 1 and not causal:
        raise NotImplementedError("multi-row queries are supported with causal=True only")
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    out = paged_attention(q.reshape(B * s, Hq, D), k_cache, v_cache, block_table,
                          cache_seqlens.to(torch.int32), softmax_scale, n_q=s)
    return out.view(B, s, Hq, D)


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                           dropout_p=0.0, softmax_scale=None, causal=False, block_table=None,
                           **unused):
    """The subset of flash-attn's ``flash_attn_varlen_func`` used for speculative verify at
    ``attention.py:67-70``: paged K/V (``block_table``), causal, every sequence with the
    same number of query rows (``max_seqlen_q``; ``model_runner.py:582``).  The cache
    length of sequence b is ``cu_seqlens_k[b+1] - cu_seqlens_k[b]`` (computed on the
    device, no host read)."""
    if block_table is None:
        raise NotImplementedError("dense (non-paged) prefill attention is outside this library")
    if not causal:
        raise NotImplementedError("verify attention is causal")
    if dropout_p:
        raise NotImplementedError("dropout is not supported")
    B = cu_seqlens_q.numel() - 1
    n_q = int(max_seqlen_q)
    if q.shape[0] != B * n_q:
        raise NotImplementedError(
            f"query rows must be uniform per sequence: {q.shape[0]} rows for {B} sequences of {n_q}")
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    seqlens = (cu_seqlens_k[1:] - cu_seqlens_k[:-1]).to(torch.int32)
    return paged_attention(q, k, v, block_table, seqlens, softmax_scale, n_q=n_q)


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Mirror of ``nanovllm/layers/attention.py:33-40``: row i -> slot slot_mapping[i], -1 skipped."""
    _lib.require_cuda(key, value, k_cache, v_cache, slot_mapping)
    N, Hkv, D = key.shape
    nb, page, hkv2, d2, sb, sp, sh = _kv_geometry(k_cache)
    if (hkv2, d2) != (Hkv, D) or value.shape != key.shape:
        raise ValueError("key/value/cache shapes disagree")
    if slot_mapping.numel() != N:
        raise AssertionError("slot_mapping must have one entry per row")
    if key.stride(-1) != 1 or value.stride(-1) != 1:
        raise AssertionError("key/value rows must be contiguous")
    slots = slot_mapping.to(torch.int32).contiguous()
    ws = _lib.WORKSPACES.get(key.device, "attention", 256)
    rc = _lib.lib().sdb_store_kvcache(
        key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0),
        value.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), sb, sp, sh, slots.data_ptr(), N,
        Hkv, D, page, nb, _lib.DTYPE_CODE[key.dtype], ws.data_ptr(), _lib.stream_of(key))
    _lib.check(rc, "sdb_store_kvcache")


class Attention(nn.Module):
    """Mirror of ``nanovllm/layers/attention.py:43-82``."""

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        has_cache = bool(k_cache.numel() and v_cache.numel())
        if has_cache and context.block_tables is not None and context.slot_mapping is not None:
            # decode / verify: the store of this step's rows runs inside the attention launch
            if context.is_prefill:
                B = context.cu_seqlens_q.numel() - 1
                n_q = int(context.max_seqlen_q)
                if q.shape[0] == B * n_q:
                    seqlens = (context.cu_seqlens_k[1:] - context.cu_seqlens_k[:-1]).to(torch.int32)
                    return paged_attention(q, k_cache, v_cache, context.block_tables, seqlens,
                                           self.scale, n_q=n_q, k_new=k, v_new=v,
                                           slot_mapping=context.slot_mapping)
            else:
                q3 = q.unsqueeze(0) if q.dim() == 2 else q
                k3 = k.unsqueeze(0) if k.dim() == 2 else k
                v3 = v.unsqueeze(0) if v.dim() == 2 else v
                out = paged_attention(q3, k_cache, v_cache, context.block_tables,
                                      context.context_lens.to(torch.int32), self.scale, n_q=1,
                                      k_new=k3, v_new=v3, slot_mapping=context.slot_mapping)
                # the reference's shape: (B, 1, Hq, D), also for a single (Hq, D) query
                return out.view(q3.shape[0], 1, *q3.shape[1:])
        if has_cache:
            store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
        if context.is_prefill:
            if context.block_tables is None:
                raise NotImplementedError("dense prefill attention is outside this library")
            return flash_attn_varlen_func(q, k_cache, v_cache, context.cu_seqlens_q,
                                          context.cu_seqlens_k, context.max_seqlen_q,
                                          context.max_seqlen_k, softmax_scale=self.scale,
                                          causal=True, block_table=context.block_tables)
        # decode: q is (B, Hq, D), or (Hq, D) for a single sequence (attention.py:72-77)
        q_in = q.unsqueeze(0).unsqueeze(0) if q.dim() == 2 else q.unsqueeze(1)
        return flash_attn_with_kvcache(q_in, k_cache, v_cache, cache_seqlens=context.context_lens,
                                       block_table=context.block_tables,
                                       softmax_scale=self.scale, causal=True)
