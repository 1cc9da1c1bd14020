"""Bit-level float helpers for the oracle (numpy has no bfloat16).  Test infrastructure only."""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x) -> np.ndarray:
    """Round float32 -> bfloat16 with round-to-nearest-even; returns uint16 bits.

    This is the IEEE conversion torch's ``.to(torch.bfloat16)`` performs (NaN is
    kept quiet).
    """
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    rounded = ((u + 0x7FFF + lsb) >> 16).astype(np.uint32)
    nan = np.isnan(x)
    rounded = np.where(nan, (u >> 16).astype(np.uint32) | 0x40, rounded)
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 value (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_f16(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def allclose_report(got, want, rtol, atol):
    """(ok, max_abs_err, max_violation) with torch.allclose semantics."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    viol = err - bound
    finite = np.isfinite(got).all()
    return bool(finite and (viol <= 0).all()), float(err.max(initial=0.0)), float(viol.max(initial=-1.0))
