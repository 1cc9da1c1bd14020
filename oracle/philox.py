"""Counter-based random numbers shared bit-for-bit by the oracle and the GPU sampler.

Test infrastructure only.  The GPU samplers (``csrc/philox.cuh``, used by
``csrc/verify_sample.cu`` and ``csrc/sampler.cu``) carry their own CUDA
restatement of exactly these operations; this module is the checker.

Philox4x32-10 is the published generator of Salmon, Moraes, Dror and Shaw,
"Parallel random numbers: as easy as 1, 2, 3" (SC'11): 10 rounds of
multiply-hi/lo with the multipliers 0xD2511F53 / 0xCD9E8D57 and the Weyl key
increments 0x9E3779B9 / 0xBB67AE85.

Stream layout (this project's own convention; the reference draws with
``torch.rand`` at ``nanovllm/spec_decode/verify.py:120`` and
``exponential_`` at :209, which no second implementation can reproduce, so the
reference parity tests inject both draws instead):

    counter = (col // 4, row, stream, offset)   key = (seed & 0xffffffff, seed >> 32)
    value   = word (col % 4) of philox(counter, key)
    stream 0: acceptance uniforms u[b, j]     -> u = (w >> 8) * 2^-24        in [0, 1)
    stream 1: bonus exponentials  E[b, i]     -> E = -log(((w >> 8) + 1) * 2^-24)  in [0, 16.64]
    stream 2: sampler exponentials E[b, i]    -> same transform (``sample``, the draw of
              ``nanovllm/layers/sampler.py:11`` and ``draft_proposer.py:509``)

``log`` here is a fixed sequence of correctly rounded float32 operations (no
fused multiply-add), so numpy and CUDA (``__fadd_rn``/``__fmul_rn``/
``__fdiv_rn``) produce identical bits:  x = m * 2^e with m in [sqrt(1/2), sqrt(2)),
s = (m - 1) / (m + 1), log m = 2 s (1 + s^2/3 + s^4/5 + ... + s^10/11) (the
atanh series), log x = e*ln2_hi + (log m + e*ln2_lo).
"""

from __future__ import annotations

import numpy as np

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = np.uint32(0x9E3779B9)
W1 = np.uint32(0xBB67AE85)
MASK32 = np.uint64(0xFFFFFFFF)

STREAM_UNIFORM = 0
STREAM_EXPONENTIAL = 1
STREAM_SAMPLE = 2


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32-10.  All inputs uint32 arrays (broadcastable)."""
    c0 = np.asarray(c0, dtype=np.uint32).astype(np.uint64)
    c1 = np.asarray(c1, dtype=np.uint32).astype(np.uint64)
    c2 = np.asarray(c2, dtype=np.uint32).astype(np.uint64)
    c3 = np.asarray(c3, dtype=np.uint32).astype(np.uint64)
    k0 = np.uint64(np.uint32(k0))
    k1 = np.uint64(np.uint32(k1))
    c0, c1, c2, c3 = np.broadcast_arrays(c0, c1, c2, c3)
    c0, c1, c2, c3 = c0.copy(), c1.copy(), c2.copy(), c3.copy()
    w0 = np.uint64(W0)
    w1 = np.uint64(W1)
    for _ in range(10):
        p0 = c0 * M0
        p1 = c2 * M1
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK32
        n0 = hi1 ^ c1 ^ k0
        n2 = hi0 ^ c3 ^ k1
        c0, c1, c2, c3 = n0, lo1, n2, lo0
        k0 = (k0 + w0) & MASK32
        k1 = (k1 + w1) & MASK32
    return (c0.astype(np.uint32), c1.astype(np.uint32),
            c2.astype(np.uint32), c3.astype(np.uint32))


def philox_words(seed: int, offset: int, stream: int, rows: int, cols: int) -> np.ndarray:
    """uint32 words [rows, cols] of one stream."""
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    k0, k1 = seed & 0xFFFFFFFF, seed >> 32
    ncol4 = (cols + 3) // 4
    r = np.arange(rows, dtype=np.uint32)[:, None]
    c = np.arange(ncol4, dtype=np.uint32)[None, :]
    w = philox4x32_10(c, r, np.uint32(stream), np.uint32(offset & 0xFFFFFFFF), k0, k1)
    out = np.stack(w, axis=-1).reshape(rows, ncol4 * 4)
    return out[:, :cols]


def words_to_uniform(w) -> np.ndarray:
    """[0, 1) with 24 random bits."""
    return ((np.asarray(w, dtype=np.uint32) >> np.uint32(8)).astype(np.float32)
            * np.float32(2.0 ** -24))


def words_to_open_uniform(w) -> np.ndarray:
    """(0, 1] with 24 random bits."""
    return (((np.asarray(w, dtype=np.uint32) >> np.uint32(8)) + np.uint32(1)).astype(np.float32)
            * np.float32(2.0 ** -24))


def _f32(bits: int) -> np.float32:
    return np.array([bits], dtype=np.uint32).view(np.float32)[0]


# Constants by bit pattern so no decimal-to-binary rounding can differ between
# numpy and nvcc.
_SQRT2 = _f32(0x3FB504F3)   # sqrt(2) rounded to float32
_LN2_HI = _f32(0x3F317200)  # 0.693145751953125, 16 significant bits: e*LN2_HI is exact
_LN2_LO = _f32(0x35BFBE8E)  # ln 2 - LN2_HI
_C = [_f32(b) for b in (0x3DBA2E8C, 0x3DE38E39, 0x3E124925, 0x3E4CCCCD, 0x3EAAAAAB)]  # 1/11 1/9 1/7 1/5 1/3


def log_f32(x) -> np.ndarray:
    """Natural log of positive normal float32 values by fixed float32 operations."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = x.view(np.uint32)
    e = ((bits >> np.uint32(23)) & np.uint32(0xFF)).astype(np.int32) - 127
    m = ((bits & np.uint32(0x7FFFFF)) | np.uint32(0x3F800000)).view(np.float32)
    big = m > _SQRT2
    m = np.where(big, m * np.float32(0.5), m).astype(np.float32)
    e = np.where(big, e + 1, e)
    one = np.float32(1.0)
    s = ((m - one) / (m + one)).astype(np.float32)
    z = (s * s).astype(np.float32)
    r = np.full_like(z, _C[0])
    for c in _C[1:]:
        r = (r * z + c).astype(np.float32)
    r = (r * z + one).astype(np.float32)
    lm = ((s + s) * r).astype(np.float32)
    ef = e.astype(np.float32)
    return (ef * _LN2_HI + (lm + ef * _LN2_LO)).astype(np.float32)


def uniforms(seed: int, offset: int, B: int, k: int) -> np.ndarray:
    """Acceptance uniforms u[b, j] (the draw of ``verify.py:120``)."""
    return words_to_uniform(philox_words(seed, offset, STREAM_UNIFORM, B, k))


def exponentials(seed: int, offset: int, B: int, V: int, stream: int | None = None) -> np.ndarray:
    """Exp(1) noise E[b, i] before its clamp_min: by default stream 1, the draw of
    ``verify.py:209``; ``STREAM_SAMPLE`` gives the sampler's draw (``sampler.py:11``)."""
    st = STREAM_EXPONENTIAL if stream is None else stream
    u = words_to_open_uniform(philox_words(seed, offset, st, B, V))
    return (-log_f32(u)).astype(np.float32)
