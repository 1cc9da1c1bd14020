"""Philox4x32-10 known-answer vectors and the fixed-operation float32 log."""

import math

import numpy as np

from oracle import philox


def _kat(ctr, key):
    out = philox.philox4x32_10(*[np.uint32(c) for c in ctr], key[0], key[1])
    return [int(w) for w in out]


def test_philox_known_answers():
    # Published known-answer vectors of Philox4x32-10 (Random123 distribution, kat_vectors).
    assert _kat([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert _kat([0xFFFFFFFF] * 4, [0xFFFFFFFF, 0xFFFFFFFF]) == \
        [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert _kat([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_log_f32_accuracy_on_every_open_uniform_exponent():
    # all values the sampler can feed it: ((w >> 8) + 1) * 2^-24
    u = (np.arange(1, 1 << 24, 257, dtype=np.float64) * 2.0 ** -24).astype(np.float32)
    got = philox.log_f32(u).astype(np.float64)
    want = np.log(u.astype(np.float64))
    ulp = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
    ulp = np.maximum(ulp, 2.0 ** -149)
    assert np.max(np.abs(got - want) / ulp) <= 3.0
    assert philox.log_f32(np.float32(1.0)) == 0.0


def test_streams_shape_and_range():
    u = philox.uniforms(5, 3, 7, 6)
    assert u.shape == (7, 6) and u.dtype == np.float32
    assert (u >= 0).all() and (u < 1).all()
    e = philox.exponentials(5, 3, 3, 1001)
    assert e.shape == (3, 1001)
    assert (e >= 0).all() and (e <= 24 * math.log(2) + 1e-5).all()
    # Exp(1): mean 1
    assert abs(float(philox.exponentials(1, 0, 64, 4096).mean()) - 1.0) < 0.01
    # offsets and streams decorrelate
    assert not np.array_equal(philox.uniforms(5, 4, 7, 6), u)
