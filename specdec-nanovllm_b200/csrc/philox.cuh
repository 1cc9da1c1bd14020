// Counter-based random numbers shared by the samplers (verify_batch, sample):
// Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3",
// SC'11), counter (col / 4, row, stream, offset), key (seed lo, seed hi); uniform
// draws U = (w >> 8) * 2^-24 in [0, 1) and open draws ((w >> 8) + 1) * 2^-24 in
// (0, 1]; exponentials E = -log(U_open) with log computed by a fixed sequence of
// correctly rounded float32 operations, so a CPU restatement reproduces every bit.
// Streams: 0 acceptance uniforms and 1 bonus exponentials of verify_batch, 2 the
// exponentials of sample.
#pragma once

#include "common.cuh"

namespace sdb {
namespace rng {

SDB_DEV void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c[0];
        const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]);
        const uint32_t lo1 = 0xCD9E8D57u * c[2];
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]);
        const uint32_t n0 = hi1 ^ c[1] ^ k0;
        const uint32_t n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}

SDB_DEV uint32_t philox_word(uint32_t seed_lo, uint32_t seed_hi, uint32_t offset, uint32_t stream,
                             uint32_t row, uint32_t col) {
    uint32_t c[4] = {col >> 2, row, stream, offset};
    philox(c, seed_lo, seed_hi);
    return c[col & 3];
}

SDB_DEV float word_to_uniform(uint32_t w) { return __fmul_rn((float)(w >> 8), 5.9604644775390625e-08f); }
SDB_DEV float word_to_open_uniform(uint32_t w) {
    return __fmul_rn((float)((w >> 8) + 1u), 5.9604644775390625e-08f);
}

// Natural log of a positive normal float by fixed float32 operations (the atanh
// series of log m on m in [sqrt(1/2), sqrt(2)) plus e*ln2 split in hi/lo).
// Constants are given by bit pattern so host and device agree on every bit.
SDB_DEV float log_fixed(float x) {
    const uint32_t bits = __float_as_uint(x);
    int e = (int)((bits >> 23) & 0xFFu) - 127;
    float m = __uint_as_float((bits & 0x7FFFFFu) | 0x3F800000u);
    if (m > __uint_as_float(0x3FB504F3u)) {  // sqrt(2)
        m = __fmul_rn(m, 0.5f);
        e += 1;
    }
    const float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
    const float z = __fmul_rn(s, s);
    float r = __uint_as_float(0x3DBA2E8Cu);                          // 1/11
    r = __fadd_rn(__fmul_rn(r, z), __uint_as_float(0x3DE38E39u));   // 1/9
    r = __fadd_rn(__fmul_rn(r, z), __uint_as_float(0x3E124925u));   // 1/7
    r = __fadd_rn(__fmul_rn(r, z), __uint_as_float(0x3E4CCCCDu));   // 1/5
    r = __fadd_rn(__fmul_rn(r, z), __uint_as_float(0x3EAAAAABu));   // 1/3
    r = __fadd_rn(__fmul_rn(r, z), 1.0f);
    const float lm = __fmul_rn(__fadd_rn(s, s), r);
    const float ef = (float)e;
    const float ln2_hi = __uint_as_float(0x3F317200u), ln2_lo = __uint_as_float(0x35BFBE8Eu);
    return __fadd_rn(__fmul_rn(ef, ln2_hi), __fadd_rn(lm, __fmul_rn(ef, ln2_lo)));
}

// Bounds of E = -log(U) for the open uniform U of a word, widened by the few ulps by
// which log_fixed may sit on either side: -log U in [1 - U, (1 - U)(3 - 2U)] for
// U >= 1/2 and <= 17 always (U >= 2^-24); 1 - U is exact (U is a multiple of 2^-24).
// Both bounds are clamped like the samplers' max(E, 1e-10).
SDB_DEV void exp_bounds(float U, float& Elo, float& Ehi) {
    Elo = fmaxf((1.0f - U) * 0.99999f, 1e-10f);
    Ehi = U >= 0.5f ? fmaxf((1.0f - U) * (3.0f - 2.0f * U) * 1.00002f, 1e-10f) : 17.0f;
}

// max(-log U, 1e-10) exactly as the CPU restatement computes it.
SDB_DEV float exp_draw(uint32_t w) { return fmaxf(-log_fixed(word_to_open_uniform(w)), 1e-10f); }

}  // namespace rng
}  // namespace sdb
