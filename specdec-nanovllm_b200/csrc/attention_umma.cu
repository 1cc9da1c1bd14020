// Paged decode / verify attention on the 5th-generation tensor cores (tcgen05).
//
// Same contract and semantics as pa_mma_kernel (csrc/attention.cu, reference
// behaviour nanovllm/layers/attention.py:64-81); this kernel takes the shapes
// with 16-bit KV, head_dim 128, page % 128 == 0 and at most 32 query rows per
// (sequence, kv head) -- Qwen3 decode (4 rows) and k <= 7 verify (k+1 rows of a
// GQA-4 group).
//
// Formulation (transposed, so the 128-row tensor-core tile is the key axis):
//   S^T[key, row] = K[key, :] . Q[row, :]        M = 128 keys, N = 32 rows, K = 128 dims
//   O^T[dim, row] += V^T[dim, key] . P^T[key, row] M = 128 dims, N = 32 rows, K = 128 keys
// Both accumulators live in tensor memory (TMEM): S^T double-buffered in
// columns [0, 64), O^T in [64, 96).  K and V tiles arrive by TMA in the
// 128-byte-swizzled layout the MMA descriptors read directly (K as a K-major A
// operand, V as an MN-major A operand); Q^T and P^T are written by the softmax
// warps as K-major B operands.  P is split into a 16-bit head and a 16-bit
// residual and both multiply V, so the probabilities keep ~16 significant bits.
//
// Warp roles (192 threads, one CTA per SM, persistent over work items):
//   warp 0      TMA producer: K/V tiles of 128 keys into a 3-stage ring
//   warp 1      TMEM owner and MMA issuer (one thread)
//   warps 2..5  softmax: thread = one TMEM lane (a key of S^T, a dim of O^T);
//               column max / sum by an in-warp transpose reduction + a 4-warp
//               exchange; lazy rescale (O is rescaled only when a row max grows
//               by more than 2^8, exact because the reference point is kept).
// Work items (split, kv head, sequence) are strided over the persistent CTAs;
// the producer streams the next item's tiles while the current one finishes.
// Every wait is bounded and reports SDB_KERR_TIMEOUT instead of hanging.
#include <cfloat>

#include "attention_common.cuh"
#include "umma.cuh"

namespace sdb {
namespace attn {
namespace umma {

constexpr int UBN = 128;                  // keys per tile
constexpr int UHALF = UBN * 128;          // one 64-dim half of a K or V tile: 16 KB
constexpr int UTILE = 2 * UHALF;          // 32 KB
constexpr int USTAGE = 2 * UTILE;         // K + V: 64 KB
constexpr int UNS = 3;                    // stages
constexpr int NROW = 32;                  // MMA N: query rows per (sequence, kv head)
constexpr int QHALF = NROW * 128;         // 4 KB
constexpr int PHALF = NROW * 128;         // 4 KB (64 keys of 32 rows)
constexpr int OFF_Q = UNS * USTAGE;
constexpr int OFF_PHI = OFF_Q + 2 * QHALF;
constexpr int OFF_PLO = OFF_PHI + 2 * PHALF;
constexpr int OFF_RED = OFF_PLO + 2 * PHALF;          // red_max[4][32], red_sum[4][32]
constexpr int OFF_BAR = OFF_RED + 2 * 4 * 32 * 4;
// barriers: full[3] empty[3] s_full[2] s_free[2] p_full o_done q_ready fin
constexpr int NBAR = UNS * 2 + 2 + 2 + 4;
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;  // + alignment slack
constexpr int kMaxUmmaSplits = 16;
constexpr uint32_t TMEM_COLS = 128;
constexpr int THREADS = 192;

struct Bars {
    uint32_t full0, empty0, sfull0, sfree0, pfull, odone, qready, fin;
};

SDB_DEV Bars bars_at(uint32_t base) {
    Bars b;
    b.full0 = base;
    b.empty0 = base + 8 * UNS;
    b.sfull0 = base + 16 * UNS;
    b.sfree0 = b.sfull0 + 16;
    b.pfull = b.sfree0 + 16;
    b.odone = b.pfull + 8;
    b.qready = b.odone + 8;
    b.fin = b.qready + 8;
    return b;
}

struct Item {
    int b, kvh, split, L, k0, k1, ntiles;
};

SDB_DEV Item item_at(const Params& p, int it) {
    Item x;
    x.split = it % p.splits;
    const int rest = it / p.splits;
    x.kvh = rest % p.Hkv;
    x.b = rest / p.Hkv;
    x.L = load_len(p, x.b);
    x.k0 = x.split * p.chunk;
    x.k1 = min(x.k0 + p.chunk, x.L);
    x.ntiles = x.k1 > x.k0 ? (x.k1 - x.k0 + UBN - 1) / UBN : 0;
    return x;
}

// Wait that becomes a no-op once this thread has seen a timeout: the softmax warps
// keep executing the same sequence of named barriers after a failure (never
// leaving a loop early), so one warp giving up can never strand the others.
SDB_DEV bool wait_or_skip(uint32_t bar, uint32_t parity, bool& ok) {
    if (!ok) return false;
    if (!mbar_wait(bar, parity)) ok = false;
    return ok;
}

// In-warp transpose reduction: lane c ends with op over the 32 lanes of v[c].
template <bool MAX>
SDB_DEV float transpose_reduce(float (&v)[32], int lane) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
            const float send = upper ? v[i] : v[i + off];
            const float keep = upper ? v[i + off] : v[i];
            const float recv = __shfl_xor_sync(0xffffffffu, send, off);
            v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
        }
    }
    return v[0];
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1)
    pa_umma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const Params p, int total_items) {
    using H = Half16<T>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const Bars bar = bars_at(sbase + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);
    float* red_max = reinterpret_cast<float*>(smem + OFF_RED);
    float* red_sum = red_max + 4 * 32;
    __shared__ int last_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < UNS; ++s) {
            mbar_init(bar.full0 + 8 * s, 1);
            mbar_init(bar.empty0 + 8 * s, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar.sfull0 + 8 * i, 1);
            mbar_init(bar.sfree0 + 8 * i, 128);
        }
        mbar_init(bar.pfull, 128);
        mbar_init(bar.odone, 1);
        mbar_init(bar.qready, 128);
        mbar_init(bar.fin, 1);
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
            const uint64_t pol = l2_policy_evict_first();
            int gt = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < total_items && ok; it += gridDim.x) {
                const Item x = item_at(p, it);
                const int* btrow = p.bt + (int64_t)x.b * p.bt_stride;
                for (int t = 0; t < x.ntiles; ++t, ++gt) {
                    const int s = gt % UNS;
                    if (gt >= UNS && !mbar_wait(bar.empty0 + 8 * s, ((gt / UNS) - 1) & 1)) {
                        atomicOr(p.err, SDB_KERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                    const int j = x.k0 + t * UBN;
                    int blk = btrow[j / p.page];
                    if (blk < 0 || blk >= p.num_blocks) {
                        atomicOr(p.err, SDB_KERR_BLOCK_ID);
                        blk = 0;
                    }
                    const int off = j % p.page;
                    const uint32_t kdst = sbase + s * USTAGE;
                    const uint32_t vdst = kdst + UTILE;
                    const uint32_t fb = bar.full0 + 8 * s;
                    mbar_arrive_expect_tx(fb, USTAGE);
                    tma_load_4d(kdst, &kmap, fb, 0, x.kvh, off, blk, pol);
                    tma_load_4d(kdst + UHALF, &kmap, fb, 64, x.kvh, off, blk, pol);
                    tma_load_4d(vdst, &vmap, fb, 0, x.kvh, off, blk, pol);
                    tma_load_4d(vdst + UHALF, &vmap, fb, 64, x.kvh, off, blk, pol);
                }
            }
            for (int g = gt - UNS > 0 ? gt - UNS : 0; g < gt; ++g) {  // drain own copies
                if (!mbar_wait(bar.full0 + 8 * (g % UNS), (g / UNS) & 1)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            constexpr uint32_t IDESC_S = idesc_f16(BF, false, false, 128, NROW);
            constexpr uint32_t IDESC_PV = idesc_f16(BF, true, false, 128, NROW);
            int gt = 0, nitem = 0;
            bool ok = true;
            auto pv = [&](int g, bool first) -> bool {
                if (!mbar_wait(bar.pfull, g & 1)) return false;
                tc_fence_after();
                const uint32_t vbase = sbase + (g % UNS) * USTAGE + UTILE;
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    const uint32_t pbase = sbase + (part == 0 ? OFF_PHI : OFF_PLO);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t a = sdesc_sw128(vbase + ks * 2048, UHALF, 1024);
                        const uint64_t b = sdesc_sw128(pbase + (ks >> 2) * PHALF + (ks & 3) * 32, 16, 1024);
                        umma_f16_ss(tmem + 64, a, b, IDESC_PV, (first && part == 0 && ks == 0) ? 0u : 1u);
                    }
                }
                umma_commit(bar.odone);
                umma_commit(bar.empty0 + 8 * (g % UNS));
                return true;
            };
            for (int it = blockIdx.x; it < total_items && ok; it += gridDim.x, ++nitem) {
                const Item x = item_at(p, it);
                if (!mbar_wait(bar.qready, nitem & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int t = 0; t < x.ntiles; ++t, ++gt) {
                    const int s = gt % UNS, sb = gt & 1;
                    if (!mbar_wait(bar.full0 + 8 * s, (gt / UNS) & 1) ||
                        (gt >= 2 && !mbar_wait(bar.sfree0 + 8 * sb, ((gt >> 1) - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t kbase = sbase + s * USTAGE;
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t a = sdesc_sw128(kbase + (ks >> 2) * UHALF + (ks & 3) * 32, 16, 1024);
                        const uint64_t b = sdesc_sw128(sbase + OFF_Q + (ks >> 2) * QHALF + (ks & 3) * 32, 16, 1024);
                        umma_f16_ss(tmem + sb * 32, a, b, IDESC_S, ks > 0 ? 1u : 0u);
                    }
                    umma_commit(bar.sfull0 + 8 * sb);
                    if (t >= 1 && !pv(gt - 1, t == 1)) {
                        ok = false;
                        break;
                    }
                }
                if (ok && x.ntiles >= 1 && !pv(gt - 1, x.ntiles == 1)) ok = false;
            }
            if (!ok) atomicOr(p.err, SDB_KERR_TIMEOUT);
            // every MMA this thread issued has completed before TMEM is released
            umma_commit(bar.fin);
            if (!mbar_wait(bar.fin, 0)) atomicOr(p.err, SDB_KERR_TIMEOUT);
        }
    } else {
        // ------------------------------------------------------------- softmax warps
        const int st = threadIdx.x - 64;   // 0..127
        const int qt = warp & 3;           // TMEM lane quarter of this warp
        const uint32_t lane_addr = (uint32_t)(32 * qt) << 16;
        const int R = p.R;
        const float sl2 = p.scale_log2;
        int gt = 0;
        bool ok = true;
        T* obase = reinterpret_cast<T*>(p.out);
        const T* qbase = reinterpret_cast<const T*>(p.q);
        for (int it = blockIdx.x; it < total_items; it += gridDim.x) {
            const Item x = item_at(p, it);
            // ---- Q^T of this item into the K-major swizzled B operand (rows >= R are zero)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int u = st + 128 * i;
                const int c = u >> 4, ch = u & 15;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (c < R) {
                    const int r = c / p.G, g = c % p.G;
                    v = __ldg(reinterpret_cast<const uint4*>(qbase + (int64_t)(x.b * p.n_q + r) * p.q_srow +
                                                             (int64_t)(x.kvh * p.G + g) * p.q_shead + ch * 8));
                }
                *reinterpret_cast<uint4*>(smem + OFF_Q + (ch >> 3) * QHALF + c * 128 + (((ch & 7) ^ (c & 7)) << 4)) =
                    v;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar.qready);

            // per-row (column) softmax state, held by lane c of every softmax warp
            float mb = NEG_INF, lsum = 0.f;
            const int lbase = x.L - p.n_q + 1;  // keys visible to row r: j < lbase + r
            for (int t = 0; t < x.ntiles; ++t, ++gt) {
                const int sb = gt & 1, s = gt % UNS;
                const int j0 = x.k0 + t * UBN;
                wait_or_skip(bar.sfull0 + 8 * sb, (gt >> 1) & 1, ok);
                tc_fence_after();
                uint32_t sr[32];
                tmem_ld32(tmem + lane_addr + sb * 32, sr);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(bar.sfree0 + 8 * sb);

                const int key = j0 + 32 * qt + lane;
                const bool masked = (j0 + UBN > min(lbase, x.k1)) || R < NROW;
                float xv[32];
                {
                    int r = 0, g = 0;
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        float v = __uint_as_float(sr[c]) * sl2;
                        if (masked) {
                            const bool vis = c < R && key < min(lbase + r, x.k1);
                            v = vis ? v : NEG_INF;
                            if (++g == p.G) {
                                g = 0;
                                ++r;
                            }
                        }
                        xv[c] = v;
                    }
                }
                // column max over the tile's 128 keys
                float tmp[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) tmp[c] = xv[c];
                red_max[qt * 32 + lane] = transpose_reduce<true>(tmp, lane);
                named_barrier_sync(1, 128);
                const float M = fmaxf(fmaxf(red_max[lane], red_max[32 + lane]),
                                      fmaxf(red_max[64 + lane], red_max[96 + lane]));
                // lazy rescale: move the reference point only when the max grows by > 2^8
                const float nb = (M > mb + 8.0f) ? M : mb;
                const float alpha = (nb != mb) ? ex2(mb - nb) : 1.0f;
                const bool rescale = __any_sync(0xffffffffu, nb != mb && lsum > 0.f);
                mb = nb;
                float pv[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float mc = __shfl_sync(0xffffffffu, mb, c);
                    pv[c] = ex2(xv[c] - (mc == NEG_INF ? 0.f : mc));
                }
#pragma unroll
                for (int c = 0; c < 32; ++c) tmp[c] = pv[c];
                red_sum[qt * 32 + lane] = transpose_reduce<false>(tmp, lane);
                named_barrier_sync(1, 128);
                lsum = lsum * alpha + (red_sum[lane] + red_sum[32 + lane]) + (red_sum[64 + lane] + red_sum[96 + lane]);

                // the previous tile's P.V has finished: P buffer free, O up to date
                if (t >= 1) {
                    wait_or_skip(bar.odone, (gt - 1) & 1, ok);
                    tc_fence_after();
                    if (rescale) {
                        uint32_t orr[32];
                        tmem_ld32(tmem + lane_addr + 64, orr);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; ++c) {
                            const float a = __shfl_sync(0xffffffffu, alpha, c);
                            orr[c] = __float_as_uint(__uint_as_float(orr[c]) * a);
                        }
                        tmem_st32(tmem + lane_addr + 64, orr);
                        tmem_wait_st();
                    }
                }
                // keys past the split end: zero their V rows (unwritten cache may hold NaN)
                const int kin = 32 * qt + lane;
                if (j0 + UBN > x.k1) {
                    wait_or_skip(bar.full0 + 8 * s, (gt / UNS) & 1, ok);
                    if (j0 + kin >= x.k1) {
                        uint8_t* vrow = smem + s * USTAGE + UTILE + kin * 128;
#pragma unroll
                        for (int h = 0; h < 2; ++h)
#pragma unroll
                            for (int cc = 0; cc < 8; ++cc)
                                *reinterpret_cast<uint4*>(vrow + h * UHALF + cc * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                // P^T (head and residual) into the K-major swizzled B operands
                {
                    const int half = kin >> 6, kk = kin & 63;
                    const int chunk = kk >> 3, byte = (kk & 7) * 2;
                    uint8_t* phi = smem + OFF_PHI + half * PHALF + byte;
                    uint8_t* plo = smem + OFF_PLO + half * PHALF + byte;
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const uint32_t packed = H::pack(pv[c], 0.f);
                        const uint32_t resid = H::pack_residual(pv[c], 0.f, packed);
                        const int o = c * 128 + ((chunk ^ (c & 7)) << 4);
                        *reinterpret_cast<uint16_t*>(phi + o) = (uint16_t)(packed & 0xffffu);
                        *reinterpret_cast<uint16_t*>(plo + o) = (uint16_t)(resid & 0xffffu);
                    }
                }
                fence_proxy_async_smem();
                tc_fence_before();
                mbar_arrive(bar.pfull);
            }

            // ---- item epilogue: O^T column c is row c; this thread holds dim 32*qt + lane
            float o[32];
            if (x.ntiles > 0) {
                wait_or_skip(bar.odone, (gt - 1) & 1, ok);
                tc_fence_after();
                uint32_t orr[32];
                tmem_ld32(tmem + lane_addr + 64, orr);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; ++c) o[c] = __uint_as_float(orr[c]);
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) o[c] = 0.f;
            }
            const int dim = 32 * qt + lane;
            if (p.splits == 1) {
                int r = 0, g = 0;
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float lc = __shfl_sync(0xffffffffu, lsum, c);
                    if (c < R) {
                        T* dst = obase + (int64_t)(x.b * p.n_q + r) * p.o_srow +
                                 (int64_t)(x.kvh * p.G + g) * p.o_shead + dim;
                        *dst = from_f32<T>(lc > 0.f ? o[c] / lc : 0.f);
                    }
                    if (++g == p.G) {
                        g = 0;
                        ++r;
                    }
                }
                continue;
            }
            const int pair = x.b * p.Hkv + x.kvh;
            const int64_t slot = (int64_t)pair * p.splits + x.split;
            float* po = p.part_o + slot * R * D;
            float* pml = p.part_ml + slot * R * 2;
#pragma unroll
            for (int c = 0; c < 32; ++c)
                if (c < R) __stcg(po + c * D + dim, o[c]);
            if (st < 32 && lane < R) __stcg(reinterpret_cast<float2*>(pml + lane * 2), make_float2(mb, lsum));
            __threadfence();
            named_barrier_sync(2, 128);
            if (st == 0) last_flag = atomicAdd(p.counters + pair, 1) == p.splits - 1;
            named_barrier_sync(2, 128);
            if (!last_flag) continue;
            __threadfence();
            // last CTA of this (sequence, kv head): LSE-merge the splits, one dim per thread
            const float* ml = p.part_ml + (int64_t)pair * p.splits * R * 2;
            const float* pob = p.part_o + (int64_t)pair * p.splits * R * D;
            int r = 0, g = 0;
            for (int c = 0; c < R; ++c) {
                float Mx = NEG_INF;
                for (int s2 = 0; s2 < p.splits; ++s2) Mx = fmaxf(Mx, __ldcg(ml + (s2 * R + c) * 2));
                const float Bm = Mx == NEG_INF ? 0.f : Mx;
                float Ls = 0.f, acc = 0.f;
                for (int s2 = 0; s2 < p.splits; ++s2) {
                    const float w = ex2(__ldcg(ml + (s2 * R + c) * 2) - Bm);
                    Ls += w * __ldcg(ml + (s2 * R + c) * 2 + 1);
                    acc += w * __ldcg(pob + ((int64_t)s2 * R + c) * D + dim);
                }
                T* dst = obase + (int64_t)(x.b * p.n_q + r) * p.o_srow + (int64_t)(x.kvh * p.G + g) * p.o_shead + dim;
                *dst = from_f32<T>(Ls > 0.f ? acc / Ls : 0.f);
                if (++g == p.G) {
                    g = 0;
                    ++r;
                }
            }
            named_barrier_sync(2, 128);
            if (st == 0) p.counters[pair] = 0;
        }
        if (!ok && lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace umma

// ------------------------------------------------------------------------- host
bool umma_path(int dtype, int D_, int page, int R) {
    return (dtype == SDB_BF16 || dtype == SDB_F16) && D_ == D && page % umma::UBN == 0 && R <= umma::NROW;
}

// Splits for the persistent grid: minimise (items per CTA) x (tiles per item), from static shape only.
int pick_umma_splits(int B, int R, int Hkv, int page, int max_blocks, int sms) {
    const long long max_ctx = (long long)max_blocks * page;
    const long long tiles = (max_ctx + umma::UBN - 1) / umma::UBN;
    const long long pairs = (long long)B * Hkv;
    int best = 1;
    double best_cost = 1e300;
    for (int s = 1; s <= umma::kMaxUmmaSplits; ++s) {
        const long long chunk_tiles = (tiles + s - 1) / s;
        if (s > 1 && chunk_tiles < 2) break;
        const long long items = pairs * s;
        const long long grid = items < sms ? items : sms;
        const long long per_cta = (items + grid - 1) / grid;
        double cost = (double)per_cta * (chunk_tiles * (double)umma::USTAGE + 4096.0);
        if (s > 1) cost += (double)per_cta * R * (D + 2) * 8.0;
        if (cost < best_cost * 0.995) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

int launch_umma(const void* k_cache, const void* v_cache, int dtype, int64_t sb, int64_t sp, int64_t sh,
                Params& p, void* workspace, size_t workspace_bytes, int splits, cudaStream_t st) {
    const int sms = device_sm_count();
    if (splits <= 0) splits = pick_umma_splits(p.B, p.R, p.Hkv, p.page, p.max_blocks, sms);
    if (splits > umma::kMaxUmmaSplits) splits = umma::kMaxUmmaSplits;
    const long long max_ctx = (long long)p.max_blocks * p.page;
    long long chunk = ((max_ctx + splits - 1) / splits + umma::UBN - 1) / umma::UBN * umma::UBN;
    if (chunk < umma::UBN) chunk = umma::UBN;
    splits = (int)((max_ctx + chunk - 1) / chunk);
    if (splits < 1) splits = 1;
    WsLayout w = ws_layout(p.B, p.R, p.Hkv, splits);
    if (workspace_bytes < w.total) {
        set_last_error("workspace too small: need %zu bytes, got %zu", w.total, workspace_bytes);
        return SDB_ERR_WORKSPACE;
    }
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    p.err = reinterpret_cast<int*>(ws + w.err);
    p.counters = reinterpret_cast<int*>(ws + w.counters);
    p.part_ml = reinterpret_cast<float*>(ws + w.part_ml);
    p.part_o = reinterpret_cast<float*>(ws + w.part_o);
    p.splits = splits;
    p.chunk = (int)chunk;
    const CUtensorMapDataType dt = dtype == SDB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)p.Hkv, (cuuint64_t)p.page, (cuuint64_t)p.num_blocks};
    cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)sp * 2, (cuuint64_t)sb * 2};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)umma::UBN, 1};
    CUtensorMap km, vm;
    int rc = encode_tensor_map(&km, dt, 4, const_cast<void*>(k_cache), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tensor_map(&vm, dt, 4, const_cast<void*>(v_cache), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const int total_items = p.B * p.Hkv * splits;
    const int grid = total_items < sms ? total_items : sms;
    if (dtype == SDB_BF16) {
        auto kern = umma::pa_umma_kernel<__nv_bfloat16>;
        rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), umma::SMEM_BYTES, 40);
        if (rc) return rc;
        kern<<<grid, umma::THREADS, umma::SMEM_BYTES, st>>>(km, vm, p, total_items);
    } else {
        auto kern = umma::pa_umma_kernel<__half>;
        rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), umma::SMEM_BYTES, 41);
        if (rc) return rc;
        kern<<<grid, umma::THREADS, umma::SMEM_BYTES, st>>>(km, vm, p, total_items);
    }
    return cuda_status(cudaGetLastError(), "pa_umma_kernel launch");
}

}  // namespace attn
}  // namespace sdb
