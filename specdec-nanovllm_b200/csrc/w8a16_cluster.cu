// W8A16 linear for 17 to 128 tokens on tcgen05, split-K inside thread-block clusters:
// y = x @ (q * s)^T (+ bias), int8 weights q [N, K], per-channel scales s [N], 16-bit x [M, K].
//
// Reference: int8_linear / _int8_dequant_gemm_kernel, nanovllm/layers/quant.py:165-310
// (weights dequantised on the fly, fp32 accumulation, scale applied per output channel).
//
// At these token counts the call streams its weights once: the cost is the weight bytes,
// the launch ramp and the split-K reduction.  The design takes all three on:
//   * Transposed tensor-core tile, as in w8a16_umma.cu: Y^T[128 features, Npad tokens] +=
//     W[128 features, 16 k] . X^T[16 k, Npad tokens], fp32 accumulators in TMEM.
//   * The A operand (the converted weights) lives in TMEM, not shared memory: eight converter
//     warps turn each 128 x 128 int8 tile into 16-bit values in registers and store them with
//     tcgen05.st (one 32-column store per thread); the MMA reads A from TMEM and only the
//     token tile from shared memory.  Shared-memory traffic per tile drops from ~96 KB
//     (int8 read, 16-bit write, MMA read of both operands) to ~32 KB.
//   * Split-K without a global round trip: the (feature tile, k tile) units of a group of
//     tiles are split evenly over the CTAs of one cluster (1..8 CTAs, sized on the host so
//     that the whole grid is resident at once); each CTA leaves its per-tile partial sums in
//     its own shared memory and the cluster sums them over DSMEM in rank order
//     (deterministic), applies scale and bias and writes y.  No partial buffer, no second
//     launch.
//   * Programmatic dependent launch: a CTA lets the next kernel launch at once and sets up
//     (barriers, TMEM, tensor-map prefetch) while the preceding kernel drains; it waits
//     (griddepcontrol.wait) before its first load and before it writes y.
//
//
// Per CTA, 352 threads (each waiting role in a warp of its own, so that no role's blocked
// mbarrier wait holds up another's issue):
//   warp 0       weight producer (TMA loads into a ring of 16 KB stages, one 128 k x 128 row
//                box, 128-byte swizzle)
//   warp 1       TMEM owner (512 columns) and MMA issuer (one thread)
//   warp 2       token producer (128 k of the token rows per unit, two 64-k boxes, 128-byte
//                swizzle)
//   warps 3..10  converters (warp w: TMEM lane quarter w % 4, k half (w - 3) / 4), then
//                the accumulator dump to shared memory and the cluster reduction
// Measured limits (B200): one tcgen05.mma of M = 128, K = 16 occupies the tensor pipe for
// ~100 cycles whether N is 16 or 64, so a unit's 8 MMAs take ~0.43 us and a CTA streams
// at most ~37 GB/s of int8 weights; the converter / MMA hand-off through the A buffers and
// the completion commits add about as much again.  Eight converter warps, three A buffers
// up to 64 tokens and one accumulator per tile measured best (16 converter warps and
// 2-4 interleaved accumulators did not help).
// Every wait is bounded and reports SDB_KERR_TIMEOUT; every thread passes both cluster
// barriers on every path.
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "umma.cuh"
#include "w8a16_convert.cuh"

namespace sdb {
namespace w8c {

constexpr int FROWS = 128;           // features per tile (MMA M)
constexpr int KT = 128;              // k per unit
constexpr int WSTAGE = FROWS * KT;   // int8 weight stage: 16 KB
constexpr int CONV_THREADS = 256;
constexpr int CONV_WARP0 = 3;  // warps 0..2: weight producer, MMA issuer, token producer
constexpr int THREADS = 32 * CONV_WARP0 + CONV_THREADS;
constexpr int MAXNPAD = 128;
constexpr int MAXNW = 14, MAXNX = 8, MAXNA = 3;
constexpr int RED_TOK = 4;  // tokens per reduction item (4 measured best of 2 / 4 / 8)
constexpr int MAXC = 8;
constexpr int kRingBudget = 220 * 1024;
constexpr int TMEM_COLS = 512;

struct Params {
    const void* s;
    int s_dtype;
    const void* bias;
    void* y;
    int64_t y_srow;
    int M, N, K, Npad, FT, KTN, C, G, NW, NX, NA, vec_y;
    int* err;
};

// Cluster g holds feature tiles [tile_lo(g), tile_lo(g + 1)).
SDB_DEV int tile_lo(const Params& p, int g) { return (int)((long long)g * p.FT / p.G); }
// First unit of rank r when U units are split over C ranks.
SDB_DEV int ustart(int U, int C, int r) { return (int)((long long)r * U / C); }
// Rank whose unit range holds unit u.
SDB_DEV int uowner(int U, int C, int u) { return (int)(((long long)(u + 1) * C + U - 1) / U) - 1; }

struct Ring {
    int slot = 0;
    uint32_t phase = 0;
    SDB_DEV void next(int n) {
        if (++slot == n) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

template <typename T>
SDB_DEV void store4(const Params& p, int m, int n0, const float (&v)[4]) {
    T* y = reinterpret_cast<T*>(p.y) + (int64_t)m * p.y_srow + n0;
    if (p.vec_y && n0 + 3 < p.N) {
        union {
            T h[4];
            uint2 u;
        } pk;
#pragma unroll
        for (int j = 0; j < 4; ++j) pk.h[j] = from_f32<T>(v[j]);
        *reinterpret_cast<uint2*>(y) = pk.u;
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (n0 + j < p.N) y[j] = from_f32<T>(v[j]);
    }
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1)
    w8a16_cluster_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                         const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t bar_mem[2 * MAXNW + 2 * MAXNX + 2 * MAXNA + 1];
    __shared__ uint32_t tmem_slot;
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = (int)cluster_ctarank(), g = (int)cluster_id_x();
    const int t0 = tile_lo(p, g), nt = tile_lo(p, g + 1) - t0;
    const int KTN = p.KTN, U = nt * KTN;
    const int u0 = ustart(U, p.C, rank), u1 = ustart(U, p.C, rank + 1);
    const int nseg = u1 > u0 ? (u1 - 1) / KTN - u0 / KTN + 1 : 0;
    const int NW = p.NW, NX = p.NX, NA = p.NA, Npad = p.Npad;
    const int xbox = Npad * 128, xstage = 2 * xbox;
    const uint32_t wfull0 = smem_u32(bar_mem), wempty0 = wfull0 + 8 * MAXNW;
    const uint32_t xfull0 = wempty0 + 8 * MAXNW, xempty0 = xfull0 + 8 * MAXNX;
    const uint32_t afull0 = xempty0 + 8 * MAXNX, aempty0 = afull0 + 8 * MAXNA;
    const uint32_t accfull = aempty0 + 8 * MAXNA;
    uint8_t* wring = smem;
    uint8_t* xring = smem + NW * WSTAGE;
    const int acc_col = NA * 64;  // A buffers: 64 columns (128 k of 16-bit values) each

    if (threadIdx.x == 0) {
        for (int i = 0; i < NW; ++i) {
            mbar_init(wfull0 + 8 * i, 1);
            mbar_init(wempty0 + 8 * i, CONV_THREADS / 32);
        }
        for (int i = 0; i < NX; ++i) {
            mbar_init(xfull0 + 8 * i, 1);
            mbar_init(xempty0 + 8 * i, 1);
        }
        for (int i = 0; i < NA; ++i) {
            mbar_init(afull0 + 8 * i, CONV_THREADS / 32);
            mbar_init(aempty0 + 8 * i, 1);
        }
        mbar_init(accfull, 1);
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------ weight producer
            prefetch_tensormap(&wmap);
            pdl_wait();  // weights stay unread until the preceding kernel has completed
            const uint64_t pol = l2_policy_evict_first();
            Ring r;
            int issued = 0;
            for (int u = u0; u < u1; ++u, ++issued) {
                if (issued >= NW && !mbar_wait(wempty0 + 8 * r.slot, r.phase ^ 1u)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
                const uint32_t fb = wfull0 + 8 * r.slot;
                mbar_arrive_expect_tx(fb, (uint32_t)WSTAGE);
                tma_load_2d(smem_u32(wring + r.slot * WSTAGE), &wmap, fb, (u % KTN) * KT, (t0 + u / KTN) * FROWS,
                            pol);
                r.next(NW);
            }
            Ring d;  // own copies land before the stages are reused or the CTA exits
            for (int i = 0; i < issued; ++i) {
                if (i >= issued - NW && !mbar_wait(wfull0 + 8 * d.slot, d.phase)) break;
                d.next(NW);
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // ------------------------------------------------------- token producer
            prefetch_tensormap(&xmap);
            pdl_wait();  // x is the preceding kernel's output
            const uint64_t pol = l2_policy_evict_normal();  // every CTA re-reads x
            Ring r;
            int issued = 0;
            for (int u = u0; u < u1; ++u, ++issued) {
                if (issued >= NX && !mbar_wait(xempty0 + 8 * r.slot, r.phase ^ 1u)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
                const uint32_t fb = xfull0 + 8 * r.slot;
                const uint32_t st = smem_u32(xring + r.slot * xstage);
                mbar_arrive_expect_tx(fb, (uint32_t)xstage);
                tma_load_2d(st, &xmap, fb, (u % KTN) * KT, 0, pol);
                tma_load_2d(st + xbox, &xmap, fb, (u % KTN) * KT + 64, 0, pol);
                r.next(NX);
            }
            Ring d;
            for (int i = 0; i < issued; ++i) {
                if (i >= issued - NX && !mbar_wait(xfull0 + 8 * d.slot, d.phase)) break;
                d.next(NX);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            const uint32_t idesc = idesc_f16(BF, false, false, FROWS, Npad);
            bool ok = true;
            Ring xr, ar;
            for (int u = u0; u < u1; ++u) {
                if (!mbar_wait(xfull0 + 8 * xr.slot, xr.phase) || !mbar_wait(afull0 + 8 * ar.slot, ar.phase)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const bool first = u == u0 || u % KTN == 0;
                const uint32_t a = tmem + (uint32_t)(ar.slot * 64);
                const uint32_t d = tmem + (uint32_t)(acc_col + (u / KTN - u0 / KTN) * Npad);
                const uint32_t xb = smem_u32(xring + xr.slot * xstage);
#pragma unroll
                for (int ks = 0; ks < KT / 16; ++ks) {
                    const uint64_t bd = sdesc_sw128(xb + (ks >> 2) * xbox + (ks & 3) * 32, 16, 1024);
                    umma_f16_ts(d, a + 8 * ks, bd, idesc, (first && ks == 0) ? 0u : 1u);
                }
                umma_commit(xempty0 + 8 * xr.slot);  // token stage consumed
                umma_commit(aempty0 + 8 * ar.slot);  // A buffer consumed
                xr.next(NX);
                ar.next(NA);
            }
            if (!ok) atomicOr(p.err, SDB_KERR_TIMEOUT);
            umma_commit(accfull);  // every MMA issued above has completed
        }
    } else {
        // ---------------------------------------------------------------- converters
        const int q = warp & 3;             // TMEM lane quarter this warp may access
        const int row = 32 * q + lane;      // feature row of the tile
        const int kh = (warp - CONV_WARP0) >> 2;  // which 64 k of each unit this thread converts
        const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
        const int sw = row & 7;
        bool ok = true;
        Ring wr, ar;
        int i = 0;
        for (int u = u0; u < u1; ++u, ++i) {
            if (ok && !mbar_wait(wfull0 + 8 * wr.slot, wr.phase)) ok = false;
            // row `row` of the stage: 128 B, 16-byte chunk j (k 16j .. 16j+15) at j ^ (row & 7)
            const uint8_t* src = wring + wr.slot * WSTAGE + row * 128;
            uint4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = *reinterpret_cast<const uint4*>(src + (((4 * kh + j) ^ sw) << 4));
            uint32_t o[32];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                w8cv::i8x4<T>(v[j].x, o[8 * j + 0], o[8 * j + 1]);
                w8cv::i8x4<T>(v[j].y, o[8 * j + 2], o[8 * j + 3]);
                w8cv::i8x4<T>(v[j].z, o[8 * j + 4], o[8 * j + 5]);
                w8cv::i8x4<T>(v[j].w, o[8 * j + 6], o[8 * j + 7]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(wempty0 + 8 * wr.slot);  // the stage's bytes are in registers
            if (ok && i >= NA && !mbar_wait(aempty0 + 8 * ar.slot, ar.phase ^ 1u)) ok = false;
            tc_fence_after();
            tmem_st32(tmem + lane_addr + (uint32_t)(ar.slot * 64 + 32 * kh), o);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(afull0 + 8 * ar.slot);
            wr.next(NW);
            ar.next(NA);
        }
        // ---- accumulator dump: red[seg][token][feature row] fp32, over the rings (every copy
        // has landed and every MMA has completed once accfull fires)
        if (ok && !mbar_wait(accfull, 0)) ok = false;
        tc_fence_after();
        float* red = reinterpret_cast<float*>(smem);
        for (int s = 0; s < nseg; ++s) {
            for (int mc = 16 * kh; mc < Npad; mc += 32) {
                uint32_t rr[16];
                tmem_ld16(tmem + lane_addr + (uint32_t)(acc_col + s * Npad + mc), rr);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) red[((s * Npad) + mc + j) * FROWS + row] = __uint_as_float(rr[j]);
            }
        }
        tc_fence_before();
        if (!ok && lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
    }

    cluster_sync_all();  // every CTA's partial sums are in its shared memory
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
    if (warp >= CONV_WARP0) {
        // ------------------------------------------------------------ cluster reduction
        // item = (tile, group of RED_TOK tokens, group of 4 features): the thread sums the
        // contributing ranks' partials in rank order, RED_TOK independent loads per rank
        pdl_wait();  // y may still be read by the preceding kernel
        const int ct = threadIdx.x - 32 * CONV_WARP0;
        const int nmc = (p.M + RED_TOK - 1) / RED_TOK;
        const int total = nt * nmc * 32;
        const T* bias = reinterpret_cast<const T*>(p.bias);
        for (int idx = rank * CONV_THREADS + ct; idx < total; idx += p.C * CONV_THREADS) {
            const int f4 = idx & 31;
            const int rest = idx >> 5;
            const int m0 = (rest % nmc) * RED_TOK, tl = rest / nmc;
            const int n0 = (t0 + tl) * FROWS + 4 * f4;
            float sc[4], bn[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + j;
                sc[j] = n < p.N ? w8cv::scale_value(p.s, p.s_dtype, n) : 0.f;
                bn[j] = (bias && n < p.N) ? to_f32(bias[n]) : 0.f;
            }
            const int r_lo = uowner(U, p.C, tl * KTN), r_hi = uowner(U, p.C, tl * KTN + KTN - 1);
            float4 acc[RED_TOK];
#pragma unroll
            for (int i = 0; i < RED_TOK; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = r_lo; r <= r_hi; ++r) {
                const int seg = tl - ustart(U, p.C, r) / KTN;
                const float4* src = reinterpret_cast<const float4*>(dsmem_map(smem, (uint32_t)r)) +
                                    ((seg * Npad + m0) * FROWS + 4 * f4) / 4;
                float4 v[RED_TOK];
#pragma unroll
                for (int i = 0; i < RED_TOK; ++i) v[i] = src[i * (FROWS / 4)];  // rows past M are padding
#pragma unroll
                for (int i = 0; i < RED_TOK; ++i) {
                    acc[i].x += v[i].x;
                    acc[i].y += v[i].y;
                    acc[i].z += v[i].z;
                    acc[i].w += v[i].w;
                }
            }
#pragma unroll
            for (int i = 0; i < RED_TOK; ++i) {
                if (m0 + i < p.M) {
                    const float out[4] = {acc[i].x * sc[0] + bn[0], acc[i].y * sc[1] + bn[1],
                                          acc[i].z * sc[2] + bn[2], acc[i].w * sc[3] + bn[3]};
                    store4<T>(p, m0 + i, n0, out);
                }
            }
        }
    }
    cluster_sync_all();  // the cluster's reads of this CTA's shared memory are done
}

}  // namespace w8c
}  // namespace sdb

namespace sdb {
namespace w8c {

struct Geometry {
    int Npad, FT, KTN, C, G, NW, NX, NA, smem, umax;
};

static void rings(int Npad, Geometry& g) {
    g.NA = Npad <= 64 ? 3 : 2;
    g.NX = Npad <= 16 ? 8 : (Npad <= 32 ? 6 : (Npad <= 64 ? 4 : 3));
    g.NW = (kRingBudget - g.NX * 2 * Npad * 128) / WSTAGE;
    if (g.NW > MAXNW) g.NW = MAXNW;
    g.smem = g.NW * WSTAGE + g.NX * 2 * Npad * 128 + 1024;
}

template <typename T>
static const void* kernel_ptr() {
    return reinterpret_cast<const void*>(w8a16_cluster_kernel<T>);
}

// Largest number of clusters of `C` CTAs (1 per SM at this shared-memory size) that are
// resident at once; cached per (dtype, C).
static int max_clusters(bool bf16, int C, int smem) {
    static int cache[64][2][MAXC + 1];
    static std::mutex mu;
    const int dev = device_index();
    if (dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    int& c = cache[dev][bf16 ? 0 : 1][C];
    if (c != 0) return c;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * 64, 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const void* kern = bf16 ? kernel_ptr<__nv_bfloat16>() : kernel_ptr<__half>();
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = -1;
    }
    c = n;
    return c;
}

// Cluster size and grouping: the fewest units on the busiest CTA over C = 1..8, with
// every cluster resident at once and at most `segmax` tiles touched per CTA (their
// accumulator chains must fit TMEM beside the A buffers, and their partial sums the
// rings).  False when no C qualifies.
static bool plan(int M, int N, int K, bool bf16, Geometry& g) {
    if (M <= 16 || M > MAXNPAD || K % KT != 0 || N < 1) return false;
    g.Npad = (M + 15) / 16 * 16;
    g.FT = (N + FROWS - 1) / FROWS;
    g.KTN = K / KT;
    rings(g.Npad, g);
    if (g.NW < 4 || g.NX < 2 || g.smem > 227 * 1024 - 1024) return false;
    int segmax = (TMEM_COLS - g.NA * 64) / g.Npad;
    while (segmax > 0 && (long long)segmax * g.Npad * FROWS * 4 > g.smem - 1024) --segmax;
    if (ensure_smem_attr(bf16 ? kernel_ptr<__nv_bfloat16>() : kernel_ptr<__half>(), g.smem, bf16 ? 72 : 73) != SDB_OK)
        return false;
    long long best = -1;
    for (int C = 1; C <= MAXC; ++C) {
        const int gmax = max_clusters(bf16, C, g.smem);
        if (gmax <= 0) continue;
        const int G = g.FT < gmax ? g.FT : gmax;
        const int tmin = g.FT / G, tmax = (g.FT + G - 1) / G;
        if ((long long)tmin * g.KTN < C) continue;  // every CTA gets at least one unit
        const long long u = ((long long)tmax * g.KTN + C - 1) / C;
        long long segs = (u + g.KTN - 1) / g.KTN + 1;
        if (segs > tmax) segs = tmax;
        if (segs > segmax) continue;
        // units on the busiest CTA; a reduction step for C > 1 costs about a fifth of a unit
        const long long cost = 10 * u + (C > 1 ? 2 : 0);
        if (best < 0 || cost < best) {
            best = cost;
            g.C = C;
            g.G = G;
            g.umax = (int)u;
        }
    }
    return best >= 0;
}

}  // namespace w8c

// Taken when a resident cluster plan exists and its busiest CTA carries fewer than 3 units
// more than an even split of all units over the SMs (what the stream-K kernel of
// w8a16_umma.cu gets).  Measured (B200, 32-128 tokens): the cluster kernel is faster on the
// Qwen3-4B qkv, o and down projections (busiest CTA 1-2 units above the even split), the
// stream-K kernel on gate_up (152 feature tiles: 24 units on the busiest CTA against 21),
// by 3-5 us per call either way.
// With require_balance false: whenever a resident cluster plan exists.
bool w8a16_cluster_eligible(int M, int N, int K, int group, int act_dtype, bool require_balance) {
    if (group != 0 || M > w8c::MAXNPAD || K % w8c::KT != 0) return false;
    w8c::Geometry g;
    if (!w8c::plan(M, N, K, act_dtype == SDB_BF16, g)) return false;
    if (!require_balance) return true;
    const long long total = (long long)g.FT * g.KTN;
    const int sms = device_sm_count();
    const long long even = (total + sms - 1) / sms;
    return g.umax - even < 3;
}

int w8a16_cluster_launch(const void* x, int64_t x_srow, const int8_t* w, const void* s, int s_dtype, const void* bias,
                         void* y, int64_t y_srow, int M, int N, int K, int act_dtype, int* err, cudaStream_t st) {
    const bool bf = act_dtype == SDB_BF16;
    w8c::Geometry g;
    if (!w8c::plan(M, N, K, bf, g)) {
        set_last_error("w8a16 cluster kernel: no resident cluster plan for M=%d N=%d K=%d", M, N, K);
        return SDB_ERR_UNSUPPORTED;
    }
    CUtensorMap wm, xm;
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
        cuuint64_t strides[1] = {(cuuint64_t)K};
        cuuint32_t box[2] = {(cuuint32_t)w8c::KT, (cuuint32_t)w8c::FROWS};
        int rc = encode_tensor_map(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w), dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        cuuint64_t strides[1] = {(cuuint64_t)x_srow * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)g.Npad};
        int rc = encode_tensor_map(&xm, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                   const_cast<void*>(x), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    w8c::Params p{};
    p.s = s;
    p.s_dtype = s_dtype;
    p.bias = bias;
    p.y = y;
    p.y_srow = y_srow;
    p.M = M;
    p.N = N;
    p.K = K;
    p.Npad = g.Npad;
    p.FT = g.FT;
    p.KTN = g.KTN;
    p.C = g.C;
    p.G = g.G;
    p.NW = g.NW;
    p.NX = g.NX;
    p.NA = g.NA;
    p.vec_y = (reinterpret_cast<uintptr_t>(y) % 8 == 0 && y_srow % 4 == 0) ? 1 : 0;
    p.err = err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g.G * g.C, 1, 1);
    cfg.blockDim = dim3(w8c::THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = g.C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = bf ? cudaLaunchKernelEx(&cfg, w8c::w8a16_cluster_kernel<__nv_bfloat16>, wm, xm, p)
                       : cudaLaunchKernelEx(&cfg, w8c::w8a16_cluster_kernel<__half>, wm, xm, p);
    return cuda_status(e, "w8a16_cluster_kernel launch");
}

}  // namespace sdb
