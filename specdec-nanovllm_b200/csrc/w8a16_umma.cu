// W8A16 linear on the 5th-generation tensor cores (tcgen05): y = x @ (q * s)^T (+ bias)
// with int8 weights q [N, K], per-channel scales s [N], 16-bit activations x [M, K].
//
// Reference: int8_linear / _int8_dequant_gemm_kernel, nanovllm/layers/quant.py:165-310
// (weights dequantised on the fly, fp32 accumulation, scale applied per output channel).
//
// Transposed so the 128-row tensor-core tile is the feature axis:
//   Y^T[128 features, N_pad tokens] += W[128 features, 16 k] . X^T[16 k, N_pad tokens]
// (M = 128, N = tokens padded to a multiple of 16, at most 256 per launch, more tokens in
// balanced blocks, 448 = 2 x 224; K = 16 per instruction).  The accumulator (columns
// 0..N_pad) and the converted A operand (three 64-column buffers from column 256) live in
// TMEM, so shared memory holds only the raw stages: three of 72 KB at 224 tokens.
//
// Per CTA (persistent, one per SM), 320 threads:
//   warp 0      TMA producer: per 128 k, the 128 x 128 int8 weights as one box (16 KB,
//               128-byte swizzle) and the matching 128 k of the token rows (two boxes,
//               128-byte swizzle) into a ring of raw stages
//   warp 1      TMEM owner and MMA issuer (one thread)
//   warps 2..9  converters: two threads per feature row (64 k each, the row being the
//               TMEM lane the warp may access); int8 -> bf16/f16 exactly in registers,
//               stored to the A buffer with one tcgen05.st (A read by the MMA from TMEM);
//               after each segment they read the accumulator back (the two warps of a
//               TMEM lane quarter take alternate 16-token column groups) and write y, or
//               an fp32 partial
// Work: the (feature tile, k tile) space is split evenly over the CTAs; a feature tile
// cut by a CTA boundary leaves one partial per CTA, summed in slot order by
// w8a16_umma_merge_kernel (a programmatic dependent launch).  The main kernel is a
// programmatic dependent launch too: it sets up while the preceding kernel drains and
// waits (griddepcontrol.wait) before its first load and before it writes.  Every wait is
// bounded and reports SDB_KERR_TIMEOUT.
#include <type_traits>

#include "common.cuh"
#include "umma.cuh"
#include "w8a16_convert.cuh"

namespace sdb {
namespace w8u {

constexpr int FROWS = 128;               // features per tile (MMA M)
constexpr int KT = 128;                  // k per tile (one converter hand-off)
constexpr int WBOX = FROWS * 64;         // one 64-k box of int8 weights: 8 KB
constexpr int MAXNA = 3;                 // converted-tile buffers in TMEM (64 columns each)
constexpr int MAXN = 256;                // tokens per launch (larger M: balanced blocks)
constexpr int TMEM_COLS = 512;           // accumulator in columns [0, Npad), A buffers from A_COL
constexpr int A_COL = 256;
constexpr int CONV_THREADS = 256;
constexpr int THREADS = 64 + CONV_THREADS;
constexpr int kSmemBudget = 224 * 1024;
constexpr int MAXNR = 8;
constexpr int MERGE_TOK = 8;  // tokens per merge thread (4 measured equal, 2 slower)

struct Params {
    const void* s;
    int s_dtype;
    const void* bias;
    void* y;
    int64_t y_srow;
    int M, N, K, Npad;
    int KTN, slots, grid, NR, NA, raw_bytes, xbox;
    long long total;
    float* part;  // [FT][slots][Npad][128]
    int* err;
};

SDB_DEV long long fstart(const Params& p, int c) { return (long long)c * p.total / p.grid; }
SDB_DEV int fcta(const Params& p, long long f) {
    int c = (int)(f * p.grid / p.total);
    if (c + 1 < p.grid && fstart(p, c + 1) <= f) ++c;
    return c;
}

SDB_DEV float scale_at(const Params& p, int n) { return w8cv::scale_value(p.s, p.s_dtype, n); }
using w8cv::i8x4;

struct Bars {
    uint32_t rfull0, rempty0, afull0, aempty0, accfull, accempty, fin;
};

// Position in a ring of n slots: slot index and the parity of its current phase.
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
__global__ void __launch_bounds__(THREADS, 1)
    w8a16_umma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t bar_mem[2 * MAXNR + 2 * MAXNA + 3];
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NR = p.NR, NA = p.NA;
    // the partial merge (a programmatic dependent launch) may become resident now; it
    // waits for this grid's completion before reading anything
    asm volatile("griddepcontrol.launch_dependents;");
    Bars bar;
    bar.rfull0 = smem_u32(bar_mem);
    bar.rempty0 = bar.rfull0 + 8 * MAXNR;
    bar.afull0 = bar.rempty0 + 8 * MAXNR;
    bar.aempty0 = bar.afull0 + 8 * MAXNA;
    bar.accfull = bar.aempty0 + 8 * MAXNA;
    bar.accempty = bar.accfull + 8;
    bar.fin = bar.accempty + 8;
    uint8_t* rraw = smem;  // NR raw stages: [W 16 KB][x 2 x Npad x 128 B]
    const uint32_t tcols = TMEM_COLS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NR; ++s) {
            mbar_init(bar.rfull0 + 8 * s, 1);
            mbar_init(bar.rempty0 + 8 * s, 1);
        }
        for (int i = 0; i < NA; ++i) {
            mbar_init(bar.afull0 + 8 * i, CONV_THREADS / 32);
            mbar_init(bar.aempty0 + 8 * i, 1);
        }
        mbar_init(bar.accfull, 1);
        mbar_init(bar.accempty, CONV_THREADS / 32);
        mbar_init(bar.fin, 1);
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), tcols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const int f0 = (int)fstart(p, blockIdx.x), f1 = (int)fstart(p, blockIdx.x + 1);

    if (warp == 0) {
        // ------------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tensormap(&wmap);
            prefetch_tensormap(&xmap);
            pdl_wait();  // the preceding kernel (a PDL launch of this one) has completed
            const uint64_t wpol = l2_policy_evict_first();
            const uint64_t xpol = l2_policy_evict_normal();  // every feature tile re-reads x
            Ring r;
            int issued = 0;
            int ft = f0 / p.KTN, kt = f0 % p.KTN;
            for (int f = f0; f < f1; ++f, ++issued) {
                if (issued >= NR && !mbar_wait(bar.rempty0 + 8 * r.slot, r.phase ^ 1u)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
                const uint32_t st = smem_u32(rraw + r.slot * p.raw_bytes);
                const uint32_t fb = bar.rfull0 + 8 * r.slot;
                mbar_arrive_expect_tx(fb, (uint32_t)p.raw_bytes);
                tma_load_2d(st, &wmap, fb, kt * KT, ft * FROWS, wpol);
                tma_load_2d(st + 2 * WBOX, &xmap, fb, kt * KT, 0, xpol);
                tma_load_2d(st + 2 * WBOX + p.xbox, &xmap, fb, kt * KT + 64, 0, xpol);
                r.next(NR);
                if (++kt == p.KTN) {
                    kt = 0;
                    ++ft;
                }
            }
            // own copies land before exit: the last min(issued, NR) fills
            Ring d;
            for (int q = 0; q < issued; ++q) {
                if (q >= issued - NR && !mbar_wait(bar.rfull0 + 8 * d.slot, d.phase)) break;
                d.next(NR);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            const uint32_t idesc = idesc_f16(BF, false, false, FROWS, p.Npad);
            bool ok = true;
            Ring r, a;
            uint32_t accph = 0;
            int seg = 0;
            int f = f0;
            while (f < f1 && ok) {
                const int kt0 = f % p.KTN;
                const int kt1 = min(p.KTN, kt0 + (f1 - f));
                // the accumulator of the previous segment has been read back
                if (seg >= 1 && !mbar_wait(bar.accempty, accph)) {
                    ok = false;
                    break;
                }
                if (seg >= 1) accph ^= 1u;
                tc_fence_after();
                for (int kt = kt0; kt < kt1; ++kt) {
                    if (!mbar_wait(bar.rfull0 + 8 * r.slot, r.phase) || !mbar_wait(bar.afull0 + 8 * a.slot, a.phase)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t abase = tmem + (uint32_t)(A_COL + a.slot * 64);
                    const uint32_t xbase = smem_u32(rraw + r.slot * p.raw_bytes + 2 * WBOX);
#pragma unroll
                    for (int ks = 0; ks < KT / 16; ++ks) {
                        const uint64_t bd = sdesc_sw128(xbase + (ks >> 2) * p.xbox + (ks & 3) * 32, 16, 1024);
                        umma_f16_ts(tmem, abase + 8 * ks, bd, idesc, (kt == kt0 && ks == 0) ? 0u : 1u);
                    }
                    umma_commit(bar.aempty0 + 8 * a.slot);  // converted tile consumed
                    umma_commit(bar.rempty0 + 8 * r.slot);  // token tile consumed
                    r.next(NR);
                    a.next(NA);
                }
                if (!ok) break;
                umma_commit(bar.accfull);
                f += kt1 - kt0;
                ++seg;
            }
            if (!ok) atomicOr(p.err, SDB_KERR_TIMEOUT);
            // every MMA this thread issued has completed before TMEM is released
            umma_commit(bar.fin);
            if (!mbar_wait(bar.fin, 0)) atomicOr(p.err, SDB_KERR_TIMEOUT);
        }
    } else {
        // ------------------------------------------------------------- converters / epilogue
        pdl_wait();  // y and the partials may still be read by the preceding kernel
        const int q = warp & 3;           // TMEM lane quarter of this warp
        const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
        const int row_epi = 32 * q + lane;  // feature row this thread converts and reads back
        const int cr = row_epi;
        const int kh = (warp - 2) >> 2;   // which 64 k of the tile this thread converts
        const int sw = cr & 7;
        bool ok = true;
        Ring r, a;
        int ga = 0;  // converted tiles so far
        uint32_t accph = 0;
        int f = f0;
        while (f < f1) {
            const int ft = f / p.KTN, kt0 = f % p.KTN;
            const int kt1 = min(p.KTN, kt0 + (f1 - f));
            for (int kt = kt0; kt < kt1; ++kt, ++ga) {
                if (ok && !mbar_wait(bar.rfull0 + 8 * r.slot, r.phase)) ok = false;
                if (ok && ga >= NA && !mbar_wait(bar.aempty0 + 8 * a.slot, a.phase ^ 1u)) ok = false;
                // raw row cr: 128 B, 16-byte chunk j (k 16j .. 16j+15) at j ^ (cr & 7); the
                // 64 converted k of half kh go to TMEM lane cr, 32 columns from A_COL + 64 slot + 32 kh
                const uint8_t* wr = rraw + r.slot * p.raw_bytes + cr * 128;
                uint4 v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) v[j] = *reinterpret_cast<const uint4*>(wr + (((4 * kh + j) ^ sw) << 4));
                uint32_t o[32];
#pragma unroll
                for (int j = 0; j < 4; ++j) {  // k 16j .. 16j+15 of this half
                    i8x4<T>(v[j].x, o[8 * j + 0], o[8 * j + 1]);
                    i8x4<T>(v[j].y, o[8 * j + 2], o[8 * j + 3]);
                    i8x4<T>(v[j].z, o[8 * j + 4], o[8 * j + 5]);
                    i8x4<T>(v[j].w, o[8 * j + 6], o[8 * j + 7]);
                }
                tc_fence_after();
                tmem_st32(tmem + lane_addr + (uint32_t)(A_COL + a.slot * 64 + 32 * kh), o);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar.afull0 + 8 * a.slot);
                r.next(NR);
                a.next(NA);
            }
            // ---- segment epilogue: tokens are TMEM columns, this thread's feature is a lane
            if (ok && !mbar_wait(bar.accfull, accph)) ok = false;
            accph ^= 1u;
            tc_fence_after();
            const int n = ft * FROWS + row_epi;
            const bool whole = kt0 == 0 && kt1 == p.KTN;
            const float sc = n < p.N ? scale_at(p, n) : 0.f;
            const T* bias = reinterpret_cast<const T*>(p.bias);
            const float bn = (bias && n < p.N) ? to_f32(bias[n]) : 0.f;
            T* y = reinterpret_cast<T*>(p.y);
            float* pt = nullptr;
            if (!whole) {
                const int slot = (int)blockIdx.x - fcta(p, (long long)ft * p.KTN);
                pt = p.part + ((int64_t)ft * p.slots + slot) * p.Npad * FROWS;
            }
            for (int mc = 16 * kh; mc < p.Npad; mc += 32) {  // this warp's column groups
                uint32_t rr[16];
                tmem_ld16(tmem + lane_addr + mc, rr);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int m = mc + i;
                    const float v = __uint_as_float(rr[i]);
                    if (whole) {
                        if (m < p.M && n < p.N) y[(int64_t)m * p.y_srow + n] = from_f32<T>(v * sc + bn);
                    } else {
                        __stcg(pt + (int64_t)m * FROWS + row_epi, v);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar.accempty);  // the MMA may overwrite the accumulator
            f += kt1 - kt0;
        }
        if (!ok && lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
    }
    __syncwarp();  // warps reconverge (role lanes and idle lanes) before the block barrier
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, tcols);
}

// Sums the partials of the feature tiles that a CTA boundary cut (slot order, so the
// result does not depend on timing), then scale and bias.  grid (feature tiles, token
// groups of MERGE_TOK), 128 threads = the tile's features.
template <typename T>
__global__ void __launch_bounds__(FROWS) w8a16_umma_merge_kernel(const Params p) {
    pdl_launch_dependents();  // the next call may set up; it waits for this grid itself
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int ft = blockIdx.x;
    const long long a = (long long)ft * p.KTN;
    const int c0 = fcta(p, a);
    const int nseg = fcta(p, a + p.KTN - 1) - c0 + 1;
    if (nseg == 1) return;  // one CTA held the whole tile and wrote y itself
    const int n = ft * FROWS + threadIdx.x;
    if (n >= p.N) return;
    const float sc = scale_at(p, n);
    const T* bias = reinterpret_cast<const T*>(p.bias);
    const float bn = bias ? to_f32(bias[n]) : 0.f;
    const float* pt = p.part + (int64_t)ft * p.slots * p.Npad * FROWS + threadIdx.x;
    const int m0 = blockIdx.y * MERGE_TOK;
    float v[MERGE_TOK];
#pragma unroll
    for (int i = 0; i < MERGE_TOK; ++i) v[i] = 0.f;
    for (int s2 = 0; s2 < nseg; ++s2)
#pragma unroll
        for (int i = 0; i < MERGE_TOK; ++i)
            if (m0 + i < p.M) v[i] += __ldcg(pt + ((int64_t)s2 * p.Npad + m0 + i) * FROWS);
    T* y = reinterpret_cast<T*>(p.y);
#pragma unroll
    for (int i = 0; i < MERGE_TOK; ++i)
        if (m0 + i < p.M) y[(int64_t)(m0 + i) * p.y_srow + n] = from_f32<T>(v[i] * sc + bn);
}

struct Geometry {
    int Npad, FT, KTN, grid, slots, NR, NA, raw_bytes, xbox, smem;
    long long total;
};

static Geometry geometry(int Mblk, int N, int K) {
    Geometry g;
    g.Npad = (Mblk + 15) / 16 * 16;
    g.FT = (N + FROWS - 1) / FROWS;
    g.KTN = K / KT;
    g.total = (long long)g.FT * g.KTN;
    const int sms = device_sm_count();
    g.grid = (int)(g.total < sms ? g.total : sms);
    const long long m = g.total / g.grid;
    long long slots = (g.KTN + m - 1) / m + 1;
    if (slots > g.grid) slots = g.grid;
    g.slots = (int)slots;
    g.xbox = g.Npad * 128;
    g.raw_bytes = 2 * WBOX + 2 * g.xbox;  // multiple of 1024: Npad % 16 == 0
    g.NA = MAXNA;
    g.NR = kSmemBudget / g.raw_bytes;
    if (g.NR > MAXNR) g.NR = MAXNR;
    g.smem = g.NR * g.raw_bytes + 1024;
    return g;
}

}  // namespace w8u

// tcgen05 path: per-channel scales, K % 128 == 0; tokens are processed in blocks of 256.
// (M <= 16 goes to the register kernel of w8a16.cu, measured faster there.)
bool w8a16_umma_eligible(int M, int N, int K, int group) {
    return group == 0 && M > 16 && N >= 1 && K % w8u::KT == 0 &&
           (long long)((N + w8u::FROWS - 1) / w8u::FROWS) * (K / w8u::KT) < (1LL << 31);
}

size_t w8a16_umma_partial_bytes(int M, int N, int K) {
    const w8u::Geometry g = w8u::geometry(M < w8u::MAXN ? M : w8u::MAXN, N, K);
    return sizeof(float) * (size_t)g.FT * g.slots * g.Npad * w8u::FROWS;
}

int w8a16_umma_launch(const void* x, int64_t x_srow, const int8_t* w, const void* s, int s_dtype, const void* bias,
                      void* y, int64_t y_srow, int M, int N, int K, int act_dtype, float* part, int* err,
                      cudaStream_t st) {
    const int esz = 2;
    CUtensorMap wm;
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
        cuuint64_t strides[1] = {(cuuint64_t)K};
        cuuint32_t box[2] = {(cuuint32_t)w8u::KT, (cuuint32_t)w8u::FROWS};  // 128 k x 128 rows, full 128-B rows
        int rc = encode_tensor_map(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w), dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    const CUtensorMapDataType dt = act_dtype == SDB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    // balanced token blocks of at most MAXN (448 -> 2 x 224: three raw stages fit at 224
    // tokens, two at 256); they share the partial region in turn
    const int nblk = (M + w8u::MAXN - 1) / w8u::MAXN;
    const int Mblk = (M + nblk - 1) / nblk;
    for (int m0 = 0; m0 < M; m0 += Mblk) {
        const int Mb = M - m0 < Mblk ? M - m0 : Mblk;
        const w8u::Geometry g = w8u::geometry(Mb, N, K);
        CUtensorMap xm;
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)Mb};
        cuuint64_t strides[1] = {(cuuint64_t)x_srow * esz};
        cuuint32_t box[2] = {64, (cuuint32_t)g.Npad};
        const uint8_t* xb = reinterpret_cast<const uint8_t*>(x) + (int64_t)m0 * x_srow * esz;
        int rc = encode_tensor_map(&xm, dt, 2, const_cast<uint8_t*>(xb), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        w8u::Params p{};
        p.s = s;
        p.s_dtype = s_dtype;
        p.bias = bias;
        p.y = reinterpret_cast<uint8_t*>(y) + (int64_t)m0 * y_srow * esz;
        p.y_srow = y_srow;
        p.M = Mb;
        p.N = N;
        p.K = K;
        p.Npad = g.Npad;
        p.KTN = g.KTN;
        p.slots = g.slots;
        p.grid = g.grid;
        p.NR = g.NR;
        p.NA = g.NA;
        p.raw_bytes = g.raw_bytes;
        p.xbox = g.xbox;
        p.total = g.total;
        p.part = part;
        p.err = err;
        cudaLaunchConfig_t mcfg = {};
        mcfg.gridDim = dim3(g.grid, 1, 1);
        mcfg.blockDim = dim3(w8u::THREADS, 1, 1);
        mcfg.dynamicSmemBytes = (size_t)g.smem;
        mcfg.stream = st;
        cudaLaunchAttribute mattr[1];
        mattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        mattr[0].val.programmaticStreamSerializationAllowed = 1;
        mcfg.attrs = mattr;
        mcfg.numAttrs = 1;
        cudaError_t me;
        if (act_dtype == SDB_BF16) {
            auto kern = w8u::w8a16_umma_kernel<__nv_bfloat16>;
            rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), g.smem, 70);
            if (rc) return rc;
            me = cudaLaunchKernelEx(&mcfg, kern, wm, xm, p);
        } else {
            auto kern = w8u::w8a16_umma_kernel<__half>;
            rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), g.smem, 71);
            if (rc) return rc;
            me = cudaLaunchKernelEx(&mcfg, kern, wm, xm, p);
        }
        rc = cuda_status(me, "w8a16_umma_kernel launch");
        if (rc) return rc;
        if (g.grid > 1) {  // some feature tile may be cut by a CTA boundary
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(g.FT, (Mb + w8u::MERGE_TOK - 1) / w8u::MERGE_TOK, 1);
            cfg.blockDim = dim3(w8u::FROWS, 1, 1);
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaError_t e = act_dtype == SDB_BF16 ? cudaLaunchKernelEx(&cfg, w8u::w8a16_umma_merge_kernel<__nv_bfloat16>, p)
                                                  : cudaLaunchKernelEx(&cfg, w8u::w8a16_umma_merge_kernel<__half>, p);
            rc = cuda_status(e, "w8a16_umma_merge_kernel launch");
            if (rc) return rc;
        }
    }
    return SDB_OK;
}

}  // namespace sdb
