// W8A16 linear for the bandwidth-bound range (M <= 64 tokens, per-channel scales):
// y = x @ (q * s)^T (+ bias).
//
// Reference: int8_linear / _int8_dequant_gemm_kernel, nanovllm/layers/quant.py:165-310.
//
// The int8 weights stream through shared memory by TMA: tiles of 128 output features
// x 128 k (16 KB, 128-byte swizzle) together with the matching 128 k of the M token
// rows (bf16/f16, two 64-k boxes, 128-byte swizzle), in a ring of stages filled by one
// producer warp.  Eight consumer warps take 16 features each; per 64-k chunk a lane
// reads 16 contiguous weight bytes of its two rows and 32 contiguous activation bytes
// of its token, i.e. the same k permutation inside the chunk for both operands as the
// register kernel in w8a16.cu (the dot products are unchanged), converts int8 ->
// 16-bit exactly and runs mma.m16n8k16 with the features as the M side.
//
// Work: the (feature tile, k tile) space is split evenly over persistent CTAs, so
// every CTA streams the same number of weight bytes; a feature tile cut by a CTA
// boundary is finished by its last contributor (atomic counter at a fixed workspace
// offset, reset after use), which sums the fp32 partials in slot order.
#include <type_traits>

#include "common.cuh"

namespace sdb {
namespace w8s {

constexpr int FROWS = 128;                 // features per tile
constexpr int KT = 128;                    // k per tile (bytes of int8)
constexpr int WTILE = FROWS * KT;          // 16 KB
constexpr int CONS = 8;                    // consumer warps, 16 features each
constexpr int THREADS = 32 * (CONS + 1);
constexpr int kCounterCap = 65536;         // feature tiles (shared region with w8a16.cu)
constexpr int kSmemBudget = 200 * 1024;

struct Params {
    const void* s;
    int s_dtype;
    const void* bias;
    void* y;
    int64_t y_srow;
    int M, N, K;
    int FT, KTN, slots, grid, NS;
    long long total;
    float* part;    // [FT][slots][M_pad][128]
    int* counters;  // [FT]
    int* err;
};

SDB_DEV long long fstart(const Params& p, int c) { return (long long)c * p.total / p.grid; }
SDB_DEV int fcta(const Params& p, long long f) {
    int c = (int)(f * p.grid / p.total);
    if (c + 1 < p.grid && fstart(p, c + 1) <= f) ++c;
    return c;
}

template <typename T>
SDB_DEV void i8x4_pairs(uint32_t w, uint32_t& lo, uint32_t& hi);
template <>
SDB_DEV void i8x4_pairs<__half>(uint32_t w, uint32_t& lo, uint32_t& hi) {
    // 0x64XX as f16 is 1024 + XX; bias the signed byte by 128 and subtract 1152 (exact)
    const uint32_t u = w ^ 0x80808080u;
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
    lo = *reinterpret_cast<uint32_t*>(&ha);
    hi = *reinterpret_cast<uint32_t*>(&hb);
}
template <>
SDB_DEV void i8x4_pairs<__nv_bfloat16>(uint32_t w, uint32_t& lo, uint32_t& hi) {
    // 0x4B0000XX as f32 is 2^23 + XX; bias by 128, subtract 2^23 + 128 (exact in bf16)
    const uint32_t u = w ^ 0x80808080u;
    uint32_t f0, f1, f2, f3;
    asm("prmt.b32 %0, %1, %2, 0x7540;" : "=r"(f0) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7541;" : "=r"(f1) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7542;" : "=r"(f2) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7543;" : "=r"(f3) : "r"(u), "r"(0x4B000000u));
    const float c = 8388736.0f;
    __nv_bfloat162 pa = __floats2bfloat162_rn(__uint_as_float(f0) - c, __uint_as_float(f1) - c);
    __nv_bfloat162 pb = __floats2bfloat162_rn(__uint_as_float(f2) - c, __uint_as_float(f3) - c);
    lo = *reinterpret_cast<uint32_t*>(&pa);
    hi = *reinterpret_cast<uint32_t*>(&pb);
}

SDB_DEV float scale_at(const Params& p, int n) {
    if (p.s_dtype == SDB_F32) return reinterpret_cast<const float*>(p.s)[n];
    if (p.s_dtype == SDB_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.s)[n]);
    return __half2float(reinterpret_cast<const __half*>(p.s)[n]);
}

// Stage layout: [weights 16 KB][activations k 0..63: M_pad x 128 B][k 64..127: M_pad x 128 B]
template <int NT>
struct Stage {
    static constexpr int XBOX = 8 * NT * 128;
    static constexpr int BYTES = WTILE + 2 * XBOX;
};

template <typename T, int NT>
__global__ void __launch_bounds__(THREADS, 1)
    w8a16_stream_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                        const Params p) {
    using H = Half16<T>;
    using S = Stage<NT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    __shared__ __align__(8) uint64_t bars[2 * 16];
    __shared__ int last_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * 16;
    const int NS = p.NS;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, CONS);
        }
        fence_mbarrier_init();
    }
    __syncthreads();
    const long long f0 = fstart(p, blockIdx.x), f1 = fstart(p, blockIdx.x + 1);

    if (warp == CONS) {
        // ------------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tensormap(&wmap);
            prefetch_tensormap(&xmap);
            const uint64_t wpol = l2_policy_evict_first();
            const uint64_t xpol = l2_policy_evict_normal();  // every feature tile re-reads x
            int g = 0;
            for (long long f = f0; f < f1; ++f, ++g) {
                const int s = g % NS;
                if (g >= NS && !mbar_wait(empty0 + 8 * s, ((g / NS) - 1) & 1)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
                const int ft = (int)(f / p.KTN), kt = (int)(f % p.KTN);
                const uint32_t st = smem_u32(smem + s * S::BYTES);
                const uint32_t fb = full0 + 8 * s;
                mbar_arrive_expect_tx(fb, S::BYTES);
                tma_load_2d(st, &wmap, fb, kt * KT, ft * FROWS, wpol);
                tma_load_2d(st + WTILE, &xmap, fb, kt * KT, 0, xpol);
                tma_load_2d(st + WTILE + S::XBOX, &xmap, fb, kt * KT + 64, 0, xpol);
            }
            for (int q = g - NS > 0 ? g - NS : 0; q < g; ++q)  // own copies land before exit
                if (!mbar_wait(full0 + 8 * (q % NS), (q / NS) & 1)) break;
        }
        return;
    }

    // ----------------------------------------------------------------- consumers
    const int gq = lane >> 2, t = lane & 3;
    bool ok = true;
    float acc[NT][4];
    int g = 0;
    long long f = f0;
    while (f < f1) {
        const int ft = (int)(f / p.KTN), kt0 = (int)(f % p.KTN);
        const int kt1 = (int)min((long long)p.KTN, kt0 + (f1 - f));
#pragma unroll
        for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        for (int kt = kt0; kt < kt1; ++kt, ++g) {
            const int s = g % NS;
            if (ok && !mbar_wait(full0 + 8 * s, (g / NS) & 1)) {
                ok = false;
                if (lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
            }
            const uint8_t* ws = smem + s * S::BYTES;
            const uint8_t* r0 = ws + (warp * 16 + gq) * 128;      // row & 7 == gq for both rows
            const uint8_t* r1 = r0 + 8 * 128;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int ch = ((c * 4 + t) ^ gq) << 4;
                const uint4 wa = *reinterpret_cast<const uint4*>(r0 + ch);
                const uint4 wb = *reinterpret_cast<const uint4*>(r1 + ch);
                uint32_t a[4][4];
                const uint32_t wa32[4] = {wa.x, wa.y, wa.z, wa.w};
                const uint32_t wb32[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    i8x4_pairs<T>(wa32[k], a[k][0], a[k][2]);
                    i8x4_pairs<T>(wb32[k], a[k][1], a[k][3]);
                }
                const uint8_t* xs = ws + WTILE + c * S::XBOX;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int m = nt * 8 + gq;  // token row of the box (m & 7 == gq)
                    const uint4 x0 = *reinterpret_cast<const uint4*>(xs + m * 128 + (((2 * t) ^ gq) << 4));
                    const uint4 x1 = *reinterpret_cast<const uint4*>(xs + m * 128 + (((2 * t + 1) ^ gq) << 4));
                    const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) H::mma(acc[nt], a[k], xw[2 * k], xw[2 * k + 1]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * s);
        }
        // C fragment: acc[nt][0..1] -> feature row gq, tokens nt*8 + 2t (+1); [2..3] -> row gq + 8
        const int nloc0 = warp * 16 + gq;
        const bool whole = kt0 == 0 && kt1 == p.KTN;
        if (!whole) {
            const int c0 = fcta(p, (long long)ft * p.KTN);
            const int nseg = fcta(p, (long long)ft * p.KTN + p.KTN - 1) - c0 + 1;
            const int slot = (int)blockIdx.x - c0;
            float* pt = p.part + ((int64_t)ft * p.slots) * (8 * NT) * FROWS;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int m = nt * 8 + 2 * t + (e & 1);
                    const int nl = nloc0 + (e < 2 ? 0 : 8);
                    __stcg(pt + ((int64_t)slot * (8 * NT) + m) * FROWS + nl, acc[nt][e]);
                }
            __threadfence();
            named_barrier_sync(1, 32 * CONS);
            if (threadIdx.x == 0) last_flag = atomicAdd(p.counters + ft, 1) == nseg - 1;
            named_barrier_sync(1, 32 * CONS);
            const bool last = last_flag;
            if (!last) {
                f += kt1 - kt0;
                continue;
            }
            __threadfence();
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int m = nt * 8 + 2 * t + (e & 1);
                    const int nl = nloc0 + (e < 2 ? 0 : 8);
                    float v = 0.f;
                    for (int s2 = 0; s2 < nseg; ++s2) v += __ldcg(pt + ((int64_t)s2 * (8 * NT) + m) * FROWS + nl);
                    acc[nt][e] = v;
                }
            if (threadIdx.x == 0) p.counters[ft] = 0;
        }
        // epilogue: per-channel scale, bias, round to the activation type
        const int n0 = ft * FROWS + nloc0, n1 = n0 + 8;
        const float sc0 = n0 < p.N ? scale_at(p, n0) : 0.f, sc1 = n1 < p.N ? scale_at(p, n1) : 0.f;
        const T* bias = reinterpret_cast<const T*>(p.bias);
        const float b0 = (bias && n0 < p.N) ? to_f32(bias[n0]) : 0.f;
        const float b1 = (bias && n1 < p.N) ? to_f32(bias[n1]) : 0.f;
        T* y = reinterpret_cast<T*>(p.y);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = nt * 8 + 2 * t + (e & 1);
                const int n = e < 2 ? n0 : n1;
                if (m < p.M && n < p.N)
                    y[(int64_t)m * p.y_srow + n] = from_f32<T>(acc[nt][e] * (e < 2 ? sc0 : sc1) + (e < 2 ? b0 : b1));
            }
        f += kt1 - kt0;
    }
}

// ----------------------------------------------------------------- host
struct Geometry {
    int NT, FT, KTN, grid, slots, NS, smem;
    long long total;
};

static Geometry geometry(int M, int N, int K) {
    Geometry g;
    g.NT = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
    g.FT = (N + FROWS - 1) / FROWS;
    g.KTN = K / KT;
    g.total = (long long)g.FT * g.KTN;
    const int sms = device_sm_count();
    g.grid = (int)(g.total < sms ? g.total : sms);
    const long long m = g.total / g.grid;  // shortest CTA range, >= 1
    long long slots = (g.KTN + m - 1) / m + 1;
    if (slots > g.grid) slots = g.grid;
    g.slots = (int)slots;
    const int stage = WTILE + 2 * 8 * g.NT * 128;
    g.NS = kSmemBudget / stage;
    if (g.NS > 16) g.NS = 16;
    g.smem = g.NS * stage + 1024;
    return g;
}

}  // namespace w8s

// The streaming path takes per-channel scales, 16 < M <= 64 and K % 128 == 0 (for
// M <= 16 the register kernel of w8a16.cu measured faster).
bool w8a16_stream_eligible(int M, int N, int K, int group) {
    return group == 0 && M > 16 && M <= 64 && K % w8s::KT == 0 && N >= 1 &&
           (N + w8s::FROWS - 1) / w8s::FROWS <= w8s::kCounterCap;
}

// Workspace bytes beyond the fixed counter region (at offset 0).
size_t w8a16_stream_partial_bytes(int M, int N, int K) {
    const w8s::Geometry g = w8s::geometry(M, N, K);
    return sizeof(float) * (size_t)g.FT * g.slots * 8 * g.NT * w8s::FROWS;
}

int w8a16_stream_launch(const void* x, int64_t x_srow, const int8_t* w, const void* s, int s_dtype, const void* bias,
                        void* y, int64_t y_srow, int M, int N, int K, int act_dtype, int* counters, float* part,
                        int* err, cudaStream_t st) {
    const w8s::Geometry g = w8s::geometry(M, N, K);
    w8s::Params p{};
    p.s = s;
    p.s_dtype = s_dtype;
    p.bias = bias;
    p.y = y;
    p.y_srow = y_srow;
    p.M = M;
    p.N = N;
    p.K = K;
    p.FT = g.FT;
    p.KTN = g.KTN;
    p.slots = g.slots;
    p.grid = g.grid;
    p.NS = g.NS;
    p.total = g.total;
    p.part = part;
    p.counters = counters;
    p.err = err;
    CUtensorMap wm, xm;
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
        cuuint64_t strides[1] = {(cuuint64_t)K};
        cuuint32_t box[2] = {(cuuint32_t)w8s::KT, (cuuint32_t)w8s::FROWS};
        int rc = encode_tensor_map(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w), dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        const CUtensorMapDataType dt =
            act_dtype == SDB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        cuuint64_t strides[1] = {(cuuint64_t)x_srow * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)(8 * g.NT)};
        int rc = encode_tensor_map(&xm, dt, 2, const_cast<void*>(x), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    int rc = SDB_OK;
#define SDB_W8S(TT, NTV, SLOT)                                                                          \
    do {                                                                                                \
        auto kern = w8s::w8a16_stream_kernel<TT, NTV>;                                                  \
        rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), g.smem, SLOT);                       \
        if (rc) return rc;                                                                              \
        kern<<<g.grid, w8s::THREADS, g.smem, st>>>(wm, xm, p);                                          \
    } while (0)
    const bool bf = act_dtype == SDB_BF16;
    switch (g.NT) {
        case 1: if (bf) SDB_W8S(__nv_bfloat16, 1, 60); else SDB_W8S(__half, 1, 61); break;
        case 2: if (bf) SDB_W8S(__nv_bfloat16, 2, 62); else SDB_W8S(__half, 2, 63); break;
        case 4: if (bf) SDB_W8S(__nv_bfloat16, 4, 64); else SDB_W8S(__half, 4, 65); break;
        default: if (bf) SDB_W8S(__nv_bfloat16, 8, 66); else SDB_W8S(__half, 8, 67); break;
    }
#undef SDB_W8S
    return cuda_status(cudaGetLastError(), "w8a16_stream_kernel launch");
}

}  // namespace sdb
