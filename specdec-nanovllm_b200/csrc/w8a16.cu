// W8A16 linear on B200 (sm_100a): y = x @ (q * s)^T (+ bias), int8 weights
// dequantised in registers.
//
// Reference: int8_linear / _int8_dequant_gemm_kernel / _splitk_reduce_kernel,
// nanovllm/layers/quant.py:165-310 (Triton, W read as [BN, BK] k-contiguous,
// dequant in registers, fp32 accumulate, split-K partials + reduce for M <= 64).
//
// This kernel swaps the operands of mma.m16n8k16: the 16 output features of a
// warp are the M side (A = W rows, converted int8 -> 16-bit exactly: |q| <= 127),
// eight tokens are the N side (B = x^T), so a decode step (M = 1..8 tokens) wastes
// no weight bandwidth on padding.  Inside each 64-wide k chunk the k order is
// permuted so that a lane's A and B fragments for four consecutive k16 steps are
// one contiguous 16-byte load of W and one 32-byte load of x (the permutation is
// applied identically to both operands, so the dot products are unchanged).
// Per-channel scales (and bias) are applied once in the epilogue; per-group
// scales are applied to each group's fp32 partial sum.  Split-K partials go to
// the caller's workspace and the last CTA of an output tile (atomic counter,
// reset after use) sums them in a fixed order.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "common.cuh"

namespace sdb {
namespace w8 {

constexpr int WARPS = 4;
constexpr int FEAT = WARPS * 16;  // output features per CTA
constexpr int KC = 64;            // k chunk
constexpr int UNROLL = 4;         // chunks whose W loads are in flight together

struct Params {
    const void* x;
    int64_t x_srow;
    const int8_t* w;
    const void* s;
    int s_dtype, group;  // group 0: per channel
    const void* bias;
    void* y;
    int64_t y_srow;
    int M, N, K, SK, chunks_per_split;
    float* part;   // [SK][M][N]
    int* counters; // [ntile_n * ntile_m]
};

// int8x4 -> two packed 16-bit pairs (bytes 0,1 and bytes 2,3), exact.
template <typename T>
SDB_DEV void i8x4_to_pairs(uint32_t w, uint32_t& lo, uint32_t& hi);

template <>
SDB_DEV void i8x4_to_pairs<__half>(uint32_t w, uint32_t& lo, uint32_t& hi) {
    // 0x64XX as f16 is 1024 + XX; bias the signed byte by 128 and subtract 1152.
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
SDB_DEV void i8x4_to_pairs<__nv_bfloat16>(uint32_t w, uint32_t& lo, uint32_t& hi) {
    // 0x4B0000XX as f32 is 2^23 + XX; bias by 128, subtract 2^23 + 128, pack to bf16 (exact).
    const uint32_t u = w ^ 0x80808080u;
    uint32_t f0, f1, f2, f3;
    asm("prmt.b32 %0, %1, %2, 0x7540;" : "=r"(f0) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7541;" : "=r"(f1) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7542;" : "=r"(f2) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7543;" : "=r"(f3) : "r"(u), "r"(0x4B000000u));
    const float c = 8388736.0f;
    const float v0 = __uint_as_float(f0) - c, v1 = __uint_as_float(f1) - c;
    const float v2 = __uint_as_float(f2) - c, v3 = __uint_as_float(f3) - c;
    __nv_bfloat162 pa = __floats2bfloat162_rn(v0, v1);
    __nv_bfloat162 pb = __floats2bfloat162_rn(v2, v3);
    lo = *reinterpret_cast<uint32_t*>(&pa);
    hi = *reinterpret_cast<uint32_t*>(&pb);
}

SDB_DEV float load_scale(const void* s, int dt, int64_t i) {
    if (dt == SDB_F32) return reinterpret_cast<const float*>(s)[i];
    if (dt == SDB_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(s)[i]);
    return __half2float(reinterpret_cast<const __half*>(s)[i]);
}

template <typename T, int NT, bool GROUPED>
__global__ void __launch_bounds__(WARPS * 32) w8a16_kernel(const Params p) {
    using H = Half16<T>;
    __shared__ int last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * FEAT + warp * 16;
    const int m0 = blockIdx.y * (8 * NT);
    const int sk = blockIdx.z;
    const int nchunks = p.K / KC;
    const int c0 = sk * p.chunks_per_split;
    const int c1 = min(c0 + p.chunks_per_split, nchunks);

    const int row0 = n0 + g, row1 = n0 + g + 8;
    const bool ok0 = row0 < p.N, ok1 = row1 < p.N;
    const int8_t* w0 = p.w + (int64_t)(ok0 ? row0 : 0) * p.K + t * 16;
    const int8_t* w1 = p.w + (int64_t)(ok1 ? row1 : 0) * p.K + t * 16;
    const T* xb = reinterpret_cast<const T*>(p.x);

    float acc[NT][4];
    float gacc[GROUPED ? NT : 1][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    if (GROUPED) {
#pragma unroll
        for (int i = 0; i < (GROUPED ? NT : 1); ++i) gacc[i][0] = gacc[i][1] = gacc[i][2] = gacc[i][3] = 0.f;
    }
    const int gchunks = GROUPED ? p.group / KC : 1;

    for (int cb = c0; cb < c1; cb += UNROLL) {
        uint4 wa[UNROLL], wb[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int c = cb + u;
            if (c < c1) {
                wa[u] = ok0 ? __ldcs(reinterpret_cast<const uint4*>(w0 + c * KC)) : make_uint4(0, 0, 0, 0);
                wb[u] = ok1 ? __ldcs(reinterpret_cast<const uint4*>(w1 + c * KC)) : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int c = cb + u;
            if (c >= c1) break;
            uint32_t a[4][4];
            const uint32_t wa32[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
            const uint32_t wb32[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                i8x4_to_pairs<T>(wa32[s], a[s][0], a[s][2]);
                i8x4_to_pairs<T>(wb32[s], a[s][1], a[s][3]);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m = m0 + nt * 8 + g;
                uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
                if (m < p.M) {
                    const uint4* xp = reinterpret_cast<const uint4*>(xb + (int64_t)m * p.x_srow + c * KC + t * 16);
                    x0 = __ldg(xp);
                    x1 = __ldg(xp + 1);
                }
                const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                float* dst = GROUPED ? gacc[GROUPED ? nt : 0] : acc[nt];
#pragma unroll
                for (int s = 0; s < 4; ++s) H::mma(dst, a[s], xw[2 * s], xw[2 * s + 1]);
            }
            if (GROUPED && (((c + 1) % gchunks) == 0 || c + 1 == c1)) {
                const int grp = c / gchunks;
                const int ng = p.K / p.group;
                const float s0 = ok0 ? load_scale(p.s, p.s_dtype, (int64_t)row0 * ng + grp) : 0.f;
                const float s1 = ok1 ? load_scale(p.s, p.s_dtype, (int64_t)row1 * ng + grp) : 0.f;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    acc[nt][0] += gacc[GROUPED ? nt : 0][0] * s0;
                    acc[nt][1] += gacc[GROUPED ? nt : 0][1] * s0;
                    acc[nt][2] += gacc[GROUPED ? nt : 0][2] * s1;
                    acc[nt][3] += gacc[GROUPED ? nt : 0][3] * s1;
                    gacc[GROUPED ? nt : 0][0] = gacc[GROUPED ? nt : 0][1] = 0.f;
                    gacc[GROUPED ? nt : 0][2] = gacc[GROUPED ? nt : 0][3] = 0.f;
                }
            }
        }
    }

    // C fragment: acc[nt][0..1] -> feature row0, tokens m0 + nt*8 + 2t (+1); [2..3] -> row1.
    if (p.SK > 1) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = m0 + nt * 8 + 2 * t + (e & 1);
                const int n = e < 2 ? row0 : row1;
                if (m < p.M && n < p.N) __stcg(p.part + ((int64_t)sk * p.M + m) * p.N + n, acc[nt][e]);
            }
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = atomicAdd(p.counters + blockIdx.y * gridDim.x + blockIdx.x, 1) == p.SK - 1;
        __syncthreads();
        if (!last) return;
        __threadfence();
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = m0 + nt * 8 + 2 * t + (e & 1);
                const int n = e < 2 ? row0 : row1;
                float v = 0.f;
                if (m < p.M && n < p.N)
                    for (int s2 = 0; s2 < p.SK; ++s2) v += __ldcg(p.part + ((int64_t)s2 * p.M + m) * p.N + n);
                acc[nt][e] = v;
            }
        }
        if (threadIdx.x == 0) p.counters[blockIdx.y * gridDim.x + blockIdx.x] = 0;
    }

    // epilogue: per-channel scale, bias, round to the activation type
    const float sc0 = (!GROUPED && ok0) ? load_scale(p.s, p.s_dtype, row0) : 1.f;
    const float sc1 = (!GROUPED && ok1) ? load_scale(p.s, p.s_dtype, row1) : 1.f;
    const T* bias = reinterpret_cast<const T*>(p.bias);
    const float b0 = (bias && ok0) ? to_f32(bias[row0]) : 0.f;
    const float b1 = (bias && ok1) ? to_f32(bias[row1]) : 0.f;
    T* y = reinterpret_cast<T*>(p.y);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int m = m0 + nt * 8 + 2 * t + (e & 1);
            const bool first = e < 2;
            const int n = first ? row0 : row1;
            if (m < p.M && n < p.N) {
                const float v = acc[nt][e] * (first ? sc0 : sc1) + (first ? b0 : b1);
                y[(int64_t)m * p.y_srow + n] = from_f32<T>(v);
            }
        }
    }
}

// quantize_weight (quant.py:123-148): one CTA per (group, row); scale =
// max(amax/127, 1e-8) in f32, q = clamp(rint(w / scale), -127, 127), the stored
// scale rounded once to the scale dtype.
template <typename TW>
__global__ void __launch_bounds__(128) quantize_kernel(const TW* w, int8_t* q, void* s, int s_dtype, int K, int G) {
    __shared__ float red[4];
    const int grp = blockIdx.x, n = blockIdx.y;
    const TW* src = w + (int64_t)n * K + (int64_t)grp * G;
    float amax = 0.f;
    for (int i = threadIdx.x; i < G; i += 128) amax = fmaxf(amax, fabsf(to_f32(src[i])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    int8_t* dst = q + (int64_t)n * K + (int64_t)grp * G;
    for (int i = threadIdx.x; i < G; i += 128) {
        int v = __float2int_rn(__fdiv_rn(to_f32(src[i]), scale));
        v = v > 127 ? 127 : (v < -127 ? -127 : v);
        dst[i] = (int8_t)v;
    }
    if (threadIdx.x == 0) {
        const int64_t idx = (int64_t)n * gridDim.x + grp;
        if (s_dtype == SDB_F32) reinterpret_cast<float*>(s)[idx] = scale;
        else if (s_dtype == SDB_BF16) reinterpret_cast<__nv_bfloat16*>(s)[idx] = __float2bfloat16_rn(scale);
        else reinterpret_cast<__half*>(s)[idx] = __float2half_rn(scale);
    }
}

struct Plan {
    int NT, mt, nt_n, SK, cps;
};

static Plan plan(int M, int N, int K) {
    Plan pl;
    pl.NT = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
    pl.mt = (M + 8 * pl.NT - 1) / (8 * pl.NT);
    pl.nt_n = (N + FEAT - 1) / FEAT;
    const int nchunks = K / KC;
    const long long ctas = (long long)pl.mt * pl.nt_n;
    const long long target = (long long)device_sm_count() * 4;
    int sk = (int)((target + ctas - 1) / ctas);
    if (sk > nchunks / 2) sk = nchunks / 2;
    if (sk < 1) sk = 1;
    pl.cps = (nchunks + sk - 1) / sk;
    pl.SK = (nchunks + pl.cps - 1) / pl.cps;
    return pl;
}

struct WsLayout {
    size_t counters, part, total;
};

}  // namespace w8

bool w8a16_umma_eligible(int M, int N, int K, int group);
size_t w8a16_umma_partial_bytes(int M, int N, int K);
int w8a16_umma_launch(const void* x, int64_t x_srow, const int8_t* w, const void* s, int s_dtype, const void* bias,
                      void* y, int64_t y_srow, int M, int N, int K, int act_dtype, float* part, int* err,
                      cudaStream_t st);
bool w8a16_cluster_eligible(int M, int N, int K, int group, int act_dtype, bool require_balance);
bool w8a16_gemv_eligible(int M, int N, int K, int group);
int w8a16_gemv_launch(const void* x, int64_t x_srow, const int8_t* w, const void* s, int s_dtype, const void* bias,
                      void* y, int64_t y_srow, int M, int N, int K, int act_dtype, cudaStream_t st);
int w8a16_cluster_launch(const void* x, int64_t x_srow, const int8_t* w, const void* s, int s_dtype, const void* bias,
                         void* y, int64_t y_srow, int M, int N, int K, int act_dtype, int* err, cudaStream_t st);

namespace w8 {

// Split-K counters at a fixed offset with a fixed capacity: one workspace serves
// calls of any shape in any order (counters are never aliased by partials and
// every call leaves them at 0).
constexpr int kCounterCap = 65536;  // output tiles

// Workspace layout shared by the three kernels: split-K counters (register kernel) at a
// fixed offset with a fixed capacity, then the error word of the tcgen05 kernels (bounded
// waits report there), then the split-K partials of whichever kernel runs.  Nothing but
// the tcgen05 kernels' timeouts writes the error word.
constexpr size_t kUmmaErrOffset = 256 * 1024;  // == align_up(4 * kCounterCap, 256)
constexpr size_t kUmmaPartOffset = kUmmaErrOffset + 256;

static WsLayout ws_layout(int M, int N, int K) {
    Plan pl = plan(M, N, K);
    WsLayout w;
    w.counters = 0;
    size_t off = kUmmaPartOffset;
    w.part = off;
    if (pl.SK > 1) off = align_up(off + sizeof(float) * (size_t)pl.SK * M * N, 256);
    w.total = off;
    return w;
}

static size_t umma_ws_bytes(int M, int N, int K) {
    return align_up(kUmmaPartOffset + w8a16_umma_partial_bytes(M, N, K), 256);
}

// Kernel choice (per-channel scales, K % 128 == 0): for 17 to 128 tokens the cluster
// split-K tcgen05 kernel (w8a16_cluster.cu) unless its plan leaves the busiest CTA 3 or
// more units above an even split (then the stream-K kernel, w8a16_umma.cu); the stream-K
// kernel above 128 tokens.  Up to 16 tokens the weight-stream kernel (w8a16_gemv.cu) for
// the shapes whose token rows fit its shared memory, at 13-16 tokens only up to 8192
// features (above that the register kernel measured faster: gate_up at 16 tokens 25.4
// against 28.8 us); the register kernel for the other shapes up to 16 tokens and for
// grouped scales.
// SDB_W8A16_KERNEL=cluster takes the cluster kernel wherever it has a plan, =umma skips it,
// =mma forces the register kernel, =gemv takes the weight-stream kernel wherever it has a
// plan (read per call: tests switch it).
enum class Kern { Cluster, Umma, Mma, Gemv };
static Kern choose(int M, int N, int K, int group, int act_dtype, const void* w) {
    const char* e = getenv("SDB_W8A16_KERNEL");
    if (e && !strcmp(e, "mma")) return Kern::Mma;
    const bool w32 = (reinterpret_cast<uintptr_t>(w) & 31) == 0;  // 256-bit weight loads
    const bool gemv_ok = w32 && w8a16_gemv_eligible(M, N, K, group);
    if (e && !strcmp(e, "gemv") && gemv_ok) return Kern::Gemv;
    if (!e && gemv_ok && (M <= 12 || N <= 8192)) return Kern::Gemv;
    const bool no_cluster = e && !strcmp(e, "umma");
    const bool any_cluster = e && !strcmp(e, "cluster");
    if (!no_cluster && w8a16_cluster_eligible(M, N, K, group, act_dtype, !any_cluster)) return Kern::Cluster;
    if (w8a16_umma_eligible(M, N, K, group)) return Kern::Umma;
    return Kern::Mma;
}

template <typename T>
static int launch(const Params& p, const Plan& pl, cudaStream_t st, bool grouped) {
    dim3 grid(pl.nt_n, pl.mt, pl.SK);
#define SDB_W8(NT)                                                                               \
    do {                                                                                         \
        if (grouped) w8a16_kernel<T, NT, true><<<grid, WARPS * 32, 0, st>>>(p);                  \
        else w8a16_kernel<T, NT, false><<<grid, WARPS * 32, 0, st>>>(p);                         \
    } while (0)
    switch (pl.NT) {
        case 1: SDB_W8(1); break;
        case 2: SDB_W8(2); break;
        case 4: SDB_W8(4); break;
        default: SDB_W8(8); break;
    }
#undef SDB_W8
    return cuda_status(cudaGetLastError(), "w8a16_kernel launch");
}

}  // namespace w8
}  // namespace sdb

using namespace sdb;

extern "C" size_t sdb_w8a16_workspace_size(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0 || K % w8::KC) return 256;
    size_t total = w8::ws_layout(M, N, K).total;
    if (w8a16_umma_eligible(M, N, K, 0)) {
        const size_t s = w8::umma_ws_bytes(M, N, K);
        if (s > total) total = s;
    }
    return total;
}

extern "C" int sdb_w8a16_linear(const void* x, int64_t x_srow, const int8_t* qweight, const void* scale,
                                int scale_dtype, int group_size, const void* bias, void* y, int64_t y_srow, int M,
                                int N, int K, int act_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    if (!x || !qweight || !scale || !y || !workspace) {
        set_last_error("null pointer argument");
        return SDB_ERR_INVALID_ARG;
    }
    if (M <= 0 || N <= 0 || K <= 0 || x_srow < K || y_srow < N) {
        set_last_error("bad sizes M=%d N=%d K=%d", M, N, K);
        return SDB_ERR_INVALID_ARG;
    }
    if (K % w8::KC != 0 || (group_size != 0 && (group_size % w8::KC != 0 || K % group_size != 0))) {
        set_last_error("need K %% 64 == 0 and group_size 0 or a multiple of 64 dividing K");
        return SDB_ERR_UNSUPPORTED;
    }
    if (act_dtype != SDB_BF16 && act_dtype != SDB_F16) {
        set_last_error("activations must be bf16 or f16");
        return SDB_ERR_UNSUPPORTED;
    }
    if (scale_dtype != SDB_F32 && scale_dtype != SDB_BF16 && scale_dtype != SDB_F16) {
        set_last_error("scale dtype must be f32, bf16 or f16");
        return SDB_ERR_UNSUPPORTED;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (x_srow % 8) || (reinterpret_cast<uintptr_t>(qweight) & 15) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255)) {
        set_last_error("x and qweight must be 16-byte aligned with x row stride %% 8 == 0; workspace 256-aligned");
        return SDB_ERR_INVALID_ARG;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const w8::Kern kern = w8::choose(M, N, K, group_size, act_dtype, qweight);
    if (kern == w8::Kern::Gemv)
        return w8a16_gemv_launch(x, x_srow, qweight, scale, scale_dtype, bias, y, y_srow, M, N, K, act_dtype, st);
    if (kern == w8::Kern::Cluster) {
        if (workspace_bytes < w8::kUmmaPartOffset) {
            set_last_error("workspace too small: need %zu bytes, got %zu", w8::kUmmaPartOffset, workspace_bytes);
            return SDB_ERR_WORKSPACE;
        }
        return w8a16_cluster_launch(x, x_srow, qweight, scale, scale_dtype, bias, y, y_srow, M, N, K, act_dtype,
                                    reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) + w8::kUmmaErrOffset),
                                    st);
    }
    if (kern == w8::Kern::Umma) {
        const size_t need = w8::umma_ws_bytes(M, N, K);
        if (workspace_bytes < need) {
            set_last_error("workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
            return SDB_ERR_WORKSPACE;
        }
        uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
        return w8a16_umma_launch(x, x_srow, qweight, scale, scale_dtype, bias, y, y_srow, M, N, K, act_dtype,
                                 reinterpret_cast<float*>(ws + w8::kUmmaPartOffset),
                                 reinterpret_cast<int*>(ws + w8::kUmmaErrOffset), st);
    }
    w8::WsLayout wl = w8::ws_layout(M, N, K);
    if (workspace_bytes < wl.total) {
        set_last_error("workspace too small: need %zu bytes, got %zu", wl.total, workspace_bytes);
        return SDB_ERR_WORKSPACE;
    }
    w8::Plan pl = w8::plan(M, N, K);
    if ((long long)pl.mt * pl.nt_n > w8::kCounterCap) {
        set_last_error("M x N too large: %d output tiles (max %d)", pl.mt * pl.nt_n, w8::kCounterCap);
        return SDB_ERR_UNSUPPORTED;
    }
    w8::Params p{};
    p.x = x;
    p.x_srow = x_srow;
    p.w = qweight;
    p.s = scale;
    p.s_dtype = scale_dtype;
    p.group = group_size;
    p.bias = bias;
    p.y = y;
    p.y_srow = y_srow;
    p.M = M;
    p.N = N;
    p.K = K;
    p.SK = pl.SK;
    p.chunks_per_split = pl.cps;
    p.counters = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) + wl.counters);
    p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + wl.part);
    if (act_dtype == SDB_BF16) return w8::launch<__nv_bfloat16>(p, pl, st, group_size != 0);
    return w8::launch<__half>(p, pl, st, group_size != 0);
}

extern "C" int sdb_quantize_weight(const void* w, int w_dtype, int8_t* q, void* scale, int scale_dtype, int N, int K,
                                   int group_size, void* stream) {
    if (!w || !q || !scale || N <= 0 || K <= 0) {
        set_last_error("bad arguments to sdb_quantize_weight");
        return SDB_ERR_INVALID_ARG;
    }
    const int G = group_size > 0 ? group_size : K;
    if (K % G != 0) {
        set_last_error("group_size must divide K");
        return SDB_ERR_INVALID_ARG;
    }
    dim3 grid(K / G, N);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (w_dtype == SDB_F32)
        w8::quantize_kernel<float><<<grid, 128, 0, st>>>(reinterpret_cast<const float*>(w), q, scale, scale_dtype, K, G);
    else if (w_dtype == SDB_BF16)
        w8::quantize_kernel<__nv_bfloat16>
            <<<grid, 128, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(w), q, scale, scale_dtype, K, G);
    else if (w_dtype == SDB_F16)
        w8::quantize_kernel<__half><<<grid, 128, 0, st>>>(reinterpret_cast<const __half*>(w), q, scale, scale_dtype, K, G);
    else {
        set_last_error("w dtype must be f32, bf16 or f16");
        return SDB_ERR_UNSUPPORTED;
    }
    return cuda_status(cudaGetLastError(), "quantize_kernel launch");
}
