// Token sampling (Gumbel-max with exponential noise) on B200 (sm_100a).
//
// Reference: Sampler.forward, nanovllm/layers/sampler.py:8-12, and the draft
// proposer's per-step sampling, nanovllm/spec_decode/draft_proposer.py:505-510:
//     tokens = argmax(softmax(logits.float() / T) / max(E, 1e-10)),   E ~ Exp(1)
// (the draft step also keeps an fp32 copy of the logits, :505).  Two launches
// instead of ~6 torch kernels that each read and write the (B, V) fp32 tensor:
//
//   1. smp_chunk  one CTA per (row, chunk of 4096): the one read of every logit (and
//      the optional fp32 copy); per chunk its max m_c, the sum
//      S_c = sum 2^((x/T - m_c) log2 e), and the few columns that can hold the
//      chunk's largest value (bounds below).
//   2. smp_pick   one warp per row (programmatic dependent launch): m = max m_c,
//      S = sum S_c 2^((m_c - m) log2 e), the exact value
//      (expf(x/T - m) / S) / max(E, 1e-10) of every candidate, argmax with the
//      first index on ties (torch.argmax).
//
// Candidates.  With a = 2^((x/T - m_c) log2 e) (hardware exponential) every value
// of the chunk is a common factor times a / E up to a relative 2^-16 or so (the
// rounding of x/T - m in expf's argument dominates: |x/T - m| <= 104 for any value
// that does not underflow); the band 2^-12 covers that.  Since -log U >= 1 - U, the
// Philox word alone gives E_lo = max((1 - U)(1 - 1e-5), 1e-10) and an upper bound
// a (1 + band) / E_lo of every column; the column of each thread's largest upper
// bound gets its exact E (one log per thread), and the CTA's largest
// a (1 - band) / E over those bounds the chunk's maximum from below.  The columns
// whose upper bound reaches it go to a shared list, get their exact E (one per
// thread), and the ones within the band of the best (normally one) go to pass 2.  A
// chunk with more than CAP candidates (ties, e.g. constant logits) or more than
// LIVE_CAP listed columns is marked and pass 2 evaluates all its columns.
//
// The noise generation is most of the work: one Philox4x32-10 block (10 rounds) per
// four columns, about 25 of the ~45 instructions a column costs, so the pass is
// bound by instruction issue rather than by HBM.
//
// Noise: caller-provided E (B, V) (parity with the reference given identical draws)
// or Philox stream 2 keyed by (seed, offset), E = -log(U_open) (rng::exp_draw).
#include <cfloat>
#include <climits>

#include "common.cuh"
#include "philox.cuh"

namespace sdb {
namespace smp {

using namespace rng;

constexpr int THREADS = 256;
constexpr int EPT = 16;                 // logits per thread
constexpr int CHUNK = THREADS * EPT;    // 4096 logits per CTA
constexpr int CAP = 8;                  // candidate columns kept per chunk
constexpr int LIVE_CAP = THREADS;       // columns surviving the first bound test
constexpr int PICK_WARPS = 8;           // rows per pass-2 CTA
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kBand = 2.44140625e-4f;  // 2^-12

struct Params {
    const void* logits;
    int64_t ls;              // row stride (elements)
    const float* temps;      // (B) or null
    const float* e;          // (B, V) or null
    uint32_t seed_lo, seed_hi, offset;
    const uint64_t* offset_dev;  // graph-safe form: the offset read from device memory
    float* copy;             // fp32 copy of the logits (B rows of stride cs) or null
    int64_t cs;
    int64_t* tokens;         // token of row b at tokens[b * ts]
    int64_t ts;
    int B, V, C;
    int vec;                 // 16-byte vector loads / stores allowed
    float2* stats;           // [B][C] (m_c, S_c)
    int* ncand;              // [B][C] candidate count, CAP + 1 = evaluate the whole chunk
    int* cand;               // [B][C][CAP]
};

template <typename T>
SDB_DEV float to_f32(T v);
template <>
SDB_DEV float to_f32<float>(float v) { return v; }
template <>
SDB_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
SDB_DEV float to_f32<__half>(__half v) { return __half2float(v); }

SDB_DEV bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// The Philox offset of this call: the host value, or the device-resident one of the
// graph-safe entry point (unchanged while the call's kernels run).
SDB_DEV uint32_t draw_offset(const Params& p) { return p.offset_dev ? (uint32_t)*p.offset_dev : p.offset; }

template <typename F>
SDB_DEV float block_reduce(float v, F op, float* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, s));
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    v = sh[0];
    for (int i = 1; i < THREADS / 32; ++i) v = op(v, sh[i]);
    return v;
}

// Column of element j (0..31) of this thread.  Vector form: VEC consecutive columns
// per 16-byte load, loads strided by the CTA; scalar form: one column per load.
template <int VEC>
SDB_DEV int column(int base, int j, bool vec) {
    return vec ? base + ((j / VEC) * THREADS + (int)threadIdx.x) * VEC + (j % VEC)
               : base + j * THREADS + (int)threadIdx.x;
}

// Sum and max over the CTA in one pass of barriers.
SDB_DEV float2 block_reduce_sum_max(float s, float m, float* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    __syncthreads();
    if (lane == 0) {
        sh[w] = s;
        sh[THREADS / 32 + w] = m;
    }
    __syncthreads();
    s = sh[0];
    m = sh[THREADS / 32];
    for (int i = 1; i < THREADS / 32; ++i) {
        s += sh[i];
        m = fmaxf(m, sh[THREADS / 32 + i]);
    }
    return make_float2(s, m);
}

template <typename T>
__global__ void __launch_bounds__(THREADS) smp_chunk(const Params p) {
    constexpr int VEC = 16 / sizeof(T);
    __shared__ float sh[2 * (THREADS / 32)];
    __shared__ int nlive, ncand;
    __shared__ int live_col[LIVE_CAP];
    __shared__ float live_a[LIVE_CAP];
    __shared__ int cands[CAP];
    asm volatile("griddepcontrol.launch_dependents;");
    const int b = blockIdx.x / p.C, c = blockIdx.x - (blockIdx.x / p.C) * p.C;
    const int base = c * CHUNK;
    const bool vec = p.vec != 0;
    const T* row = reinterpret_cast<const T*>(p.logits) + (int64_t)b * p.ls;
    if (threadIdx.x == 0) {
        nlive = 0;
        ncand = 0;
    }

    float x[EPT];
    if (vec) {
#pragma unroll
        for (int q = 0; q < EPT / VEC; ++q) {
            const int i0 = base + (q * THREADS + (int)threadIdx.x) * VEC;
            if (i0 < p.V) {  // V % 8 == 0: a vector is wholly inside or outside the row
                const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(row + i0));
                const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
                for (int e = 0; e < VEC; ++e) x[q * VEC + e] = to_f32<T>(v[e]);
                if (p.copy) {
                    float* dst = p.copy + (int64_t)b * p.cs + i0;
#pragma unroll
                    for (int e = 0; e < VEC; e += 4)
                        __stcs(reinterpret_cast<float4*>(dst + e),
                               make_float4(x[q * VEC + e], x[q * VEC + e + 1], x[q * VEC + e + 2], x[q * VEC + e + 3]));
                }
            } else {
#pragma unroll
                for (int e = 0; e < VEC; ++e) x[q * VEC + e] = -INFINITY;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
            const int i = base + j * THREADS + (int)threadIdx.x;
            x[j] = -INFINITY;
            if (i < p.V) {
                x[j] = to_f32<T>(row[i]);
                if (p.copy) p.copy[(int64_t)b * p.cs + i] = x[j];
            }
        }
    }
    const float T_ = p.temps ? p.temps[b] : 1.0f;
    if (T_ != 1.0f) {  // x / T as torch divides (IEEE), one uniform branch per CTA
#pragma unroll
        for (int j = 0; j < EPT; ++j) x[j] = __fdiv_rn(x[j], T_);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < EPT; ++j) mx = fmaxf(mx, x[j]);
    const float mc = block_reduce(mx, [](float a, float b2) { return fmaxf(a, b2); }, sh);

    // a_j = 2^((x - m_c) log2 e) in place of x (an out-of-range column gives 0), their
    // sum, and upper bounds ub_j = a_j (1 + band) / E_lo,j with E_lo from the word alone
    // (1 - U = (2^24 - 1 - (w >> 8)) 2^-24 exactly).  The column of the thread's largest
    // upper bound gets its exact E: a_j (1 - band) / E_j is a value of the chunk up to
    // the band, so the CTA's largest such product bounds the chunk's maximum from below.
    float sum = 0.f, ub[EPT];
    float best_ub = -1.f, best_a = 0.f;
    uint32_t best_w = 0u;
    int best_col = -1;
#pragma unroll
    for (int g = 0; g < EPT / 4; ++g) {
        uint32_t w4[4] = {0u, 0u, 0u, 0u};
        const int i0 = column<VEC>(base, 4 * g, vec);
        if (vec && !p.e && i0 < p.V) {  // four consecutive columns from one Philox block
            w4[0] = (uint32_t)i0 >> 2;
            w4[1] = (uint32_t)b;
            w4[2] = 2u;
            w4[3] = draw_offset(p);
            philox(w4, p.seed_lo, p.seed_hi);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = 4 * g + e;
            const int i = column<VEC>(base, j, vec);
            const float a = ex2((x[j] - mc) * kLog2e);
            x[j] = a;
            sum += a;
            uint32_t w = w4[e];
            float Elo;
            if (p.e) {
                Elo = i < p.V ? fmaxf(p.e[(int64_t)b * p.V + i], 1e-10f) : 1.f;
            } else {
                if (!vec) w = i < p.V ? philox_word(p.seed_lo, p.seed_hi, draw_offset(p), 2u, (uint32_t)b, (uint32_t)i) : 0u;
                Elo = fmaxf((float)(0xFFFFFFu - (w >> 8)) * (5.9604644775390625e-08f * 0.99999f), 1e-10f);
            }
            ub[j] = __fdividef(a * (1.f + kBand), Elo);
            if (ub[j] > best_ub) {
                best_ub = ub[j];
                best_a = a;
                best_w = w;
                best_col = i;
            }
        }
    }
    float lb = 0.f;
    if (best_col >= 0 && best_a > 0.f) {
        const float E = p.e ? fmaxf(p.e[(int64_t)b * p.V + best_col], 1e-10f) : exp_draw(best_w);
        lb = __fdividef(best_a * (1.f - kBand), E);
    }
    const float2 sl = block_reduce_sum_max(sum, lb, sh);
    const float sc = sl.x, LB1 = sl.y;

    // the columns that can still be the chunk's argmax go to a shared list
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        if (x[j] > 0.f && ub[j] >= LB1) {
            const int slot = atomicAdd(&nlive, 1);
            if (slot < LIVE_CAP) {
                live_col[slot] = column<VEC>(base, j, vec);
                live_a[slot] = x[j];
            }
        }
    }
    __syncthreads();
    // second pass, one list entry per thread: the exact E narrows the list to the columns
    // within the band of the best (normally one)
    const int nl = nlive;
    float lb2 = 0.f, ub2 = -1.f;
    int col2 = -1;
    if ((int)threadIdx.x < min(nl, LIVE_CAP)) {
        col2 = live_col[threadIdx.x];
        const float a = live_a[threadIdx.x];
        const float E = p.e ? fmaxf(p.e[(int64_t)b * p.V + col2], 1e-10f)
                            : exp_draw(philox_word(p.seed_lo, p.seed_hi, draw_offset(p), 2u, (uint32_t)b, (uint32_t)col2));
        lb2 = __fdividef(a * (1.f - kBand), E);
        ub2 = __fdividef(a * (1.f + kBand), E);
    }
    const float LB2 = block_reduce(lb2, [](float a, float b2) { return fmaxf(a, b2); }, sh);
    if (col2 >= 0 && ub2 >= LB2) {
        const int slot = atomicAdd(&ncand, 1);
        if (slot < CAP) cands[slot] = col2;
    }
    __syncthreads();
    const int nc = ncand;
    if (threadIdx.x == 0) {
        const int idx = b * p.C + c;
        p.stats[idx] = make_float2(mc, sc);
        p.ncand[idx] = (nc > CAP || nl > LIVE_CAP) ? CAP + 1 : nc;
    }
    if ((int)threadIdx.x < min(nc, CAP)) p.cand[(int64_t)(b * p.C + c) * CAP + threadIdx.x] = cands[threadIdx.x];
}

template <typename T>
__global__ void __launch_bounds__(PICK_WARPS * 32) smp_pick(const Params p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // pass 1 complete and visible
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * PICK_WARPS + (threadIdx.x >> 5);
    if (b >= p.B) return;
    const T* row = reinterpret_cast<const T*>(p.logits) + (int64_t)b * p.ls;
    float m = -INFINITY;
    for (int c = lane; c < p.C; c += 32) m = fmaxf(m, p.stats[b * p.C + c].x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float S = 0.f;
    for (int c = lane; c < p.C; c += 32) {
        const float2 st = p.stats[b * p.C + c];
        S += st.y * ex2((st.x - m) * kLog2e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    const float T_ = p.temps ? p.temps[b] : 1.0f;
    float best = -INFINITY;
    int bidx = INT_MAX;
    // exact value of column i: (expf(x/T - m) / S) / max(E, 1e-10), as the reference
    // evaluates softmax then the division (sampler.py:10-11)
    auto eval = [&](int i) {
        float xt = to_f32<T>(row[i]);
        if (T_ != 1.0f) xt = __fdiv_rn(xt, T_);
        const float E = p.e ? fmaxf(p.e[(int64_t)b * p.V + i], 1e-10f)
                            : exp_draw(philox_word(p.seed_lo, p.seed_hi, draw_offset(p), 2u, (uint32_t)b, (uint32_t)i));
        const float v = __fdiv_rn(__fdiv_rn(expf(xt - m), S), E);
        if (better(v, i, best, bidx)) {
            best = v;
            bidx = i;
        }
    };
    for (int c0 = 0; c0 < p.C; c0 += 32) {  // lane c: the candidates of chunk c0 + c
        const int c = c0 + lane;
        const int n = c < p.C ? p.ncand[b * p.C + c] : 0;
        if (n <= CAP)
            for (int k = 0; k < n; ++k) eval(p.cand[(int64_t)(b * p.C + c) * CAP + k]);
        unsigned whole = __ballot_sync(0xffffffffu, n > CAP);  // chunks to evaluate in full
        while (whole) {  // rare: ties; the whole warp walks the chunk
            const int cc = c0 + __ffs(whole) - 1;
            whole &= whole - 1;
            const int hi = min(p.V, (cc + 1) * CHUNK);
            for (int i = cc * CHUNK + lane; i < hi; i += 32) eval(i);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (better(ov, oi, best, bidx)) {
            best = ov;
            bidx = oi;
        }
    }
    if (lane == 0) p.tokens[(int64_t)b * p.ts] = bidx == INT_MAX ? 0 : bidx;
}

struct WsLayout {
    size_t stats, ncand, cand, total;
};

static WsLayout ws_layout(int B, int V) {
    const size_t C = (size_t)((V + CHUNK - 1) / CHUNK);
    WsLayout w;
    size_t off = 256;  // error word kept at offset 0 like the other workspaces
    w.stats = off;
    off = align_up(off + sizeof(float2) * (size_t)B * C, 256);
    w.ncand = off;
    off = align_up(off + sizeof(int) * (size_t)B * C, 256);
    w.cand = off;
    off = align_up(off + sizeof(int) * (size_t)B * C * CAP, 256);
    w.total = off;
    return w;
}

template <typename T>
static int launch(const Params& p, cudaStream_t st) {
    smp_chunk<T><<<(unsigned)((long long)p.C * p.B), THREADS, 0, st>>>(p);
    int rc = cuda_status(cudaGetLastError(), "smp_chunk launch");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.B + PICK_WARPS - 1) / PICK_WARPS, 1, 1);
    cfg.blockDim = dim3(PICK_WARPS * 32, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, smp_pick<T>, p), "smp_pick launch");
}

}  // namespace smp
}  // namespace sdb

using namespace sdb;

extern "C" size_t sdb_sample_workspace_size(int B, int V) {
    if (B <= 0 || V <= 0) return 256;
    return smp::ws_layout(B, V).total;
}

namespace {
int sample_impl(const void* logits, int64_t logits_stride_row, int dtype, const float* temperatures,
                const float* exponentials, uint64_t seed, uint64_t offset, uint64_t* offset_dev, int64_t* tokens,
                int64_t tokens_stride, float* logits_f32, int64_t logits_f32_stride_row, int B, int V,
                void* workspace, size_t workspace_bytes, void* stream) {
    if (B == 0) return SDB_OK;
    if (!logits || !tokens || !workspace || B < 0 || V <= 0 || logits_stride_row < V || tokens_stride < 1 ||
        (logits_f32 && logits_f32_stride_row < V) ||
        (long long)B * ((V + smp::CHUNK - 1) / smp::CHUNK) > INT_MAX) {
        set_last_error("bad arguments to sdb_sample");
        return SDB_ERR_INVALID_ARG;
    }
    if (dtype != SDB_F32 && dtype != SDB_BF16 && dtype != SDB_F16) {
        set_last_error("dtype %d not supported", dtype);
        return SDB_ERR_UNSUPPORTED;
    }
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) {
        set_last_error("workspace must be 256-byte aligned");
        return SDB_ERR_WORKSPACE;
    }
    const smp::WsLayout w = smp::ws_layout(B, V);
    if (workspace_bytes < w.total) {
        set_last_error("workspace too small: need %zu bytes, got %zu", w.total, workspace_bytes);
        return SDB_ERR_WORKSPACE;
    }
    const int elem = dtype == SDB_F32 ? 4 : 2;
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    smp::Params p{};
    p.logits = logits;
    p.ls = logits_stride_row;
    p.temps = temperatures;
    p.e = exponentials;
    p.seed_lo = (uint32_t)(seed & 0xffffffffu);
    p.seed_hi = (uint32_t)(seed >> 32);
    p.offset = (uint32_t)offset;
    p.copy = logits_f32;
    p.cs = logits_f32_stride_row;
    p.tokens = tokens;
    p.ts = tokens_stride;
    p.B = B;
    p.V = V;
    p.C = (V + smp::CHUNK - 1) / smp::CHUNK;
    p.vec = (V % 8 == 0) && al16(logits) && ((logits_stride_row * elem) % 16 == 0) &&
            (!logits_f32 || (al16(logits_f32) && (logits_f32_stride_row * 4) % 16 == 0));
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    p.stats = reinterpret_cast<float2*>(ws + w.stats);
    p.ncand = reinterpret_cast<int*>(ws + w.ncand);
    p.cand = reinterpret_cast<int*>(ws + w.cand);
    p.offset_dev = offset_dev;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int rc;
    if (dtype == SDB_F32) rc = smp::launch<float>(p, st);
    else if (dtype == SDB_BF16) rc = smp::launch<__nv_bfloat16>(p, st);
    else rc = smp::launch<__half>(p, st);
    if (rc || !offset_dev) return rc;
    return launch_advance_offset(offset_dev, st);
}
}  // namespace

extern "C" int sdb_sample(const void* logits, int64_t logits_stride_row, int dtype, const float* temperatures,
                          const float* exponentials, uint64_t seed, uint64_t offset, int64_t* tokens,
                          int64_t tokens_stride, float* logits_f32, int64_t logits_f32_stride_row, int B, int V,
                          void* workspace, size_t workspace_bytes, void* stream) {
    return sample_impl(logits, logits_stride_row, dtype, temperatures, exponentials, seed, offset, nullptr, tokens,
                       tokens_stride, logits_f32, logits_f32_stride_row, B, V, workspace, workspace_bytes, stream);
}

extern "C" int sdb_sample_dev_offset(const void* logits, int64_t logits_stride_row, int dtype,
                                     const float* temperatures, uint64_t seed, uint64_t* offset_dev,
                                     int64_t* tokens, int64_t tokens_stride, float* logits_f32,
                                     int64_t logits_f32_stride_row, int B, int V, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    if (!offset_dev || (reinterpret_cast<uintptr_t>(offset_dev) & 7)) {
        set_last_error("sdb_sample_dev_offset needs an 8-byte aligned device offset");
        return SDB_ERR_INVALID_ARG;
    }
    return sample_impl(logits, logits_stride_row, dtype, temperatures, nullptr, seed, 0, offset_dev, tokens,
                       tokens_stride, logits_f32, logits_f32_stride_row, B, V, workspace, workspace_bytes, stream);
}
