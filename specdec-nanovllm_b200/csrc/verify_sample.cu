// verify_batch rejection sampling on B200 (sm_100a).
//
// Reference: nanovllm/spec_decode/verify.py:42-209.  Same arithmetic, four
// launches instead of ~8 passes of generic torch kernels plus a q_pad copy:
//
//   1. vs_row_stats   grid (rows, chunks of 8192): per chunk of every draft and
//      target row, max and sum of exp(x/T - max) (one HBM read of every logit --
//      the floor of this path; 32 logits per thread held in registers).
//   2. vs_decide      one warp per sequence: merges the row statistics and makes
//      the k acceptance decisions (candidate j against target row j, ratio =
//      min(1, p/q), u < ratio, verify.py:109-129).
//   3. vs_resid_sums  grid (B, chunks): sums resid = max(p[a] - q_pad[a], 0) and
//      p[a] over its chunk of row a = accepted (verify.py:141-151).
//   4. vs_bonus       grid (B, chunks): partial argmax of (resid / Z) / max(E, 1e-10)
//      (verify.py:152, :167, :203-209), first index on ties; the last CTA of a
//      sequence (atomic counter, reset after use) finishes the argmax and writes
//      the bonus token.
//
// The draws: acceptance uniforms u[b, j] and exponentials E[b, i] are either
// caller-provided (parity with the reference given identical draws) or
// generated in-kernel from Philox4x32-10 (Salmon et al., SC'11), stream 0 / 1,
// counter (col/4, row, stream, offset), key (seed lo, seed hi), with
// E = -log(U), U = ((w >> 8) + 1) * 2^-24, and log computed by a fixed
// sequence of correctly rounded float32 operations (no contraction) so a CPU
// restatement reproduces every bit.
#include <cfloat>
#include <type_traits>

#include "common.cuh"
#include "philox.cuh"

namespace sdb {
namespace vs {

using namespace rng;

constexpr int THREADS = 256;
constexpr int EPT = 32;                    // logits per thread held in registers (pass 1)
constexpr int CHUNK1 = THREADS * EPT;      // 8192 logits per chunk in pass 1
constexpr int EPT2 = 16;                   // logits per thread in passes 3-4
constexpr int CHUNK2 = THREADS * EPT2;     // 4096 logits per CTA in passes 3-4
// pass 1, streaming form: persistent CTAs, one producer warp moving 32 KB chunks of
// a row into a shared-memory ring by bulk copy, 16 consumer warps reducing them
constexpr int SUB = 16;                    // (max, sum) partials per chunk: one per consumer warp
constexpr int BS_STAGES = 3;               // x 32 KB, two CTAs per SM
constexpr int BS_CONSUMERS = SUB;          // warps, 512 logits of each chunk apiece
constexpr int BS_EPT = CHUNK1 / (32 * BS_CONSUMERS);
constexpr int BS_THREADS = 32 * (BS_CONSUMERS + 1);
constexpr int BS_SMEM = BS_STAGES * CHUNK1 * 4;
// fused residual + bonus pass: candidate columns kept per chunk, and the columns whose
// upper bound reaches the chunk's lower bound that get an exact evaluation
constexpr int RB_CAP = 8;
constexpr int RB_LIVE = 64;

struct Params {
    const void* draft;     // (B, k, V)
    const void* target;    // (B, Tr, V)
    int dkind, tkind;      // element type of draft / target: 0 float32, 1 bfloat16, 2 float16
    int vec;               // passes 3-4 read rows in 16-byte vectors (group_col layout)
    const int64_t* tokens; // (B, k)
    const float* temps;    // (B) or null
    const float* u;        // (B, k) or null
    const float* e;        // (B, V) or null
    uint32_t seed_lo, seed_hi, offset;
    const uint64_t* offset_dev;  // graph-safe form: the offset read from device memory
    int point_mass;
    int64_t* out_acc;
    int64_t* out_bonus;
    uint8_t* out_mask;
    int B, k, Tr, V, C1, C2;
    float2* stats;         // [rows][C1 * SUB]  (max, sumexp) per chunk and warp
    float2* rsum;          // [B][C2]     (sum resid, sum p[a])
    float2* amax;          // [B][C2]     (value, index as float bits)
    int* ncand;            // [B][C2]     fused residual + bonus pass: candidates kept, RB_CAP + 1 = all
    int* cand;             // [B][C2][RB_CAP] their columns
    int* counters;         // [B], zero between calls
    struct Decision* dec;  // [B]
    int* err;
    // vocabulary-parallel form (the LM head split by columns across tp ranks): this
    // rank holds global columns [col0, col0 + V) of Vg; `gathered` holds the previous
    // exchange of all tp ranks (rank-major), `send` receives this rank's next one.
    // Single-device calls: col0 = 0, Vg = V, shard = 0.
    int col0, Vg, tp, shard;
    const float* gathered;
    float* send;
};

// The Philox offset of this call: the host value, or the device-resident one of the
// graph-safe entry point (unchanged while the call's kernels run).
SDB_DEV uint32_t draw_offset(const Params& p) { return p.offset_dev ? (uint32_t)*p.offset_dev : p.offset; }

SDB_DEV float accept_uniform(const Params& p, int b, int j) {
    if (p.u) return p.u[b * p.k + j];
    return word_to_uniform(philox_word(p.seed_lo, p.seed_hi, draw_offset(p), 0u, (uint32_t)b, (uint32_t)j));
}

// x / T exactly as torch divides (IEEE); T == 1 is the identity.
SDB_DEV float scale_t(float x, float T) { return T == 1.0f ? x : __fdiv_rn(x, T); }

// One row of logits of any of the three element types, read as float32 exactly (the
// reference converts with .float(), verify.py:194).  The type is uniform per call,
// so the branches below never diverge.
SDB_DEV float half_bits_to_f32(uint32_t h, int kind) {
    return kind == 1 ? __uint_as_float(h << 16) : __half2float(__ushort_as_half((unsigned short)h));
}
// Two packed 16-bit logits -> float32 (kind 1 bfloat16, 2 float16), one branch per pair.
SDB_DEV float2 unpack2(uint32_t u, int kind) {
    if (kind == 1) return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
struct Row {
    const uint8_t* p;  // null: no row
    int kind;
    SDB_DEV float at(int64_t i) const {
        if (kind == 0) return __ldg(reinterpret_cast<const float*>(p) + i);
        return half_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(p) + i), kind);
    }
    // four logits from i (i % 4 == 0; rows 8-byte aligned for 16-bit types)
    SDB_DEV float4 at4(int64_t i) const {
        if (kind == 0) return __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const unsigned short*>(p) + i));
        const float2 a = unpack2(u.x, kind), b = unpack2(u.y, kind);
        return make_float4(a.x, a.y, b.x, b.y);
    }
    // eight logits from i (i % 8 == 0), in two groups of four: one 16-byte load for
    // 16-bit rows (16-byte aligned: V % 8 == 0), two for float32 rows; `left` logits
    // of the row remain from i (a float32 row may end after the first group)
    SDB_DEV void at8(int64_t i, int left, float4& g0, float4& g1) const {
        if (kind == 0) {
            const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
            g0 = __ldg(q);
            if (left > 4) g1 = __ldg(q + 1);
            return;
        }
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned short*>(p) + i));
        const float2 a = unpack2(u.x, kind), b = unpack2(u.y, kind), c = unpack2(u.z, kind), d = unpack2(u.w, kind);
        g0 = make_float4(a.x, a.y, b.x, b.y);
        g1 = make_float4(c.x, c.y, d.x, d.y);
    }
};

// Column of group q (four consecutive logits) of this thread in the vector form of
// passes 3-4: pairs of groups are adjacent, so one 16-byte load covers a pair of
// 16-bit groups.
SDB_DEV int group_col(int q) { return (q >> 1) * THREADS * 8 + (int)threadIdx.x * 8 + (q & 1) * 4; }
SDB_DEV int elem_bytes(int kind) { return kind == 0 ? 4 : 2; }
SDB_DEV Row draft_row(const Params& p, int64_t row) {
    return Row{reinterpret_cast<const uint8_t*>(p.draft) + row * p.V * elem_bytes(p.dkind), p.dkind};
}
SDB_DEV Row target_row(const Params& p, int64_t row) {
    return Row{reinterpret_cast<const uint8_t*>(p.target) + row * p.V * elem_bytes(p.tkind), p.tkind};
}

// ------------------------------------------------------------------ reductions
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

struct Decision {
    int a;          // accepted prefix length
    unsigned mask;  // accept bits (k <= 32)
    float Mp, ip;   // max and 1/sum of target row min(a, Tr-1)
    float Mq, iq;   // same for draft row a (a < k, not point mass)
};

// ------------------------------------------------------------------ pass 1
// Sum of exp(x - max) by the hardware base-2 exponential: relative error ~2^-22 per
// term, far below what the decisions can resolve (they compare against uniforms).
__global__ void __launch_bounds__(THREADS, 4) vs_row_stats(const Params p) {
    __shared__ float sh[THREADS / 32];
    const int nd = p.B * p.k;
    // point-mass drafts need no statistics: the grid then starts at the target rows
    const int row = blockIdx.x + (p.point_mass ? nd : 0);
    const int c = blockIdx.y;
    Row src;
    int b;
    if (row < nd) {
        src = draft_row(p, row);
        b = row / p.k;
    } else {
        src = target_row(p, row - nd);
        b = (row - nd) / p.Tr;
    }
    const float T = p.temps ? p.temps[b] : 1.0f;
    const int base = c * CHUNK1;
    const int n = min(CHUNK1, p.V - base);
    float v[EPT];
    if ((p.V & 3) == 0) {
#pragma unroll
        for (int it = 0; it < EPT / 4; ++it) {
            const int idx = it * THREADS * 4 + threadIdx.x * 4;
            float4 x = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            if (idx < n) x = src.at4(base + idx);
            v[it * 4 + 0] = idx < n ? x.x : -INFINITY;
            v[it * 4 + 1] = idx < n ? x.y : -INFINITY;
            v[it * 4 + 2] = idx < n ? x.z : -INFINITY;
            v[it * 4 + 3] = idx < n ? x.w : -INFINITY;
        }
    } else {
#pragma unroll
        for (int it = 0; it < EPT; ++it) {
            const int idx = it * THREADS + threadIdx.x;
            v[it] = idx < n ? src.at(base + idx) : -INFINITY;
        }
    }
    if (T != 1.0f) {  // x / T as torch divides (IEEE), one uniform branch per CTA
#pragma unroll
        for (int i = 0; i < EPT; ++i) v[i] = __fdiv_rn(v[i], T);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPT; ++i) mx = fmaxf(mx, v[i]);
    mx = block_reduce(mx, [](float a, float b2) { return fmaxf(a, b2); }, sh);
    float s = 0.f;
    if (mx != -INFINITY) {
        constexpr float kLog2e = 1.4426950408889634f;
        const float off = -mx * kLog2e;
#pragma unroll
        for (int i = 0; i < EPT; ++i) s += ex2(fmaf(v[i], kLog2e, off));
    }
    s = block_reduce(s, [](float a, float b2) { return a + b2; }, sh);
    if (threadIdx.x < SUB)
        __stcg(p.stats + ((int64_t)row * p.C1 + c) * SUB + threadIdx.x,
               threadIdx.x == 0 ? make_float2(mx, s) : make_float2(-INFINITY, 0.f));
}

// Pass 1 for 16-byte-aligned rows with V % 4 == 0: items (row, chunk) strided over
// persistent CTAs; the last warp streams each item's 32 KB into the stage ring with one
// bulk copy, the consumer warps reduce it from shared memory and release the stage.
SDB_DEV Row logits_row(const Params& p, int row, int& b) {
    const int nd = p.B * p.k;
    if (row < nd) {
        b = row / p.k;
        return draft_row(p, row);
    }
    b = (row - nd) / p.Tr;
    return target_row(p, row - nd);
}

__global__ void __launch_bounds__(BS_THREADS, 2) vs_row_stats_bulk(const Params p, int row0, int nrows) {
    extern __shared__ __align__(128) uint8_t ring[];
    __shared__ __align__(8) uint64_t bars[2 * BS_STAGES];
    // per stage, written by the producer before it arms the stage: the item's row and
    // chunk, its logit count and element type, and the row's temperature, so the
    // consumers do no index arithmetic (integer divisions) per item
    __shared__ int meta_row[BS_STAGES], meta_c[BS_STAGES], meta_n[BS_STAGES], meta_kind[BS_STAGES];
    __shared__ float meta_t[BS_STAGES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = nrows * p.C1;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * BS_STAGES;
    if (threadIdx.x == 0) {
        for (int s = 0; s < BS_STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, BS_CONSUMERS);
        }
        fence_mbarrier_init();
    }
    __syncthreads();
    if (warp == BS_CONSUMERS) {
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int g = 0;
            for (int it = blockIdx.x; it < total; it += gridDim.x, ++g) {
                const int s = g % BS_STAGES;
                if (g >= BS_STAGES && !mbar_wait_sleep(empty0 + 8 * s, ((g / BS_STAGES) - 1) & 1)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
                int b;
                const int c = it % p.C1, row = row0 + it / p.C1;
                const Row r = logits_row(p, row, b);
                const int esz = elem_bytes(r.kind);
                const uint8_t* src = r.p + (int64_t)c * CHUNK1 * esz;
                const int n = min(CHUNK1, p.V - c * CHUNK1);
                const uint32_t bytes = (uint32_t)esz * (uint32_t)n;
                meta_row[s] = row;
                meta_c[s] = c;
                meta_n[s] = n;
                meta_kind[s] = r.kind;
                meta_t[s] = p.temps ? p.temps[b] : 1.0f;
                mbar_arrive_expect_tx(full0 + 8 * s, bytes);  // release: the consumers see the metadata
                bulk_load(smem_u32(ring + s * CHUNK1 * 4), src, bytes, full0 + 8 * s, pol);
            }
            for (int q = g - BS_STAGES > 0 ? g - BS_STAGES : 0; q < g; ++q)  // own copies land before exit
                if (!mbar_wait(full0 + 8 * (q % BS_STAGES), (q / BS_STAGES) & 1)) break;
        }
        return;
    }
    // consumer warp w reduces logits [512 w, 512 w + 512) of each chunk on its own
    bool ok = true;
    int g = 0;
    for (int it = blockIdx.x; it < total; it += gridDim.x, ++g) {
        const int s = g % BS_STAGES;
        if (ok && !mbar_wait_sleep(full0 + 8 * s, (g / BS_STAGES) & 1)) {
            ok = false;
            if (lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
        }
        const int row = meta_row[s], c = meta_c[s], n = meta_n[s], kind = meta_kind[s];
        const float T = meta_t[s];
        // this warp's 512 logits of the chunk (the assignment of logits to lanes is free:
        // only their max and sum are formed): float32 as 4 x 16 bytes per lane, 16-bit
        // types as 2 x 16 bytes per lane; the type branch is uniform per item
        const uint8_t* sb = ring + s * CHUNK1 * 4;
        float v[BS_EPT];
        if (kind == 0) {
            const float4* st = reinterpret_cast<const float4*>(sb) + warp * (CHUNK1 / 4 / SUB);
#pragma unroll
            for (int q = 0; q < BS_EPT / 4; ++q) {
                const int i4 = q * 32 + lane;
                const bool in = 4 * (warp * (CHUNK1 / 4 / SUB) + i4) < n;
                const float4 x = st[i4];
                v[4 * q + 0] = in ? x.x : -INFINITY;
                v[4 * q + 1] = in ? x.y : -INFINITY;
                v[4 * q + 2] = in ? x.z : -INFINITY;
                v[4 * q + 3] = in ? x.w : -INFINITY;
            }
        } else {
            const uint4* st = reinterpret_cast<const uint4*>(sb) + warp * (CHUNK1 / 8 / SUB);
            uint4 u[BS_EPT / 8];
            bool in[BS_EPT / 8];
#pragma unroll
            for (int q = 0; q < BS_EPT / 8; ++q) {
                const int i8 = q * 32 + lane;
                in[q] = 8 * (warp * (CHUNK1 / 8 / SUB) + i8) < n;  // n % 8 == 0 on this path
                u[q] = st[i8];
            }
            if (kind == 1) {
#pragma unroll
                for (int q = 0; q < BS_EPT / 8; ++q) {
                    const uint32_t w[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        v[8 * q + 2 * e] = in[q] ? __uint_as_float(w[e] << 16) : -INFINITY;
                        v[8 * q + 2 * e + 1] = in[q] ? __uint_as_float(w[e] & 0xffff0000u) : -INFINITY;
                    }
                }
            } else {
#pragma unroll
                for (int q = 0; q < BS_EPT / 8; ++q) {
                    const uint32_t w[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
                        v[8 * q + 2 * e] = in[q] ? f2.x : -INFINITY;
                        v[8 * q + 2 * e + 1] = in[q] ? f2.y : -INFINITY;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
        if (T != 1.0f) {  // x / T as torch divides (IEEE); -inf / T stays -inf
#pragma unroll
            for (int i = 0; i < BS_EPT; ++i) v[i] = __fdiv_rn(v[i], T);
        }
        float m4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
        for (int i = 4; i < BS_EPT; ++i) m4[i & 3] = fmaxf(m4[i & 3], v[i]);
        float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        if (mx != -INFINITY) {
            constexpr float kLog2e = 1.4426950408889634f;
            const float off = -mx * kLog2e;
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < BS_EPT; ++i) s4[i & 3] += ex2(fmaf(v[i], kLog2e, off));
            sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (ok && lane == 0) __stcg(p.stats + ((int64_t)row * p.C1 + c) * SUB + warp, make_float2(mx, sum));
    }
}

// ------------------------------------------------------------------ pass 2
// One CTA per sequence: warp w merges the chunk statistics of rows w, w + 16, ...
// (the k draft rows, then the target rows) into (max, 1/sum); warp 0 then makes the
// k acceptance decisions, one candidate per lane:
// ratio = where(q_tok > 0, min(p_tok / max(q_tok, 1e-10), 1), 0); accept = u < ratio
// (verify.py:109-121); accepted = first rejection or k (:125-129).
constexpr int DECIDE_THREADS = 512;

// (max, sum exp(x - max)) of global row `grow` from its chunk partials, on every lane
// of the calling warp.
SDB_DEV float2 merge_row_stats(const Params& p, int grow, int lane) {
    const float2* st = p.stats + (int64_t)grow * p.C1 * SUB;
    const int np = p.C1 * SUB;
    constexpr int kHeld = 16;  // partials per lane kept in registers (V up to 2^22)
    float2 h[kHeld];
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < kHeld; ++j) {
        const int c = lane + 32 * j;
        h[j] = c < np ? __ldcg(st + c) : make_float2(-INFINITY, 0.f);
        M = fmaxf(M, h[j].x);
    }
    for (int c = lane + 32 * kHeld; c < np; c += 32) M = fmaxf(M, __ldcg(st + c).x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float S = 0.f;
#pragma unroll
    for (int j = 0; j < kHeld; ++j)
        if (h[j].x != -INFINITY) S += h[j].y * expf(h[j].x - M);
    for (int c = lane + 32 * kHeld; c < np; c += 32) {
        const float2 v = __ldcg(st + c);
        if (v.x != -INFINITY) S += v.y * expf(v.x - M);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    return make_float2(M, S);
}

// Warp-wide: the k acceptance decisions of sequence b given every row's max sM and
// inverse sum sI (draft rows 0..k-1, target rows k..k+Tr-1) and, on lane j < k, the
// draft and target logits of candidate j (verify.py:109-129); writes the Decision and
// the outputs.
SDB_DEV void decide_from(const Params& p, int b, int lane, const float* sM, const float* sI, float xq, float xp) {
    const float T = p.temps ? p.temps[b] : 1.0f;
    bool acc = true;
    if (lane < p.k) {
        const float q_tok = p.point_mass ? xq : expf(scale_t(xq, T) - sM[lane]) * sI[lane];
        const float p_tok = expf(scale_t(xp, T) - sM[p.k + lane]) * sI[p.k + lane];
        const float ratio = q_tok > 0.f ? fminf(__fdiv_rn(p_tok, fmaxf(q_tok, 1e-10f)), 1.0f) : 0.f;
        acc = accept_uniform(p, b, lane) < ratio;
        p.out_mask[b * p.k + lane] = acc ? 1 : 0;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, acc);
    const unsigned low = p.k >= 32 ? 0xffffffffu : ((1u << p.k) - 1u);
    const unsigned rej = ~bal & low;
    const int a = rej ? __ffs(rej) - 1 : p.k;
    if (lane == 0) {
        Decision d;
        d.a = a;
        d.mask = bal & low;
        const int tr = p.k + min(a, p.Tr - 1);  // verify.py:143
        d.Mp = sM[tr];
        d.ip = sI[tr];
        const bool hq = a < p.k && !p.point_mass;
        d.Mq = hq ? sM[a] : 0.f;
        d.iq = hq ? sI[a] : 0.f;
        p.dec[b] = d;
        p.out_acc[b] = a;
    }
}

// Candidate j's token, range-checked against the (global) vocabulary.
SDB_DEV int64_t candidate_token(const Params& p, int b, int j) {
    int64_t tok = p.tokens[b * p.k + j];
    if (tok < 0 || tok >= p.Vg) {
        atomicOr(p.err, SDB_KERR_TOKEN);
        tok = 0;
    }
    return tok;
}

__global__ void __launch_bounds__(DECIDE_THREADS) vs_decide(const Params p) {
    __shared__ float sM[65], sI[65];
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nd = p.B * p.k;
    const int nrows = p.k + p.Tr;
    for (int r = warp; r < nrows; r += DECIDE_THREADS / 32) {
        if (r < p.k && p.point_mass) continue;
        const int grow = r < p.k ? b * p.k + r : nd + b * p.Tr + (r - p.k);
        const float2 ms = merge_row_stats(p, grow, lane);
        if (lane == 0) {
            sM[r] = ms.x;
            sI[r] = 1.0f / ms.y;
        }
    }
    __syncthreads();
    if (warp != 0) return;
    float xq = 0.f, xp = 0.f;
    if (lane < p.k) {
        const int64_t tok = candidate_token(p, b, lane);
        xq = draft_row(p, b * p.k + lane).at(tok);
        xp = target_row(p, b * p.Tr + lane).at(tok);
    }
    decide_from(p, b, lane, sM, sI, xq, xp);
}

// ------------------------------------------------------------------ vocabulary-parallel form
// Exchange 1 (this rank -> all): per sequence, every row's local (max, sum) and, for
// each candidate, its draft and target logit if this rank owns the token's column
// (NaN otherwise).  Layout per sequence: M[k+Tr], S[k+Tr], xq[k], xp[k].
SDB_DEV int summary_floats(const Params& p) { return 2 * (p.k + p.Tr) + 2 * p.k; }

__global__ void __launch_bounds__(DECIDE_THREADS) vs_summary(const Params p) {
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nd = p.B * p.k;
    const int nrows = p.k + p.Tr;
    float* out = p.send + (int64_t)b * summary_floats(p);
    for (int r = warp; r < nrows; r += DECIDE_THREADS / 32) {
        float2 ms = make_float2(-INFINITY, 0.f);
        if (!(r < p.k && p.point_mass)) {
            const int grow = r < p.k ? b * p.k + r : nd + b * p.Tr + (r - p.k);
            ms = merge_row_stats(p, grow, lane);
        }
        if (lane == 0) {
            out[r] = ms.x;
            out[nrows + r] = ms.y;
        }
    }
    if (warp == 0 && lane < p.k) {
        const int64_t tok = candidate_token(p, b, lane);
        const bool own = tok >= p.col0 && tok < (int64_t)p.col0 + p.V;
        out[2 * nrows + lane] = own ? draft_row(p, b * p.k + lane).at(tok - p.col0) : __int_as_float(0x7fc00000);
        out[2 * nrows + p.k + lane] = own ? target_row(p, b * p.Tr + lane).at(tok - p.col0) : __int_as_float(0x7fc00000);
    }
}

// After exchange 1: every rank merges the tp summaries in rank order (so all ranks hold
// identical statistics) and makes the same decisions.  One warp per sequence.
__global__ void __launch_bounds__(32) vs_decide_shard(const Params p) {
    __shared__ float sM[65], sI[65];
    const int b = blockIdx.x, lane = threadIdx.x;
    const int nrows = p.k + p.Tr, F = summary_floats(p);
    for (int r = lane; r < nrows; r += 32) {
        float M = -INFINITY;
        for (int t = 0; t < p.tp; ++t) M = fmaxf(M, p.gathered[((int64_t)t * p.B + b) * F + r]);
        float S = 0.f;
        for (int t = 0; t < p.tp; ++t) {
            const float* g = p.gathered + ((int64_t)t * p.B + b) * F;
            if (g[r] != -INFINITY) S += g[nrows + r] * expf(g[r] - M);
        }
        sM[r] = M;
        sI[r] = 1.0f / S;
    }
    __syncwarp();
    float xq = 0.f, xp = 0.f;
    if (lane < p.k) {
        candidate_token(p, b, lane);  // the range check
        for (int t = 0; t < p.tp; ++t) {  // exactly one rank owns the column
            const float* g = p.gathered + ((int64_t)t * p.B + b) * F;
            const float q = g[2 * nrows + lane], x = g[2 * nrows + p.k + lane];
            if (!isnan(x)) {
                xq = q;
                xp = x;
            }
        }
    }
    decide_from(p, b, lane, sM, sI, xq, xp);
}

// Exchange 2: this rank's residual and p sums of row a (the chunk sums of pass 3).
__global__ void __launch_bounds__(256) vs_rsum_total(const Params p) {
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= p.B) return;
    float sr = 0.f, sp = 0.f;
    for (int cc = lane; cc < p.C2; cc += 32) {
        const float2 v = __ldcg(p.rsum + b * p.C2 + cc);
        sr += v.x;
        sp += v.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sr += __shfl_xor_sync(0xffffffffu, sr, o);
        sp += __shfl_xor_sync(0xffffffffu, sp, o);
    }
    if (lane == 0) {
        p.send[2 * b] = sr;
        p.send[2 * b + 1] = sp;
    }
}

// After exchange 3 (each rank's (best value, global column) of the bonus argmax): the
// first index among the largest values, ranks holding increasing column ranges.
__global__ void vs_bonus_finish(const Params p) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= p.B) return;
    float gb = -INFINITY;
    int gi = 0x7fffffff;
    for (int t = 0; t < p.tp; ++t) {
        const float v = p.gathered[((int64_t)t * p.B + b) * 2];
        const int i = __float_as_int(p.gathered[((int64_t)t * p.B + b) * 2 + 1]);
        if (v > gb || (v == gb && i < gi)) {
            gb = v;
            gi = i;
        }
    }
    p.out_bonus[b] = gi == 0x7fffffff ? 0 : gi;
}

// resid_i and p_i of row a (verify.py:141-148): q_pad[k] = 0, p index clamped.
// UNIT: temperature 1 (x / T is x); the callers branch once per CTA so no division
// is evaluated for the common case.
template <bool UNIT>
SDB_DEV void resid_of(const Params& p, const Decision& d, float T, float xt, float xd, float& r, float& pv) {
    pv = expf((UNIT ? xt : __fdiv_rn(xt, T)) - d.Mp) * d.ip;
    float qv = 0.f;
    if (d.a < p.k) qv = p.point_mass ? xd : expf((UNIT ? xd : __fdiv_rn(xd, T)) - d.Mq) * d.iq;
    r = fmaxf(pv - qv, 0.f);
}

SDB_DEV Decision load_decision(const Params& p, int b) {
    const int* src = reinterpret_cast<const int*>(p.dec + b);
    Decision d;
    int* dst = reinterpret_cast<int*>(&d);
#pragma unroll
    for (int i = 0; i < (int)(sizeof(Decision) / 4); ++i) dst[i] = __ldcg(src + i);
    return d;
}

// Row a of the target (clamped) and of the draft (none when a == k) for sequence b.
SDB_DEV Row target_row_a(const Params& p, int b, const Decision& d) {
    return target_row(p, b * p.Tr + min(d.a, p.Tr - 1));
}
SDB_DEV Row draft_row_a(const Params& p, int b, const Decision& d) {
    return d.a < p.k ? draft_row(p, b * p.k + d.a) : Row{nullptr, p.dkind};
}

// Visits the logits of this CTA's chunk of row a as (index, target logit, draft
// logit): float4 loads issued together when V % 4 == 0, scalar loads otherwise.
template <typename F>
SDB_DEV void for_chunk(const Params& p, const Row& tr, const Row& dr, int base, F f) {
    const int n = min(CHUNK2, p.V - base);
    if (p.vec) {
        float4 xt[EPT2 / 4], xd[EPT2 / 4];
#pragma unroll
        for (int it = 0; it < EPT2 / 4; ++it) {
            xt[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            xd[it] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q2 = 0; q2 < EPT2 / 8; ++q2) {
            const int idx = group_col(2 * q2);
            if (idx < n) {
                tr.at8(base + idx, n - idx, xt[2 * q2], xt[2 * q2 + 1]);
                if (dr.p) dr.at8(base + idx, n - idx, xd[2 * q2], xd[2 * q2 + 1]);
            }
        }
#pragma unroll
        for (int it = 0; it < EPT2 / 4; ++it) {
            const int idx = group_col(it);
            if (idx < n) f(base + idx, xt[it], xd[it]);
        }
    } else {
        for (int idx = threadIdx.x; idx < n; idx += THREADS) {
            const float4 t1 = make_float4(tr.at(base + idx), 0.f, 0.f, 0.f);
            const float4 d1 = make_float4(dr.p ? dr.at(base + idx) : 0.f, 0.f, 0.f, 0.f);
            f(base + idx, t1, d1);  // only .x is meaningful: lanes of one logit
        }
    }
}

// ------------------------------------------------------------------ pass 3
__global__ void __launch_bounds__(THREADS) vs_resid_sums(const Params p) {
    __shared__ float sh[THREADS / 32];
    const int b = blockIdx.x, c = blockIdx.y;
    const Decision d = load_decision(p, b);
    const float T = p.temps ? p.temps[b] : 1.0f;
    const Row tr = target_row_a(p, b, d);
    const Row dr = draft_row_a(p, b, d);
    const int cnt = p.vec ? 4 : 1;
    float sr = 0.f, sp = 0.f;
    auto body = [&](auto unit) {
        for_chunk(p, tr, dr, c * CHUNK2, [&](int, const float4& xt, const float4& xd) {
            const float t4[4] = {xt.x, xt.y, xt.z, xt.w}, d4[4] = {xd.x, xd.y, xd.z, xd.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < cnt) {
                    float r, pv;
                    resid_of<decltype(unit)::value>(p, d, T, t4[e], d4[e], r, pv);
                    sr += r;
                    sp += pv;
                }
        });
    };
    if (T == 1.0f) body(std::true_type{});
    else body(std::false_type{});
    sr = block_reduce(sr, [](float a, float b2) { return a + b2; }, sh);
    sp = block_reduce(sp, [](float a, float b2) { return a + b2; }, sh);
    if (threadIdx.x == 0) __stcg(p.rsum + b * p.C2 + c, make_float2(sr, sp));
}

SDB_DEV bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// max(E, 1e-10) for global columns i .. i + cnt - 1 of sequence b (cnt = 4: i % 4 == 0,
// one Philox block gives the four words).
SDB_DEV void exp_noise4(const Params& p, int b, int i, int cnt, float (&E)[4]) {
    if (p.e) {
#pragma unroll
        for (int e = 0; e < 4; ++e) E[e] = e < cnt ? p.e[(int64_t)b * p.Vg + i + e] : 1.f;
    } else if (cnt == 4) {
        uint32_t c[4] = {(uint32_t)i >> 2, (uint32_t)b, 1u, draw_offset(p)};
        philox(c, p.seed_lo, p.seed_hi);
#pragma unroll
        for (int e = 0; e < 4; ++e) E[e] = -log_fixed(word_to_open_uniform(c[e]));
    } else {
        E[0] = -log_fixed(word_to_open_uniform(philox_word(p.seed_lo, p.seed_hi, draw_offset(p), 1u, (uint32_t)b, (uint32_t)i)));
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) E[e] = fmaxf(E[e], 1e-10f);  // clamp_min_(1e-10), verify.py:209
}

// ------------------------------------------------------------------ pass 4
__global__ void __launch_bounds__(THREADS) vs_bonus(const Params p) {
    __shared__ float zsh;
    __shared__ int use_p;
    __shared__ float bv[THREADS / 32];
    __shared__ int bi[THREADS / 32];
    const int b = blockIdx.x, c = blockIdx.y;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (threadIdx.x < 32) {  // the chunk sums of pass 3 (every rank's totals in the
                             // vocabulary-parallel form), loaded by all lanes at once
        float sr = 0.f, sp = 0.f;
        if (p.shard) {
            for (int t = lane; t < p.tp; t += 32) {
                sr += p.gathered[((int64_t)t * p.B + b) * 2];
                sp += p.gathered[((int64_t)t * p.B + b) * 2 + 1];
            }
        } else {
            for (int cc = lane; cc < p.C2; cc += 32) {
                const float2 v = __ldcg(p.rsum + b * p.C2 + cc);
                sr += v.x;
                sp += v.y;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sr += __shfl_xor_sync(0xffffffffu, sr, o);
            sp += __shfl_xor_sync(0xffffffffu, sp, o);
        }
        if (lane == 0) {
            use_p = !(sr > 0.f);                   // fallback to p[a], verify.py:151
            zsh = fmaxf(use_p ? sp : sr, 1e-10f);  // normaliser, verify.py:152
        }
    }
    __syncthreads();
    const Decision d = load_decision(p, b);
    const float T = p.temps ? p.temps[b] : 1.0f;
    const float Z = zsh;
    const bool up = use_p != 0;
    const Row tr = target_row_a(p, b, d);
    const Row dr = draft_row_a(p, b, d);
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    // Exact value of column i: (v / Z) / max(E, 1e-10) with v = p[a] or resid[a].
    auto exact = [&](auto unit, int i, float xt, float xd, float E) {
        float r, pv;
        resid_of<decltype(unit)::value>(p, d, T, xt, xd, r, pv);
        const float v = up ? pv : r;
        const float x = v != 0.f ? __fdiv_rn(__fdiv_rn(v, Z), E) : 0.f;  // 0 / Z / E is +0
        if (better(x, p.col0 + i, best, bidx)) {  // global column
            best = x;
            bidx = p.col0 + i;
        }
    };
    auto body = [&](auto unit) {
        if (!p.vec) {
            for_chunk(p, tr, dr, c * CHUNK2, [&](int i, const float4& xt, const float4& xd) {
                float E[4];
                exp_noise4(p, b, p.col0 + i, 1, E);
                exact(unit, i, xt.x, xd.x, E[0]);
            });
            return;
        }
        // vector form: every lane holds 16 columns (4 runs of 4).  Cheap bounds first:
        // v in [v_lo, v_hi] from fast exponentials (within 2^-10 of expf above
        // exponent -8192; the residual max(p - q, 0) from p_lo - q_hi and p_hi) and
        // E = max(-log U, 1e-10) in [max(1 - U, 1e-10), max((1 - U) / U, 1e-10)].  The
        // warp's largest v_lo / E_hi is a lower bound of its best value; only columns
        // whose v_hi / E_lo reaches it are evaluated exactly, and the others are
        // strictly below an evaluated one, so the argmax (first index on ties) is the
        // one of the exact values.  The winner has U near 1, where the E bounds meet.
        const int base = c * CHUNK2;
        const int n = min(CHUNK2, p.V - base);
        float4 xt[EPT2 / 4], xd[EPT2 / 4];
#pragma unroll
        for (int q = 0; q < EPT2 / 4; ++q) {
            xt[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            xd[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q2 = 0; q2 < EPT2 / 8; ++q2) {
            const int idx = group_col(2 * q2);
            if (idx < n) {
                tr.at8(base + idx, n - idx, xt[2 * q2], xt[2 * q2 + 1]);
                if (dr.p) dr.at8(base + idx, n - idx, xd[2 * q2], xd[2 * q2 + 1]);
            }
        }
        constexpr float kLog2e = 1.4426950408889634f;
        const bool has_q = d.a < p.k;
        float vhi[EPT2], elo[EPT2];
        float lbmax = 0.f;
#pragma unroll
        for (int q = 0; q < EPT2 / 4; ++q) {
            const int idx = group_col(q);
            const bool in = idx < n;
            const float t4[4] = {xt[q].x, xt[q].y, xt[q].z, xt[q].w};
            const float d4[4] = {xd[q].x, xd[q].y, xd[q].z, xd[q].w};
            uint32_t w4[4] = {(uint32_t)(p.col0 + base + idx) >> 2, (uint32_t)b, 1u, draw_offset(p)};
            if (!p.e && in) philox(w4, p.seed_lo, p.seed_hi);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * q + e;
                float Elo, Ehi;
                if (p.e) {
                    Elo = Ehi = in ? fmaxf(p.e[(int64_t)b * p.Vg + p.col0 + base + idx + e], 1e-10f) : 1.f;
                } else {
                    // -log U in [1 - U, (1 - U)(3 - 2U)] for U >= 1/2 and <= 17 always
                    // (U >= 2^-24); 1 - U is exact (U is a multiple of 2^-24); the factors
                    // cover the few ulps by which log_fixed may sit on either side
                    const float U = word_to_open_uniform(w4[e]);
                    Elo = fmaxf((1.0f - U) * 0.99999f, 1e-10f);
                    Ehi = U >= 0.5f ? fmaxf((1.0f - U) * (3.0f - 2.0f * U) * 1.00002f, 1e-10f) : 17.0f;
                }
                const float xs = decltype(unit)::value ? t4[e] : __fdiv_rn(t4[e], T);
                const float pf = ex2((xs - d.Mp) * kLog2e) * d.ip;
                float hi = fmaxf(pf * 1.001f, FLT_MIN);
                float lo = pf * 0.999f;
                if (!up && has_q) {
                    const float xq = decltype(unit)::value || p.point_mass ? d4[e] : __fdiv_rn(d4[e], T);
                    const float qf = p.point_mass ? xq : ex2((xq - d.Mq) * kLog2e) * d.iq;
                    lo = fmaxf(lo - fmaxf(qf * 1.001f, FLT_MIN), 0.f);
                    if (p.point_mass) hi += fmaxf(-qf, 0.f) * 1.001f;  // a negative draft value raises r
                }
                vhi[j] = in ? hi : -1.f;
                elo[j] = Elo;
                if (in) lbmax = fmaxf(lbmax, __fdividef(lo, Ehi) * 0.9999f);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lbmax = fmaxf(lbmax, __shfl_xor_sync(0xffffffffu, lbmax, o));
        const float thr = lbmax * 0.9999f;  // slack for the rounding of these bounds
        uint32_t live = 0;  // columns whose v_hi / E_lo reaches the threshold
#pragma unroll
        for (int j = 0; j < EPT2; ++j)
            if (vhi[j] >= 0.f && !(vhi[j] < thr * elo[j])) live |= 1u << j;
        // the exact evaluation exists once in the code (not per unrolled column): the
        // few live columns reload their two logits from cache
        while (live) {
            const int j = __ffs(live) - 1;
            live &= live - 1;
            const int i = base + group_col(j >> 2) + (j & 3);
            const float E = p.e ? fmaxf(p.e[(int64_t)b * p.Vg + p.col0 + i], 1e-10f)
                                : fmaxf(-log_fixed(word_to_open_uniform(philox_word(
                                            p.seed_lo, p.seed_hi, draw_offset(p), 1u, (uint32_t)b, (uint32_t)(p.col0 + i)))),
                                        1e-10f);
            exact(unit, i, tr.at(i), dr.p ? dr.at(i) : 0.f, E);
        }
    };
    if (T == 1.0f) body(std::true_type{});
    else body(std::false_type{});
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, s);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, s);
        if (better(ov, oi, best, bidx)) {
            best = ov;
            bidx = oi;
        }
    }
    if (lane == 0) {
        bv[w] = best;
        bi[w] = bidx;
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    __shared__ int last;
    if (lane == 0) {
        for (int i = 1; i < THREADS / 32; ++i)
            if (better(bv[i], bi[i], best, bidx)) {
                best = bv[i];
                bidx = bi[i];
            }
        __stcg(p.amax + b * p.C2 + c, make_float2(best, __int_as_float(bidx)));
        __threadfence();
        last = atomicAdd(p.counters + b, 1) == p.C2 - 1;
    }
    __syncwarp();
    if (!last) return;
    // last CTA of sequence b: finish the argmax (first index on ties, torch.argmax)
    __threadfence();
    float gb = -INFINITY;
    int gi = 0x7fffffff;
    for (int cc = lane; cc < p.C2; cc += 32) {
        const float2 v = __ldcg(p.amax + b * p.C2 + cc);
        const int vi = __float_as_int(v.y);
        if (better(v.x, vi, gb, gi)) {
            gb = v.x;
            gi = vi;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, gb, o);
        const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
        if (better(ov, oi, gb, gi)) {
            gb = ov;
            gi = oi;
        }
    }
    if (lane == 0) {
        if (p.shard) {  // exchange 3: this rank's best value and its global column
            p.send[2 * b] = gb;
            p.send[2 * b + 1] = __int_as_float(gi);
        } else {
            p.out_bonus[b] = gi == 0x7fffffff ? 0 : gi;
        }
        p.counters[b] = 0;
    }
}

// ------------------------------------------------------------------ passes 3 + 4 fused
// One read of row a (single device, vector form).  Per chunk: the residual and p sums in
// the order of vs_resid_sums (so the normaliser Z is the same float), and the columns
// that can hold the chunk's bonus argmax without knowing Z.  With exact v (the residual)
// and exact E the bonus value is x = fl(fl(v / Z) / E), i.e. y = v / E times the positive
// constant 1 / Z up to a relative 2^-23; so a column with fl(v / E) below the chunk's
// best by more than the band 2^-20 cannot be the argmax, and the kept columns (normally
// one) are re-evaluated exactly once Z is known.  E comes from the Philox word alone as
// bounds (as in vs_bonus), exactly only for columns whose bound reaches the chunk's
// lower bound.  A chunk whose residuals are all zero keeps its first column (every x
// there is 0); a chunk with more than RB_CAP candidates or RB_LIVE live columns, and the
// p fallback (zero residual mass, verify.py:151), are evaluated in full by the last CTA
// of the sequence, which writes the bonus token.
__global__ void __launch_bounds__(THREADS) vs_resid_bonus(const Params p) {
    __shared__ float sh[THREADS / 32];
    __shared__ int nlive, nkeep, last;
    __shared__ int live_col[RB_LIVE];
    __shared__ float live_y[RB_LIVE];
    __shared__ float zsh;
    __shared__ int use_p, any_ovf;
    __shared__ float bv[THREADS / 32];
    __shared__ int bi[THREADS / 32];
    const int b = blockIdx.x, c = blockIdx.y;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        nlive = 0;
        nkeep = 0;
        any_ovf = 0;
    }
    const Decision d = load_decision(p, b);
    const float T = p.temps ? p.temps[b] : 1.0f;
    const Row tr = target_row_a(p, b, d);
    const Row dr = draft_row_a(p, b, d);
    const int base = c * CHUNK2;
    const int n = min(CHUNK2, p.V - base);
    float4 xt[EPT2 / 4], xd[EPT2 / 4];
#pragma unroll
    for (int q = 0; q < EPT2 / 4; ++q) {
        xt[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        xd[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int q2 = 0; q2 < EPT2 / 8; ++q2) {
        const int idx = group_col(2 * q2);
        if (idx < n) {
            tr.at8(base + idx, n - idx, xt[2 * q2], xt[2 * q2 + 1]);
            if (dr.p) dr.at8(base + idx, n - idx, xd[2 * q2], xd[2 * q2 + 1]);
        }
    }
    float sr = 0.f, sp = 0.f;
    float rv[EPT2], yhi[EPT2];
    float lbmax = 0.f;
    auto sweep = [&](auto unit) {
#pragma unroll
        for (int q = 0; q < EPT2 / 4; ++q) {
            const int idx = group_col(q);
            const bool in = idx < n;
            const float t4[4] = {xt[q].x, xt[q].y, xt[q].z, xt[q].w};
            const float d4[4] = {xd[q].x, xd[q].y, xd[q].z, xd[q].w};
            uint32_t w4[4] = {(uint32_t)(base + idx) >> 2, (uint32_t)b, 1u, draw_offset(p)};
            if (!p.e && in) philox(w4, p.seed_lo, p.seed_hi);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * q + e;
                float r = 0.f, pv = 0.f;
                if (in) {
                    resid_of<decltype(unit)::value>(p, d, T, t4[e], d4[e], r, pv);
                    sr += r;
                    sp += pv;
                }
                float Elo, Ehi;
                if (p.e) {
                    Elo = Ehi = in ? fmaxf(p.e[(int64_t)b * p.Vg + base + idx + e], 1e-10f) : 1.f;
                } else {
                    // -log U in [1 - U, (1 - U)(3 - 2U)] for U >= 1/2 and <= 17 always (see vs_bonus)
                    const float U = word_to_open_uniform(w4[e]);
                    Elo = fmaxf((1.0f - U) * 0.99999f, 1e-10f);
                    Ehi = U >= 0.5f ? fmaxf((1.0f - U) * (3.0f - 2.0f * U) * 1.00002f, 1e-10f) : 17.0f;
                }
                rv[j] = in ? r : -1.f;
                yhi[j] = in ? __fdividef(r, Elo) * 1.0001f : -1.f;
                if (in) lbmax = fmaxf(lbmax, __fdividef(r, Ehi) * 0.9999f);
            }
        }
    };
    if (T == 1.0f) sweep(std::true_type{});
    else sweep(std::false_type{});
    // chunk sums, reduced as vs_resid_sums reduces them
    const float csr = block_reduce(sr, [](float a, float b2) { return a + b2; }, sh);
    const float csp = block_reduce(sp, [](float a, float b2) { return a + b2; }, sh);
    const float LB = block_reduce(lbmax, [](float a, float b2) { return fmaxf(a, b2); }, sh);
    float ymax_hi = -1.f;
#pragma unroll
    for (int j = 0; j < EPT2; ++j) ymax_hi = fmaxf(ymax_hi, yhi[j]);
    const float YH = block_reduce(ymax_hi, [](float a, float b2) { return fmaxf(a, b2); }, sh);
    float rpos = 0.f;
#pragma unroll
    for (int j = 0; j < EPT2; ++j) rpos = fmaxf(rpos, rv[j]);
    // a positive residual whose bounds underflowed to 0: evaluate the chunk in full
    bool overflow = YH <= 0.f && block_reduce(rpos, [](float a, float b2) { return fmaxf(a, b2); }, sh) > 0.f;
    if (YH > 0.f) {
        // live columns: an upper bound of v / E that reaches the chunk's lower bound
        const float thr = LB * 0.9999f;
#pragma unroll
        for (int j = 0; j < EPT2; ++j) {
            if (rv[j] > 0.f && yhi[j] >= thr) {
                const int col = base + group_col(j >> 2) + (j & 3);
                const int slot = atomicAdd(&nlive, 1);
                if (slot < RB_LIVE) {
                    const float E = p.e ? fmaxf(p.e[(int64_t)b * p.Vg + col], 1e-10f)
                                        : fmaxf(-log_fixed(word_to_open_uniform(philox_word(
                                                    p.seed_lo, p.seed_hi, draw_offset(p), 1u, (uint32_t)b, (uint32_t)col))),
                                                1e-10f);
                    live_col[slot] = col;
                    live_y[slot] = __fdiv_rn(rv[j], E);
                }
            }
        }
        __syncthreads();
        const int nl = nlive;
        if (nl > RB_LIVE) {
            overflow = true;
        } else {
            float ybest = 0.f;
            for (int i = 0; i < nl; ++i) ybest = fmaxf(ybest, live_y[i]);
            const float keep_thr = ybest * (1.0f - 1.0f / (1 << 20));
            if ((int)threadIdx.x < nl && live_y[threadIdx.x] >= keep_thr) {
                const int slot = atomicAdd(&nkeep, 1);
                if (slot < RB_CAP) p.cand[((int64_t)b * p.C2 + c) * RB_CAP + slot] = live_col[threadIdx.x];
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int cnt;
        if (YH > 0.f || overflow) cnt = (overflow || nkeep > RB_CAP) ? RB_CAP + 1 : nkeep;
        else {  // every residual of the chunk is 0: its first column stands for all of them
            p.cand[((int64_t)b * p.C2 + c) * RB_CAP] = base;
            cnt = 1;
        }
        __stcg(p.ncand + b * p.C2 + c, cnt);
        __stcg(p.rsum + b * p.C2 + c, make_float2(csr, csp));
        __threadfence();
        last = atomicAdd(p.counters + b, 1) == p.C2 - 1;
    }
    __syncthreads();
    if (!last) return;
    // ---- last CTA of sequence b: the normaliser, then the exact values of the candidates
    __threadfence();
    if (threadIdx.x < 32) {
        float s1 = 0.f, s2 = 0.f;
        for (int cc = lane; cc < p.C2; cc += 32) {
            const float2 v = __ldcg(p.rsum + b * p.C2 + cc);
            s1 += v.x;
            s2 += v.y;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        if (lane == 0) {
            use_p = !(s1 > 0.f);                   // fallback to p[a], verify.py:151
            zsh = fmaxf(use_p ? s2 : s1, 1e-10f);  // normaliser, verify.py:152
        }
    }
    __syncthreads();
    const float Z = zsh;
    const bool up = use_p != 0;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    auto eval = [&](auto unit, int i) {
        float r, pv;
        resid_of<decltype(unit)::value>(p, d, T, tr.at(i), dr.p ? dr.at(i) : 0.f, r, pv);
        const float v = up ? pv : r;
        const float E = p.e ? fmaxf(p.e[(int64_t)b * p.Vg + i], 1e-10f)
                            : fmaxf(-log_fixed(word_to_open_uniform(
                                        philox_word(p.seed_lo, p.seed_hi, draw_offset(p), 1u, (uint32_t)b, (uint32_t)i))),
                                    1e-10f);
        const float x = v != 0.f ? __fdiv_rn(__fdiv_rn(v, Z), E) : 0.f;  // 0 / Z / E is +0
        if (better(x, i, best, bidx)) {
            best = x;
            bidx = i;
        }
    };
    auto finish = [&](auto unit) {
        if (up) {  // rare: no residual mass; every column of the row, v = p[a]
            for (int i = threadIdx.x; i < p.V; i += THREADS) eval(unit, i);
            return;
        }
        // the kept columns of every chunk, (chunk, slot) pairs spread over the threads
        for (int u = threadIdx.x; u < p.C2 * RB_CAP; u += THREADS) {
            const int cc = u / RB_CAP, sl = u - cc * RB_CAP;
            const int cnt = __ldcg(p.ncand + b * p.C2 + cc);
            if (cnt > RB_CAP) {
                if (sl == 0) any_ovf = 1;
            } else if (sl < cnt) {
                eval(unit, __ldcg(p.cand + ((int64_t)b * p.C2 + cc) * RB_CAP + sl));
            }
        }
        __syncthreads();
        if (!any_ovf) return;
        for (int cc = 0; cc < p.C2; ++cc) {  // rare: ties or a flat chunk; all of its columns
            if (__ldcg(p.ncand + b * p.C2 + cc) <= RB_CAP) continue;
            const int hi = min(p.V, (cc + 1) * CHUNK2);
            for (int i = cc * CHUNK2 + threadIdx.x; i < hi; i += THREADS) eval(unit, i);
        }
    };
    if (T == 1.0f) finish(std::true_type{});
    else finish(std::false_type{});
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (better(ov, oi, best, bidx)) {
            best = ov;
            bidx = oi;
        }
    }
    if (lane == 0) {
        bv[w] = best;
        bi[w] = bidx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < THREADS / 32; ++i)
            if (better(bv[i], bi[i], best, bidx)) {
                best = bv[i];
                bidx = bi[i];
            }
        p.out_bonus[b] = bidx == 0x7fffffff ? 0 : bidx;
        p.counters[b] = 0;  // graph-replay safe: ready for the next call
    }
}

struct WsLayout {
    size_t err, counters, dec, stats, rsum, amax, ncand, cand, total;
};

constexpr int kCounterCap = 1 << 19;  // sequences per call

static WsLayout ws_layout(int B, int k, int Tr, int V) {
    const int C1 = (V + CHUNK1 - 1) / CHUNK1;
    const int C2 = (V + CHUNK2 - 1) / CHUNK2;
    WsLayout w;
    size_t off = 0;
    w.err = off;
    off += 256;
    w.counters = off;  // fixed offset and capacity: never aliased by another call's data
    off = align_up(off + sizeof(int) * (size_t)kCounterCap, 256);
    w.dec = off;
    off = align_up(off + sizeof(Decision) * B, 256);
    w.stats = off;
    off = align_up(off + sizeof(float2) * (size_t)B * (k + Tr) * C1 * SUB, 256);
    w.rsum = off;
    off = align_up(off + sizeof(float2) * (size_t)B * C2, 256);
    w.amax = off;
    off = align_up(off + sizeof(float2) * (size_t)B * C2, 256);
    w.ncand = off;
    off = align_up(off + sizeof(int) * (size_t)B * C2, 256);
    w.cand = off;
    off = align_up(off + sizeof(int) * (size_t)B * C2 * RB_CAP, 256);
    w.total = off;
    return w;
}

__global__ void philox_fill_kernel(float* out, int rows, int cols, uint32_t slo, uint32_t shi, uint32_t off,
                                   int stream) {
    const int64_t n = (int64_t)rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / cols), c = (int)(i % cols);
        const uint32_t w = philox_word(slo, shi, off, (uint32_t)stream, (uint32_t)r, (uint32_t)c);
        out[i] = stream == 0 ? word_to_uniform(w) : -log_fixed(word_to_open_uniform(w));
    }
}

}  // namespace vs
}  // namespace sdb

using namespace sdb;

extern "C" size_t sdb_verify_workspace_size(int B, int k, int target_rows, int V) {
    if (B <= 0 || k <= 0 || target_rows <= 0 || V <= 0) return 256;
    return vs::ws_layout(B, k, target_rows, V).total;
}

namespace {

// Validation and parameter block shared by the single-device and the
// vocabulary-parallel entry points.  V is this rank's column count, [col0, col0 + V)
// its columns of the Vg-wide vocabulary.
int setup(vs::Params& p, const void* draft, int draft_dtype, const void* target, int target_dtype,
          const int64_t* tokens, const float* temps, const float* uniforms, const float* exponentials, uint64_t seed,
          uint64_t offset, int point_mass, int64_t* out_acc, int64_t* out_bonus, uint8_t* out_mask, int B, int k,
          int Tr, int V, int col0, int Vg, void* workspace, size_t workspace_bytes) {
    if (!draft || !target || !tokens || !out_acc || !out_bonus || !out_mask || !workspace) {
        set_last_error("null pointer argument");
        return SDB_ERR_INVALID_ARG;
    }
    if (B <= 0 || B > vs::kCounterCap || k <= 0 || k > 32 || V <= 0 || !(Tr == k || Tr == k + 1) || col0 < 0 ||
        (long long)col0 + V > Vg) {
        set_last_error("bad sizes B=%d k=%d target_rows=%d V=%d columns [%d, %lld) of %d (need B <= %d, "
                       "1<=k<=32, target_rows in {k, k+1})",
                       B, k, Tr, V, col0, (long long)col0 + V, Vg, vs::kCounterCap);
        return SDB_ERR_INVALID_ARG;
    }
    auto kind_of = [](int dt) { return dt == SDB_F32 ? 0 : (dt == SDB_BF16 ? 1 : (dt == SDB_F16 ? 2 : -1)); };
    const int dkind = kind_of(draft_dtype), tkind = kind_of(target_dtype);
    if (dkind < 0 || tkind < 0) {
        set_last_error("logits dtypes %d / %d not supported (float32, bfloat16, float16)", draft_dtype, target_dtype);
        return SDB_ERR_UNSUPPORTED;
    }
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) ||
        ((V & 3) == 0 && ((reinterpret_cast<uintptr_t>(draft) & 15) || (reinterpret_cast<uintptr_t>(target) & 15)))) {
        set_last_error("workspace must be 256-byte aligned and logits 16-byte aligned");
        return SDB_ERR_INVALID_ARG;
    }
    vs::WsLayout w = vs::ws_layout(B, k, Tr, V);
    if (workspace_bytes < w.total) {
        set_last_error("workspace too small: need %zu bytes, got %zu", w.total, workspace_bytes);
        return SDB_ERR_WORKSPACE;
    }
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    p = vs::Params{};
    p.draft = draft;
    p.target = target;
    p.dkind = dkind;
    p.tkind = tkind;
    p.tokens = tokens;
    p.temps = temps;
    p.u = uniforms;
    p.e = exponentials;
    p.seed_lo = (uint32_t)(seed & 0xffffffffu);
    p.seed_hi = (uint32_t)(seed >> 32);
    p.offset = (uint32_t)offset;
    p.point_mass = point_mass ? 1 : 0;
    p.out_acc = out_acc;
    p.out_bonus = out_bonus;
    p.out_mask = out_mask;
    p.B = B;
    p.k = k;
    p.Tr = Tr;
    p.V = V;
    p.col0 = col0;
    p.Vg = Vg;
    p.tp = 1;
    p.C1 = (V + vs::CHUNK1 - 1) / vs::CHUNK1;
    p.C2 = (V + vs::CHUNK2 - 1) / vs::CHUNK2;
    p.err = reinterpret_cast<int*>(ws + w.err);
    p.counters = reinterpret_cast<int*>(ws + w.counters);
    p.dec = reinterpret_cast<vs::Decision*>(ws + w.dec);
    p.stats = reinterpret_cast<float2*>(ws + w.stats);
    p.rsum = reinterpret_cast<float2*>(ws + w.rsum);
    p.amax = reinterpret_cast<float2*>(ws + w.amax);
    p.ncand = reinterpret_cast<int*>(ws + w.ncand);
    p.cand = reinterpret_cast<int*>(ws + w.cand);
    // passes 3-4 read 16-byte vectors when every row they read is 16-byte aligned (the
    // point-mass draft is read too: its residual row) and Philox groups of four columns
    // start on this rank's group boundaries
    p.vec = (V & 3) == 0 && (col0 & 3) == 0 && (dkind == 0 || (V & 7) == 0) && (tkind == 0 || (V & 7) == 0);
    return SDB_OK;
}

// Pass 1 over this rank's rows.
int launch_stats(const vs::Params& p, cudaStream_t st) {
    const int row0 = p.point_mass ? p.B * p.k : 0;
    const int nrows = p.B * ((p.point_mass ? 0 : p.k) + p.Tr);
    // bulk copies need every streamed row to be a whole number of 16-byte units (the
    // bases were checked): V % 4 == 0 for float32 rows, V % 8 == 0 for 16-bit ones
    const bool draft_rows_ok = p.point_mass || ((p.V * (p.dkind == 0 ? 4 : 2)) % 16 == 0);
    const bool target_rows_ok = (p.V * (p.tkind == 0 ? 4 : 2)) % 16 == 0;
    if ((p.V & 3) == 0 && draft_rows_ok && target_rows_ok) {
        int rc = ensure_smem_attr(reinterpret_cast<const void*>(vs::vs_row_stats_bulk), vs::BS_SMEM, 50);
        if (rc) return rc;
        const long long items = (long long)nrows * p.C1;
        const int slots = 2 * device_sm_count();
        const int grid = (int)(items < slots ? items : slots);
        vs::vs_row_stats_bulk<<<grid, vs::BS_THREADS, vs::BS_SMEM, st>>>(p, row0, nrows);
        return cuda_status(cudaGetLastError(), "vs_row_stats_bulk launch");
    }
    vs::vs_row_stats<<<dim3(nrows, p.C1), vs::THREADS, 0, st>>>(p);
    return cuda_status(cudaGetLastError(), "vs_row_stats launch");
}

}  // namespace

namespace {
int verify_impl(const void* draft, int draft_dtype, const void* target, int target_dtype, const int64_t* tokens,
                const float* temps, const float* uniforms, const float* exponentials, uint64_t seed, uint64_t offset,
                uint64_t* offset_dev, int point_mass, int64_t* out_acc, int64_t* out_bonus, uint8_t* out_mask, int B,
                int k, int Tr, int V, void* workspace, size_t workspace_bytes, cudaStream_t st);
}  // namespace

extern "C" int sdb_verify_batch_ex(const void* draft, int draft_dtype, const void* target, int target_dtype,
                                   const int64_t* tokens, const float* temps, const float* uniforms,
                                   const float* exponentials, uint64_t seed, uint64_t offset, int point_mass,
                                   int64_t* out_acc, int64_t* out_bonus, uint8_t* out_mask, int B, int k, int Tr,
                                   int V, void* workspace, size_t workspace_bytes, void* stream) {
    return verify_impl(draft, draft_dtype, target, target_dtype, tokens, temps, uniforms, exponentials, seed, offset,
                       nullptr, point_mass, out_acc, out_bonus, out_mask, B, k, Tr, V, workspace, workspace_bytes,
                       reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sdb_verify_batch_dev_offset(const void* draft, int draft_dtype, const void* target, int target_dtype,
                                           const int64_t* tokens, const float* temps, uint64_t seed,
                                           uint64_t* offset_dev, int point_mass, int64_t* out_acc,
                                           int64_t* out_bonus, uint8_t* out_mask, int B, int k, int Tr, int V,
                                           void* workspace, size_t workspace_bytes, void* stream) {
    if (!offset_dev || (reinterpret_cast<uintptr_t>(offset_dev) & 7)) {
        set_last_error("sdb_verify_batch_dev_offset needs an 8-byte aligned device offset");
        return SDB_ERR_INVALID_ARG;
    }
    return verify_impl(draft, draft_dtype, target, target_dtype, tokens, temps, nullptr, nullptr, seed, 0, offset_dev,
                       point_mass, out_acc, out_bonus, out_mask, B, k, Tr, V, workspace, workspace_bytes,
                       reinterpret_cast<cudaStream_t>(stream));
}

namespace {
int verify_impl(const void* draft, int draft_dtype, const void* target, int target_dtype, const int64_t* tokens,
                const float* temps, const float* uniforms, const float* exponentials, uint64_t seed, uint64_t offset,
                uint64_t* offset_dev, int point_mass, int64_t* out_acc, int64_t* out_bonus, uint8_t* out_mask, int B,
                int k, int Tr, int V, void* workspace, size_t workspace_bytes, cudaStream_t st) {
    vs::Params p;
    int rc = setup(p, draft, draft_dtype, target, target_dtype, tokens, temps, uniforms, exponentials, seed, offset,
                   point_mass, out_acc, out_bonus, out_mask, B, k, Tr, V, 0, V, workspace, workspace_bytes);
    if (rc) return rc;
    p.offset_dev = offset_dev;
    rc = launch_stats(p, st);
    if (rc) return rc;
    vs::vs_decide<<<B, vs::DECIDE_THREADS, 0, st>>>(p);
    rc = cuda_status(cudaGetLastError(), "vs_decide launch");
    if (rc) return rc;
    if (p.vec) {  // one pass over row a: sums, candidates, and the bonus by the last CTA
        vs::vs_resid_bonus<<<dim3(B, p.C2), vs::THREADS, 0, st>>>(p);
        rc = cuda_status(cudaGetLastError(), "vs_resid_bonus launch");
    } else {
        vs::vs_resid_sums<<<dim3(B, p.C2), vs::THREADS, 0, st>>>(p);
        rc = cuda_status(cudaGetLastError(), "vs_resid_sums launch");
        if (rc) return rc;
        vs::vs_bonus<<<dim3(B, p.C2), vs::THREADS, 0, st>>>(p);
        rc = cuda_status(cudaGetLastError(), "vs_bonus launch");
    }
    if (rc || !offset_dev) return rc;
    return launch_advance_offset(offset_dev, st);
}
}  // namespace

extern "C" size_t sdb_verify_shard_send_floats(int B, int k, int target_rows, int phase) {
    if (B <= 0 || k <= 0 || target_rows <= 0) return 0;
    if (phase == 1) return (size_t)B * (2 * (k + target_rows) + 2 * k);
    if (phase == 2 || phase == 3) return (size_t)B * 2;
    return 0;
}

extern "C" int sdb_verify_batch_shard(int phase, const void* draft, int draft_dtype, const void* target,
                                      int target_dtype, const int64_t* tokens, const float* temps,
                                      const float* uniforms, const float* exponentials, uint64_t seed,
                                      uint64_t offset, int point_mass, int64_t* out_acc, int64_t* out_bonus,
                                      uint8_t* out_mask, int B, int k, int Tr, int V_local, int vocab_start,
                                      int V_total, int tp, const float* gathered, float* send, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    if (phase < 1 || phase > 4 || tp < 1 || (phase > 1 && !gathered) || (phase < 4 && !send)) {
        set_last_error("bad phase %d / tp %d / exchange buffers for sdb_verify_batch_shard", phase, tp);
        return SDB_ERR_INVALID_ARG;
    }
    vs::Params p;
    int rc = setup(p, draft, draft_dtype, target, target_dtype, tokens, temps, uniforms, exponentials, seed, offset,
                   point_mass, out_acc, out_bonus, out_mask, B, k, Tr, V_local, vocab_start, V_total, workspace,
                   workspace_bytes);
    if (rc) return rc;
    p.tp = tp;
    p.shard = 1;
    p.gathered = gathered;
    p.send = send;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (phase) {
        case 1:  // local statistics -> exchange 1
            rc = launch_stats(p, st);
            if (rc) return rc;
            vs::vs_summary<<<B, vs::DECIDE_THREADS, 0, st>>>(p);
            return cuda_status(cudaGetLastError(), "vs_summary launch");
        case 2:  // decisions from exchange 1, local residual sums -> exchange 2
            vs::vs_decide_shard<<<B, 32, 0, st>>>(p);
            rc = cuda_status(cudaGetLastError(), "vs_decide_shard launch");
            if (rc) return rc;
            vs::vs_resid_sums<<<dim3(B, p.C2), vs::THREADS, 0, st>>>(p);
            rc = cuda_status(cudaGetLastError(), "vs_resid_sums launch");
            if (rc) return rc;
            vs::vs_rsum_total<<<(B + 7) / 8, 256, 0, st>>>(p);
            return cuda_status(cudaGetLastError(), "vs_rsum_total launch");
        case 3:  // local bonus argmax with the global normaliser of exchange 2 -> exchange 3
            vs::vs_bonus<<<dim3(B, p.C2), vs::THREADS, 0, st>>>(p);
            return cuda_status(cudaGetLastError(), "vs_bonus launch");
        default:  // the bonus token from exchange 3
            vs::vs_bonus_finish<<<(B + 127) / 128, 128, 0, st>>>(p);
            return cuda_status(cudaGetLastError(), "vs_bonus_finish launch");
    }
}

extern "C" int sdb_verify_batch(const float* draft, const float* target, const int64_t* tokens, const float* temps,
                                const float* uniforms, const float* exponentials, uint64_t seed, uint64_t offset,
                                int point_mass, int64_t* out_acc, int64_t* out_bonus, uint8_t* out_mask, int B,
                                int k, int Tr, int V, void* workspace, size_t workspace_bytes, void* stream) {
    return sdb_verify_batch_ex(draft, SDB_F32, target, SDB_F32, tokens, temps, uniforms, exponentials, seed, offset,
                               point_mass, out_acc, out_bonus, out_mask, B, k, Tr, V, workspace, workspace_bytes,
                               stream);
}

extern "C" int sdb_philox_fill(float* out, int rows, int cols, uint64_t seed, uint64_t offset, int stream_id,
                               void* stream) {
    if (!out || rows <= 0 || cols <= 0 || stream_id < 0 || stream_id > 2) {
        set_last_error("bad arguments to sdb_philox_fill");
        return SDB_ERR_INVALID_ARG;
    }
    const int64_t n = (int64_t)rows * cols;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    vs::philox_fill_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        out, rows, cols, (uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32), (uint32_t)offset, stream_id);
    return cuda_status(cudaGetLastError(), "philox_fill launch");
}
