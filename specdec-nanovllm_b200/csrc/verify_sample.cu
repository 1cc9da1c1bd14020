// verify_batch rejection sampling on B200 (sm_100a).
//
// Reference: nanovllm/spec_decode/verify.py:42-209.  Same arithmetic, three
// launches instead of ~8 passes of generic torch kernels plus a q_pad copy:
//
//   1. vs_row_stats   grid (rows, chunks): per chunk of every draft and target
//      row, max and sum of exp(x/T - max) from values held in registers
//      (one HBM read of every logit -- the floor of this path).
//   2. vs_resid_sums  grid (B, chunks): every CTA merges the row statistics of
//      its sequence, recomputes the k acceptance decisions (candidate j against
//      target row j, ratio = min(1, p/q), u < ratio, verify.py:109-129) and sums
//      resid = max(p[a] - q_pad[a], 0) and p[a] over its chunk of row a = accepted
//      (verify.py:141-151).
//   3. vs_bonus       grid (B, chunks): partial argmax of (resid / Z) / max(E, 1e-10)
//      (verify.py:152, :167, :203-209), first index on ties; the last CTA of a
//      sequence (atomic counter, reset after use) finishes the argmax and writes
//      accepted / accept_mask / bonus.
//
// The draws: acceptance uniforms u[b, j] and exponentials E[b, i] are either
// caller-provided (parity with the reference given identical draws) or
// generated in-kernel from Philox4x32-10 (Salmon et al., SC'11), stream 0 / 1,
// counter (col/4, row, stream, offset), key (seed lo, seed hi), with
// E = -log(U), U = ((w >> 8) + 1) * 2^-24, and log computed by a fixed
// sequence of correctly rounded float32 operations (no contraction) so a CPU
// restatement reproduces every bit.
#include <cfloat>

#include "common.cuh"

namespace sdb {
namespace vs {

constexpr int THREADS = 256;
constexpr int EPT = 64;                    // logits per thread held in registers (pass 1)
constexpr int CHUNK1 = THREADS * EPT;      // 16384 logits per CTA in pass 1
constexpr int CHUNK2 = THREADS * 32;       // 8192 logits per CTA in passes 2-3

struct Params {
    const float* draft;    // (B, k, V)
    const float* target;   // (B, Tr, V)
    const int64_t* tokens; // (B, k)
    const float* temps;    // (B) or null
    const float* u;        // (B, k) or null
    const float* e;        // (B, V) or null
    uint32_t seed_lo, seed_hi, offset;
    int point_mass;
    int64_t* out_acc;
    int64_t* out_bonus;
    uint8_t* out_mask;
    int B, k, Tr, V, C1, C2;
    float2* stats;         // [rows][C1]  (max, sumexp)
    float2* rsum;          // [B][C2]     (sum resid, sum p[a])
    float2* amax;          // [B][C2]     (value, index as float bits)
    int* counters;         // [B], zero between calls
    struct Decision* dec;  // [B]
    int* err;
};

// ------------------------------------------------------------------ Philox
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

SDB_DEV float exp_noise(const Params& p, int b, int i) {
    float E;
    if (p.e) {
        E = p.e[(int64_t)b * p.V + i];
    } else {
        const uint32_t w = philox_word(p.seed_lo, p.seed_hi, p.offset, 1u, (uint32_t)b, (uint32_t)i);
        E = -log_fixed(word_to_open_uniform(w));
    }
    return fmaxf(E, 1e-10f);  // clamp_min_(1e-10), verify.py:209
}

SDB_DEV float accept_uniform(const Params& p, int b, int j) {
    if (p.u) return p.u[b * p.k + j];
    return word_to_uniform(philox_word(p.seed_lo, p.seed_hi, p.offset, 0u, (uint32_t)b, (uint32_t)j));
}

// x / T exactly as torch divides (IEEE); T == 1 is the identity.
SDB_DEV float scale_t(float x, float T) { return T == 1.0f ? x : __fdiv_rn(x, T); }

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

// Merged (max, 1/sum) of one row from its per-chunk statistics.
SDB_DEV void row_norm(const Params& p, int row, float& M, float& inv) {
    const float2* st = p.stats + (int64_t)row * p.C1;
    M = -INFINITY;
    for (int c = 0; c < p.C1; ++c) M = fmaxf(M, __ldcg(st + c).x);
    float S = 0.f;
    for (int c = 0; c < p.C1; ++c) {
        const float2 v = __ldcg(st + c);
        if (v.x != -INFINITY) S += v.y * expf(v.x - M);
    }
    inv = 1.0f / S;
}

// The k acceptance decisions of sequence b, one candidate per lane (warp-wide).
// ratio = where(q_tok > 0, min(p_tok / max(q_tok, 1e-10), 1), 0); accept = u < ratio
// (verify.py:109-121); accepted = first rejection or k (:125-129).
SDB_DEV void decide_warp(const Params& p, int b, Decision* out) {
    const int lane = threadIdx.x & 31;
    const int nd = p.B * p.k;
    const float T = p.temps ? p.temps[b] : 1.0f;
    bool acc = true;
    if (lane < p.k) {
        int64_t tok = p.tokens[b * p.k + lane];
        if (tok < 0 || tok >= p.V) {
            atomicOr(p.err, SDB_KERR_TOKEN);
            tok = 0;
        }
        const int drow = b * p.k + lane;
        float q_tok;
        if (p.point_mass) {
            q_tok = p.draft[(int64_t)drow * p.V + tok];
        } else {
            float M, inv;
            row_norm(p, drow, M, inv);
            q_tok = expf(scale_t(p.draft[(int64_t)drow * p.V + tok], T) - M) * inv;
        }
        float Mt, it;
        row_norm(p, nd + b * p.Tr + lane, Mt, it);
        const float p_tok = expf(scale_t(p.target[(int64_t)(b * p.Tr + lane) * p.V + tok], T) - Mt) * it;
        const float ratio = q_tok > 0.f ? fminf(__fdiv_rn(p_tok, fmaxf(q_tok, 1e-10f)), 1.0f) : 0.f;
        acc = accept_uniform(p, b, lane) < ratio;
        p.out_mask[b * p.k + lane] = acc ? 1 : 0;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, acc);
    const unsigned low = p.k >= 32 ? 0xffffffffu : ((1u << p.k) - 1u);
    const unsigned rej = ~bal & low;
    const int a = rej ? __ffs(rej) - 1 : p.k;
    float Mp = 0.f, ip = 0.f, Mq = 0.f, iq = 0.f;
    if (lane == 0) row_norm(p, nd + b * p.Tr + min(a, p.Tr - 1), Mp, ip);  // verify.py:143
    if (lane == 1 && a < p.k && !p.point_mass) row_norm(p, b * p.k + a, Mq, iq);
    Mq = __shfl_sync(0xffffffffu, Mq, 1);
    iq = __shfl_sync(0xffffffffu, iq, 1);
    if (lane == 0) {
        Decision d;
        d.a = a;
        d.mask = bal & low;
        d.Mp = Mp;
        d.ip = ip;
        d.Mq = Mq;
        d.iq = iq;
        *out = d;
        p.out_acc[b] = a;
    }
}

// ------------------------------------------------------------------ pass 1
__global__ void __launch_bounds__(THREADS) vs_row_stats(const Params p) {
    __shared__ float sh[THREADS / 32];
    __shared__ int last;
    const int nd = p.B * p.k;
    // point-mass drafts need no statistics: the grid then starts at the target rows
    const int row = blockIdx.x + (p.point_mass ? nd : 0);
    const int c = blockIdx.y;
    const float* src;
    int b;
    if (row < nd) {
        src = p.draft + (int64_t)row * p.V;
        b = row / p.k;
    } else {
        src = p.target + (int64_t)(row - nd) * p.V;
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
            if (idx < n) x = __ldcs(reinterpret_cast<const float4*>(src + base + idx));
            v[it * 4 + 0] = idx < n ? scale_t(x.x, T) : -INFINITY;
            v[it * 4 + 1] = idx < n ? scale_t(x.y, T) : -INFINITY;
            v[it * 4 + 2] = idx < n ? scale_t(x.z, T) : -INFINITY;
            v[it * 4 + 3] = idx < n ? scale_t(x.w, T) : -INFINITY;
        }
    } else {
#pragma unroll
        for (int it = 0; it < EPT; ++it) {
            const int idx = it * THREADS + threadIdx.x;
            v[it] = idx < n ? scale_t(__ldcs(src + base + idx), T) : -INFINITY;
        }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPT; ++i) mx = fmaxf(mx, v[i]);
    mx = block_reduce(mx, [](float a, float b2) { return fmaxf(a, b2); }, sh);
    float s = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
        for (int i = 0; i < EPT; ++i) s += expf(v[i] - mx);
    }
    s = block_reduce(s, [](float a, float b2) { return a + b2; }, sh);
    if (threadIdx.x == 0) {
        __stcg(p.stats + (int64_t)row * p.C1 + c, make_float2(mx, s));
        __threadfence();
        const int expect = (p.point_mass ? p.Tr : p.k + p.Tr) * p.C1;
        last = atomicAdd(p.counters + b, 1) == expect - 1;
    }
    __syncthreads();
    if (!last) return;
    // last statistics CTA of sequence b: decide once for the whole sequence
    __threadfence();
    if (threadIdx.x < 32) {
        decide_warp(p, b, p.dec + b);
        if (threadIdx.x == 0) p.counters[b] = 0;
    }
}

// resid_i and p_i of row a (verify.py:141-148): q_pad[k] = 0, p index clamped.
SDB_DEV void resid_at(const Params& p, int b, const Decision& d, float T, int i, float& r, float& pv) {
    const int pa = min(d.a, p.Tr - 1);
    pv = expf(scale_t(__ldg(p.target + (int64_t)(b * p.Tr + pa) * p.V + i), T) - d.Mp) * d.ip;
    float qv = 0.f;
    if (d.a < p.k) {
        const float x = __ldg(p.draft + (int64_t)(b * p.k + d.a) * p.V + i);
        qv = p.point_mass ? x : expf(scale_t(x, T) - d.Mq) * d.iq;
    }
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

// ------------------------------------------------------------------ pass 2
__global__ void __launch_bounds__(THREADS) vs_resid_sums(const Params p) {
    __shared__ float sh[THREADS / 32];
    const int b = blockIdx.x, c = blockIdx.y;
    const Decision d = load_decision(p, b);
    const float T = p.temps ? p.temps[b] : 1.0f;
    float sr = 0.f, sp = 0.f;
    const int base = c * CHUNK2;
    const int end = min(base + CHUNK2, p.V);
    for (int i = base + threadIdx.x; i < end; i += THREADS) {
        float r, pv;
        resid_at(p, b, d, T, i, r, pv);
        sr += r;
        sp += pv;
    }
    sr = block_reduce(sr, [](float a, float b2) { return a + b2; }, sh);
    sp = block_reduce(sp, [](float a, float b2) { return a + b2; }, sh);
    if (threadIdx.x == 0) __stcg(p.rsum + b * p.C2 + c, make_float2(sr, sp));
}

SDB_DEV bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// ------------------------------------------------------------------ pass 3
__global__ void __launch_bounds__(THREADS) vs_bonus(const Params p) {
    __shared__ float zsh;
    __shared__ int use_p;
    __shared__ float bv[THREADS / 32];
    __shared__ int bi[THREADS / 32];
    const int b = blockIdx.x, c = blockIdx.y;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        float sr = 0.f, sp = 0.f;
        for (int cc = 0; cc < p.C2; ++cc) {
            const float2 v = __ldcg(p.rsum + b * p.C2 + cc);
            sr += v.x;
            sp += v.y;
        }
        use_p = !(sr > 0.f);                   // fallback to p[a], verify.py:151
        zsh = fmaxf(use_p ? sp : sr, 1e-10f);  // normaliser, verify.py:152
    }
    __syncthreads();
    const Decision d = load_decision(p, b);
    const float T = p.temps ? p.temps[b] : 1.0f;
    const float Z = zsh;
    const bool up = use_p != 0;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    const int base = c * CHUNK2;
    const int end = min(base + CHUNK2, p.V);
    for (int i = base + threadIdx.x; i < end; i += THREADS) {
        float r, pv;
        resid_at(p, b, d, T, i, r, pv);
        const float x = __fdiv_rn(__fdiv_rn(up ? pv : r, Z), exp_noise(p, b, i));
        if (better(x, i, best, bidx)) {
            best = x;
            bidx = i;
        }
    }
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
    if (threadIdx.x != 0) return;
    for (int i = 1; i < THREADS / 32; ++i)
        if (better(bv[i], bi[i], best, bidx)) {
            best = bv[i];
            bidx = bi[i];
        }
    __stcg(p.amax + b * p.C2 + c, make_float2(best, __int_as_float(bidx)));
    __threadfence();
    if (atomicAdd(p.counters + b, 1) != p.C2 - 1) return;
    // last CTA of sequence b: finish the argmax (first index on ties, torch.argmax)
    __threadfence();
    float gb = -INFINITY;
    int gi = 0x7fffffff;
    for (int cc = 0; cc < p.C2; ++cc) {
        const float2 v = __ldcg(p.amax + b * p.C2 + cc);
        const int vi = __float_as_int(v.y);
        if (better(v.x, vi, gb, gi)) {
            gb = v.x;
            gi = vi;
        }
    }
    p.out_bonus[b] = gi == 0x7fffffff ? 0 : gi;
    p.counters[b] = 0;
}

struct WsLayout {
    size_t err, counters, dec, stats, rsum, amax, total;
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
    off = align_up(off + sizeof(float2) * (size_t)B * (k + Tr) * C1, 256);
    w.rsum = off;
    off = align_up(off + sizeof(float2) * (size_t)B * C2, 256);
    w.amax = off;
    off = align_up(off + sizeof(float2) * (size_t)B * C2, 256);
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

extern "C" int sdb_verify_batch(const float* draft, const float* target, const int64_t* tokens, const float* temps,
                                const float* uniforms, const float* exponentials, uint64_t seed, uint64_t offset,
                                int point_mass, int64_t* out_acc, int64_t* out_bonus, uint8_t* out_mask, int B,
                                int k, int Tr, int V, void* workspace, size_t workspace_bytes, void* stream) {
    if (!draft || !target || !tokens || !out_acc || !out_bonus || !out_mask || !workspace) {
        set_last_error("null pointer argument");
        return SDB_ERR_INVALID_ARG;
    }
    if (B <= 0 || B > vs::kCounterCap || k <= 0 || k > 32 || V <= 0 || !(Tr == k || Tr == k + 1)) {
        set_last_error("bad sizes B=%d k=%d target_rows=%d V=%d (need B <= %d, 1<=k<=32, target_rows in {k, k+1})",
                       B, k, Tr, V, vs::kCounterCap);
        return SDB_ERR_INVALID_ARG;
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
    vs::Params p{};
    p.draft = draft;
    p.target = target;
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
    p.C1 = (V + vs::CHUNK1 - 1) / vs::CHUNK1;
    p.C2 = (V + vs::CHUNK2 - 1) / vs::CHUNK2;
    p.err = reinterpret_cast<int*>(ws + w.err);
    p.counters = reinterpret_cast<int*>(ws + w.counters);
    p.dec = reinterpret_cast<vs::Decision*>(ws + w.dec);
    p.stats = reinterpret_cast<float2*>(ws + w.stats);
    p.rsum = reinterpret_cast<float2*>(ws + w.rsum);
    p.amax = reinterpret_cast<float2*>(ws + w.amax);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    vs::vs_row_stats<<<dim3(B * ((point_mass ? 0 : k) + Tr), p.C1), vs::THREADS, 0, st>>>(p);
    int rc = cuda_status(cudaGetLastError(), "vs_row_stats launch");
    if (rc) return rc;
    vs::vs_resid_sums<<<dim3(B, p.C2), vs::THREADS, 0, st>>>(p);
    rc = cuda_status(cudaGetLastError(), "vs_resid_sums launch");
    if (rc) return rc;
    vs::vs_bonus<<<dim3(B, p.C2), vs::THREADS, 0, st>>>(p);
    return cuda_status(cudaGetLastError(), "vs_bonus launch");
}

extern "C" int sdb_philox_fill(float* out, int rows, int cols, uint64_t seed, uint64_t offset, int stream_id,
                               void* stream) {
    if (!out || rows <= 0 || cols <= 0 || (stream_id != 0 && stream_id != 1)) {
        set_last_error("bad arguments to sdb_philox_fill");
        return SDB_ERR_INVALID_ARG;
    }
    const int64_t n = (int64_t)rows * cols;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    vs::philox_fill_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        out, rows, cols, (uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32), (uint32_t)offset, stream_id);
    return cuda_status(cudaGetLastError(), "philox_fill launch");
}
