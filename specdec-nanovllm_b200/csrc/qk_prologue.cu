// Attention prologue of a Qwen3 layer in one launch: split of the fused QKV
// projection, per-head RMSNorm of q and k, rotary embedding of q and k, and the
// store of the step's k / v rows into the paged cache.
//
// Reference: Qwen3Attention.forward, nanovllm/models/qwen3.py:77-86 --
//   q, k, v = qkv.split(...)                         (:78-81)
//   q = q_norm(q); k = k_norm(k)                     (:82-84, RMSNorm.rms_forward,
//                                                     nanovllm/layers/layernorm.py:16-25)
//   q, k = rotary_emb(positions, q, k)               (:85, rotary_embedding.py:38-50, :6-14)
// followed by store_kvcache(k, v, ...) inside Attention.forward (attention.py:59-63).
// The reference runs these as separate torch / Triton kernels, each reading and
// writing the activations.
//
// One warp per (token, head) row of head_dim D = 32 * EPL: lane l holds elements
// [EPL l, EPL (l + 1)), so the rotate-half partner of a lane is lane l ^ 16.
//   RMSNorm (eager torch semantics): x in float32, var = sum(x^2) / D, x * (1 / sqrt(var
//   + eps)) rounded to the model dtype, times the weight, rounded again.
//   Rotary: x in float32, y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin with every product
//   and sum rounded separately (no contraction), rounded to the model dtype; cos / sin
//   are read from the caller's cos_sin_cache (the module's own buffer).
// v rows are copied unchanged.  Slot -1 skips a row's store (graph padding).
#include "common.cuh"

namespace sdb {
namespace qkp {

constexpr int WARPS = 8;

struct Params {
    const void* qkv;
    int64_t qkv_stok;          // elements between tokens
    const void* qw;            // q_norm weight (D) or null (no norm)
    const void* kw;            // k_norm weight (D) or null
    float eps;
    const float* cs;           // cos_sin_cache rows: [cos(D/2) | sin(D/2)]
    int64_t cs_spos;
    const int64_t* pos;        // (T)
    void* q_out;
    int64_t q_stok, q_shead;
    void* k_out;               // (T, Hkv, D) or null
    void* v_out;
    int64_t kv_stok, kv_shead;
    void* kc;                  // caches or null
    void* vc;
    int64_t sb, sp, sh;
    const int* slots;
    int T, Hq, Hkv, page, num_blocks, max_pos;
    int* err;
};

template <typename T>
SDB_DEV float ld_f32(const T* p) { return to_f32(*p); }

template <typename T, int EPL>
__global__ void __launch_bounds__(WARPS * 32) qk_prologue_kernel(const Params p) {
    constexpr int D = 32 * EPL;
    const int lane = threadIdx.x & 31;
    const int heads = p.Hq + 2 * p.Hkv;
    const long long r = (long long)blockIdx.x * WARPS + (threadIdx.x >> 5);
    if (r >= (long long)p.T * heads) return;
    const int t = (int)(r / heads), h = (int)(r % heads);
    const T* src = reinterpret_cast<const T*>(p.qkv) + (int64_t)t * p.qkv_stok + (int64_t)h * D + lane * EPL;
    float x[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = to_f32(src[i]);
    const bool is_q = h < p.Hq, is_v = h >= p.Hq + p.Hkv;
    const int hk = is_q ? h : (is_v ? h - p.Hq - p.Hkv : h - p.Hq);
    if (!is_v) {
        const T* w = reinterpret_cast<const T*>(is_q ? p.qw : p.kw);
        if (w) {  // RMSNorm
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < EPL; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
            const float var = __fmul_rn(ss, 1.0f / D);  // exact: D is a power of two
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
#pragma unroll
            for (int i = 0; i < EPL; ++i) {
                const float xn = to_f32(from_f32<T>(__fmul_rn(x[i], inv)));
                x[i] = to_f32(from_f32<T>(__fmul_rn(xn, to_f32(w[lane * EPL + i]))));
            }
        }
        // rotary embedding, rotate-half form
        int64_t ps = p.pos[t];
        if (ps < 0 || ps >= p.max_pos) {
            if (lane == 0) atomicOr(p.err, SDB_KERR_SEQLEN);
            ps = ps < 0 ? 0 : p.max_pos - 1;
        }
        const float* cs = p.cs + ps * p.cs_spos;
        const bool lo = lane < 16;
        const int d0 = (lane & 15) * EPL;  // index into the D/2 cos / sin entries
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const float other = __shfl_xor_sync(0xffffffffu, x[i], 16);
            const float c = cs[d0 + i], s = cs[D / 2 + d0 + i];
            const float xc = __fmul_rn(x[i], c), os = __fmul_rn(other, s);
            x[i] = to_f32(from_f32<T>(lo ? __fsub_rn(xc, os) : __fadd_rn(xc, os)));
        }
    }
    // outputs
    T* dst = nullptr;
    if (is_q) {
        dst = reinterpret_cast<T*>(p.q_out) + (int64_t)t * p.q_stok + (int64_t)hk * p.q_shead;
    } else if (!is_v ? p.k_out != nullptr : p.v_out != nullptr) {
        dst = reinterpret_cast<T*>(is_v ? p.v_out : p.k_out) + (int64_t)t * p.kv_stok + (int64_t)hk * p.kv_shead;
    }
    if (dst) {
#pragma unroll
        for (int i = 0; i < EPL; ++i) dst[lane * EPL + i] = from_f32<T>(x[i]);
    }
    if (!is_q && p.slots) {
        const int slot = p.slots[t];
        if (slot >= 0) {
            const int blk = slot / p.page, off = slot % p.page;
            if (blk >= p.num_blocks) {
                if (lane == 0) atomicOr(p.err, SDB_KERR_BLOCK_ID);
            } else {
                T* c = reinterpret_cast<T*>(is_v ? p.vc : p.kc) + (int64_t)blk * p.sb + (int64_t)off * p.sp +
                       (int64_t)hk * p.sh;
#pragma unroll
                for (int i = 0; i < EPL; ++i) c[lane * EPL + i] = from_f32<T>(x[i]);
            }
        }
    }
}

template <typename T>
static int launch(const Params& p, int D, cudaStream_t st) {
    const long long rows = (long long)p.T * (p.Hq + 2 * p.Hkv);
    const unsigned grid = (unsigned)((rows + WARPS - 1) / WARPS);
    switch (D) {
        case 64: qk_prologue_kernel<T, 2><<<grid, WARPS * 32, 0, st>>>(p); break;
        case 128: qk_prologue_kernel<T, 4><<<grid, WARPS * 32, 0, st>>>(p); break;
        default: qk_prologue_kernel<T, 8><<<grid, WARPS * 32, 0, st>>>(p); break;
    }
    return cuda_status(cudaGetLastError(), "qk_prologue_kernel launch");
}

}  // namespace qkp
}  // namespace sdb

using namespace sdb;

extern "C" int sdb_qk_norm_rope_store(const void* qkv, int64_t qkv_stride_tok, const void* q_norm_weight,
                                      const void* k_norm_weight, float eps, const float* cos_sin_cache,
                                      int64_t cos_sin_stride_pos, int max_position, const int64_t* positions,
                                      void* q_out, int64_t q_stride_tok, int64_t q_stride_head, void* k_out,
                                      void* v_out, int64_t kv_stride_tok, int64_t kv_stride_head, void* k_cache,
                                      void* v_cache, int64_t kv_stride_block, int64_t kv_stride_page,
                                      int64_t kv_stride_head_cache, const int32_t* slot_mapping, int T, int Hq,
                                      int Hkv, int D, int page, int num_blocks, int dtype, void* workspace,
                                      void* stream) {
    if (T == 0) return SDB_OK;
    if (!qkv || !cos_sin_cache || !positions || !q_out || !workspace || T < 0 || Hq <= 0 || Hkv <= 0 ||
        max_position <= 0 || qkv_stride_tok < (int64_t)(Hq + 2 * Hkv) * D || q_stride_head < D ||
        cos_sin_stride_pos < D || ((k_out || v_out) && kv_stride_head < D)) {
        set_last_error("bad arguments to sdb_qk_norm_rope_store");
        return SDB_ERR_INVALID_ARG;
    }
    if (slot_mapping && (!k_cache || !v_cache || page <= 0 || num_blocks <= 0 || kv_stride_head_cache < D)) {
        set_last_error("sdb_qk_norm_rope_store: a store needs both caches, page and num_blocks");
        return SDB_ERR_INVALID_ARG;
    }
    if (D != 64 && D != 128 && D != 256) {
        set_last_error("head_dim %d not supported (64, 128 or 256)", D);
        return SDB_ERR_UNSUPPORTED;
    }
    if (dtype != SDB_BF16 && dtype != SDB_F16 && dtype != SDB_F32) {
        set_last_error("dtype %d not supported", dtype);
        return SDB_ERR_UNSUPPORTED;
    }
    qkp::Params p{};
    p.qkv = qkv;
    p.qkv_stok = qkv_stride_tok;
    p.qw = q_norm_weight;
    p.kw = k_norm_weight;
    p.eps = eps;
    p.cs = cos_sin_cache;
    p.cs_spos = cos_sin_stride_pos;
    p.pos = positions;
    p.q_out = q_out;
    p.q_stok = q_stride_tok;
    p.q_shead = q_stride_head;
    p.k_out = k_out;
    p.v_out = v_out;
    p.kv_stok = kv_stride_tok;
    p.kv_shead = kv_stride_head;
    p.kc = k_cache;
    p.vc = v_cache;
    p.sb = kv_stride_block;
    p.sp = kv_stride_page;
    p.sh = kv_stride_head_cache;
    p.slots = slot_mapping;
    p.T = T;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.page = page;
    p.num_blocks = num_blocks;
    p.max_pos = max_position;
    p.err = reinterpret_cast<int*>(workspace);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == SDB_BF16) return qkp::launch<__nv_bfloat16>(p, D, st);
    if (dtype == SDB_F16) return qkp::launch<__half>(p, D, st);
    return qkp::launch<float>(p, D, st);
}
