// The two elementwise steps of a Qwen3 decoder layer around the projections, one launch
// each (the reference runs them as torch.compile'd torch code):
//
//   sdb_rms_norm   RMSNorm.rms_forward / add_rms_forward, nanovllm/layers/layernorm.py:17-43:
//                  s = x (+ residual) in float32, residual_out = s rounded to the model
//                  dtype, y = (s * rsqrt(mean(s^2) + eps)) rounded to the model dtype,
//                  times the weight, rounded again.
//   sdb_silu_mul   SiluAndMul.forward, nanovllm/layers/activation.py:8-13: for the
//                  (T, 2F) gate|up rows, y = silu(gate) * up, silu(x) = x / (1 + e^-x),
//                  each product of two model-dtype values rounded to the model dtype as
//                  torch's elementwise ops round them.
//
// Both are HBM-bound single passes: one CTA per token row, 16-byte loads and stores.
#include "common.cuh"

namespace sdb {
namespace lops {

constexpr int THREADS = 256;

template <typename T>
SDB_DEV void load8(const T* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32(e[i]);
}

template <typename T>
SDB_DEV void store8(T* p, const float (&v)[8]) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = u;
}

SDB_DEV float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) s += red[w];
    return s;
}

// Row t: up to kMaxVec 8-element groups per thread are held in registers between the
// statistics and the output.
constexpr int kMaxVec = 4;  // H <= 256 threads x 4 x 8 = 8192

template <typename T>
__global__ void __launch_bounds__(THREADS) rms_norm_kernel(const T* x, int64_t xs, const T* res_in, int64_t ris,
                                                           T* out, int64_t os, T* res_out, int64_t ros,
                                                           const T* w, int H, float eps) {
    __shared__ float red[THREADS / 32];
    const int t = blockIdx.x;
    const int nvec = H / 8;
    float v[kMaxVec][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        const int c = (threadIdx.x + i * THREADS) * 8;
        if (c < H) {
            load8(x + (int64_t)t * xs + c, v[i]);
            if (res_in) {
                float r[8];
                load8(res_in + (int64_t)t * ris + c, r);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] += r[j];
            }
            if (res_out) store8(res_out + (int64_t)t * ros + c, v[i]);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
    }
    (void)nvec;
    const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        const int c = (threadIdx.x + i * THREADS) * 8;
        if (c < H) {
            float wv[8], y[8];
            load8(w + c, wv);
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] = to_f32(from_f32<T>(v[i][j] * inv)) * wv[j];
            store8(out + (int64_t)t * os + c, y);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(THREADS) silu_mul_kernel(const T* gu, int64_t gs, T* out, int64_t os, int F) {
    const int t = blockIdx.y;
    const int c = (blockIdx.x * THREADS + threadIdx.x) * 8;
    if (c >= F) return;
    float g[8], u[8], y[8];
    load8(gu + (int64_t)t * gs + c, g);
    load8(gu + (int64_t)t * gs + F + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float a = to_f32(from_f32<T>(g[j] / (1.0f + expf(-g[j]))));  // silu, rounded like torch
        y[j] = a * u[j];
    }
    store8(out + (int64_t)t * os + c, y);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace lops
}  // namespace sdb

using namespace sdb;

extern "C" int sdb_rms_norm(const void* x, int64_t x_stride, const void* residual_in, int64_t residual_in_stride,
                            void* out, int64_t out_stride, void* residual_out, int64_t residual_out_stride,
                            const void* weight, int T, int H, float eps, int dtype, void* stream) {
    if (!x || !out || !weight || T < 0 || H <= 0) {
        set_last_error("bad arguments to sdb_rms_norm");
        return SDB_ERR_INVALID_ARG;
    }
    if (T == 0) return SDB_OK;
    if (dtype != SDB_BF16 && dtype != SDB_F16) {
        set_last_error("sdb_rms_norm: dtype must be bf16 or f16");
        return SDB_ERR_UNSUPPORTED;
    }
    if (H % 8 || H > lops::THREADS * lops::kMaxVec * 8) {
        set_last_error("sdb_rms_norm: hidden size %d must be a multiple of 8 and at most %d", H,
                       lops::THREADS * lops::kMaxVec * 8);
        return SDB_ERR_UNSUPPORTED;
    }
    if (!lops::aligned16(x) || !lops::aligned16(out) || !lops::aligned16(weight) ||
        (residual_in && !lops::aligned16(residual_in)) || (residual_out && !lops::aligned16(residual_out)) ||
        (x_stride % 8) || (out_stride % 8) || (residual_in && residual_in_stride % 8) ||
        (residual_out && residual_out_stride % 8)) {
        set_last_error("sdb_rms_norm: rows must be 16-byte aligned");
        return SDB_ERR_INVALID_ARG;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == SDB_BF16) {
        using T_ = __nv_bfloat16;
        lops::rms_norm_kernel<T_><<<T, lops::THREADS, 0, st>>>(
            reinterpret_cast<const T_*>(x), x_stride, reinterpret_cast<const T_*>(residual_in), residual_in_stride,
            reinterpret_cast<T_*>(out), out_stride, reinterpret_cast<T_*>(residual_out), residual_out_stride,
            reinterpret_cast<const T_*>(weight), H, eps);
    } else {
        using T_ = __half;
        lops::rms_norm_kernel<T_><<<T, lops::THREADS, 0, st>>>(
            reinterpret_cast<const T_*>(x), x_stride, reinterpret_cast<const T_*>(residual_in), residual_in_stride,
            reinterpret_cast<T_*>(out), out_stride, reinterpret_cast<T_*>(residual_out), residual_out_stride,
            reinterpret_cast<const T_*>(weight), H, eps);
    }
    return cuda_status(cudaGetLastError(), "rms_norm_kernel launch");
}

extern "C" int sdb_silu_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride, int T,
                            int F, int dtype, void* stream) {
    if (!gate_up || !out || T < 0 || F <= 0) {
        set_last_error("bad arguments to sdb_silu_mul");
        return SDB_ERR_INVALID_ARG;
    }
    if (T == 0) return SDB_OK;
    if (dtype != SDB_BF16 && dtype != SDB_F16) {
        set_last_error("sdb_silu_mul: dtype must be bf16 or f16");
        return SDB_ERR_UNSUPPORTED;
    }
    if (F % 8 || !lops::aligned16(gate_up) || !lops::aligned16(out) || gate_up_stride % 8 || out_stride % 8) {
        set_last_error("sdb_silu_mul: F must be a multiple of 8 and rows 16-byte aligned");
        return SDB_ERR_INVALID_ARG;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    dim3 grid((F / 8 + lops::THREADS - 1) / lops::THREADS, T);
    if (dtype == SDB_BF16)
        lops::silu_mul_kernel<__nv_bfloat16><<<grid, lops::THREADS, 0, st>>>(
            reinterpret_cast<const __nv_bfloat16*>(gate_up), gate_up_stride, reinterpret_cast<__nv_bfloat16*>(out),
            out_stride, F);
    else
        lops::silu_mul_kernel<__half><<<grid, lops::THREADS, 0, st>>>(
            reinterpret_cast<const __half*>(gate_up), gate_up_stride, reinterpret_cast<__half*>(out), out_stride, F);
    return cuda_status(cudaGetLastError(), "silu_mul_kernel launch");
}
