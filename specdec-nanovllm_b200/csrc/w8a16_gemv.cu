// W8A16 linear for 1-16 tokens with per-channel scales: a weight stream.
//
// Reference: int8_linear, nanovllm/layers/quant.py:165-310 (decode steps and small
// verify batches run it with M = batch or batch x (k+1) tokens; at these sizes the
// call is one pass over the int8 weights).
//
// Decomposition.  The N output features are split over the CTAs in contiguous row
// ranges (1-row granularity: every CTA streams the same number of weight bytes to
// within one row), two CTAs per SM where their shared memory fits.  A CTA's rows are
// cut into T tiles of at most 16 rows (the M side of mma.m16n8k16), its (tile, 128-k
// block) units are split evenly over its 8 warps in tile-major order, and each warp
// accumulates its consecutive blocks in registers; a warp's partial sum for a tile
// goes to shared memory when the warp leaves the tile, and the CTA adds the partials
// of each tile in warp order at the end (deterministic).  There is no split-K across
// CTAs, no workspace and no fix-up launch.
//
// Per 128-k block a lane loads 32 contiguous weight bytes of two rows (g and g + 8)
// with one 256-bit load each, so one warp instruction reads eight full 128-byte
// lines.  Inside the block the k order is permuted (identically for both operands)
// so that lane t's 32 bytes are its A fragments for the block's eight k16 steps:
// byte j of lane t is k = 32 t + j, and step m takes bytes 4m..4m+3.  The matching
// token fragments are 64 contiguous bytes of the token row, read from shared memory
// where the tokens of the whole call sit (loaded once per CTA with cp.async).  The
// int8 -> 16-bit conversion is exact, as in the other W8A16 kernels.
//
// Each warp keeps D blocks of weights in flight in a ring of D + 1 register slots (a
// slot is refilled with the block D ahead once the previous block has been consumed,
// so no register copies are needed).  The kernel is a programmatic dependent launch:
// it lets the next kernel launch at once, and before it waits for the preceding
// kernel it issues its first D + 1 weight blocks and reads its rows' scales and bias
// (the tokens are that kernel's output; the weights and scales are not).
#include <type_traits>

#include "common.cuh"
#include "w8a16_convert.cuh"

namespace sdb {
namespace w8g {

constexpr int KBLK = 128;  // k per unit

struct Params {
    const void* x;
    int64_t x_srow;
    const int8_t* w;
    const void* s;
    int s_dtype;
    const void* bias;
    void* y;
    int64_t y_srow;
    int M, N, K;
    int kb;       // 128-k blocks per row
    int J;        // partial slots per warp
    int x_bytes;     // shared-memory bytes of the token rows
    int part_bytes;  // shared-memory bytes of the warps' partial sums
};

// 32 contiguous weight bytes if `ok`, not kept in L1; the L2 fetch is promoted to 256
// bytes (the warp reads the following 128 bytes of each row with its next block).
// Predicated inside the instruction, so the call site has no branch.  If `ok` is false, r
// keeps whatever bits its registers held: every 32-bit pattern converts to four finite
// int8 values, and they only reach accumulator rows of missing weight rows, or blocks past
// the warp's range that are never consumed.
SDB_DEV void ldg256(const int8_t* p, bool ok, uint32_t (&r)[8]) {
    asm volatile(
        "{\n.reg .pred q;\nsetp.ne.b32 q, %9, 0;\n"
        "@q ld.global.nc.L1::no_allocate.L2::256B.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n}"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "l"(p), "r"((int)ok));
}

SDB_DEV void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// First row (relative to the CTA's first row) of tile t when R rows are cut into T tiles.
SDB_DEV int tile_lo(int t, int R, int T) { return t * R / T; }

// Where a warp's next weight load points: the block within the tile, the two row
// pointers (advanced 128 bytes per block) and whether the rows exist.  A row past the
// tile's end is not loaded: its registers keep stale weights, and the rows of the
// accumulator they feed are never written out.
struct Cursor {
    int t, b;
    const int8_t* p0;
    const int8_t* p1;
    bool ok0, ok1;
};

SDB_DEV void cursor_tile(Cursor& c, const Params& p, int r0, int R, int T, int g, int t4) {
    const int lo = tile_lo(c.t, R, T), hi = tile_lo(c.t + 1, R, T);
    c.ok0 = lo + g < hi;
    c.ok1 = lo + g + 8 < hi;
    c.p0 = p.w + (int64_t)(r0 + lo + g) * p.K + t4 * 32 + c.b * KBLK;
    c.p1 = c.p0 + (int64_t)8 * p.K;
}

SDB_DEV void load_block(Cursor& c, bool go, const Params& p, int r0, int R, int T, int g, int t4, uint32_t (&a)[8],
                        uint32_t (&b)[8]) {
    ldg256(c.p0, go && c.ok0, a);
    ldg256(c.p1, go && c.ok1, b);
    c.p0 += KBLK;
    c.p1 += KBLK;
    if (++c.b == p.kb) {
        c.b = 0;
        ++c.t;
        cursor_tile(c, p, r0, R, T, g, t4);
    }
}

template <typename E, int NT, int WARPS, int D, int MINB>
__global__ void __launch_bounds__(WARPS * 32, MINB) w8a16_gemv_kernel(const Params p) {
    using H = Half16<E>;
    constexpr int S = D + 1;  // register slots: D blocks in flight while one is consumed
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int r0 = (int)((int64_t)blockIdx.x * p.N / gridDim.x);
    const int R = (int)((int64_t)(blockIdx.x + 1) * p.N / gridDim.x) - r0;
    if (R <= 0) return;
    const int T = (R + 15) / 16;
    const int U = T * p.kb;
    const int u0 = (int)((int64_t)warp * U / WARPS), u1 = (int)((int64_t)(warp + 1) * U / WARPS);

    // the first S = D + 1 weight blocks: independent of the preceding kernel
    uint32_t ra[S][8], rb[S][8];
#pragma unroll
    for (int i = 0; i < S; ++i)
#pragma unroll
        for (int k = 0; k < 8; ++k) ra[i][k] = rb[i][k] = 0u;
    Cursor lc;
    lc.t = u0 / p.kb;
    lc.b = u0 - lc.t * p.kb;
    cursor_tile(lc, p, r0, R, T, g, t4);
#pragma unroll
    for (int i = 0; i < S; ++i) load_block(lc, u0 + i < u1, p, r0, R, T, g, t4, ra[i], rb[i]);
    // per-channel scales and bias of the CTA's rows (constant: the first WARPS * 32 are read
    // into registers before the wait and stored to shared memory after it, so no thread
    // waits for them on its way to the wait)
    float* sc = reinterpret_cast<float*>(smem + p.x_bytes + p.part_bytes);
    const E* bias = reinterpret_cast<const E*>(p.bias);
    float s_first = 0.f, b_first = 0.f;
    if ((int)threadIdx.x < R) {
        s_first = w8cv::scale_value(p.s, p.s_dtype, r0 + threadIdx.x);
        if (bias) b_first = to_f32(bias[r0 + threadIdx.x]);
    }

    pdl_wait();
    {  // the call's token rows -> shared memory, row n at n * 2K bytes
        const int upr = p.K / 8;  // 16-byte units per row
        const E* xg = reinterpret_cast<const E*>(p.x);
        const uint32_t sbase = smem_u32(smem);
        for (int i = threadIdx.x; i < p.M * upr; i += WARPS * 32) {
            const int n = i / upr, u = i - n * upr;
            cp_async16(sbase + (uint32_t)(n * p.K * 2 + u * 16), xg + (int64_t)n * p.x_srow + u * 8);
        }
        if ((int)threadIdx.x < R) {
            sc[threadIdx.x] = s_first;
            sc[R + threadIdx.x] = b_first;
        }
        for (int r = threadIdx.x + WARPS * 32; r < R; r += WARPS * 32) {
            sc[r] = w8cv::scale_value(p.s, p.s_dtype, r0 + r);
            sc[R + r] = bias ? to_f32(bias[r0 + r]) : 0.f;
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();

    // token fragments of block b for lane (g, t4): 64 bytes at row n, byte 256 b + 64 t4
    // (the quarter-warp's lanes t4 = 0 and 2 share banks: a 2-way conflict on 4 loads per block)
    const uint8_t* xp[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int n = nt * 8 + g;
        xp[nt] = smem + (n < p.M ? n : 0) * p.K * 2 + t4 * 64 + (u0 - (u0 / p.kb) * p.kb) * 256;
    }

    float* part = reinterpret_cast<float*>(smem + p.x_bytes);  // [WARPS][J][NT][16][8]
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    int cb = u0 - (u0 / p.kb) * p.kb;  // block of the unit being consumed
    int jt = 0;                        // its tile, counted from the warp's first tile

    for (int base = u0; base < u1; base += S) {
#pragma unroll
        for (int i = 0; i < S; ++i) {
            const int u = base + i;
            if (u >= u1) break;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                uint32_t xw[16];
                if (nt * 8 + g < p.M) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint4 v = *reinterpret_cast<const uint4*>(xp[nt] + q * 16);
                        xw[4 * q] = v.x;
                        xw[4 * q + 1] = v.y;
                        xw[4 * q + 2] = v.z;
                        xw[4 * q + 3] = v.w;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 16; ++q) xw[q] = 0u;
                }
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    uint32_t a[4];
                    w8cv::i8x4<E>(ra[i][m], a[0], a[2]);
                    w8cv::i8x4<E>(rb[i][m], a[1], a[3]);
                    H::mma(acc[nt], a, xw[2 * m], xw[2 * m + 1]);
                }
                xp[nt] += 256;
            }
            // the slot is converted: refill it with the unit S ahead (D others stay in flight)
            load_block(lc, u + S < u1, p, r0, R, T, g, t4, ra[i], rb[i]);
            if (++cb == p.kb) {  // tile done: partial sums to shared memory
                float* pp = part + ((warp * p.J + jt) * NT) * 128;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    *reinterpret_cast<float2*>(pp + nt * 128 + g * 8 + 2 * t4) = make_float2(acc[nt][0], acc[nt][1]);
                    *reinterpret_cast<float2*>(pp + nt * 128 + (g + 8) * 8 + 2 * t4) =
                        make_float2(acc[nt][2], acc[nt][3]);
                    acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
                    xp[nt] -= p.K * 2;
                }
                ++jt;
                cb = 0;
            }
        }
    }
    if (cb != 0) {
        float* pp = part + ((warp * p.J + jt) * NT) * 128;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            *reinterpret_cast<float2*>(pp + nt * 128 + g * 8 + 2 * t4) = make_float2(acc[nt][0], acc[nt][1]);
            *reinterpret_cast<float2*>(pp + nt * 128 + (g + 8) * 8 + 2 * t4) = make_float2(acc[nt][2], acc[nt][3]);
        }
    }
    __syncthreads();

    // each output: the partials of the warps that covered its tile, in warp order
    E* y = reinterpret_cast<E*>(p.y);
    for (int o = threadIdx.x; o < R * p.M; o += WARPS * 32) {
        const int n = o / R, row = o - n * R;
        int t = row * T / R;
        while (t + 1 < T && tile_lo(t + 1, R, T) <= row) ++t;
        while (tile_lo(t, R, T) > row) --t;
        const int lr = row - tile_lo(t, R, T);
        float v = 0.f;
#pragma unroll 1
        for (int w = 0; w < WARPS; ++w) {
            const int a0 = (int)((int64_t)w * U / WARPS), a1 = (int)((int64_t)(w + 1) * U / WARPS);
            if (a0 < a1 && a0 < (t + 1) * p.kb && a1 > t * p.kb) {
                const int j = t - a0 / p.kb;
                v += part[(((w * p.J + j) * NT + (n >> 3)) * 16 + lr) * 8 + (n & 7)];
            }
        }
        y[(int64_t)n * p.y_srow + r0 + row] = from_f32<E>(v * sc[row] + sc[R + row]);
    }
}

constexpr int kWarps = 8;
constexpr int kDepth1 = 4, kDepth2 = 2;    // weight blocks in flight per warp (1 / 2 token fragments)
constexpr int kCtasPerSm = 2;              // register budget of the launch bounds
constexpr size_t kSmemCap = 200 * 1024;
constexpr size_t kSmemPerSm = 228 * 1024;  // shared memory of one SM (1 KB reserved per CTA)

struct Plan {
    int NT, G, J;
    size_t x_bytes, part_bytes, smem;
};

// One CTA per SM for each CTA that fits (2 by registers, fewer when the token rows are
// large), rows split evenly over them; J = the most tiles one warp's unit range can touch.
static bool plan(int M, int N, int K, Plan& pl) {
    if (M < 1 || M > 16 || N < 1 || K < KBLK || K % KBLK) return false;
    pl.NT = M <= 8 ? 1 : 2;
    const int kb = K / KBLK;
    pl.x_bytes = align_up((size_t)M * K * 2, 128);
    int per_sm = kCtasPerSm;
    for (;; --per_sm) {
        const int sms = device_sm_count() * per_sm;
        pl.G = N / 8 < sms ? (N / 8 > 0 ? N / 8 : 1) : sms;
        const int rmax = (N + pl.G - 1) / pl.G;
        const int tmax = (rmax + 15) / 16;
        const long long umax = (long long)tmax * kb;
        const long long per_warp = (umax + kWarps - 1) / kWarps;
        long long j = per_warp > 0 ? (per_warp + kb - 2) / kb + 1 : 1;
        if (j > tmax) j = tmax;
        pl.J = (int)j;
        pl.part_bytes = (size_t)kWarps * pl.J * pl.NT * 128 * sizeof(float);
        pl.smem = pl.x_bytes + pl.part_bytes + align_up(2 * sizeof(float) * (size_t)rmax, 128);
        if (per_sm == 1 || (pl.smem + 1024) * per_sm <= kSmemPerSm) break;
    }
    return pl.smem <= kSmemCap;
}

template <typename E, int NT>
static int launch_t(const Params& p, const Plan& pl, cudaStream_t st) {
    auto kern = w8a16_gemv_kernel<E, NT, kWarps, NT == 1 ? kDepth1 : kDepth2, kCtasPerSm>;
    const int slot = 80 + (std::is_same<E, __nv_bfloat16>::value ? 0 : 2) + (NT - 1);
    int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)pl.smem, slot);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.G, 1, 1);
    cfg.blockDim = dim3(kWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, p), "w8a16_gemv_kernel launch");
}

}  // namespace w8g

bool w8a16_gemv_eligible(int M, int N, int K, int group) {
    w8g::Plan pl;
    return group == 0 && w8g::plan(M, N, K, pl);
}

int w8a16_gemv_launch(const void* x, int64_t x_srow, const int8_t* w, const void* s, int s_dtype, const void* bias,
                      void* y, int64_t y_srow, int M, int N, int K, int act_dtype, cudaStream_t st) {
    w8g::Plan pl;
    if (!w8g::plan(M, N, K, pl)) {
        set_last_error("w8a16_gemv: no plan for M=%d N=%d K=%d", M, N, K);
        return SDB_ERR_UNSUPPORTED;
    }
    w8g::Params p{};
    p.x = x;
    p.x_srow = x_srow;
    p.w = w;
    p.s = s;
    p.s_dtype = s_dtype;
    p.bias = bias;
    p.y = y;
    p.y_srow = y_srow;
    p.M = M;
    p.N = N;
    p.K = K;
    p.kb = K / w8g::KBLK;
    p.J = pl.J;
    p.x_bytes = (int)pl.x_bytes;
    p.part_bytes = (int)pl.part_bytes;
    const bool bf = act_dtype == SDB_BF16;
    if (pl.NT == 1)
        return bf ? w8g::launch_t<__nv_bfloat16, 1>(p, pl, st) : w8g::launch_t<__half, 1>(p, pl, st);
    return bf ? w8g::launch_t<__nv_bfloat16, 2>(p, pl, st) : w8g::launch_t<__half, 2>(p, pl, st);
}

}  // namespace sdb
