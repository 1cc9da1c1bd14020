// Paged decode / speculative-verify attention for B200 (sm_100a).
//
// One CTA per (KV split, kv head, sequence).  Reference behaviour being
// replaced: flash_attn_with_kvcache (decode, nanovllm/layers/attention.py:78-81),
// flash_attn_varlen_func(causal=True, block_table) (verify, attention.py:67-70),
// and the reference's own split-K design (paged_decode_attn_cuda.cu:792-1064,
// host :1388-1453): grid (kv heads, splits, sequences), chunk =
// round_up(ceil(max_blocks*page/splits), BN) from the STATIC table width (no
// device->host read of the lengths), LSE merge of the splits by the last CTA
// to arrive (:1047-1063).
//
// B200 structure (16-bit KV, head_dim 128):
//   * warp NC (the producer) streams K and V tiles of BN = 64 keys with 4-D TMA
//     (cp.async.bulk.tensor, SWIZZLE_128B, L2 evict-first) into an NS-stage ring
//     guarded by full/empty mbarriers.  A tile never crosses a page because
//     page % 64 == 0, so one block-table lookup feeds four TMA boxes.
//   * the GQA group of query heads times the n_q query rows of the sequence form
//     the M dimension: rows rho = r*G + g, padded to MT m16 tiles.  MT x KG = 4
//     consumer warps: warp (mt, kg) owns m-tile mt and a 64/KG-key slice of every
//     tile; every consumer waits for and releases every stage, and the KG
//     partial softmax states are merged through shared memory at the end.
//   * P is split into a 16-bit head and a 16-bit residual (P = P_hi + P_lo) and
//     both multiply V, so the probabilities keep ~16 significant bits: the
//     rows of a short verify window (a few visible keys) would otherwise carry
//     the 8-bit rounding of P straight into the output.
//     S = Q K^T and O += P V run on mma.m16n8k16 with fp32 accumulators; P is
//     re-packed from the S accumulators in registers; the row max / row sum use
//     quad shuffles; exp is MUFU ex2 on log2-scaled logits.
//   * causal rule per row: key j is visible to row r iff j <= L - n_q + r.
//   * keys past the split end can be garbage (unwritten cache slots, possibly
//     NaN): their logits are masked by select and their V rows are zeroed in the
//     B fragments, so 0 * NaN never reaches an accumulator.
// fp32 KV (the CPU-runnable reference config) uses the CUDA-core kernel at the
// bottom of this file.
#include <cfloat>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "attention_common.cuh"

namespace sdb {
namespace attn {

// Producer: stream the tiles of [k0, k0 + ntiles*BN) for (b, kvh) into the ring.
template <int NS, int NCONS_PER_STAGE>
SDB_DEV void produce(const Params& p, const CUtensorMap* kmap, const CUtensorMap* vmap,
                     uint32_t stage0, uint32_t full0, uint32_t empty0, int b, int kvh, int k0,
                     int ntiles) {
    prefetch_tensormap(kmap);
    prefetch_tensormap(vmap);
    const uint64_t pol = l2_policy_evict_first();
    const int* btrow = p.bt + (int64_t)b * p.bt_stride;
    int issued = 0;
    for (int t = 0; t < ntiles; ++t) {
        const int s = t % NS;
        const int round = t / NS;
        if (round > 0 && !mbar_wait(empty0 + 8 * s, (round - 1) & 1)) {
            atomicOr(p.err, SDB_KERR_TIMEOUT);
            break;
        }
        const int j = k0 + t * BN;
        int blk = btrow[j / p.page];
        if (blk < 0 || blk >= p.num_blocks) {
            atomicOr(p.err, SDB_KERR_BLOCK_ID);
            blk = 0;
        }
        const int off = j % p.page;
        const uint32_t kdst = stage0 + s * STAGE_BYTES;
        const uint32_t vdst = kdst + TILE_BYTES;
        const uint32_t bar = full0 + 8 * s;
        mbar_arrive_expect_tx(bar, STAGE_BYTES);
        tma_load_4d(kdst, kmap, bar, 0, kvh, off, blk, pol);
        tma_load_4d(kdst + HALF_BYTES, kmap, bar, 64, kvh, off, blk, pol);
        tma_load_4d(vdst, vmap, bar, 0, kvh, off, blk, pol);
        tma_load_4d(vdst + HALF_BYTES, vmap, bar, 64, kvh, off, blk, pol);
        issued = t + 1;
    }
    // Drain: every copy this thread issued has landed before it leaves.
    for (int t = issued - NS > 0 ? issued - NS : 0; t < issued; ++t) {
        if (!mbar_wait(full0 + 8 * (t % NS), (t / NS) & 1)) {
            atomicOr(p.err, SDB_KERR_TIMEOUT);
            break;
        }
    }
}

// Byte address of 16-byte chunk c (0..15) of row `row` in a swizzled 64-row tile.
SDB_DEV uint32_t tile_addr(uint32_t base, int row, int c) {
    return base + (c >> 3) * HALF_BYTES + row * 128 + (((c & 7) ^ (row & 7)) << 4);
}

template <typename T, int MT, int KG, int NS>
__global__ void __launch_bounds__((MT * KG + 1) * 32)
    pa_mma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const Params p) {
    using H = Half16<T>;
    // Consumer warp (mt, kg) = warp mt + MT*kg owns m-tile mt and keys
    // [kg*SK, (kg+1)*SK) of every tile.  Every consumer warp waits for and
    // releases every stage, so each stage's phases are awaited in order.
    constexpr int NC = MT * KG;
    constexpr int SK = BN / KG;       // keys per warp per tile: 64, 32 or 16
    constexpr int NKT = SK / 8;       // n8 tiles of keys in S
    constexpr int NKK = SK / 16;      // k16 steps of keys in P.V
    static_assert(SK % 16 == 0, "key slice must hold whole k16 steps");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NS * STAGE_BYTES);
    int* sflag = reinterpret_cast<int*>(bars + 2 * NS);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;

    const int L = load_len(p, b);
    const int k0 = split * p.chunk;
    const int k1 = min(k0 + p.chunk, L);
    const int ntiles = k1 > k0 ? (k1 - k0 + BN - 1) / BN : 0;

    const uint32_t stage0 = smem_u32(smem);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + NS);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, NC);
        }
        fence_mbarrier_init();
    }
    __syncthreads();

    if (warp == NC) {
        if (lane == 0 && ntiles > 0) produce<NS, NC>(p, &kmap, &vmap, stage0, full0, empty0, b, kvh, k0, ntiles);
        return;
    }

    // ------------------------------------------------------------ consumers
    const int mt = warp % MT;
    const int kg = warp / MT;
    const int R = p.R;
    const int rho0 = mt * 16 + (lane >> 2);
    const int rho1 = rho0 + 8;
    const int cq = 2 * (lane & 3);
    const int kbase = kg * SK;  // first key of this warp's slice inside a tile

    // Q fragments (A operand) straight from global: rows rho0 / rho1.
    uint32_t qa[8][4];
    int lim0 = k1, lim1 = k1;
    {
        const T* qbase = reinterpret_cast<const T*>(p.q);
        const uint32_t* q0 = nullptr;
        const uint32_t* q1 = nullptr;
        if (rho0 < R) {
            const int r = rho0 / p.G, g = rho0 % p.G;
            q0 = reinterpret_cast<const uint32_t*>(qbase + (int64_t)(b * p.n_q + r) * p.q_srow +
                                                   (int64_t)(kvh * p.G + g) * p.q_shead);
            lim0 = min(L - p.n_q + r + 1, k1);
        }
        if (rho1 < R) {
            const int r = rho1 / p.G, g = rho1 % p.G;
            q1 = reinterpret_cast<const uint32_t*>(qbase + (int64_t)(b * p.n_q + r) * p.q_srow +
                                                   (int64_t)(kvh * p.G + g) * p.q_shead);
            lim1 = min(L - p.n_q + r + 1, k1);
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int e0 = (ks * 16 + cq) >> 1;
            const int e1 = (ks * 16 + 8 + cq) >> 1;
            qa[ks][0] = q0 ? __ldg(q0 + e0) : 0u;
            qa[ks][2] = q0 ? __ldg(q0 + e1) : 0u;
            qa[ks][1] = q1 ? __ldg(q1 + e0) : 0u;
            qa[ks][3] = q1 ? __ldg(q1 + e1) : 0u;
        }
    }

    float m0 = NEG_INF, m1 = NEG_INF, l0 = 0.f, l1 = 0.f;
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    const float sl2 = p.scale_log2;
    for (int t = 0; t < ntiles; ++t) {
        const int s = t % NS;
        if (!mbar_wait(full0 + 8 * s, (t / NS) & 1)) {
            if (lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
            break;
        }
        const uint32_t kb = stage0 + s * STAGE_BYTES;
        const uint32_t vb = kb + TILE_BYTES;
        const int j0 = k0 + t * BN + kbase;  // first key of this warp's slice

        // ---- S = Q K^T over the slice (16 x SK per warp)
        float sc[NKT][4];
#pragma unroll
        for (int i = 0; i < NKT; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
            for (int np = 0; np < NKT / 2; ++np) {
                const int key = kbase + np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int c = ks * 2 + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, tile_addr(kb, key, c));
                H::mma(sc[2 * np], qa[ks], b0, b1);
                H::mma(sc[2 * np + 1], qa[ks], b2, b3);
            }
        }

        // ---- scale, mask, online softmax
        const bool masked = (j0 + SK > lim0) || (j0 + SK > lim1);
        float mx0 = NEG_INF, mx1 = NEG_INF;
#pragma unroll
        for (int nt = 0; nt < NKT; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float x0 = sc[nt][e] * sl2;
                float x1 = sc[nt][2 + e] * sl2;
                if (masked) {
                    const int j = j0 + nt * 8 + cq + e;
                    x0 = j < lim0 ? x0 : NEG_INF;
                    x1 = j < lim1 ? x1 : NEG_INF;
                }
                sc[nt][e] = x0;
                sc[nt][2 + e] = x1;
                mx0 = fmaxf(mx0, x0);
                mx1 = fmaxf(mx1, x1);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float base0 = mn0 == NEG_INF ? 0.f : mn0;
        const float base1 = mn1 == NEG_INF ? 0.f : mn1;
        const float a0 = ex2(m0 - base0), a1 = ex2(m1 - base1);
        m0 = mn0;
        m1 = mn1;
        float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < NKT; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                sc[nt][e] = ex2(sc[nt][e] - base0);
                sc[nt][2 + e] = ex2(sc[nt][2 + e] - base1);
                ls0 += sc[nt][e];
                ls1 += sc[nt][2 + e];
            }
        }
        l0 = l0 * a0 + ls0;
        l1 = l1 * a1 + ls1;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            o[i][0] *= a0;
            o[i][1] *= a0;
            o[i][2] *= a1;
            o[i][3] *= a1;
        }

        // ---- O += P V with P = P_hi + P_lo (both 16-bit): the second product
        // carries the rounding residual of P, so O keeps ~16 bits of P.
        const bool vmask = j0 + SK > k1;
#pragma unroll
        for (int kk = 0; kk < NKK; ++kk) {
            uint32_t ph[4], pl[4];
            {
                const float* c0 = sc[2 * kk];
                const float* c1 = sc[2 * kk + 1];
                ph[0] = H::pack(c0[0], c0[1]);
                ph[1] = H::pack(c0[2], c0[3]);
                ph[2] = H::pack(c1[0], c1[1]);
                ph[3] = H::pack(c1[2], c1[3]);
                pl[0] = H::pack_residual(c0[0], c0[1], ph[0]);
                pl[1] = H::pack_residual(c0[2], c0[3], ph[1]);
                pl[2] = H::pack_residual(c1[0], c1[1], ph[2]);
                pl[3] = H::pack_residual(c1[2], c1[3], ph[3]);
            }
            // keys of this lane's B-fragment halves: kb0, kb0+1 (regs 0/2), +8 (regs 1/3)
            const int kb0 = j0 + kk * 16 + cq;
            uint32_t keep_lo = 0xffffffffu, keep_hi = 0xffffffffu;
            if (vmask) {
                keep_lo = (kb0 < k1 ? 0x0000ffffu : 0u) | (kb0 + 1 < k1 ? 0xffff0000u : 0u);
                keep_hi = (kb0 + 8 < k1 ? 0x0000ffffu : 0u) | (kb0 + 9 < k1 ? 0xffff0000u : 0u);
            }
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {
                const int key = kbase + kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int c = dp * 2 + (lane >> 4);
                uint32_t r0, r1, r2, r3;
                ldsm_x4_t(r0, r1, r2, r3, tile_addr(vb, key, c));
                r0 &= keep_lo;
                r2 &= keep_lo;
                r1 &= keep_hi;
                r3 &= keep_hi;
                H::mma(o[2 * dp], ph, r0, r1);
                H::mma(o[2 * dp + 1], ph, r2, r3);
                H::mma(o[2 * dp], pl, r0, r1);
                H::mma(o[2 * dp + 1], pl, r2, r3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
    }

    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // ------------------------------------------ merge the key groups (stage ring reused)
    if (KG > 1) {
        named_barrier_sync(1, NC * 32);  // every consumer is past its last stage read
        float* scr = reinterpret_cast<float*>(smem);  // [(KG-1)][MT][16][D+2]
        constexpr int ROWF = D + 2;
        const int ra = lane >> 2, rb = ra + 8;
        if (kg > 0) {
            float* base = scr + ((kg - 1) * MT + mt) * 16 * ROWF;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                *reinterpret_cast<float2*>(base + ra * ROWF + i * 8 + cq) = make_float2(o[i][0], o[i][1]);
                *reinterpret_cast<float2*>(base + rb * ROWF + i * 8 + cq) = make_float2(o[i][2], o[i][3]);
            }
            if ((lane & 3) == 0) {
                base[ra * ROWF + D] = m0;
                base[ra * ROWF + D + 1] = l0;
                base[rb * ROWF + D] = m1;
                base[rb * ROWF + D + 1] = l1;
            }
        }
        named_barrier_sync(1, NC * 32);
        if (kg > 0) return;
        for (int g2 = 1; g2 < KG; ++g2) {
            const float* base = scr + ((g2 - 1) * MT + mt) * 16 * ROWF;
            const float om0 = base[ra * ROWF + D], ol0 = base[ra * ROWF + D + 1];
            const float om1 = base[rb * ROWF + D], ol1 = base[rb * ROWF + D + 1];
            const float M0 = fmaxf(m0, om0), M1 = fmaxf(m1, om1);
            const float B0 = M0 == NEG_INF ? 0.f : M0, B1 = M1 == NEG_INF ? 0.f : M1;
            const float w0 = ex2(m0 - B0), v0 = ex2(om0 - B0);
            const float w1 = ex2(m1 - B1), v1 = ex2(om1 - B1);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float2 x = *reinterpret_cast<const float2*>(base + ra * ROWF + i * 8 + cq);
                const float2 y = *reinterpret_cast<const float2*>(base + rb * ROWF + i * 8 + cq);
                o[i][0] = o[i][0] * w0 + x.x * v0;
                o[i][1] = o[i][1] * w0 + x.y * v0;
                o[i][2] = o[i][2] * w1 + y.x * v1;
                o[i][3] = o[i][3] * w1 + y.y * v1;
            }
            l0 = l0 * w0 + ol0 * v0;
            l1 = l1 * w1 + ol1 * v1;
            m0 = M0;
            m1 = M1;
        }
    }

    // ------------------------------------------ epilogue
    T* obase = reinterpret_cast<T*>(p.out);
    if (p.splits == 1) {
        const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
        const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
        if (rho0 < R) {
            const int r = rho0 / p.G, g = rho0 % p.G;
            T* dst = obase + (int64_t)(b * p.n_q + r) * p.o_srow + (int64_t)(kvh * p.G + g) * p.o_shead;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                *reinterpret_cast<uint32_t*>(dst + i * 8 + cq) = H::pack(o[i][0] * inv0, o[i][1] * inv0);
        }
        if (rho1 < R) {
            const int r = rho1 / p.G, g = rho1 % p.G;
            T* dst = obase + (int64_t)(b * p.n_q + r) * p.o_srow + (int64_t)(kvh * p.G + g) * p.o_shead;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                *reinterpret_cast<uint32_t*>(dst + i * 8 + cq) = H::pack(o[i][2] * inv1, o[i][3] * inv1);
        }
        return;
    }

    const int pair = b * p.Hkv + kvh;
    const int64_t slot = (int64_t)pair * p.splits + split;
    float* po = p.part_o + slot * R * D;
    float* pml = p.part_ml + slot * R * 2;
    if (rho0 < R) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
            __stcg(reinterpret_cast<float2*>(po + rho0 * D + i * 8 + cq), make_float2(o[i][0], o[i][1]));
        if ((lane & 3) == 0) __stcg(reinterpret_cast<float2*>(pml + rho0 * 2), make_float2(m0, l0));
    }
    if (rho1 < R) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
            __stcg(reinterpret_cast<float2*>(po + rho1 * D + i * 8 + cq), make_float2(o[i][2], o[i][3]));
        if ((lane & 3) == 0) __stcg(reinterpret_cast<float2*>(pml + rho1 * 2), make_float2(m1, l1));
    }
    __threadfence();
    named_barrier_sync(2, MT * 32);
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(p.counters + pair, 1);
        *sflag = (prev == p.splits - 1);
    }
    named_barrier_sync(2, MT * 32);
    if (!*sflag) return;
    __threadfence();

    // Last CTA of this (sequence, kv head): LSE-merge the splits.
    float* coef = reinterpret_cast<float*>(smem);  // [splits][R]
    const float* ml = p.part_ml + (int64_t)pair * p.splits * R * 2;
    const float* pob = p.part_o + (int64_t)pair * p.splits * R * D;
    for (int rho = threadIdx.x; rho < R; rho += MT * 32) {
        float M = NEG_INF;
        for (int s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(ml + (s * R + rho) * 2));
        const float Bm = M == NEG_INF ? 0.f : M;
        float Lsum = 0.f;
        for (int s = 0; s < p.splits; ++s) {
            const float w = ex2(__ldcg(ml + (s * R + rho) * 2) - Bm);
            coef[s * R + rho] = w;
            Lsum += w * __ldcg(ml + (s * R + rho) * 2 + 1);
        }
        const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
        for (int s = 0; s < p.splits; ++s) coef[s * R + rho] *= inv;
    }
    named_barrier_sync(2, MT * 32);
    for (int idx = threadIdx.x; idx < R * (D / 4); idx += MT * 32) {
        const int rho = idx / (D / 4);
        const int d4 = idx % (D / 4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < p.splits; ++s) {
            const float c = coef[s * R + rho];
            const float4 x = __ldcg(reinterpret_cast<const float4*>(pob + ((int64_t)s * R + rho) * D) + d4);
            acc.x += c * x.x;
            acc.y += c * x.y;
            acc.z += c * x.z;
            acc.w += c * x.w;
        }
        const int r = rho / p.G, g = rho % p.G;
        T* dst = obase + (int64_t)(b * p.n_q + r) * p.o_srow + (int64_t)(kvh * p.G + g) * p.o_shead + d4 * 4;
        uint2 v;
        v.x = H::pack(acc.x, acc.y);
        v.y = H::pack(acc.z, acc.w);
        *reinterpret_cast<uint2*>(dst) = v;
    }
    if (threadIdx.x == 0) p.counters[pair] = 0;  // graph-replay safe: ready for the next call
}

// Memory floor: same grid, same TMA stream of every visible K/V tile, no math.
template <int NS>
__global__ void __launch_bounds__(2 * 32)
    pa_readonly_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NS * STAGE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int L = load_len(p, b);
    const int k0 = split * p.chunk;
    const int k1 = min(k0 + p.chunk, L);
    const int ntiles = k1 > k0 ? (k1 - k0 + BN - 1) / BN : 0;
    const uint32_t stage0 = smem_u32(smem), full0 = smem_u32(bars), empty0 = smem_u32(bars + NS);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        fence_mbarrier_init();
    }
    __syncthreads();
    if (warp == 1) {
        if (lane == 0 && ntiles > 0) produce<NS, 1>(p, &kmap, &vmap, stage0, full0, empty0, b, kvh, k0, ntiles);
        return;
    }
    unsigned acc = 0;
    for (int t = 0; t < ntiles; ++t) {
        const int s = t % NS;
        if (!mbar_wait(full0 + 8 * s, (t / NS) & 1)) {
            if (lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
            break;
        }
        acc ^= *reinterpret_cast<const unsigned*>(smem + s * STAGE_BYTES + lane * 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
    }
    acc = __reduce_xor_sync(0xffffffffu, acc);
    if (lane == 0) p.checksum[(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x] = acc;
}

// ---------------------------------------------------------------------------
// CUDA-core path: fp32 (or 16-bit) KV with any page size and head_dim 64/128/256.
// grid (Hkv, B), 4 warps striding over keys; lane owns DPL = D/32 dims; rows are
// processed RC at a time.  Online softmax per key in fp32.
// ---------------------------------------------------------------------------
template <typename T, int DPL, int RC>
__global__ void __launch_bounds__(128)
    pa_simt_kernel(const Params p, const T* __restrict__ kc, const T* __restrict__ vc, int64_t sb,
                   int64_t sp, int64_t sh) {
    constexpr int DD = DPL * 32;
    __shared__ float sm_o[4][RC][DD];
    __shared__ float sm_ml[4][RC][2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = blockIdx.x, b = blockIdx.y;
    const int L = load_len(p, b);
    const int R = p.R;
    const int* btrow = p.bt + (int64_t)b * p.bt_stride;
    const T* qbase = reinterpret_cast<const T*>(p.q);
    T* obase = reinterpret_cast<T*>(p.out);

    for (int rc0 = 0; rc0 < R; rc0 += RC) {
        float q[RC][DPL], o[RC][DPL], m[RC], l[RC];
        int lim[RC];
#pragma unroll
        for (int i = 0; i < RC; ++i) {
            const int rho = rc0 + i;
            m[i] = NEG_INF;
            l[i] = 0.f;
            lim[i] = 0;
#pragma unroll
            for (int d = 0; d < DPL; ++d) o[i][d] = q[i][d] = 0.f;
            if (rho < R) {
                const int r = rho / p.G, g = rho % p.G;
                const T* qr = qbase + (int64_t)(b * p.n_q + r) * p.q_srow + (int64_t)(kvh * p.G + g) * p.q_shead;
#pragma unroll
                for (int d = 0; d < DPL; ++d) q[i][d] = to_f32(qr[lane * DPL + d]);
                lim[i] = min(L - p.n_q + r + 1, L);
            }
        }
        for (int j = warp; j < L; j += 4) {
            int blk = btrow[j / p.page];
            if (blk < 0 || blk >= p.num_blocks) {
                if (lane == 0) atomicOr(p.err, SDB_KERR_BLOCK_ID);
                blk = 0;
            }
            const int64_t off = (int64_t)blk * sb + (int64_t)(j % p.page) * sp + (int64_t)kvh * sh + lane * DPL;
            float kr[DPL], vr[DPL];
#pragma unroll
            for (int d = 0; d < DPL; ++d) {
                kr[d] = to_f32(kc[off + d]);
                vr[d] = to_f32(vc[off + d]);
            }
#pragma unroll
            for (int i = 0; i < RC; ++i) {
                float dot = 0.f;
#pragma unroll
                for (int d = 0; d < DPL; ++d) dot = fmaf(q[i][d], kr[d], dot);
#pragma unroll
                for (int sft = 16; sft > 0; sft >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, sft);
                if (j < lim[i]) {
                    const float x = dot * p.scale_log2;
                    const float mn = fmaxf(m[i], x);
                    const float a = exp2f(m[i] - mn);
                    const float e = exp2f(x - mn);
                    l[i] = l[i] * a + e;
#pragma unroll
                    for (int d = 0; d < DPL; ++d) o[i][d] = o[i][d] * a + e * vr[d];
                    m[i] = mn;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < RC; ++i) {
#pragma unroll
            for (int d = 0; d < DPL; ++d) sm_o[warp][i][lane * DPL + d] = o[i][d];
            if (lane == 0) {
                sm_ml[warp][i][0] = m[i];
                sm_ml[warp][i][1] = l[i];
            }
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < RC * DD; idx += 128) {
            const int i = idx / DD, d = idx % DD;
            const int rho = rc0 + i;
            if (rho >= R) continue;
            float M = NEG_INF;
            for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[w][i][0]);
            float acc = 0.f, Ls = 0.f;
            if (M != NEG_INF) {
                for (int w = 0; w < 4; ++w) {
                    const float c = exp2f(sm_ml[w][i][0] - M);
                    acc += c * sm_o[w][i][d];
                    Ls += c * sm_ml[w][i][1];
                }
            }
            const int r = rho / p.G, g = rho % p.G;
            T* dst = obase + (int64_t)(b * p.n_q + r) * p.o_srow + (int64_t)(kvh * p.G + g) * p.o_shead;
            dst[d] = from_f32<T>(Ls > 0.f ? acc / Ls : 0.f);
        }
        __syncthreads();
    }
}


// store_kvcache (nanovllm/layers/attention.py:10-40): row i of key/value goes to
// cache slot slot_mapping[i] = block * page + offset; slot -1 is skipped (graph
// padding rows, nanovllm/spec_decode/graph_pad.py:33-40).  One CTA per token,
// 16-byte vectors over the Hkv*D elements of the row.
__global__ void store_kvcache_kernel(const uint8_t* __restrict__ key, int64_t ks_tok, int64_t ks_head,
                                     const uint8_t* __restrict__ val, int64_t vs_tok, int64_t vs_head,
                                     uint8_t* kc, uint8_t* vc, int64_t sb, int64_t sp, int64_t sh,
                                     const int* __restrict__ slots, int Hkv, int row_bytes, int page,
                                     int num_blocks, int elem, int* err) {
    const int i = blockIdx.x;
    const int slot = slots[i];
    if (slot < 0) return;
    const int blk = slot / page, off = slot % page;
    if (blk >= num_blocks) {
        if (threadIdx.x == 0) atomicOr(err, SDB_KERR_BLOCK_ID);
        return;
    }
    const int vec_per_head = row_bytes / 16;
    for (int v = threadIdx.x; v < Hkv * vec_per_head; v += blockDim.x) {
        const int h = v / vec_per_head, c = v % vec_per_head;
        const int64_t dst = ((int64_t)blk * sb + (int64_t)off * sp + (int64_t)h * sh) * elem + c * 16;
        const uint4 kx = *reinterpret_cast<const uint4*>(key + ((int64_t)i * ks_tok + (int64_t)h * ks_head) * elem + c * 16);
        const uint4 vx = *reinterpret_cast<const uint4*>(val + ((int64_t)i * vs_tok + (int64_t)h * vs_head) * elem + c * 16);
        *reinterpret_cast<uint4*>(kc + dst) = kx;
        *reinterpret_cast<uint4*>(vc + dst) = vx;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Stage count of the K/V ring: 3 stages of 32 KB -> 2 CTAs per SM.
template <int MT>
struct Stages {
    static constexpr int NS = 3;
};
constexpr int kSmemPerSM = 233472;  // 228 KB on sm_100
// splits x R (<= 64) fp32 merge coefficients must fit the smallest stage ring (64 KB)
constexpr int kMaxSplits = 256;
static_assert(kMaxSplits * 64 * 4 <= 2 * STAGE_BYTES, "merge scratch exceeds the stage ring");

static int smem_bytes_ring(int ns) { return ns * STAGE_BYTES + 1024 + 2 * ns * 8 + 16; }
static int smem_bytes_ro() { return 4 * STAGE_BYTES + 1024 + 2 * 4 * 8 + 16; }
static int mt_for_rows(int R) { return R <= 16 ? 1 : (R <= 32 ? 2 : 4); }
static int ctas_per_sm(int R) {
    const int ns = mt_for_rows(R) == 1 ? Stages<1>::NS : Stages<2>::NS;
    const int c = kSmemPerSM / (smem_bytes_ring(ns) + 1024);
    return c < 1 ? 1 : c;
}

static bool mma_path(int dtype, int D_, int page, int R) {
    return (dtype == SDB_BF16 || dtype == SDB_F16) && D_ == D && page % BN == 0 && R <= 64;
}

static int pick_splits(int B, int R, int Hkv, int page, int max_blocks, int sms) {
    // Minimise (waves x keys per split) + merge traffic, from static shape only.
    const long long max_ctx = (long long)max_blocks * page;
    const long long tiles = (max_ctx + BN - 1) / BN;
    const long long pairs = (long long)B * Hkv;
    const long long slots = (long long)sms * ctas_per_sm(R);
    int best = 1;
    double best_cost = 1e300;
    for (int s = 1; s <= 64; ++s) {
        const long long chunk_tiles = (tiles + s - 1) / s;
        if (s > 1 && chunk_tiles < 4) break;  // keep >= 256 keys per split
        const long long ctas = pairs * s;
        const long long waves = (ctas + slots - 1) / slots;
        // per-wave cost in bytes of one CTA's KV stream + fixed CTA overhead (~8 KB)
        double cost = (double)waves * (chunk_tiles * (double)STAGE_BYTES + 8192.0);
        if (s > 1) cost += (double)pairs * s * R * (D + 2) * 8.0 / (double)slots;
        if (cost < best_cost * 0.995) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

// Split count and key chunk the mma.sync path launches for a requested `splits`
// (0: its default): at most kMaxSplits, and no split that can never hold a key.
static int mma_launch_splits(int B, int R, int Hkv, int page, int max_blocks, int splits, long long* chunk_out) {
    if (splits <= 0) splits = pick_splits(B, R, Hkv, page, max_blocks, device_sm_count());
    // the last-CTA merge keeps splits x R coefficients in the (idle) stage ring
    if (splits > kMaxSplits) splits = kMaxSplits;
    const long long max_ctx = (long long)max_blocks * page;
    long long chunk = ((max_ctx + splits - 1) / splits + BN - 1) / BN * BN;
    if (chunk < BN) chunk = BN;
    splits = (int)((max_ctx + chunk - 1) / chunk);
    *chunk_out = chunk;
    return splits < 1 ? 1 : splits;
}

}  // namespace attn
}  // namespace sdb

using namespace sdb;
using namespace sdb::attn;

bool sdb::attn::prefer_umma() {
    const char* v = getenv("SDB_ATTN_KERNEL");
    return !(v && strcmp(v, "mma") == 0);
}

extern "C" int sdb_paged_attention_default_splits(int B, int n_q, int Hq, int Hkv, int D_, int page,
                                                  int max_blocks, int dtype) {
    if (B <= 0 || n_q <= 0 || Hkv <= 0 || Hq % Hkv != 0 || page <= 0 || max_blocks <= 0) return 1;
    const int R = n_q * (Hq / Hkv);
    if (umma_path(dtype, D_, page, R) && prefer_umma())
        return pick_umma_splits(B, R, Hkv, page, max_blocks, device_sm_count());
    if (!mma_path(dtype, D_, page, R)) return 1;
    return pick_splits(B, R, Hkv, page, max_blocks, device_sm_count());
}

extern "C" size_t sdb_paged_attention_workspace_size(int B, int n_q, int Hq, int Hkv, int D_, int splits) {
    if (B <= 0 || n_q <= 0 || Hkv <= 0 || Hq % Hkv != 0 || D_ != D) {
        // CUDA-core path needs only the error word; size the partials for D anyway.
        const int R = (Hkv > 0 && Hq % Hkv == 0) ? n_q * (Hq / Hkv) : 1;
        return ws_layout(B > 0 ? B : 1, R > 0 ? R : 1, Hkv > 0 ? Hkv : 1, splits).total;
    }
    const int R = n_q * (Hq / Hkv);
    WsLayout w = ws_layout(B, R, Hkv, splits < 1 ? 1 : splits);
    // the read-only twin stores one checksum word per CTA after the partials
    return w.total + align_up(sizeof(unsigned) * (size_t)B * Hkv * (splits < 1 ? 1 : splits), 256);
}

extern "C" const int32_t* sdb_paged_attention_error_word(const void* workspace, int, int, int, int, int, int) {
    return reinterpret_cast<const int32_t*>(workspace);
}

extern "C" size_t sdb_paged_attention_plan(int B, int n_q, int Hq, int Hkv, int D_, int page, int max_blocks,
                                           int dtype, int splits, int* kernel, int* slots) {
    int k = -1, s = 0;
    size_t need = 0;
    if (B > 0 && n_q > 0 && Hkv > 0 && Hq > 0 && Hq % Hkv == 0 && page > 0 && max_blocks > 0 && D_ > 0) {
        const int R = n_q * (Hq / Hkv);
        if (umma_path(dtype, D_, page, R) && prefer_umma()) {
            const UmmaShape u = umma_launch_shape(B, Hkv, page, max_blocks, splits);
            k = u.grouped ? SDB_ATTN_PLAN_TCGEN05_GROUPED : SDB_ATTN_PLAN_TCGEN05_STRIDED;
            s = u.slots;
            need = ws_layout(B, R, Hkv, s).total;
        } else if (mma_path(dtype, D_, page, R)) {
            long long chunk = 0;
            k = SDB_ATTN_PLAN_MMA;
            s = mma_launch_splits(B, R, Hkv, page, max_blocks, splits, &chunk);
            need = ws_layout(B, R, Hkv, s).total;
        } else {
            k = SDB_ATTN_PLAN_CUDA_CORE;
            s = 1;
            need = ws_layout(B, R, Hkv, 1).err + 256;
        }
    }
    if (kernel) *kernel = k;
    if (slots) *slots = s;
    return need;
}

namespace {

struct Common {
    int R, G, splits, chunk;
    WsLayout ws;
};

int validate(const void* q, const void* k_cache, const void* v_cache, const int32_t* bt,
             const int32_t* seqlens, int B, int n_q, int Hq, int Hkv, int D_, int page, int max_blocks,
             int num_blocks, int64_t q_srow, int64_t q_shead, int64_t sb, int64_t sp, int64_t sh,
             int64_t bt_stride, const void* workspace) {
    if (!q || !k_cache || !v_cache || !bt || !seqlens || !workspace) {
        set_last_error("null pointer argument");
        return SDB_ERR_INVALID_ARG;
    }
    if (B <= 0 || n_q <= 0 || Hq <= 0 || Hkv <= 0 || D_ <= 0 || page <= 0 || max_blocks <= 0 ||
        num_blocks <= 0 || Hq % Hkv != 0) {
        set_last_error("bad sizes B=%d n_q=%d Hq=%d Hkv=%d D=%d page=%d max_blocks=%d num_blocks=%d", B, n_q, Hq,
                       Hkv, D_, page, max_blocks, num_blocks);
        return SDB_ERR_INVALID_ARG;
    }
    // head_dim is the contiguous axis of q and of the caches; the other cache axes may
    // come in any order (the reference also supports a head-major layout).
    if (q_srow <= 0 || q_shead < D_ || sh <= 0 || sp <= 0 || sb <= 0 || bt_stride < max_blocks) {
        set_last_error("unsupported strides (need a contiguous head_dim and positive strides)");
        return SDB_ERR_INVALID_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) {
        set_last_error("workspace must be 256-byte aligned");
        return SDB_ERR_WORKSPACE;
    }
    return SDB_OK;
}

template <typename T, int MT, int KG>
int launch_mma(const CUtensorMap& km, const CUtensorMap& vm, const Params& p, dim3 grid, cudaStream_t st, int slot) {
    constexpr int NS = Stages<MT>::NS;
    auto kern = pa_mma_kernel<T, MT, KG, NS>;
    const int smem = smem_bytes_ring(NS);
    int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem, slot);
    if (rc) return rc;
    kern<<<grid, (MT * KG + 1) * 32, smem, st>>>(km, vm, p);
    return cuda_status(cudaGetLastError(), "pa_mma_kernel launch");
}

// Four consumer warps per CTA in every configuration: 1 m-tile x 4 key slices
// (decode), 2 x 2 (k+1 verify rows of a GQA-4 group), 4 x 1 (up to 64 rows).
template <typename T>
int dispatch_mma(const CUtensorMap& km, const CUtensorMap& vm, const Params& p, dim3 grid, cudaStream_t st) {
    const int base = std::is_same<T, __half>::value ? 10 : 0;
    switch (mt_for_rows(p.R)) {
        case 1: return launch_mma<T, 1, 4>(km, vm, p, grid, st, base + 0);
        case 2: return launch_mma<T, 2, 2>(km, vm, p, grid, st, base + 1);
        default: return launch_mma<T, 4, 1>(km, vm, p, grid, st, base + 2);
    }
}

int make_maps(CUtensorMap* km, CUtensorMap* vm, const void* k_cache, const void* v_cache, int dtype, int Hkv,
              int page, int num_blocks, int64_t sb, int64_t sp, int64_t sh) {
    const CUtensorMapDataType dt =
        dtype == SDB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
        ((sh * 2) & 15) || ((sp * 2) & 15) || ((sb * 2) & 15)) {
        set_last_error("KV cache base and strides must be 16-byte aligned for TMA");
        return SDB_ERR_INVALID_ARG;
    }
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)page, (cuuint64_t)num_blocks};
    cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)sp * 2, (cuuint64_t)sb * 2};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)BN, 1};
    int rc = encode_tensor_map(km, dt, 4, const_cast<void*>(k_cache), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    return encode_tensor_map(vm, dt, 4, const_cast<void*>(v_cache), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// The new rows of a fused store + attention call (strides in elements).
struct StoreArgs {
    const void* key;
    int64_t ks_tok, ks_head;
    const void* value;
    int64_t vs_tok, vs_head;
    const int32_t* slots;
};

int check_store(const void* key, int64_t ks_tok, int64_t ks_head, const void* value, int64_t vs_tok,
                int64_t vs_head, const void* k_cache, const void* v_cache, int64_t sb, int64_t sp, int64_t sh,
                const int32_t* slots, int N, int Hkv, int D_, int page, int num_blocks, int dtype,
                const void* workspace) {
    if (!key || !value || !k_cache || !v_cache || !slots || !workspace || N < 0 || Hkv <= 0 || D_ <= 0 ||
        page <= 0 || num_blocks <= 0) {
        set_last_error("bad arguments to store_kvcache");
        return SDB_ERR_INVALID_ARG;
    }
    if (dtype != SDB_F32 && dtype != SDB_BF16 && dtype != SDB_F16) {
        set_last_error("dtype %d not supported", dtype);
        return SDB_ERR_UNSUPPORTED;
    }
    const int elem = dtype == SDB_F32 ? 4 : 2;
    auto mis = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
    if (((D_ * elem) & 15) || mis(key) || mis(value) || mis(k_cache) || mis(v_cache) || ((ks_tok * elem) & 15) ||
        ((ks_head * elem) & 15) || ((vs_tok * elem) & 15) || ((vs_head * elem) & 15) || ((sb * elem) & 15) ||
        ((sp * elem) & 15) || ((sh * elem) & 15)) {
        set_last_error("store_kvcache needs 16-byte aligned rows and strides");
        return SDB_ERR_INVALID_ARG;
    }
    return SDB_OK;
}

int launch_store(const StoreArgs& a, void* k_cache, void* v_cache, int64_t sb, int64_t sp, int64_t sh, int N,
                 int Hkv, int D_, int page, int num_blocks, int dtype, void* workspace, cudaStream_t st) {
    if (N == 0) return SDB_OK;
    const int elem = dtype == SDB_F32 ? 4 : 2;
    const int row_bytes = D_ * elem;
    int threads = Hkv * (row_bytes / 16);
    threads = threads > 256 ? 256 : (threads < 32 ? 32 : threads);
    store_kvcache_kernel<<<N, threads, 0, st>>>(
        reinterpret_cast<const uint8_t*>(a.key), a.ks_tok, a.ks_head, reinterpret_cast<const uint8_t*>(a.value),
        a.vs_tok, a.vs_head, reinterpret_cast<uint8_t*>(k_cache), reinterpret_cast<uint8_t*>(v_cache), sb, sp, sh,
        a.slots, Hkv, row_bytes, page, num_blocks, elem, reinterpret_cast<int*>(workspace));
    return cuda_status(cudaGetLastError(), "store_kvcache launch");
}

int attention_impl(const void* q, int64_t q_srow, int64_t q_shead, const void* k_cache, const void* v_cache,
                   int64_t sb, int64_t sp, int64_t sh, const int32_t* block_tables, int64_t bt_stride,
                   const int32_t* cache_seqlens, void* out, int64_t o_srow, int64_t o_shead, int B, int n_q, int Hq,
                   int Hkv, int D_, int page, int max_blocks, int num_blocks, float softmax_scale, int dtype,
                   int splits, void* workspace, size_t workspace_bytes, void* stream, const StoreArgs* store) {
    int rc = validate(q, k_cache, v_cache, block_tables, cache_seqlens, B, n_q, Hq, Hkv, D_, page, max_blocks,
                      num_blocks, q_srow, q_shead, sb, sp, sh, bt_stride, workspace);
    if (rc) return rc;
    if (store) {
        rc = check_store(store->key, store->ks_tok, store->ks_head, store->value, store->vs_tok, store->vs_head,
                         k_cache, v_cache, sb, sp, sh, store->slots, B * n_q, Hkv, D_, page, num_blocks, dtype,
                         workspace);
        if (rc) return rc;
    }
    if (!out || o_shead < D_) {
        set_last_error("bad output pointer or stride");
        return SDB_ERR_INVALID_ARG;
    }
    if (dtype != SDB_F32 && dtype != SDB_BF16 && dtype != SDB_F16) {
        set_last_error("dtype %d not supported", dtype);
        return SDB_ERR_UNSUPPORTED;
    }
    const int G = Hq / Hkv;
    const int R = n_q * G;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    Params p{};
    p.q = q;
    p.q_srow = q_srow;
    p.q_shead = q_shead;
    p.out = out;
    p.o_srow = o_srow;
    p.o_shead = o_shead;
    p.bt = block_tables;
    p.bt_stride = bt_stride;
    p.seqlens = cache_seqlens;
    p.B = B;
    p.n_q = n_q;
    p.G = G;
    p.R = R;
    p.Hkv = Hkv;
    p.page = page;
    p.max_blocks = max_blocks;
    p.num_blocks = num_blocks;
    p.scale_log2 = softmax_scale * 1.4426950408889634f;

    if (umma_path(dtype, D_, page, R) && prefer_umma()) {
        if ((long long)B * Hkv > kCounterCap) {
            set_last_error("B * Hkv = %lld exceeds the supported %d (sequence, kv head) pairs", (long long)B * Hkv,
                           kCounterCap);
            return SDB_ERR_UNSUPPORTED;
        }
        if ((reinterpret_cast<uintptr_t>(q) & 15) || (q_srow % 8) || (q_shead % 8) ||
            (reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
            ((sh * 2) & 15) || ((sp * 2) & 15) || ((sb * 2) & 15)) {
            set_last_error("q rows and the KV cache must be 16-byte aligned");
            return SDB_ERR_INVALID_ARG;
        }
        if (store) {  // the attention kernel writes the new rows itself
            p.slots = store->slots;
            p.new_k = reinterpret_cast<const uint8_t*>(store->key);
            p.new_v = reinterpret_cast<const uint8_t*>(store->value);
            p.nk_stok = store->ks_tok * 2;
            p.nk_shead = store->ks_head * 2;
            p.nv_stok = store->vs_tok * 2;
            p.nv_shead = store->vs_head * 2;
            p.kc = reinterpret_cast<uint8_t*>(const_cast<void*>(k_cache));
            p.vc = reinterpret_cast<uint8_t*>(const_cast<void*>(v_cache));
            p.c_sb = sb * 2;
            p.c_sp = sp * 2;
            p.c_sh = sh * 2;
        }
        return launch_umma(k_cache, v_cache, dtype, sb, sp, sh, p, workspace, workspace_bytes, splits, st);
    }
    if (store) {  // other paths: the store kernel, then attention
        rc = launch_store(*store, const_cast<void*>(k_cache), const_cast<void*>(v_cache), sb, sp, sh, B * n_q, Hkv,
                          D_, page, num_blocks, dtype, workspace, st);
        if (rc) return rc;
    }

    if (mma_path(dtype, D_, page, R)) {
        long long chunk = 0;
        splits = mma_launch_splits(B, R, Hkv, page, max_blocks, splits, &chunk);
        if ((long long)B * Hkv > kCounterCap) {
            set_last_error("B * Hkv = %lld exceeds the supported %d (sequence, kv head) pairs", (long long)B * Hkv,
                           kCounterCap);
            return SDB_ERR_UNSUPPORTED;
        }
        WsLayout w = ws_layout(B, R, Hkv, splits);
        if (workspace_bytes < w.total) {
            set_last_error("workspace too small: need %zu bytes, got %zu", w.total, workspace_bytes);
            return SDB_ERR_WORKSPACE;
        }
        uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
        p.err = reinterpret_cast<int*>(ws + w.err);
        p.counters = reinterpret_cast<int*>(ws + w.counters);
        p.part_ml = reinterpret_cast<float*>(ws + w.part_ml);
        p.part_o = reinterpret_cast<float*>(ws + w.part_o);
        p.splits = splits;
        p.chunk = (int)chunk;
        CUtensorMap km, vm;
        rc = make_maps(&km, &vm, k_cache, v_cache, dtype, Hkv, page, num_blocks, sb, sp, sh);
        if (rc) return rc;
        dim3 grid(splits, Hkv, B);
        if (dtype == SDB_BF16) return dispatch_mma<__nv_bfloat16>(km, vm, p, grid, st);
        return dispatch_mma<__half>(km, vm, p, grid, st);
    }

    // CUDA-core path (fp32 KV, or shapes outside the tensor-core kernel)
    if (!(D_ == 32 || D_ == 64 || D_ == 128 || D_ == 256) || R > 64) {
        set_last_error("unsupported shape for the CUDA-core path: D=%d rows=%d", D_, R);
        return SDB_ERR_UNSUPPORTED;
    }
    WsLayout w = ws_layout(B, R, Hkv, 1);
    if (workspace_bytes < w.err + 256) {
        set_last_error("workspace too small");
        return SDB_ERR_WORKSPACE;
    }
    p.err = reinterpret_cast<int*>(workspace);
    p.splits = 1;
    dim3 grid(Hkv, B);
#define SDB_SIMT(T, DPL)                                                                                       \
    pa_simt_kernel<T, DPL, 8><<<grid, 128, 0, st>>>(p, reinterpret_cast<const T*>(k_cache),                 \
                                                    reinterpret_cast<const T*>(v_cache), sb, sp, sh)
    if (dtype == SDB_F32) {
        if (D_ == 32) SDB_SIMT(float, 1);
        else if (D_ == 64) SDB_SIMT(float, 2);
        else if (D_ == 128) SDB_SIMT(float, 4);
        else SDB_SIMT(float, 8);
    } else if (dtype == SDB_BF16) {
        if (D_ == 32) SDB_SIMT(__nv_bfloat16, 1);
        else if (D_ == 64) SDB_SIMT(__nv_bfloat16, 2);
        else if (D_ == 128) SDB_SIMT(__nv_bfloat16, 4);
        else SDB_SIMT(__nv_bfloat16, 8);
    } else {
        if (D_ == 32) SDB_SIMT(__half, 1);
        else if (D_ == 64) SDB_SIMT(__half, 2);
        else if (D_ == 128) SDB_SIMT(__half, 4);
        else SDB_SIMT(__half, 8);
    }
#undef SDB_SIMT
    return cuda_status(cudaGetLastError(), "pa_simt_kernel launch");
}

}  // namespace

extern "C" int sdb_paged_attention(const void* q, int64_t q_srow, int64_t q_shead, const void* k_cache,
                                   const void* v_cache, int64_t sb, int64_t sp, int64_t sh,
                                   const int32_t* block_tables, int64_t bt_stride, const int32_t* cache_seqlens,
                                   void* out, int64_t o_srow, int64_t o_shead, int B, int n_q, int Hq, int Hkv,
                                   int D_, int page, int max_blocks, int num_blocks, float softmax_scale,
                                   int dtype, int splits, void* workspace, size_t workspace_bytes, void* stream) {
    return attention_impl(q, q_srow, q_shead, k_cache, v_cache, sb, sp, sh, block_tables, bt_stride, cache_seqlens,
                          out, o_srow, o_shead, B, n_q, Hq, Hkv, D_, page, max_blocks, num_blocks, softmax_scale,
                          dtype, splits, workspace, workspace_bytes, stream, nullptr);
}

extern "C" int sdb_paged_attention_store(const void* q, int64_t q_srow, int64_t q_shead, const void* key,
                                         int64_t ks_tok, int64_t ks_head, const void* value, int64_t vs_tok,
                                         int64_t vs_head, const int32_t* slot_mapping, void* k_cache, void* v_cache,
                                         int64_t sb, int64_t sp, int64_t sh, const int32_t* block_tables,
                                         int64_t bt_stride, const int32_t* cache_seqlens, void* out, int64_t o_srow,
                                         int64_t o_shead, int B, int n_q, int Hq, int Hkv, int D_, int page,
                                         int max_blocks, int num_blocks, float softmax_scale, int dtype, int splits,
                                         void* workspace, size_t workspace_bytes, void* stream) {
    const StoreArgs a{key, ks_tok, ks_head, value, vs_tok, vs_head, slot_mapping};
    return attention_impl(q, q_srow, q_shead, k_cache, v_cache, sb, sp, sh, block_tables, bt_stride, cache_seqlens,
                          out, o_srow, o_shead, B, n_q, Hq, Hkv, D_, page, max_blocks, num_blocks, softmax_scale,
                          dtype, splits, workspace, workspace_bytes, stream, &a);
}

extern "C" int sdb_paged_attention_readonly(const void* q, int64_t q_srow, int64_t q_shead, const void* k_cache,
                                            const void* v_cache, int64_t sb, int64_t sp, int64_t sh,
                                            const int32_t* block_tables, int64_t bt_stride,
                                            const int32_t* cache_seqlens, int B, int n_q, int Hq, int Hkv, int D_,
                                            int page, int max_blocks, int num_blocks, int dtype, int splits,
                                            void* workspace, size_t workspace_bytes, void* stream) {
    int rc = validate(q, k_cache, v_cache, block_tables, cache_seqlens, B, n_q, Hq, Hkv, D_, page, max_blocks,
                      num_blocks, q_srow, q_shead, sb, sp, sh, bt_stride, workspace);
    if (rc) return rc;
    const int R = n_q * (Hq / Hkv);
    if (!mma_path(dtype, D_, page, R)) {
        set_last_error("read-only twin exists for the tensor-core path only");
        return SDB_ERR_UNSUPPORTED;
    }
    long long chunk = 0;
    splits = mma_launch_splits(B, R, Hkv, page, max_blocks, splits, &chunk);
    WsLayout w = ws_layout(B, R, Hkv, splits);
    const size_t need = w.total + align_up(sizeof(unsigned) * (size_t)B * Hkv * splits, 256);
    if (workspace_bytes < need) {
        set_last_error("workspace too small: need %zu bytes", need);
        return SDB_ERR_WORKSPACE;
    }
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    Params p{};
    p.bt = block_tables;
    p.bt_stride = bt_stride;
    p.seqlens = cache_seqlens;
    p.B = B;
    p.n_q = n_q;
    p.G = Hq / Hkv;
    p.R = R;
    p.Hkv = Hkv;
    p.page = page;
    p.max_blocks = max_blocks;
    p.num_blocks = num_blocks;
    p.splits = splits;
    p.chunk = (int)chunk;
    p.err = reinterpret_cast<int*>(ws + w.err);
    p.checksum = reinterpret_cast<unsigned*>(ws + w.total);
    CUtensorMap km, vm;
    rc = make_maps(&km, &vm, k_cache, v_cache, dtype, Hkv, page, num_blocks, sb, sp, sh);
    if (rc) return rc;
    auto kern = pa_readonly_kernel<4>;
    rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem_bytes_ro(), 30);
    if (rc) return rc;
    kern<<<dim3(splits, Hkv, B), 64, smem_bytes_ro(), reinterpret_cast<cudaStream_t>(stream)>>>(km, vm, p);
    return cuda_status(cudaGetLastError(), "pa_readonly_kernel launch");
}

extern "C" int sdb_store_kvcache(const void* key, int64_t ks_tok, int64_t ks_head, const void* value, int64_t vs_tok,
                                 int64_t vs_head, void* k_cache, void* v_cache, int64_t sb, int64_t sp, int64_t sh,
                                 const int32_t* slot_mapping, int N, int Hkv, int D_, int page, int num_blocks,
                                 int dtype, void* workspace, void* stream) {
    if (N == 0) return SDB_OK;
    int rc = check_store(key, ks_tok, ks_head, value, vs_tok, vs_head, k_cache, v_cache, sb, sp, sh, slot_mapping, N,
                         Hkv, D_, page, num_blocks, dtype, workspace);
    if (rc) return rc;
    const StoreArgs a{key, ks_tok, ks_head, value, vs_tok, vs_head, slot_mapping};
    return launch_store(a, k_cache, v_cache, sb, sp, sh, N, Hkv, D_, page, num_blocks, dtype, workspace,
                        reinterpret_cast<cudaStream_t>(stream));
}
