// Paged decode / verify attention on the 5th-generation tensor cores (tcgen05).
//
// Same contract and semantics as pa_mma_kernel (csrc/attention.cu, reference
// behaviour nanovllm/layers/attention.py:64-81); this kernel takes the shapes
// with 16-bit KV, head_dim 128, page % 128 == 0 and at most 32 query rows per
// (sequence, kv head) -- Qwen3 decode (4 rows) and k <= 7 verify (k+1 rows of a
// GQA-4 group).
//
// Formulation (transposed, so the 128-row tensor-core tile is the key axis):
//   S^T[key, row] = K[key, :] . Q[row, :]        M = 128 keys, N = 32 rows, K = 128 dims
//   O^T[dim, row] += V^T[dim, key] . P[key, row]  M = 128 dims, N = 64, K = 128 keys
// Both accumulators live in tensor memory (TMEM): S^T double-buffered in
// columns [0, 64), O^T head / residual parts in [64, 96) / [96, 128).  K, V and Q
// arrive by TMA in the 128-byte-swizzled layout the MMA descriptors read directly
// (K as a K-major A operand, V as an MN-major A operand, Q^T as a K-major B
// operand); P is written by the softmax warps key-major into its own buffer (an
// MN-major B operand).
// P is split into a 16-bit head and a 16-bit residual and both multiply V, so the
// probabilities keep ~16 significant bits.
//
// Warp roles (352 threads, one CTA per SM, persistent over work items):
//   warp 0      TMA producers: lane 0 Q of each item and K tiles of 128 keys, lane 1
//               V tiles, into two 3-slot rings (a K slot is released by S(t), a V slot
//               by P.V(t))
//   warp 1      TMEM owner and S issuer (one thread)
//   warp 10     P.V issuer (one thread): S and P.V are issued independently, so the
//               tensor core gets S(t+1) while P.V(t) still waits for the softmax
//   warps 2..9  (fused store_kvcache only) first copy the step's new K/V rows of
//               the CTA's items into the cache, then
//               softmax: thread = one TMEM lane (a key of S^T, a dim of O^T) and
//               16 of the 32 columns (rows); column max / sum by an in-warp
//               transpose reduction + a 4-warp exchange; lazy rescale (O is
//               rescaled only when a row max grows by more than 2^8, exact
//               because the reference point is kept).
// Work items (split, kv head, sequence) are strided over the persistent CTAs; the
// producer streams the next item's tiles while the current one finishes.  With several splits per sequence, pa_umma_merge_kernel
// LSE-merges the partials.  Every wait is bounded and reports SDB_KERR_TIMEOUT
// instead of hanging.
#include <cfloat>
#include <climits>

#include "attention_common.cuh"
#include "umma.cuh"

namespace sdb {
namespace attn {
namespace umma {

constexpr int UBN = 128;                  // keys per tile
constexpr int UHALF = UBN * 128;          // one 64-dim half of a K or V tile: 16 KB
constexpr int UTILE = 2 * UHALF;          // one K or V tile: 32 KB
// K and V tiles stream through two rings of UNS slots each.  A K slot is released
// when S(t) has read it and a V slot when P.V(t) has, so each ring holds a tile from
// its load until its own last use: tile t + UNS can be loaded UNS tile-intervals
// before it is needed (a shared K+V stage, released only after P.V, gave K two).
constexpr int UNS = 3;                    // slots per ring
constexpr int NROW = 32;                  // MMA N: query rows per (sequence, kv head)
constexpr int QHALF = NROW * 128;         // 4 KB
// P of tile t is written into its own buffer, as one N = 64 B operand: 128 key rows
// of 128 B, columns 0..31 the 16-bit heads of the 32 rows' probabilities, columns
// 32..63 their residuals, so a single MMA per key step reads V once and accumulates
// O_head and O_residual side by side (64 TMEM columns).  The completion of P.V(t)
// frees the buffer (p_free) before the softmax writes P(t + 1).
constexpr int PROWS = 2 * NROW;
constexpr int PBYTES = UBN * 128;         // 16 KB
constexpr int QBUF = 2 * QHALF;           // one item's Q^T (8 KB)
constexpr int OFF_K = 0;                  // K ring
constexpr int OFF_V = UNS * UTILE;        // V ring
constexpr int OFF_P = 2 * UNS * UTILE;    // P
constexpr int OFF_Q = OFF_P + PBYTES;     // two Q^T buffers: item i uses buffer i & 1
constexpr int OFF_RED = OFF_Q + 2 * QBUF;             // red_max[4][32], red_sum[4][32]
constexpr int kMaxUmmaSplits = 16;
constexpr int OFF_BAR = OFF_RED + 2 * 4 * 32 * 4;
// barriers: k_full[3] k_empty[3] v_full[3] v_empty[3] s_full[2] s_free[2] p_full
// p_free q_ready[2] q_free[2] fin stored
constexpr int NBAR = UNS * 4 + 2 + 2 + 1 + 1 + 2 + 2 + 1 + 1;
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB of shared memory a CTA may use");
// TMEM columns: S^T buffers [0, 64), O^T heads / residuals [64, 96) / [96, 128)
constexpr uint32_t TMEM_COLS = 128;
constexpr uint32_t TCOL_O = 64;
constexpr int SOFTMAX_THREADS = 256;  // 8 warps
constexpr int SOFTMAX_WARPS = SOFTMAX_THREADS / 32;  // one mbarrier arrival per warp
constexpr int GROUP_THREADS = SOFTMAX_THREADS / 2;   // the 4 softmax warps of a column half
constexpr int PV_WARP = 2 + SOFTMAX_WARPS;  // the P.V issuer, after the softmax warps
constexpr int THREADS = 64 + SOFTMAX_THREADS + 32;

struct Bars {
    uint32_t kfull0, kempty0, vfull0, vempty0, sfull0, sfree0, pfull, pfree, qready0, qfree0, fin, stored;
};

SDB_DEV Bars bars_at(uint32_t base) {
    Bars b;
    b.kfull0 = base;
    b.kempty0 = base + 8 * UNS;
    b.vfull0 = base + 16 * UNS;
    b.vempty0 = base + 24 * UNS;
    b.sfull0 = base + 32 * UNS;
    b.sfree0 = b.sfull0 + 16;
    b.pfull = b.sfree0 + 16;
    b.pfree = b.pfull + 8;
    b.qready0 = b.pfree + 8;
    b.qfree0 = b.qready0 + 16;
    b.fin = b.qfree0 + 16;
    b.stored = b.fin + 8;
    return b;
}

// A contiguous key range [k0, k1) of one (sequence b, kv head) pair processed by one
// CTA.  `direct`: the CTA holds every key of the pair and writes the output itself;
// otherwise it writes partial `slot` of the pair for pa_umma_merge_kernel.
struct Item {
    int b, kvh, slot, L, k0, k1, kend, ntiles, span;  // kend: k1 before clamping to L
    bool direct;
};

SDB_DEV Item make_item(const Params& p, int pair, int k0, int k1, int slot, bool direct, int span) {
    Item x;
    x.kvh = pair % p.Hkv;
    x.b = pair / p.Hkv;
    x.L = load_len(p, x.b);
    x.k0 = k0;
    x.kend = k1;
    x.k1 = min(k1, x.L);
    x.ntiles = x.k1 > x.k0 ? (x.k1 - x.k0 + UBN - 1) / UBN : 0;
    x.slot = slot;
    x.direct = direct;
    x.span = span;
    return x;
}

// Balanced partition in CTA groups: the CTAs form flat_grid groups of Hkv, CTA
// g * Hkv + h taking kv head h.  The sequences' tile slots (flat_T per sequence) are
// laid end to end and group g owns [start(g), start(g + 1)) with start(g) =
// floor(g * total / flat_grid): every CTA streams the same number of tiles (+-1),
// the Hkv heads of a sequence are read in lockstep by one group (the heads of a key
// row share its DRAM pages), and a sequence is split only where a group boundary
// falls inside it.
SDB_DEV long long flat_start(const Params& p, int g) { return (long long)g * p.flat_total / p.flat_grid; }
SDB_DEV int flat_group_of(const Params& p, long long f) {
    int g = (int)(f * p.flat_grid / p.flat_total);
    if (g + 1 < p.flat_grid && flat_start(p, g + 1) <= f) ++g;
    return g;
}

// The items of this CTA in order: with the balanced partition, the pieces of its slot
// range; otherwise (static splits) items blockIdx.x, blockIdx.x + gridDim.x, ... of
// the (pair, split) list, split fastest.
struct WorkIter {
    int f, f1;  // the host keeps every flat index and item count below 2^31
    SDB_DEV explicit WorkIter(const Params& p) {
        if (p.flat_T > 0) {
            const int g = blockIdx.x / p.Hkv;
            f = (int)flat_start(p, g);
            f1 = (int)flat_start(p, g + 1);
        } else {
            f = blockIdx.x;
            f1 = p.B * p.Hkv * p.splits;
        }
    }
    SDB_DEV bool valid() const { return f < f1; }
    SDB_DEV Item item(const Params& p) const {
        if (p.flat_T > 0) {
            const int b = f / p.flat_T, t0 = f % p.flat_T;
            const int t1 = min(p.flat_T, t0 + (f1 - f));
            const bool whole = t0 == 0 && t1 == p.flat_T;
            const int g = blockIdx.x / p.Hkv;
            const int slot = whole ? 0 : g - flat_group_of(p, (long long)b * p.flat_T);
            return make_item(p, b * p.Hkv + (int)blockIdx.x % p.Hkv, t0 * UBN, t1 * UBN, slot, whole, t1 - t0);
        }
        const int it = f, split = it % p.splits;
        return make_item(p, it / p.splits, split * p.chunk, split * p.chunk + p.chunk, split, p.splits == 1, 0);
    }
    SDB_DEV void next(const Params& p, const Item& x) { f += p.flat_T > 0 ? x.span : gridDim.x; }
    // next() without the item (the same span)
    SDB_DEV void skip(const Params& p) {
        f += p.flat_T > 0 ? min(p.flat_T - f % p.flat_T, f1 - f) : (int)gridDim.x;
    }
};

// Position (item, tile) in the sequence of tiles this CTA processes (items without
// tiles are skipped); valid() is false once the sequence is exhausted.
struct TileCursor {
    WorkIter w;
    Item x;
    int t;
    SDB_DEV explicit TileCursor(const Params& p) : w(p), t(-1) {
        if (w.valid()) x = w.item(p);
        advance(p);
    }
    SDB_DEV bool valid() const { return w.valid(); }
    SDB_DEV void advance(const Params& p) {
        ++t;
        while (w.valid() && t >= x.ntiles) {
            w.next(p, x);
            t = 0;
            if (w.valid()) x = w.item(p);
        }
    }
};

// Fused store_kvcache (nanovllm/layers/attention.py:10-40 followed by the attention
// of :59-81).  New token i of sequence b (row b * n_q + i of key / value) sits at
// cache position L - n_q + i.  The item whose unclamped key range [k0, kend) holds
// that position -- or key 0 for a token at a negative position -- owns the token's
// kv-head row: the key ranges of a (sequence, kv head) pair partition
// [0, max_blocks * page), so every row has exactly one owner, and only the owner's
// CTA reads the tile holding the position.  At kernel start the softmax warps of
// each CTA copy the rows of all its items to their slots (they would otherwise wait
// for the first S tile), then arrive on the `stored` barrier; the producer waits on
// it once, before the TMA load of the first tile holding a new row.  The fused form
// needs the slot of a token at position p >= 0 to be -1 or the slot the block table
// gives p; any other slot is still written but sets SDB_KERR_SLOT (the attention
// reads the position's own slot, as a separate store followed by attention would).
struct NewRows {
    int i0, i1;  // tokens [i0, i1) of the item's sequence
    int tile;    // the item's first tile holding one of their positions
};

SDB_DEV NewRows new_rows(const Params& p, const Item& x) {
    NewRows r{0, 0, 0};
    if (p.slots == nullptr) return r;
    const int lo = x.L - p.n_q;  // position of token 0
    r.i0 = x.k0 == 0 ? 0 : max(0, x.k0 - lo);
    r.i1 = min(p.n_q, x.kend - lo);
    const int first = max(max(lo, 0), x.k0);
    r.tile = (first - x.k0) / UBN;
    return r;
}

// Warp-wide copy of the item's owned rows (n_q <= 32 tokens): lane u reads token u's
// slot and checks it, then per token lanes 0..15 copy 16 bytes each of the K row and
// lanes 16..31 of the V row (head_dim 128 at 16 bits = 256 bytes), eight tokens' loads
// in flight at a time.
SDB_DEV void copy_new_rows(const Params& p, const Item& x, const NewRows& nr, int lane) {
    const int lo = x.L - p.n_q;
    const int n = nr.i1 - nr.i0;
    const int tok0 = x.b * p.n_q + nr.i0;
    int slot = -1;
    bool bad_blk = false, bad_slot = false;
    if (lane < n) {
        slot = p.slots[tok0 + lane];
        const int pos = lo + nr.i0 + lane;
        const int want = pos >= 0 ? p.bt[(int64_t)x.b * p.bt_stride + pos / p.page] * p.page + pos % p.page : slot;
        if (slot >= 0) {
            if (slot / p.page >= p.num_blocks) {
                bad_blk = true;
                slot = -1;
            } else if (want != slot) {
                bad_slot = true;
            }
        }
    }
    const unsigned bb = __ballot_sync(0xffffffffu, bad_blk), bs = __ballot_sync(0xffffffffu, bad_slot);
    if (lane == 0 && bb) atomicOr(p.err, SDB_KERR_BLOCK_ID);
    if (lane == 0 && bs) atomicOr(p.err, SDB_KERR_SLOT);
    const bool isv = lane >= 16;
    const int c = lane & 15;
    const uint8_t* src0 = (isv ? p.new_v : p.new_k) + (int64_t)x.kvh * (isv ? p.nv_shead : p.nk_shead) + c * 16;
    const int64_t src_stok = isv ? p.nv_stok : p.nk_stok;
    uint8_t* dst0 = (isv ? p.vc : p.kc) + (int64_t)x.kvh * p.c_sh + c * 16;
    for (int u0 = 0; u0 < n; u0 += 8) {
        uint4 v[8];
        uint8_t* dst[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int sl = __shfl_sync(0xffffffffu, slot, (u0 + u) & 31);
            dst[u] = nullptr;
            if (u0 + u < n && sl >= 0) {
                v[u] = __ldg(reinterpret_cast<const uint4*>(src0 + (int64_t)(tok0 + u0 + u) * src_stok));
                dst[u] = dst0 + (int64_t)(sl / p.page) * p.c_sb + (int64_t)(sl % p.page) * p.c_sp;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (dst[u]) *reinterpret_cast<uint4*>(dst[u]) = v[u];
    }
}

// Softmax warp sw (0..7) copies the new rows of items sw, sw + 8, ... of this CTA,
// then makes them visible to the async proxy (the producer's TMA loads).
SDB_DEV void store_new_rows(const Params& p, int sw, int lane) {
    int k = 0;
    for (WorkIter w(p); w.valid(); w.skip(p), ++k) {
        if (k % SOFTMAX_WARPS != sw) continue;
        const Item x = w.item(p);
        const NewRows nr = new_rows(p, x);
        if (nr.i0 < nr.i1) copy_new_rows(p, x, nr, lane);
    }
    fence_proxy_async_global();
    __syncwarp();
}

// Wait that becomes a no-op once this thread has seen a timeout: the softmax warps
// keep executing the same sequence of named barriers after a failure (never
// leaving a loop early), so one warp giving up can never strand the others.
SDB_DEV bool wait_or_skip(uint32_t bar, uint32_t parity, bool& ok) {
    if (!ok) return false;
    if (!mbar_wait(bar, parity)) ok = false;
    return ok;
}

// In-warp transpose reduction of 16 columns: lanes c and c + 16 end with op over
// the 32 lanes of v[c] (16 + 4 + ... shuffles instead of 16 x 5).
template <bool MAX>
SDB_DEV float transpose_reduce16(float (&v)[16], int lane) {
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
            const float send = upper ? v[i] : v[i + off];
            const float keep = upper ? v[i + off] : v[i];
            const float recv = __shfl_xor_sync(0xffffffffu, send, off);
            v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
        }
    }
    const float other = __shfl_xor_sync(0xffffffffu, v[0], 16);
    return MAX ? fmaxf(v[0], other) : v[0] + other;
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1)
    pa_umma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const __grid_constant__ CUtensorMap qmap, const Params p) {
    using H = Half16<T>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const Bars bar = bars_at(sbase + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);
    float* red_max = reinterpret_cast<float*>(smem + OFF_RED);
    float* red_sum = red_max + 4 * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the split merge (a programmatic dependent launch) may become resident now; it
    // waits for this grid's completion before reading anything
    asm volatile("griddepcontrol.launch_dependents;");

    if (threadIdx.x == 0) {
        for (int s = 0; s < UNS; ++s) {
            mbar_init(bar.kfull0 + 8 * s, 1);
            mbar_init(bar.kempty0 + 8 * s, 1);
            mbar_init(bar.vfull0 + 8 * s, 1);
            mbar_init(bar.vempty0 + 8 * s, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar.sfull0 + 8 * i, 1);
            mbar_init(bar.sfree0 + 8 * i, SOFTMAX_WARPS);
        }
        mbar_init(bar.pfull, SOFTMAX_WARPS);
        mbar_init(bar.pfree, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar.qready0 + 8 * i, 1);
            mbar_init(bar.qfree0 + 8 * i, 1);
        }
        mbar_init(bar.fin, 2);  // one commit from each MMA issuer
        mbar_init(bar.stored, SOFTMAX_WARPS);
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    // Q buffers: TMA writes rows 0..R-1 of each; rows R..31 (pad columns of S^T) stay zero
    for (int i = threadIdx.x; i < 2 * QBUF / 16; i += THREADS)
        reinterpret_cast<uint4*>(smem + OFF_Q)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------- producers
        // lane 0 loads Q and the K ring, lane 1 the V ring: each ring refills a slot as
        // soon as its own last reader (S for K, P.V for V) has completed, independently
        // of the other ring's waits
        if (lane < 2) {
            const bool isk = lane == 0;
            if (isk) {
                prefetch_tensormap(&kmap);
                prefetch_tensormap(&qmap);
            } else {
                prefetch_tensormap(&vmap);
            }
            const CUtensorMap* map = isk ? &kmap : &vmap;
            const uint32_t full0 = isk ? bar.kfull0 : bar.vfull0;
            const uint32_t empty0 = isk ? bar.kempty0 : bar.vempty0;
            const uint32_t ring = sbase + (isk ? OFF_K : OFF_V);
            const uint64_t pol = l2_policy_evict_first();
            const uint64_t qpol = l2_policy_evict_normal();  // every split of a sequence reads Q
            int gt = 0, nq = 0;
            bool ok = true;
            bool stored = p.slots == nullptr;  // no fused store: nothing to wait for
            int need_tile = INT_MAX;
            TileCursor ld(p);
            while (ld.valid()) {
                const int j = ld.x.k0 + ld.t * UBN;
                // the block id is read before the waits, off the slot-hold path
                int blk = p.bt[(int64_t)ld.x.b * p.bt_stride + j / p.page];
                if (ld.t == 0) {
                    if (!stored) {
                        const NewRows nr = new_rows(p, ld.x);
                        need_tile = nr.i0 < nr.i1 ? nr.tile : INT_MAX;
                    }
                    if (isk) {
                        // Q^T rows (r, g) -> row r*G + g of Q buffer nq & 1, K-major 128-byte
                        // swizzle; the buffer is free once the S MMAs of the item two before
                        // have completed
                        const int qb = nq & 1;
                        if (nq >= 2 && !mbar_wait(bar.qfree0 + 8 * qb, ((nq >> 1) - 1) & 1)) {
                            ok = false;
                            break;
                        }
                        const uint32_t qdst = sbase + OFF_Q + qb * QBUF;
                        mbar_arrive_expect_tx(bar.qready0 + 8 * qb, 2 * 128 * p.R);
                        tma_load_4d(qdst, &qmap, bar.qready0 + 8 * qb, 0, 0, ld.x.kvh, ld.x.b * p.n_q, qpol);
                        tma_load_4d(qdst + QHALF, &qmap, bar.qready0 + 8 * qb, 64, 0, ld.x.kvh, ld.x.b * p.n_q,
                                    qpol);
                        ++nq;
                    }
                }
                const int s = gt % UNS;
                // slot s is free once the last reader of tile gt - UNS has completed
                if (gt >= UNS && !mbar_wait(empty0 + 8 * s, ((gt / UNS) - 1) & 1)) {
                    ok = false;
                    break;
                }
                // the fused store's rows are in place before a tile holding one is loaded
                if (!stored && ld.t >= need_tile) {
                    if (!mbar_wait(bar.stored, 0)) {
                        ok = false;
                        break;
                    }
                    stored = true;
                }
                if (blk < 0 || blk >= p.num_blocks) {
                    if (isk) atomicOr(p.err, SDB_KERR_BLOCK_ID);
                    blk = 0;
                }
                const int off = j % p.page;
                const uint32_t dst = ring + s * UTILE;
                const uint32_t fb = full0 + 8 * s;
                mbar_arrive_expect_tx(fb, UTILE);
                tma_load_4d(dst, map, fb, 0, ld.x.kvh, off, blk, pol);
                tma_load_4d(dst + UHALF, map, fb, 64, ld.x.kvh, off, blk, pol);
                ++gt;
                ld.advance(p);
            }
            if (!ok) atomicOr(p.err, SDB_KERR_TIMEOUT);
            for (int g = gt - UNS > 0 ? gt - UNS : 0; g < gt; ++g) {  // drain own copies
                if (!mbar_wait(full0 + 8 * (g % UNS), (g / UNS) & 1)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
            }
            for (int n = nq - 2 > 0 ? nq - 2 : 0; n < nq; ++n) {
                if (!mbar_wait(bar.qready0 + 8 * (n & 1), (n >> 1) & 1)) {
                    atomicOr(p.err, SDB_KERR_TIMEOUT);
                    break;
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- S issuer
        // S^T(t) = K(t) . Q^T, one thread; P.V has its own issuer (warp PV_WARP), so an
        // S is never queued behind a P.V that waits for the softmax
        if (lane == 0) {
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            constexpr uint32_t IDESC_S = idesc_f16(BF, false, false, 128, NROW);
            int gt = 0, nitem = 0;
            bool ok = true;
            // nitem counts the items that have tiles: only those take a Q buffer / q_ready phase
            for (WorkIter w(p); w.valid() && ok;) {
                const Item x = w.item(p);
                w.next(p, x);
                if (x.ntiles == 0) continue;
                if (!mbar_wait(bar.qready0 + 8 * (nitem & 1), (nitem >> 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int t = 0; t < x.ntiles; ++t, ++gt) {
                    const int s = gt % UNS, sb = gt & 1;
                    if (!mbar_wait(bar.kfull0 + 8 * s, (gt / UNS) & 1) ||
                        (gt >= 2 && !mbar_wait(bar.sfree0 + 8 * sb, ((gt >> 1) - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t kbase = sbase + OFF_K + s * UTILE;
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t a = sdesc_sw128(kbase + (ks >> 2) * UHALF + (ks & 3) * 32, 16, 1024);
                        const uint64_t b =
                            sdesc_sw128(sbase + OFF_Q + (nitem & 1) * QBUF + (ks >> 2) * QHALF + (ks & 3) * 32, 16, 1024);
                        umma_f16_ss(tmem + sb * 32, a, b, IDESC_S, ks > 0 ? 1u : 0u);
                    }
                    umma_commit(bar.sfull0 + 8 * sb);
                    umma_commit(bar.kempty0 + 8 * s);  // K slot read
                    if (t == x.ntiles - 1) umma_commit(bar.qfree0 + 8 * (nitem & 1));  // Q buffer read
                }
                ++nitem;
            }
            if (!ok) atomicOr(p.err, SDB_KERR_TIMEOUT);
            // every MMA this thread issued has completed before TMEM is released (fin
            // completes once both issuers have committed)
            umma_commit(bar.fin);
            if (!mbar_wait(bar.fin, 0)) atomicOr(p.err, SDB_KERR_TIMEOUT);
        }
    } else if (warp == PV_WARP) {
        // ------------------------------------------------------------- P.V issuer
        // O^T += V(g)^T . P(g), heads and residuals as N = 64; completion frees V slot
        // g % UNS and the P buffer
        if (lane == 0) {
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            constexpr uint32_t IDESC_PV = idesc_f16(BF, true, true, 128, PROWS);
            int gt = 0;
            bool ok = true;
            for (WorkIter w(p); w.valid() && ok;) {
                const Item x = w.item(p);
                w.next(p, x);
                for (int t = 0; t < x.ntiles; ++t, ++gt) {
                    if (!mbar_wait(bar.pfull, gt & 1) || !mbar_wait(bar.vfull0 + 8 * (gt % UNS), (gt / UNS) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t vbase = sbase + OFF_V + (gt % UNS) * UTILE;
                    const uint32_t pbase = sbase + OFF_P;
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t a = sdesc_sw128(vbase + ks * 2048, UHALF, 1024);
                        const uint64_t b = sdesc_sw128(pbase + ks * 2048, UHALF, 1024);
                        umma_f16_ss(tmem + TCOL_O, a, b, IDESC_PV, (t == 0 && ks == 0) ? 0u : 1u);
                    }
                    umma_commit(bar.vempty0 + 8 * (gt % UNS));
                    umma_commit(bar.pfree);
                }
            }
            if (!ok) atomicOr(p.err, SDB_KERR_TIMEOUT);
            umma_commit(bar.fin);
            if (!mbar_wait(bar.fin, 0)) atomicOr(p.err, SDB_KERR_TIMEOUT);
        }
    } else {
        // ------------------------------------------------------------- softmax warps
        // 8 warps: warp w (2..9) reads TMEM lane quarter qt = w % 4 (its 32 keys of S^T,
        // its 32 dims of O^T) and column half ch = (w - 2) / 4 (16 of the 32 rows).
        //
        // Common path per tile: no reduction at all.  Every thread keeps the reference
        // point mbv[i] of each of its 16 rows; if no logit of the tile exceeds its row's
        // reference by more than 8 (log2 units, p <= 256), one vote barrier confirms it,
        // P = 2^(x - ref) is written and the row sums accumulate per thread.  Otherwise
        // (first tile of an item, or a row max that grew) the 4 warps of the column half
        // take the exact path:
        // column max over the 128 keys, new reference = max, partial sums and O rescaled.
        const int sw = warp - 2;            // 0..7
        if (p.slots != nullptr) {  // fused store_kvcache, before the first S tile arrives
            store_new_rows(p, sw, lane);
            if (lane == 0) mbar_arrive(bar.stored);
        }
        const int qt = warp & 3;
        const int ch = sw >> 2;
        const int c0 = 16 * ch;             // first column (row) of this thread
        // the 4 warps of a column half exchange maxima and sums only among themselves:
        // each half synchronises on its own named barrier (ids 1 and 2)
        const int gbar = 1 + ch;
        const int lc = lane & 15;           // column whose reference this lane owns: c0 + lc
        const uint32_t lane_addr = (uint32_t)(32 * qt) << 16;
        const int R = p.R;
        const float sl2 = p.scale_log2;
        int gt = 0;
        bool ok = true;
        T* obase = reinterpret_cast<T*>(p.out);
        // Result of an item of pair `pair` for columns cb .. cb+7 (cb = c0 or c0 + 8): the
        // output rows (slot < 0: the CTA saw every key of the pair) or partial `slot` of
        // the pair: O^T column c, the row max reference and the row sum.
        auto store8 = [&](int pair, int slot, int cb, const float (&o)[8], float lsum, float mb_own) {
            const int dim = 32 * qt + lane;
            if (slot < 0) {
                const int b = pair / p.Hkv, kvh = pair - b * p.Hkv;
                int r = cb / p.G, g = cb % p.G;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float l_i = __shfl_sync(0xffffffffu, lsum, cb - c0 + i);
                    if (cb + i < R) {
                        T* dst = obase + (int64_t)(b * p.n_q + r) * p.o_srow +
                                 (int64_t)(kvh * p.G + g) * p.o_shead + dim;
                        *dst = from_f32<T>(l_i > 0.f ? o[i] / l_i : 0.f);
                    }
                    if (++g == p.G) {
                        g = 0;
                        ++r;
                    }
                }
                return;
            }
            const int64_t sl = (int64_t)pair * p.splits + slot;
            float* po = p.part_o + sl * R * D;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (cb + i < R) __stcg(po + (cb + i) * D + dim, o[i]);
            if (cb == c0 && qt == 0 && lane < 16 && c0 + lane < R)
                __stcg(reinterpret_cast<float2*>(p.part_ml + (sl * R + c0 + lane) * 2), make_float2(mb_own, lsum));
        };
        for (WorkIter w(p); w.valid();) {
            const Item x = w.item(p);
            w.next(p, x);
            const int pair = x.b * p.Hkv + x.kvh;
            const int slot = x.direct ? -1 : x.slot;
            if (x.ntiles == 0) {
                // no keys: zero output or an empty partial (m = -inf, l = 0)
                float o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = 0.f;
                store8(pair, slot, c0, o, 0.f, NEG_INF);
                store8(pair, slot, c0 + 8, o, 0.f, NEG_INF);
                continue;
            }
            const uint32_t ocol = TCOL_O;

            float mb_own = NEG_INF;   // reference of column c0 + lc
            float mbv[16], lpart[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                mbv[i] = NEG_INF;
                lpart[i] = 0.f;
            }
            const int lbase = x.L - p.n_q + 1;  // keys visible to row r: j < lbase + r
            for (int t = 0; t < x.ntiles; ++t, ++gt) {
                const int sb = gt & 1, s = gt % UNS;
                const int j0 = x.k0 + t * UBN;
                wait_or_skip(bar.sfull0 + 8 * sb, (gt >> 1) & 1, ok);
                tc_fence_after();
                uint32_t sr[16];
                tmem_ld16(tmem + lane_addr + sb * 32 + c0, sr);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar.sfree0 + 8 * sb);

                const int key = j0 + 32 * qt + lane;
                float xv[16];
                if (j0 + UBN > min(lbase, x.k1)) {
                    // tail tile: causal limits, split end, pad rows
                    int r = c0 / p.G, g = c0 % p.G;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const bool vis = c0 + i < R && key < min(lbase + r, x.k1);
                        xv[i] = vis ? __uint_as_float(sr[i]) * sl2 : NEG_INF;
                        if (++g == p.G) {
                            g = 0;
                            ++r;
                        }
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) xv[i] = __uint_as_float(sr[i]) * sl2;
                }
                bool need = false;
#pragma unroll
                for (int i = 0; i < 16; ++i) need |= xv[i] > mbv[i] + 8.0f;
                if (barrier_or(gbar, GROUP_THREADS, need)) {
                    // exact path (uniform over the 4 warps of this column half)
                    float tmp[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) tmp[i] = xv[i];
                    const float wm = transpose_reduce16<true>(tmp, lane);
                    if (lane < 16) red_max[qt * 32 + c0 + lane] = wm;
                    named_barrier_sync(gbar, GROUP_THREADS);
                    const int cc = c0 + lc;
                    const float M =
                        fmaxf(fmaxf(red_max[cc], red_max[32 + cc]), fmaxf(red_max[64 + cc], red_max[96 + cc]));
                    const float nb = fmaxf(M, mb_own);
                    const float alpha = nb == mb_own ? 1.0f : ex2(mb_own - nb);
                    mb_own = nb;
                    float av[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        mbv[i] = __shfl_sync(0xffffffffu, mb_own, i);
                        av[i] = __shfl_sync(0xffffffffu, alpha, i);
                        lpart[i] *= av[i];
                    }
                    if (t >= 1) {
                        // P.V(t-1) complete (p_free): O is up to date, rescale it
                        wait_or_skip(bar.pfree, (gt - 1) & 1, ok);
                        tc_fence_after();
                        uint32_t oh[16], ol[16];
                        tmem_ld16(tmem + lane_addr + ocol + c0, oh);
                        tmem_ld16(tmem + lane_addr + ocol + 32 + c0, ol);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            oh[i] = __float_as_uint(__uint_as_float(oh[i]) * av[i]);
                            ol[i] = __float_as_uint(__uint_as_float(ol[i]) * av[i]);
                        }
                        tmem_st16(tmem + lane_addr + ocol + c0, oh);
                        tmem_st16(tmem + lane_addr + ocol + 32 + c0, ol);
                        tmem_wait_st();
                    }
                }
                float pv[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    pv[i] = ex2(xv[i] - (mbv[i] == NEG_INF ? 0.f : mbv[i]));
                    lpart[i] += pv[i];
                }
                // keys past the split end: zero their V rows (unwritten cache may hold NaN)
                const int kin = 32 * qt + lane;
                if (j0 + UBN > x.k1) {
                    wait_or_skip(bar.vfull0 + 8 * s, (gt / UNS) & 1, ok);
                    if (j0 + kin >= x.k1) {
                        uint8_t* vrow = smem + OFF_V + s * UTILE + kin * 128 + ch * UHALF;
#pragma unroll
                        for (int q16 = 0; q16 < 8; ++q16)
                            *reinterpret_cast<uint4*>(vrow + q16 * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                // P into the P buffer once P.V(t-1) has read it: row `key` holds 64
                // columns, heads of rows 0..31 then their residuals, 128-byte swizzle
                // (16-byte chunk j of row k at j ^ (k & 7)): the MN-major B operand of P.V
                {
                    uint32_t hw[8], lw[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) H::split2(pv[2 * i], pv[2 * i + 1], hw[i], lw[i]);
                    if (gt >= 1) {
                        wait_or_skip(bar.pfree, (gt - 1) & 1, ok);
                        tc_fence_after();
                    }
                    uint8_t* prow = smem + OFF_P + kin * 128;
                    const int sw = kin & 7;
                    *reinterpret_cast<uint4*>(prow + (((2 * ch) ^ sw) << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(prow + (((2 * ch + 1) ^ sw) << 4)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                    *reinterpret_cast<uint4*>(prow + (((4 + 2 * ch) ^ sw) << 4)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                    *reinterpret_cast<uint4*>(prow + (((5 + 2 * ch) ^ sw) << 4)) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                }
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar.pfull);
            }


            // ---- item epilogue: row sums, then O^T column c is row c (this thread: dim 32*qt + lane)
            float lsum;
            {
                const float ws = transpose_reduce16<false>(lpart, lane);
                // every warp has read the previous item's red_sum
                named_barrier_sync(gbar, GROUP_THREADS);
                if (lane < 16) red_sum[qt * 32 + c0 + lane] = ws;
                named_barrier_sync(gbar, GROUP_THREADS);
                const int cc = c0 + lc;
                lsum = (red_sum[cc] + red_sum[32 + cc]) + (red_sum[64 + cc] + red_sum[96 + cc]);
            }
            // the last P.V has completed (p_free): O^T is final
            wait_or_skip(bar.pfree, (gt - 1) & 1, ok);
            tc_fence_after();
            {
                uint32_t oh[16], ol[16];
                tmem_ld16(tmem + lane_addr + ocol + c0, oh);
                tmem_ld16(tmem + lane_addr + ocol + 32 + c0, ol);
                tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float o[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(oh[8 * h + i]) + __uint_as_float(ol[8 * h + i]);
                    store8(pair, slot, c0 + 8 * h, o, lsum, mb_own);
                }
            }
        }
        if (!ok && lane == 0) atomicOr(p.err, SDB_KERR_TIMEOUT);
    }

    // each warp reconverges first (the producer, MMA and idle lanes of warps 0, 1 and the
    // P.V warp come from different branches), so the block barrier below holds every thread
    // until the softmax warps' last TMEM reads are done
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// LSE merge of the split partials.  One thread per (pair, row, 4 dims): out =
// sum_s w_s o_s with w_s = 2^(m_s - M) / sum_s 2^(m_s - M) l_s over the pair's
// partials (independent L2 reads).  Under the balanced partition only sequences cut
// by a group boundary have partials; the grid covers just those.  Launched as a programmatic dependent of pa_umma_kernel:
// its CTAs become resident while the attention tail runs and wait
// (griddepcontrol.wait) for its results.
constexpr int MERGE_THREADS = 128;  // small enough to sit beside a pa_umma_kernel CTA
template <typename T>
__global__ void __launch_bounds__(MERGE_THREADS) pa_umma_merge_kernel(const Params p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int R = p.R;
    const int rb = (R * 32 + MERGE_THREADS - 1) / MERGE_THREADS;  // CTAs per pair
    const int u = (blockIdx.y % rb) * MERGE_THREADS + threadIdx.x;  // row * 32 + dim quad
    const int c = u >> 5, dq = u & 31;
    if (c >= R) return;
    int pair, nseg;
    if (p.flat_T > 0) {
        // grid.x: group boundaries 1 .. groups-1; the first boundary inside a sequence
        // merges it (grid.y: kv head x row block)
        const int k = blockIdx.x + 1;
        const long long f = flat_start(p, k);
        const long long b = f / p.flat_T;
        if (f % p.flat_T == 0) return;
        if (k > 1) {
            const long long fp = flat_start(p, k - 1);
            if (fp / p.flat_T == b && fp % p.flat_T != 0) return;
        }
        pair = (int)b * p.Hkv + (int)blockIdx.y / rb;
        nseg = flat_group_of(p, (b + 1) * p.flat_T - 1) - flat_group_of(p, b * p.flat_T) + 1;
    } else {
        pair = blockIdx.x;  // grid.y: row blocks
        nseg = p.splits;
    }
    const float* ml = p.part_ml + (int64_t)pair * p.splits * R * 2 + c * 2;
    const float4* po = reinterpret_cast<const float4*>(p.part_o + (int64_t)pair * p.splits * R * D + c * D) + dq;
    const int64_t sstride = (int64_t)R * D / 4;  // float4s between partials
    float Mx = NEG_INF;
#pragma unroll 4
    for (int s2 = 0; s2 < nseg; ++s2) Mx = fmaxf(Mx, __ldcg(ml + s2 * R * 2));
    const float Bm = Mx == NEG_INF ? 0.f : Mx;
    float Ls = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int s2 = 0; s2 < nseg; ++s2) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(ml + s2 * R * 2));
        const float4 o = __ldcg(po + s2 * sstride);
        const float w = ex2(v.x - Bm);
        Ls += w * v.y;
        acc.x += w * o.x;
        acc.y += w * o.y;
        acc.z += w * o.z;
        acc.w += w * o.w;
    }
    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
    const int b = pair / p.Hkv, kvh = pair % p.Hkv;
    const int r = c / p.G, g = c % p.G;
    T* dst = reinterpret_cast<T*>(p.out) + (int64_t)(b * p.n_q + r) * p.o_srow +
             (int64_t)(kvh * p.G + g) * p.o_shead + dq * 4;
    dst[0] = from_f32<T>(acc.x * inv);
    dst[1] = from_f32<T>(acc.y * inv);
    dst[2] = from_f32<T>(acc.z * inv);
    dst[3] = from_f32<T>(acc.w * inv);
}

}  // namespace umma

// ------------------------------------------------------------------------- host
bool umma_path(int dtype, int D_, int page, int R) {
    return (dtype == SDB_BF16 || dtype == SDB_F16) && D_ == D && page % umma::UBN == 0 && R <= umma::NROW;
}

// Balanced partition geometry from the static shape: tile slots per sequence, all
// slots, CTA groups, and the most groups one sequence can straddle (the partial slots
// a pair needs).  groups == 0: the kv heads do not fit the SMs as groups.
struct FlatShape {
    int T, groups, slots;
    long long total;
};
static FlatShape flat_shape(int B, int Hkv, int page, int max_blocks, int sms) {
    FlatShape f;
    const long long max_ctx = (long long)max_blocks * page;
    f.T = (int)((max_ctx + umma::UBN - 1) / umma::UBN);
    if (f.T < 1) f.T = 1;
    f.total = (long long)B * f.T;
    const long long g = sms / Hkv;
    f.groups = (int)(f.total < g ? f.total : g);
    if (f.groups < 1) {
        f.groups = 0;
        f.slots = 1;
        return f;
    }
    const long long m = f.total / f.groups;  // shortest group range, >= 1
    long long slots = (f.T + m - 1) / m + 1;
    if (slots > f.groups) slots = f.groups;
    f.slots = (int)slots;
    return f;
}

// Decomposition choice from the static shape, in tile-time units: the strided split
// count s costs its busiest CTA's tiles plus kItemCost per item it runs and, with
// s > 1, the merge (growing with the partials per pair); the grouped partition costs its (even) tiles per CTA times
// kGroupedTax (measured: its CTAs stream somewhat slower than the strided ones),
// its items and the merge.  Fitted to B200 runs of Qwen3-shaped verify / decode
// batches (B 16..128, context 2K..8K).
struct UmmaPlan {
    bool grouped;
    int splits;  // partial slots per pair (grouped) or the strided split count
};
static UmmaPlan umma_plan(int B, int Hkv, int page, int max_blocks, int sms) {
    constexpr double kItemCost = 1.5, kMergeBase = 1.5, kMergePerSlot = 0.25, kGroupedTax = 1.08;
    const FlatShape fs = flat_shape(B, Hkv, page, max_blocks, sms);
    const long long pairs = (long long)B * Hkv;
    UmmaPlan best{false, 1};
    double best_cost = 1e300;
    for (int s = 1; s <= umma::kMaxUmmaSplits; ++s) {
        const long long chunk = (fs.T + s - 1) / s;
        if (s > 1 && chunk < 2) break;
        const long long s_eff = (fs.T + chunk - 1) / chunk;
        if (s > 1 && s_eff < s) continue;  // same as a smaller s
        const long long items = pairs * s_eff;
        const long long grid = items < sms ? items : sms;
        const long long per_cta = (items + grid - 1) / grid;
        const double cost = per_cta * (chunk + kItemCost) + (s_eff > 1 ? kMergeBase + kMergePerSlot * s_eff : 0.0);
        if (cost < best_cost) {
            best_cost = cost;
            best = UmmaPlan{false, (int)s_eff};
        }
    }
    if (fs.groups > 0) {
        const double tiles = (double)((fs.total + fs.groups - 1) / fs.groups);
        const double items = tiles / fs.T + 1.0;
        const double cost =
            tiles * kGroupedTax + items * kItemCost + (fs.groups > 1 ? kMergeBase + kMergePerSlot * fs.slots : 0.0);
        if (cost < best_cost) best = UmmaPlan{true, fs.slots};
    }
    return best;
}

// Default `splits` of the tcgen05 path: the partial slots per pair its plan needs.
int pick_umma_splits(int B, int, int Hkv, int page, int max_blocks, int sms) {
    return umma_plan(B, Hkv, page, max_blocks, sms).splits;
}

// The launch decomposition for a `splits` capacity (0: the plan's default).  The grouped
// partition runs when the plan prefers it and the capacity covers it, and then uses
// exactly the slots a pair can straddle; otherwise every pair is split into `splits`
// key chunks (at most kMaxUmmaSplits, dropping chunks that can hold no key).
UmmaShape umma_launch_shape(int B, int Hkv, int page, int max_blocks, int splits) {
    const int sms = device_sm_count();
    const FlatShape fs = flat_shape(B, Hkv, page, max_blocks, sms);
    const UmmaPlan plan = umma_plan(B, Hkv, page, max_blocks, sms);
    if (splits <= 0) splits = plan.splits;
    UmmaShape u{};
    if (plan.grouped && splits >= fs.slots && fs.total < (1LL << 31)) {
        u.grouped = true;
        u.slots = fs.slots;
        u.flat_T = fs.T;
        u.flat_total = fs.total;
        u.groups = fs.groups;
        return u;
    }
    if (splits > umma::kMaxUmmaSplits) splits = umma::kMaxUmmaSplits;
    const long long max_ctx = (long long)max_blocks * page;
    long long chunk = ((max_ctx + splits - 1) / splits + umma::UBN - 1) / umma::UBN * umma::UBN;
    if (chunk < umma::UBN) chunk = umma::UBN;
    splits = (int)((max_ctx + chunk - 1) / chunk);
    u.grouped = false;
    u.slots = splits < 1 ? 1 : splits;
    u.chunk = (int)chunk;
    return u;
}

int launch_umma(const void* k_cache, const void* v_cache, int dtype, int64_t sb, int64_t sp, int64_t sh,
                Params& p, void* workspace, size_t workspace_bytes, int splits, cudaStream_t st) {
    const int sms = device_sm_count();
    const UmmaShape u = umma_launch_shape(p.B, p.Hkv, p.page, p.max_blocks, splits);
    splits = u.slots;
    int grid;
    bool merge;
    if (u.grouped) {
        p.flat_T = u.flat_T;
        p.flat_total = u.flat_total;
        p.flat_grid = u.groups;
        p.chunk = 0;
        grid = u.groups * p.Hkv;
        merge = u.groups > 1;
    } else {
        p.flat_T = 0;
        p.chunk = u.chunk;
        const long long items = (long long)p.B * p.Hkv * splits;
        grid = (int)(items < sms ? items : sms);
        merge = splits > 1;
    }
    WsLayout w = ws_layout(p.B, p.R, p.Hkv, splits);
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
    const CUtensorMapDataType dt = dtype == SDB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)p.Hkv, (cuuint64_t)p.page, (cuuint64_t)p.num_blocks};
    cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)sp * 2, (cuuint64_t)sb * 2};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)umma::UBN, 1};
    CUtensorMap km, vm;
    int rc = encode_tensor_map(&km, dt, 4, const_cast<void*>(k_cache), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tensor_map(&vm, dt, 4, const_cast<void*>(v_cache), dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    // Q viewed as (dim, head in group, kv head, query row): one box is the R = n_q * G rows
    // of one (sequence, kv head) in row order r * G + g, 64 dims each
    const int G = p.G;
    cuuint64_t qdims[4] = {(cuuint64_t)D, (cuuint64_t)G, (cuuint64_t)p.Hkv, (cuuint64_t)p.B * p.n_q};
    cuuint64_t qstrides[3] = {(cuuint64_t)p.q_shead * 2, (cuuint64_t)p.q_shead * G * 2, (cuuint64_t)p.q_srow * 2};
    cuuint32_t qbox[4] = {64, (cuuint32_t)G, 1, (cuuint32_t)p.n_q};
    CUtensorMap qm;
    rc = encode_tensor_map(&qm, dt, 4, const_cast<void*>(p.q), qdims, qstrides, qbox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (dtype == SDB_BF16) {
        auto kern = umma::pa_umma_kernel<__nv_bfloat16>;
        rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), umma::SMEM_BYTES, 40);
        if (rc) return rc;
        kern<<<grid, umma::THREADS, umma::SMEM_BYTES, st>>>(km, vm, qm, p);
    } else {
        auto kern = umma::pa_umma_kernel<__half>;
        rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), umma::SMEM_BYTES, 41);
        if (rc) return rc;
        kern<<<grid, umma::THREADS, umma::SMEM_BYTES, st>>>(km, vm, qm, p);
    }
    rc = cuda_status(cudaGetLastError(), "pa_umma_kernel launch");
    if (rc || !merge) return rc;
    cudaLaunchConfig_t cfg = {};
    const int rb = (p.R * 32 + umma::MERGE_THREADS - 1) / umma::MERGE_THREADS;
    cfg.gridDim = p.flat_T > 0 ? dim3(p.flat_grid - 1, p.Hkv * rb, 1) : dim3(p.B * p.Hkv, rb, 1);
    cfg.blockDim = dim3(umma::MERGE_THREADS, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = dtype == SDB_BF16 ? cudaLaunchKernelEx(&cfg, umma::pa_umma_merge_kernel<__nv_bfloat16>, p)
                                      : cudaLaunchKernelEx(&cfg, umma::pa_umma_merge_kernel<__half>, p);
    return cuda_status(e, "pa_umma_merge_kernel launch");
}

}  // namespace attn
}  // namespace sdb
