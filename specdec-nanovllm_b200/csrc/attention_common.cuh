// Definitions shared by the paged-attention kernels (mma.sync and tcgen05 paths).
#pragma once

#include "common.cuh"

namespace sdb {
namespace attn {

constexpr int D = 128;
constexpr int BN = 64;                 // keys per stage
constexpr int HALF_BYTES = BN * 128;   // one 64-dim half of a K or V tile (8 KB, swizzled)
constexpr int TILE_BYTES = 2 * HALF_BYTES;
constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // K + V
constexpr float NEG_INF = -INFINITY;

struct Params {
    const void* q;
    int64_t q_srow, q_shead;
    void* out;
    int64_t o_srow, o_shead;
    const int* bt;
    int64_t bt_stride;
    const int* seqlens;
    float* part_o;   // [B*Hkv*splits][R][D]
    float* part_ml;  // [B*Hkv*splits][R][2]
    int* counters;   // [B*Hkv]
    int* err;
    unsigned* checksum;  // read-only twin only
    int B, n_q, G, R, Hkv, page, max_blocks, num_blocks, splits, chunk;
    float scale_log2;
    // tcgen05 path, balanced partition: tile slots per sequence (0 = strided static
    // splits instead), all sequences' slots, and the CTA groups (Hkv CTAs each) sharing them
    int flat_T, flat_grid;
    long long flat_total;
    // tcgen05 path, fused store_kvcache: the step's new K / V rows (token b * n_q + i,
    // at cache position seqlen(b) - n_q + i) and their slots; slots == nullptr when the
    // launch stores nothing.  Strides in bytes.
    const int* slots;
    const uint8_t* new_k;
    const uint8_t* new_v;
    uint8_t* kc;
    uint8_t* vc;
    int64_t nk_stok, nk_shead, nv_stok, nv_shead;
    int64_t c_sb, c_sp, c_sh;
};

struct WsLayout {
    size_t err, counters, part_ml, part_o, total;
};

// The split-merge counters live at a fixed offset with a fixed capacity, so one
// workspace can serve calls of any shape in any order: a counter slot is never
// aliased by another call's partials, and every kernel leaves its counters at 0.
constexpr int kCounterCap = 65536;  // (sequence, kv head) pairs

inline WsLayout ws_layout(int B, int R, int Hkv, int splits) {
    WsLayout w;
    size_t off = 0;
    w.err = off;
    off += 256;
    w.counters = off;
    off = align_up(off + sizeof(int) * (size_t)kCounterCap, 256);
    const size_t slots = (size_t)B * Hkv * (splits > 1 ? splits : 0);
    w.part_ml = off;
    off = align_up(off + sizeof(float) * slots * R * 2, 256);
    w.part_o = off;
    off = align_up(off + sizeof(float) * slots * R * D, 256);
    w.total = off;
    return w;
}

// Sequence length clamped to the table capacity, error bit on violation.
SDB_DEV int load_len(const Params& p, int b) {
    int L = p.seqlens[b];
    const int cap = p.max_blocks * p.page;
    if (L < 0 || L > cap) {
        if (threadIdx.x == 0) atomicOr(p.err, SDB_KERR_SEQLEN);
        L = L < 0 ? 0 : cap;
    }
    return L;
}

// tcgen05 path (csrc/attention_umma.cu)
bool umma_path(int dtype, int D_, int page, int R);
int pick_umma_splits(int B, int R, int Hkv, int page, int max_blocks, int sms);
// The decomposition a tcgen05 launch takes: the grouped partition (flat_T / flat_total /
// groups set) or strided key chunks of `chunk` keys; `slots` partials per pair either way.
struct UmmaShape {
    bool grouped;
    int slots, chunk, flat_T, groups;
    long long flat_total;
};
UmmaShape umma_launch_shape(int B, int Hkv, int page, int max_blocks, int splits);
int launch_umma(const void* k_cache, const void* v_cache, int dtype, int64_t sb, int64_t sp, int64_t sh,
                Params& p, void* workspace, size_t workspace_bytes, int splits, cudaStream_t st);

// Kernel choice: the tcgen05 kernel for the shapes it takes unless the environment
// variable SDB_ATTN_KERNEL is "mma" (forces the mma.sync kernel, for comparison).
bool prefer_umma();

}  // namespace attn
}  // namespace sdb
