// sdb_paged_attention_noalloc: the paged decode / verify attention for callers
// that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc (or any allocator) when
// they run attention: a plugin executing inside another runtime's enqueue
// callback, where that runtime owns every device byte through its own pool and
// forbids raw allocations; a serving loop in steady state, where cudaMalloc's
// implicit device-wide synchronisation would stall every stream; a deployment
// whose device-memory budget is fixed up front.  They still pass their inputs
// and outputs, but they cannot provide the workspace that sdb_paged_attention
// wants for its split partials and merge counters.  This entry point supplies
// that workspace from a file-scope device array instead.
//
// The array is kNoAllocScratchBytes (16 MiB) and exists on every GPU that loads
// the library, until the process exits.  Shapes whose workspace would exceed it
// are rejected with SDB_ERR_WORKSPACE before anything is launched.
//
// Set-up: every call (with the target device current) looks up the array's device
// address with cudaGetSymbolAddress -- in host code the array's name is only a
// host-side stand-in, never a device address.  The first call on a device, and the
// first after the address changed (a cudaDeviceReset reloads the module), clears the
// error word and the merge counters with cudaMemsetAsync on the caller's stream; that
// call must not be made during stream capture (it is refused with
// SDB_ERR_INVALID_ARG), since the memset would only be recorded into the graph.
// Every later call reuses the same array, which keeps the last call's contents: the
// kernels return the counters to zero after each call and fully overwrite the
// partials before reading them.  The error word keeps every bit the kernels record
// until sdb_paged_attention_noalloc_error_word clears it.  Calls that overlap on the
// GPU (different streams, or different host threads) share the array and race;
// serialise them.
#include <mutex>

#include "common.cuh"

namespace sdb {
namespace {

constexpr size_t kNoAllocScratchBytes = SDB_NOALLOC_SCRATCH_BYTES;
// error word (256 B) + the fixed-capacity counter region of the attention workspace
constexpr size_t kNoAllocZeroBytes = 256 + sizeof(int) * 65536;

static __device__ __align__(256) unsigned char g_attention_scratch[kNoAllocScratchBytes];

struct ScratchSlot {
    void* ptr = nullptr;
    bool cleared = false;
};

std::mutex g_scratch_mu;
ScratchSlot g_scratch[64];

// Device address of this device's scratch array; on first use (or when the address
// moved), clear what must start at zero.
int scratch_for_current_device(cudaStream_t stream, void** out) {
    int dev = 0;
    int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) {
        set_last_error("device index %d out of range for the no-alloc scratch table", dev);
        return SDB_ERR_UNSUPPORTED;
    }
    void* p = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&p, g_attention_scratch), "cudaGetSymbolAddress");
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchSlot& s = g_scratch[dev];
    if (s.ptr != p) {
        s.ptr = p;
        s.cleared = false;
    }
    if (!s.cleared) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        rc = cuda_status(cudaStreamIsCapturing(stream, &cap), "cudaStreamIsCapturing");
        if (rc) return rc;
        if (cap != cudaStreamCaptureStatusNone) {
            set_last_error("the first no-alloc call on device %d sets up its static array and must not be made "
                           "during stream capture; make one call before capturing", dev);
            return SDB_ERR_INVALID_ARG;
        }
        rc = cuda_status(cudaMemsetAsync(s.ptr, 0, kNoAllocZeroBytes, stream), "cudaMemsetAsync (scratch set-up)");
        if (rc) return rc;
        s.cleared = true;
    }
    *out = s.ptr;
    return SDB_OK;
}

}  // namespace
}  // namespace sdb

extern "C" int sdb_paged_attention_noalloc(const void* q, int64_t q_srow, int64_t q_shead, const void* k_cache,
                                           const void* v_cache, int64_t sb, int64_t sp, int64_t sh,
                                           const int32_t* block_tables, int64_t bt_stride,
                                           const int32_t* cache_seqlens, void* out, int64_t o_srow,
                                           int64_t o_shead, int B, int n_q, int Hq, int Hkv, int D, int page,
                                           int max_blocks, int num_blocks, float softmax_scale, int dtype,
                                           int splits, void* stream) {
    using namespace sdb;
    if (B <= 0 || n_q <= 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0 || page <= 0 || max_blocks <= 0) {
        set_last_error("bad sizes B=%d n_q=%d Hq=%d Hkv=%d page=%d max_blocks=%d", B, n_q, Hq, Hkv, page, max_blocks);
        return SDB_ERR_INVALID_ARG;
    }
    // sized for the decomposition the launch will use (an explicit `splits` is clamped there)
    int kernel = -1, slots = 0;
    const size_t need =
        sdb_paged_attention_plan(B, n_q, Hq, Hkv, D, page, max_blocks, dtype, splits, &kernel, &slots);
    if (need > kNoAllocScratchBytes) {
        set_last_error("sdb_paged_attention_noalloc: this shape needs %zu bytes of scratch, more than the %zu-byte "
                       "static array (use sdb_paged_attention with a caller-provided workspace)",
                       need, kNoAllocScratchBytes);
        return SDB_ERR_WORKSPACE;
    }
    void* scratch = nullptr;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int rc = scratch_for_current_device(st, &scratch);
    if (rc) return rc;
    return sdb_paged_attention(q, q_srow, q_shead, k_cache, v_cache, sb, sp, sh, block_tables, bt_stride,
                               cache_seqlens, out, o_srow, o_shead, B, n_q, Hq, Hkv, D, page, max_blocks,
                               num_blocks, softmax_scale, dtype, splits, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int sdb_paged_attention_noalloc_error_word(int32_t* host_word, int clear, void* stream) {
    using namespace sdb;
    if (!host_word) {
        set_last_error("null host_word");
        return SDB_ERR_INVALID_ARG;
    }
    void* scratch = nullptr;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int rc = scratch_for_current_device(st, &scratch);
    if (rc) return rc;
    // the error word is the first word of the attention workspace layout
    rc = cuda_status(cudaMemcpyAsync(host_word, scratch, sizeof(int32_t), cudaMemcpyDeviceToHost, st),
                     "cudaMemcpyAsync (error word)");
    if (rc || !clear) return rc;
    return cuda_status(cudaMemsetAsync(scratch, 0, sizeof(int32_t), st), "cudaMemsetAsync (error word)");
}
