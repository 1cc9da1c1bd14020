// Shared device helpers for the sm_100a kernels of this library.
//
// Everything that waits (mbarrier phases) waits with a cycle limit and reports
// failure to the caller instead of spinning forever; callers turn a failed wait
// into SDB_KERR_TIMEOUT in the workspace error word and leave their loop.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "specdec_b200.h"

#define SDB_DEV __device__ __forceinline__

namespace sdb {

// ~2 s at the B200 boost clock: far beyond any legitimate wait in these kernels.
constexpr long long kSpinLimitCycles = 4000000000LL;

// ---------------------------------------------------------------- host side
void set_last_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* where);
int device_sm_count();
int device_index();
// Dynamic shared memory opt-in, done once per (device, kernel).
int ensure_smem_attr(const void* func, int bytes, int slot);
// One-thread launch that adds 1 to a device-resident uint64 Philox offset.
int launch_advance_offset(uint64_t* off, cudaStream_t st);

// Tensor-map encoder obtained from the driver through the runtime.
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank,
                      void* base, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                      const cuuint32_t* box, CUtensorMapSwizzle swizzle);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------- device side
SDB_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SDB_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

SDB_DEV void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

SDB_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

SDB_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

SDB_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps in the
// barrier (woken by the completing arrival) instead of spinning; for waits on HBM.
SDB_DEV bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "n"(1000000)
        : "memory");
    return ok != 0;
}
SDB_DEV bool mbar_wait_sleep(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (clock64() - t0 > kSpinLimitCycles) return false;
    }
    return true;
}

// Wait for the phase of the given parity to complete; false after ~2 s.
SDB_DEV bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kSpinLimitCycles) return false;
    }
    return true;
}

// 4-D tiled TMA load into this CTA's shared memory, completing on an mbarrier.
// No multicast: the source is always this GPU's own memory.
SDB_DEV void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                         int c2, int c3, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "l"(policy)
        : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory, completing on an mbarrier.
SDB_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
        : "memory");
}

// Contiguous bulk copy global -> this CTA's shared memory, completing on an mbarrier
// (both addresses 16-byte aligned, bytes a multiple of 16).  No multicast.
SDB_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

SDB_DEV uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

SDB_DEV uint64_t l2_policy_evict_normal() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

SDB_DEV void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- clusters and PDL
SDB_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
SDB_DEV uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
// Every thread of every CTA in the cluster arrives (release) and waits (acquire): shared
// memory written before it is visible to the cluster's other CTAs after it.
SDB_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Generic address of the same shared-memory location in the CTA of rank `rank` of this
// cluster; plain loads through it read that CTA's shared memory (DSMEM).
SDB_DEV const void* dsmem_map(const void* p, uint32_t rank) {
    uint64_t r;
    asm("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
    return reinterpret_cast<const void*>(r);
}
// Programmatic dependent launch: let the next kernel in the stream start launching, and
// wait until the preceding kernel has completed with its memory visible.
SDB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
SDB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

SDB_DEV void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier over `nthreads` threads that also ORs a predicate across them.
SDB_DEV bool barrier_or(int id, int nthreads, bool pred) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(out)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return out != 0;
}

SDB_DEV void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

SDB_DEV void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// Element-type traits for the 16-bit tensor-core path.
template <typename T>
struct Half16;

template <>
struct Half16<__nv_bfloat16> {
    static SDB_DEV uint32_t pack(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static SDB_DEV void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    // (lo - hi0, hi - hi1) rounded to bf16, where hi0/hi1 are the packed head values
    static SDB_DEV uint32_t pack_residual(float lo, float hi, uint32_t head) {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&head);
        const float2 f = __bfloat1622float2(h);
        return pack(lo - f.x, hi - f.y);
    }
    // x = hi + lo with both 16-bit: hi is x truncated to bf16 (bit mask), x - hi is
    // exact in f32 and is rounded once, so hi + lo carries ~16 significant bits of x.
    static SDB_DEV void split(float x, uint16_t& hi, uint16_t& lo) {
        const uint32_t b = __float_as_uint(x);
        hi = (uint16_t)(b >> 16);
        const float r = x - __uint_as_float(b & 0xffff0000u);
        lo = __bfloat16_as_ushort(__float2bfloat16_rn(r));
    }
    // split() of two columns at once: packed heads (x0 in the low half) and packed residuals.
    static SDB_DEV void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
        const uint32_t b0 = __float_as_uint(x0), b1 = __float_as_uint(x1);
        hi = __byte_perm(b0, b1, 0x7632);
        lo = pack(x0 - __uint_as_float(b0 & 0xffff0000u), x1 - __uint_as_float(b1 & 0xffff0000u));
    }
    static constexpr CUtensorMapDataType tmap_type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};

template <>
struct Half16<__half> {
    static SDB_DEV uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static SDB_DEV void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    static SDB_DEV uint32_t pack_residual(float lo, float hi, uint32_t head) {
        __half2 h = *reinterpret_cast<__half2*>(&head);
        const float2 f = __half22float2(h);
        return pack(lo - f.x, hi - f.y);
    }
    static SDB_DEV void split(float x, uint16_t& hi, uint16_t& lo) {
        const __half h = __float2half_rn(x);
        hi = __half_as_ushort(h);
        lo = __half_as_ushort(__float2half_rn(x - __half2float(h)));
    }
    static SDB_DEV void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
        const __half2 h = __floats2half2_rn(x0, x1);
        const float2 f = __half22float2(h);
        hi = *reinterpret_cast<const uint32_t*>(&h);
        lo = pack(x0 - f.x, x1 - f.y);
    }
    static constexpr CUtensorMapDataType tmap_type = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
};

// Hardware base-2 exponential (MUFU.EX2): ex2(-inf) = +0.
SDB_DEV float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

SDB_DEV float to_f32(float x) { return x; }
SDB_DEV float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
SDB_DEV float to_f32(__half x) { return __half2float(x); }

template <typename T>
SDB_DEV T from_f32(float x);
template <>
SDB_DEV float from_f32<float>(float x) { return x; }
template <>
SDB_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
SDB_DEV __half from_f32<__half>(float x) { return __float2half_rn(x); }

}  // namespace sdb
