// Device helpers shared by the tcgen05 W8A16 kernels: exact int8 -> 16-bit conversion
// of the weights and the per-channel scale read.
#pragma once

#include "common.cuh"

namespace sdb {
namespace w8cv {

// Per-channel scale of output feature n, stored as float32, bf16 or f16.
SDB_DEV float scale_value(const void* s, int s_dtype, int n) {
    if (s_dtype == SDB_F32) return reinterpret_cast<const float*>(s)[n];
    if (s_dtype == SDB_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(s)[n]);
    return __half2float(reinterpret_cast<const __half*>(s)[n]);
}

// 4 int8 -> 4 16-bit values (two packed pairs, the lower k in the low half), exact (|q| <= 127).
template <typename T>
SDB_DEV void i8x4(uint32_t w, uint32_t& lo, uint32_t& hi);
template <>
SDB_DEV void i8x4<__half>(uint32_t w, uint32_t& lo, uint32_t& hi) {
    // 0x64XX as f16 is 1024 + XX; bias the signed byte by 128 and subtract 1152
    const uint32_t u = w ^ 0x80808080u;
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
    lo = *reinterpret_cast<uint32_t*>(&ha);
    hi = *reinterpret_cast<uint32_t*>(&hb);
}
template <>
SDB_DEV void i8x4<__nv_bfloat16>(uint32_t w, uint32_t& lo, uint32_t& hi) {
    // 0x4B0000XX as f32 is 2^23 + XX; bias by 128, subtract 2^23 + 128, pack to bf16
    const uint32_t u = w ^ 0x80808080u;
    uint32_t f0, f1, f2, f3;
    asm("prmt.b32 %0, %1, %2, 0x7540;" : "=r"(f0) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7541;" : "=r"(f1) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7542;" : "=r"(f2) : "r"(u), "r"(0x4B000000u));
    asm("prmt.b32 %0, %1, %2, 0x7543;" : "=r"(f3) : "r"(u), "r"(0x4B000000u));
    const float c = 8388736.0f;
    __nv_bfloat162 pa = __floats2bfloat162_rn(__uint_as_float(f0) - c, __uint_as_float(f1) - c);
    __nv_bfloat162 pb = __floats2bfloat162_rn(__uint_as_float(f2) - c, __uint_as_float(f3) - c);
    lo = *reinterpret_cast<uint32_t*>(&pa);
    hi = *reinterpret_cast<uint32_t*>(&pb);
}

}  // namespace w8cv
}  // namespace sdb
