// crumpet_b200: shared device helpers for the shifted-window kernels.
//
// Integer division by run-time invariant divisors, 2/4/8/16-byte vector
// global loads and stores, and the element-type table used by every kernel.
// Written for sm_100a (B200); nothing here is architecture-generic on purpose.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace crumpet {

// ---------------------------------------------------------------------------
// Division by an invariant divisor.
//
// Granlund & Montgomery, "Division by invariant integers using
// multiplication" (PLDI 1994), Figure 4.1: for an N-bit unsigned dividend n
// and divisor d >= 1, with l = ceil(log2 d) and m = floor(2^N (2^l - d) / d) + 1,
//     t = mulhi(m, n);  q = (t + ((n - t) >> min(l,1))) >> max(l-1,0)
// is exact for every n in [0, 2^N).  The host computes (m, shifts) once per
// launch; the device pays one multiply-high, two shifts and two adds.
// ---------------------------------------------------------------------------
struct DivMod32 {
  uint32_t d;
  uint32_t m;
  uint32_t s1;
  uint32_t s2;

  static DivMod32 make(uint32_t divisor) {
    DivMod32 r;
    r.d = divisor;
    uint32_t l = 0;
    while ((uint64_t(1) << l) < divisor) ++l;
    r.m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << l) - divisor)) / divisor + 1);
    r.s1 = l < 1 ? l : 1;
    r.s2 = l > 0 ? l - 1 : 0;
    return r;
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    const uint32_t t = __umulhi(n, m);
    return (t + ((n - t) >> s1)) >> s2;
  }
  __device__ __forceinline__ void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
    q = div(n);
    r = n - q * d;
  }
};

struct DivMod64 {
  uint64_t d;
  uint64_t m;
  uint32_t s1;
  uint32_t s2;

  static DivMod64 make(uint64_t divisor) {
    DivMod64 r;
    r.d = divisor;
    uint32_t l = 0;
    while (l < 64 && ((unsigned __int128)1 << l) < divisor) ++l;
    const unsigned __int128 num =
        ((unsigned __int128)1 << 64) * (((unsigned __int128)1 << l) - divisor);
    r.m = uint64_t(num / divisor + 1);
    r.s1 = l < 1 ? l : 1;
    r.s2 = l > 0 ? l - 1 : 0;
    return r;
  }
  __device__ __forceinline__ uint64_t div(uint64_t n) const {
    const uint64_t t = __umul64hi(n, m);
    return (t + ((n - t) >> s1)) >> s2;
  }
};

// ---------------------------------------------------------------------------
// Vector global memory access.  Loads use the non-coherent path and do not
// allocate in L1 (each byte is read exactly once by these kernels).
// ---------------------------------------------------------------------------
template <int kBytes>
struct VecT;
template <>
struct VecT<16> { using type = uint4; };
template <>
struct VecT<8> { using type = uint2; };
template <>
struct VecT<4> { using type = uint32_t; };
template <>
struct VecT<2> { using type = uint16_t; };

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream(const uint2* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_stream(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ldg_stream(const uint16_t* p) {
  uint16_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void stg(uint4* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void stg(uint2* p, uint2 v) {
  asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void stg(uint32_t* p, uint32_t v) {
  asm volatile("st.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void stg(uint16_t* p, uint16_t v) {
  asm volatile("st.global.u16 [%0], %1;" ::"l"(p), "h"(v) : "memory");
}

// Element types crossing the C ABI (values match CRUMPET_DTYPE_* in
// include/crumpet_b200.h).
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

inline int dtype_size(int dt) { return dt == kF32 ? 4 : 2; }

// Bit pattern of -100.0 in each element type (exact in all three formats).
inline uint32_t neg100_bits(int dt) {
  if (dt == kF32) return 0xC2C80000u;
  if (dt == kF16) return 0xD640u;
  return 0xC2C8u;  // bf16 is the upper half of the fp32 pattern
}

}  // namespace crumpet
