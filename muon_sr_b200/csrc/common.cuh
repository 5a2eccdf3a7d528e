// Shared device helpers for the muon_sr_b200 engine (sm_100a only).
//
// * Philox4x32-10 word 0, bit-compatible with Triton's tl.randint as every muon_sr kernel
//   calls it (counter = (offset_lo32, 0, 0, 0), key = 64-bit seed), see
//   muon_sr/triton_muon_sr.py:44 and triton/language/random.py:12-110.
// * Stochastic rounding fp32 -> bf16 exactly as muon_sr/triton_adamw.py:57-67 does it:
//   int32 add of the low 16 noise bits, clear the low 16 bits.
// * Round-to-nearest-even fp32 -> bf16 (Triton / torch .to(bfloat16)).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/muon_sr_b200.h"

#if !defined(__CUDA_ARCH__) || __CUDA_ARCH__ >= 1000
#else
#error "muon_sr_b200 is written for sm_100a (B200) only"
#endif

namespace msr {

// ---------------------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC 2011) with Triton's constants and layout. Only word 0 is
// returned. Counter words 1..3 are zero, so the first two rounds fold to fewer multiplies;
// the compiler does that folding from the literal zeros.
// ---------------------------------------------------------------------------------------
struct PhiloxKey {
  uint32_t k0, k1;
};

__host__ __device__ __forceinline__ PhiloxKey make_key(uint64_t key64) {
  PhiloxKey k;
  k.k0 = static_cast<uint32_t>(key64);
  k.k1 = static_cast<uint32_t>(key64 >> 32);
  return k;
}

__device__ __forceinline__ uint32_t philox_word0(uint32_t ctr, PhiloxKey key) {
  uint32_t c0 = ctr, c1 = 0u, c2 = 0u, c3 = 0u;
  uint32_t k0 = key.k0, k1 = key.k1;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo0 = 0xD2511F53u * c0;
    const uint32_t hi2 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t lo2 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi2 ^ c1 ^ k0;
    const uint32_t n2 = hi0 ^ c3 ^ k1;
    c1 = lo2;
    c3 = lo0;
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

// ---------------------------------------------------------------------------------------
// Rounding
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// SR: (bits(x) + (rand & 0xFFFF)) & 0xFFFF0000, top half is the bf16 (integer wrap-around
// exactly like the reference's int32 arithmetic).
__device__ __forceinline__ uint16_t sr_bf16_bits(float x, uint32_t rand) {
  const uint32_t b = __float_as_uint(x) + (rand & 0xFFFFu);
  return static_cast<uint16_t>(b >> 16);
}

__device__ __forceinline__ uint16_t rne_bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// ---------------------------------------------------------------------------------------
// 16-byte vectors of 8 bf16 values
// ---------------------------------------------------------------------------------------
struct alignas(16) U16x8 {
  uint16_t v[8];
};

__device__ __forceinline__ U16x8 ld_u16x8(const void* p) {
  uint4 r = *reinterpret_cast<const uint4*>(p);
  U16x8 o;
  *reinterpret_cast<uint4*>(o.v) = r;
  return o;
}

__device__ __forceinline__ U16x8 ld_u16x8_stream(const void* p) {
  uint4 r = __ldcs(reinterpret_cast<const uint4*>(p));
  U16x8 o;
  *reinterpret_cast<uint4*>(o.v) = r;
  return o;
}

__device__ __forceinline__ void st_u16x8(void* p, const U16x8& x) {
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(x.v);
}

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Multi-tensor launch helper: map a global chunk index to (entry, chunk-in-entry) by a
// binary search over the exclusive prefix of per-entry chunk counts (uniform per CTA).
template <int MAXE>
__device__ __forceinline__ int find_entry(const int64_t (&prefix)[MAXE + 1], int count, int64_t chunk) {
  int lo = 0, hi = count;  // prefix[lo] <= chunk < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= chunk) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace msr
