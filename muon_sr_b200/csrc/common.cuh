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

// All four Philox4x32-10 output words for the 64-bit counter (ctr_lo32, ctr_hi32, 0, 0).
__device__ __forceinline__ uint4 philox4(uint64_t ctr, PhiloxKey key) {
  uint32_t c0 = static_cast<uint32_t>(ctr), c1 = static_cast<uint32_t>(ctr >> 32), c2 = 0u, c3 = 0u;
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
  return make_uint4(c0, c1, c2, c3);
}

// ---------------------------------------------------------------------------------------
// Stochastic-rounding noise streams (the low 16 bits of each value are used), one per
// msr_sr_noise mode:
//  * SrNoise<NOISE_REF>  -- the reference's: word 0 of Philox4x32-10 at the counter truncated
//    to 32 bits, one generator call per rounded value (bit-identical to muon_sr).
//  * SrNoise<NOISE_FAST> -- one generator call per 8 consecutive counters; counter c uses the
//    16-bit half (c & 1) of word ((c >> 1) & 3) of Philox4x32-10 at counter (c >> 3)
//    (64-bit). Same keys. Statistically an unbiased 16-bit uniform per value like the
//    reference's, but different bits.
//  * SrNoise<NOISE_NONE> -- no noise: round_bf16 rounds to nearest even instead.
// ---------------------------------------------------------------------------------------
enum NoiseMode : int { NOISE_REF = MSR_SR_NOISE_REFERENCE, NOISE_FAST = MSR_SR_NOISE_FAST, NOISE_NONE = MSR_SR_NOISE_NONE };

__device__ __forceinline__ uint32_t half_of(uint4 w, uint32_t k) {
  const uint32_t word = k < 2 ? w.x : (k < 4 ? w.y : (k < 6 ? w.z : w.w));
  return (word >> (16u * (k & 1u))) & 0xFFFFu;
}

template <int MODE>
struct SrNoise {
  PhiloxKey key;

  __device__ __forceinline__ uint32_t at(uint64_t ctr) const {
    if (MODE == NOISE_NONE) return 0u;
    if (MODE == NOISE_FAST) return half_of(philox4(ctr >> 3, key), static_cast<uint32_t>(ctr & 7u));
    return philox_word0(static_cast<uint32_t>(ctr), key);
  }

  // Noise for the 8 consecutive counters ctr0 .. ctr0 + 7 into r[0..7].
  __device__ __forceinline__ void eight(uint64_t ctr0, uint32_t* r) const {
    if (MODE == NOISE_NONE) {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = 0u;
      return;
    }
    if (MODE == NOISE_REF) {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = philox_word0(static_cast<uint32_t>(ctr0 + j), key);
      return;
    }
    const uint4 w0 = philox4(ctr0 >> 3, key);
    const uint32_t off = static_cast<uint32_t>(ctr0 & 7u);
    if (off == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = half_of(w0, j);
      return;
    }
    const uint4 w1 = philox4((ctr0 >> 3) + 1, key);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t k = off + j;
      r[j] = k < 8 ? half_of(w0, k) : half_of(w1, k - 8);
    }
  }
};

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

// The rounding of every SR store: stochastic with the mode's noise word, or round to
// nearest even in NOISE_NONE (the noise word is then unused).
template <int MODE>
__device__ __forceinline__ uint16_t round_bf16(float x, uint32_t rand) {
  if (MODE == NOISE_NONE) return rne_bf16_bits(x);
  return sr_bf16_bits(x, rand);
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

// Stores through an NVLink multicast address (multimem.st): the bytes land at the same offset
// in every GPU's memory bound to the multicast object. 16 bytes (8 bf16, moved as four
// 32-bit words; a store does no arithmetic on them) or 4 bytes (two bf16).
__device__ __forceinline__ void mc_st_u16x8(void* mc, const U16x8& x) {
  const uint4 r = *reinterpret_cast<const uint4*>(x.v);
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "r"(r.x), "r"(r.y), "r"(r.z), "r"(r.w)
               : "memory");
}

__device__ __forceinline__ void mc_st_u32(void* mc, uint32_t v) {
  asm volatile("multimem.st.relaxed.sys.global.b32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
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
