// Fused elementwise kernels of the optimizer step: SR gradient accumulation, Muon
// prepare (momentum + Nesterov), Muon apply (decay + scaled update) and AdamW-SR.
//
// Design (B200): multi-tensor launches. Each launch carries up to MAXE tensors in its
// kernel parameters; the work is cut into chunks of 4096 elements that never cross a
// tensor, and a persistent grid (a multiple of the SM count) walks the chunks. Each thread
// moves 8 bf16 per 16-byte access, issuing all loads of a chunk before its math so that
// every SM keeps enough bytes in flight for HBM3e. All fp32 arithmetic uses explicit
// round-to-nearest intrinsics (no contraction into FMA), in the reference's op order, so
// results are bit-identical to the reference kernels' fp32 evaluation. Every kernel is
// instantiated per noise mode (msr_set_sr_noise), and prepare / apply / AdamW once more
// (REC) for the replayable launches that read their scalars and entries from a device
// record (msr_*_rec, used inside captured CUDA graphs).
#include "common.cuh"
#include "host_common.h"

#include <algorithm>

namespace msr {
namespace {

constexpr int EW_THREADS = 256;
constexpr int EW_VEC = 8;
constexpr int EW_ITERS = 2;
constexpr int64_t EW_CHUNK = EW_THREADS * EW_VEC * EW_ITERS;  // 4096 elements
constexpr int MAXE = 64;
constexpr int EW_BLOCKS_PER_SM = 4;
// AdamW: the three Philox chains of each element need more than 64 registers. Measured on 2^30
// elements with the reference noise: 1 vector of 8 per thread and chunk at 2 CTAs per SM
// (122 registers, no spills) 1645 GB/s; 2 vectors at 2 CTAs per SM (128 registers, 40 bytes
// of spills) 1490; 1 vector at 3 or 4 CTAs per SM (80 / 64 registers, spilling) slower still.
constexpr int ADAMW_ITERS = 1;
constexpr int ADAMW_MINB = 2;
constexpr int64_t ADAMW_CHUNK = EW_THREADS * EW_VEC * ADAMW_ITERS;
// Apply: one vector per thread and chunk (60 registers, no spills) measured 2350 GB/s on 2^30
// elements against 2262 for two vectors (64 registers with 20 bytes of spills).
constexpr int APPLY_ITERS = 1;
constexpr int64_t APPLY_CHUNK = EW_THREADS * EW_VEC * APPLY_ITERS;

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }

// ---------------------------------------------------------------------------------------
// Philox test hook
// ---------------------------------------------------------------------------------------
__global__ void philox_fill_kernel(uint32_t* out, int64_t n, uint64_t ctr_base, PhiloxKey key) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = philox_word0(static_cast<uint32_t>(ctr_base + static_cast<uint64_t>(i)), key);
}

// ---------------------------------------------------------------------------------------
// SR gradient accumulation: acc <- SR(acc + g) -- muon_sr/triton_adamw.py:206-229
// ---------------------------------------------------------------------------------------
template <int NOISE>
__device__ __forceinline__ uint16_t accum_one(uint16_t a, uint16_t g, uint32_t rnd) {
  const float s = fadd(bf16_bits_to_f32(a), bf16_bits_to_f32(g));
  return round_bf16<NOISE>(s, rnd);
}

// First micro-batch: SR(0 + g) == g exactly (g is already bf16), except -0 + 0 = +0.
__device__ __forceinline__ uint16_t first_one(uint16_t g) { return g == 0x8000u ? uint16_t(0) : g; }

template <bool VEC>
__global__ __launch_bounds__(EW_THREADS) void grad_accum_first_kernel(uint16_t* __restrict__ acc,
                                                                     const uint16_t* __restrict__ g, int64_t n) {
  const int64_t nvec = VEC ? n / EW_VEC : 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    U16x8 v = ld_u16x8_stream(g + i * EW_VEC);
#pragma unroll
    for (int j = 0; j < EW_VEC; ++j) v.v[j] = first_one(v.v[j]);
    st_u16x8(acc + i * EW_VEC, v);
  }
  for (int64_t i = nvec * EW_VEC + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    acc[i] = first_one(g[i]);
}

template <bool VEC, int NOISE>
__global__ __launch_bounds__(EW_THREADS, 4) void grad_accum_kernel(uint16_t* __restrict__ acc,
                                                               const uint16_t* __restrict__ g,
                                                               int64_t n, PhiloxKey key) {
  constexpr bool FAST = NOISE == NOISE_FAST;
  const SrNoise<NOISE> nz{key};
  const int64_t nchunks = (n + EW_CHUNK - 1) / EW_CHUNK;
  for (int64_t chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
    const int64_t base = chunk * EW_CHUNK;
    if (VEC) {
      U16x8 va[EW_ITERS], vg[EW_ITERS];
#pragma unroll
      for (int it = 0; it < EW_ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          va[it] = ld_u16x8(acc + idx);
          vg[it] = ld_u16x8_stream(g + idx);
        }
      }
#pragma unroll
      for (int it = 0; it < EW_ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          U16x8 o;
          uint32_t r[EW_VEC];
          if (FAST) nz.eight(static_cast<uint64_t>(idx), r);
#pragma unroll
          for (int j = 0; j < EW_VEC; ++j)
            o.v[j] = accum_one<NOISE>(va[it].v[j], vg[it].v[j],
                                      FAST ? r[j] : nz.at(static_cast<uint64_t>(idx + j)));
          st_u16x8(acc + idx, o);
        } else {
          for (int64_t i = idx; i < n; ++i) acc[i] = accum_one<NOISE>(acc[i], g[i], nz.at(static_cast<uint64_t>(i)));
        }
      }
    } else {
      for (int it = 0; it < EW_ITERS * EW_VEC; ++it) {
        const int64_t i = base + it * EW_THREADS + threadIdx.x;
        if (i < n) acc[i] = accum_one<NOISE>(acc[i], g[i], nz.at(static_cast<uint64_t>(i)));
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Muon prepare -- muon_sr/triton_muon_sr.py:18-50
// ---------------------------------------------------------------------------------------
struct PrepareArgs {
  msr_prepare_entry e[MAXE];
  int64_t prefix[MAXE + 1];
  uint8_t vec[MAXE];
  int count;
  float beta, omb;
  int nesterov;
  // Replayable launches (msr_muon_prepare_rec): scalars and entries come from this device
  // record; src[i] is the record's index of entry i.
  const msr_prepare_record* rec;
  int32_t src[MAXE];
};

// Launch scalars and entry i of a launch, from the parameters or (REC) the device record.
template <bool REC>
__device__ __forceinline__ const msr_prepare_entry& entry_of(const PrepareArgs& a, int i) {
  if constexpr (REC) return reinterpret_cast<const msr_prepare_entry*>(a.rec + 1)[a.src[i]];
  else return a.e[i];
}
template <bool REC>
__device__ __forceinline__ float beta_of(const PrepareArgs& a) { return REC ? a.rec->beta : a.beta; }
template <bool REC>
__device__ __forceinline__ float omb_of(const PrepareArgs& a) { return REC ? a.rec->one_minus_beta : a.omb; }

// `rnd()` yields the element's noise word; it is called after the math, where the noise is
// consumed, which keeps the register allocation of the Philox chain as short as possible.
template <int NOISE, class Rnd>
__device__ __forceinline__ void prepare_one(uint16_t g_bits, uint16_t b_bits, float beta, float omb, bool nesterov,
                                            Rnd rnd, uint16_t& buf_out, uint16_t& upd_out) {
  const float g = bf16_bits_to_f32(g_bits);
  const float buf = bf16_bits_to_f32(b_bits);
  const float nb = fadd(buf, fmul(omb, fsub(g, buf)));
  const float upd = nesterov ? fadd(g, fmul(beta, fsub(nb, g))) : nb;
  buf_out = round_bf16<NOISE>(nb, rnd());
  upd_out = rne_bf16_bits(upd);
}

template <int NOISE, bool REC>
__global__ __launch_bounds__(EW_THREADS, 4) void muon_prepare_kernel(const __grid_constant__ PrepareArgs a) {
  constexpr bool FAST = NOISE == NOISE_FAST;
  const int64_t total = a.prefix[a.count];
  const bool nesterov = (REC ? a.rec->nesterov : a.nesterov) != 0;
  for (int64_t chunk = blockIdx.x; chunk < total; chunk += gridDim.x) {
    const int ei = find_entry<MAXE>(a.prefix, a.count, chunk);
    const msr_prepare_entry& E = entry_of<REC>(a, ei);
    const uint16_t* g = static_cast<const uint16_t*>(E.grad);
    uint16_t* mb = static_cast<uint16_t*>(E.momentum);
    uint16_t* up = static_cast<uint16_t*>(E.update);
    const int64_t n = E.numel;
    const SrNoise<NOISE> nz{make_key(E.key)};
    const uint64_t cb = E.ctr_base;
    const int64_t base = (chunk - a.prefix[ei]) * EW_CHUNK;
    if (a.vec[ei]) {
      U16x8 vg[EW_ITERS], vb[EW_ITERS];
#pragma unroll
      for (int it = 0; it < EW_ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          vg[it] = ld_u16x8_stream(g + idx);
          vb[it] = ld_u16x8(mb + idx);
        }
      }
#pragma unroll
      for (int it = 0; it < EW_ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          U16x8 ob, ou;
          uint32_t r[EW_VEC];
          if (FAST) nz.eight(cb + static_cast<uint64_t>(idx), r);
#pragma unroll
          for (int j = 0; j < EW_VEC; ++j)
            prepare_one<NOISE>(vg[it].v[j], vb[it].v[j], beta_of<REC>(a), omb_of<REC>(a), nesterov,
                               [&] { return FAST ? r[j] : nz.at(cb + static_cast<uint64_t>(idx + j)); }, ob.v[j],
                               ou.v[j]);
          st_u16x8(mb + idx, ob);
          st_u16x8(up + idx, ou);
        } else {
          for (int64_t i = idx; i < n; ++i) {
            uint16_t ob, ou;
            prepare_one<NOISE>(g[i], mb[i], beta_of<REC>(a), omb_of<REC>(a), nesterov, [&] { return nz.at(cb + static_cast<uint64_t>(i)); }, ob, ou);
            mb[i] = ob;
            up[i] = ou;
          }
        }
      }
    } else {
      for (int it = 0; it < EW_ITERS * EW_VEC; ++it) {
        const int64_t i = base + it * EW_THREADS + threadIdx.x;
        if (i < n) {
          uint16_t ob, ou;
          prepare_one<NOISE>(g[i], mb[i], beta_of<REC>(a), omb_of<REC>(a), nesterov, [&] { return nz.at(cb + static_cast<uint64_t>(i)); }, ob, ou);
          mb[i] = ob;
          up[i] = ou;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Muon apply -- muon_sr/triton_muon_sr.py:53-80
// ---------------------------------------------------------------------------------------
struct ApplyArgs {
  msr_apply_entry e[MAXE];
  int64_t prefix[MAXE + 1];
  uint8_t vec[MAXE];
  int count;
  float lr, decay;
  const msr_apply_record* rec;  // msr_muon_apply_rec (see PrepareArgs)
  int32_t src[MAXE];
  int any_mc;  // some entry stores its weights through a multicast address
};

template <bool REC>
__device__ __forceinline__ const msr_apply_entry& entry_of(const ApplyArgs& a, int i) {
  if constexpr (REC) return reinterpret_cast<const msr_apply_entry*>(a.rec + 1)[a.src[i]];
  else return a.e[i];
}
template <bool REC>
__device__ __forceinline__ float lr_of(const ApplyArgs& a) { return REC ? a.rec->lr : a.lr; }
template <bool REC>
__device__ __forceinline__ float decay_of(const ApplyArgs& a) { return REC ? a.rec->decay : a.decay; }

template <int NOISE>
__device__ __forceinline__ uint16_t apply_one(uint16_t p_bits, uint16_t u_bits, float scale, float lr, float decay,
                                              uint32_t rnd) {
  const float u = fmul(bf16_bits_to_f32(u_bits), scale);
  float p = fmul(bf16_bits_to_f32(p_bits), decay);
  p = fsub(p, fmul(lr, u));
  return round_bf16<NOISE>(p, rnd);
}

// Elements lo .. hi - 1 of one apply entry, one thread: plain stores, or (multicast weights)
// 4-byte pairs from an even index -- a pair past the last element writes 0 into the padding
// that follows the parameter's slot.
template <int NOISE, bool REC>
__device__ __forceinline__ void apply_tail(const ApplyArgs& a, uint16_t* p, uint16_t* pm, const uint16_t* u,
                                           float scale, const SrNoise<NOISE>& nz, int64_t lo, int64_t hi) {
  auto one = [&](int64_t i) {
    return apply_one<NOISE>(p[i], u[i], scale, lr_of<REC>(a), decay_of<REC>(a), nz.at(static_cast<uint64_t>(i)));
  };
  if (!pm) {
    for (int64_t i = lo; i < hi; ++i) p[i] = one(i);
    return;
  }
  for (int64_t i = lo; i < hi; i += 2) {
    const uint32_t v0 = one(i), v1 = i + 1 < hi ? one(i + 1) : 0u;
    mc_st_u32(pm + i, v0 | (v1 << 16));
  }
}

template <int NOISE, bool REC>
__global__ __launch_bounds__(EW_THREADS, 4) void muon_apply_kernel(const __grid_constant__ ApplyArgs a) {
  constexpr bool FAST = NOISE == NOISE_FAST;
  const int64_t total = a.prefix[a.count];
  for (int64_t chunk = blockIdx.x; chunk < total; chunk += gridDim.x) {
    const int ei = find_entry<MAXE>(a.prefix, a.count, chunk);
    const msr_apply_entry& E = entry_of<REC>(a, ei);
    uint16_t* p = static_cast<uint16_t*>(E.param);
    uint16_t* pm = static_cast<uint16_t*>(E.param_mc);  // multicast weights (sharded steps)
    const uint16_t* u = static_cast<const uint16_t*>(E.update);
    const int64_t n = E.numel;
    const SrNoise<NOISE> nz{make_key(E.key)};
    const float scale = E.scale;
    const int64_t base = (chunk - a.prefix[ei]) * APPLY_CHUNK;
    if (a.vec[ei]) {
      U16x8 vp[APPLY_ITERS], vu[APPLY_ITERS];
#pragma unroll
      for (int it = 0; it < APPLY_ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          vp[it] = ld_u16x8(p + idx);
          vu[it] = ld_u16x8_stream(u + idx);
        }
      }
#pragma unroll
      for (int it = 0; it < APPLY_ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          U16x8 o;
          uint32_t r[EW_VEC];
          if (FAST) nz.eight(static_cast<uint64_t>(idx), r);
#pragma unroll
          for (int j = 0; j < EW_VEC; ++j)
            o.v[j] = apply_one<NOISE>(vp[it].v[j], vu[it].v[j], scale, lr_of<REC>(a), decay_of<REC>(a),
                                      FAST ? r[j] : nz.at(static_cast<uint64_t>(idx + j)));
          if (pm)
            mc_st_u16x8(pm + idx, o);
          else
            st_u16x8(p + idx, o);
        } else {
          apply_tail<NOISE, REC>(a, p, pm, u, scale, nz, idx, n);
        }
      }
    } else {
      if (pm) {  // an unaligned entry with multicast weights: 4-byte pairs, thread-contiguous
        const int64_t lo = base + static_cast<int64_t>(threadIdx.x) * (APPLY_ITERS * EW_VEC);
        apply_tail<NOISE, REC>(a, p, pm, u, scale, nz, lo, lo + APPLY_ITERS * EW_VEC < n ? lo + APPLY_ITERS * EW_VEC : n);
      } else {
        for (int it = 0; it < APPLY_ITERS * EW_VEC; ++it) {
          const int64_t i = base + it * EW_THREADS + threadIdx.x;
          if (i < n) p[i] = apply_one<NOISE>(p[i], u[i], scale, lr_of<REC>(a), decay_of<REC>(a), nz.at(static_cast<uint64_t>(i)));
        }
      }
    }
  }
  if (a.any_mc) __threadfence_system();  // multicast stores ordered before the callers' barrier
}

// ---------------------------------------------------------------------------------------
// AdamW-SR -- muon_sr/triton_adamw.py:9-72
// ---------------------------------------------------------------------------------------
struct AdamWArgs {
  msr_adamw_entry e[MAXE];
  int64_t prefix[MAXE + 1];
  uint8_t vec[MAXE];
  int count;
  msr_adamw_hparams hp;
  const msr_adamw_record* rec;  // msr_adamw_sr_rec (see PrepareArgs)
  int32_t src[MAXE];
  int any_mc;  // some entry stores its weights through a multicast address
};

template <bool REC>
__device__ __forceinline__ const msr_adamw_entry& entry_of(const AdamWArgs& a, int i) {
  if constexpr (REC) return reinterpret_cast<const msr_adamw_entry*>(a.rec + 1)[a.src[i]];
  else return a.e[i];
}
template <bool REC>
__device__ __forceinline__ const msr_adamw_hparams& hp_of(const AdamWArgs& a) {
  if constexpr (REC) return a.rec->hp;
  else return a.hp;
}

template <int NOISE, class Rnd>
__device__ __forceinline__ void adamw_one(uint16_t& p_bits, uint16_t g_bits, uint16_t& m_bits, uint16_t& v_bits,
                                          const msr_adamw_hparams& hp, float step_size, float bc2s, Rnd rnd) {
  const float g = bf16_bits_to_f32(g_bits);
  float m = bf16_bits_to_f32(m_bits);
  float v = bf16_bits_to_f32(v_bits);
  float p = bf16_bits_to_f32(p_bits);
  m = fadd(fmul(hp.beta1, m), fmul(hp.one_minus_beta1, g));
  v = fadd(fmul(hp.beta2, v), fmul(fmul(hp.one_minus_beta2, g), g));
  const float denom = fadd(__fdiv_rn(__fsqrt_rn(v), bc2s), hp.eps);
  p = fmul(p, hp.decay);
  p = fsub(p, __fdiv_rn(fmul(step_size, m), denom));
  m_bits = round_bf16<NOISE>(m, rnd(0));
  v_bits = round_bf16<NOISE>(v, rnd(1));
  p_bits = round_bf16<NOISE>(p, rnd(2));
}

// Elements lo .. hi - 1 of one AdamW entry, one thread: plain stores, or (multicast weights)
// the weights in 4-byte pairs from an even index (a pair past the last element writes 0 into
// the padding that follows the parameter's slot); the moments are always local.
template <int NOISE, bool REC>
__device__ __forceinline__ void adamw_tail(const AdamWArgs& a, const msr_adamw_entry& E, const SrNoise<NOISE>& nm,
                                           const SrNoise<NOISE>& nv, const SrNoise<NOISE>& np_, int64_t lo,
                                           int64_t hi) {
  uint16_t* p = static_cast<uint16_t*>(E.param);
  uint16_t* pm = static_cast<uint16_t*>(E.param_mc);
  const uint16_t* g = static_cast<const uint16_t*>(E.grad);
  uint16_t* m = static_cast<uint16_t*>(E.exp_avg);
  uint16_t* v = static_cast<uint16_t*>(E.exp_avg_sq);
  auto one = [&](int64_t i) {
    uint16_t pb = p[i], mb = m[i], vb = v[i];
    const uint64_t c = static_cast<uint64_t>(i);
    adamw_one<NOISE>(pb, g[i], mb, vb, hp_of<REC>(a), E.step_size, E.bc2_sqrt,
                     [&](int w) { return w == 0 ? nm.at(c) : w == 1 ? nv.at(c) : np_.at(c); });
    m[i] = mb;
    v[i] = vb;
    return pb;
  };
  if (!pm) {
    for (int64_t i = lo; i < hi; ++i) p[i] = one(i);
    return;
  }
  for (int64_t i = lo; i < hi; i += 2) {
    const uint32_t v0 = one(i), v1 = i + 1 < hi ? one(i + 1) : 0u;
    mc_st_u32(pm + i, v0 | (v1 << 16));
  }
}

// ITERS vectors of 8 elements per thread and chunk; MINB CTAs per SM for the register budget.
template <int ITERS, int MINB, int NOISE, bool REC>
__global__ __launch_bounds__(EW_THREADS, MINB) void adamw_kernel(const __grid_constant__ AdamWArgs a) {
  constexpr bool FAST = NOISE == NOISE_FAST;
  constexpr int64_t CHUNK = EW_THREADS * EW_VEC * ITERS;
  const int64_t total = a.prefix[a.count];
  for (int64_t chunk = blockIdx.x; chunk < total; chunk += gridDim.x) {
    const int ei = find_entry<MAXE>(a.prefix, a.count, chunk);
    const msr_adamw_entry& E = entry_of<REC>(a, ei);
    uint16_t* p = static_cast<uint16_t*>(E.param);
    uint16_t* pm = static_cast<uint16_t*>(E.param_mc);  // multicast weights (sharded steps)
    const uint16_t* g = static_cast<const uint16_t*>(E.grad);
    uint16_t* m = static_cast<uint16_t*>(E.exp_avg);
    uint16_t* v = static_cast<uint16_t*>(E.exp_avg_sq);
    const int64_t n = E.numel;
    const SrNoise<NOISE> nm{make_key(E.key_m)}, nv{make_key(E.key_v)}, np_{make_key(E.key_p)};
    const float ss = E.step_size, bc2s = E.bc2_sqrt;
    const int64_t base = (chunk - a.prefix[ei]) * CHUNK;
    if (a.vec[ei]) {
      U16x8 vp[ITERS], vg[ITERS], vm[ITERS], vv[ITERS];
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          vp[it] = ld_u16x8(p + idx);
          vg[it] = ld_u16x8_stream(g + idx);
          vm[it] = ld_u16x8(m + idx);
          vv[it] = ld_u16x8(v + idx);
        }
      }
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const int64_t idx = base + (int64_t)(it * EW_THREADS + threadIdx.x) * EW_VEC;
        if (idx + EW_VEC <= n) {
          uint32_t rm[EW_VEC], rv[EW_VEC], rp[EW_VEC];
          if (FAST) {
            nm.eight(static_cast<uint64_t>(idx), rm);
            nv.eight(static_cast<uint64_t>(idx), rv);
            np_.eight(static_cast<uint64_t>(idx), rp);
          }
#pragma unroll
          for (int j = 0; j < EW_VEC; ++j) {
            const uint64_t c = static_cast<uint64_t>(idx + j);
            adamw_one<NOISE>(vp[it].v[j], vg[it].v[j], vm[it].v[j], vv[it].v[j], hp_of<REC>(a), ss, bc2s, [&](int w) {
              return w == 0 ? (FAST ? rm[j] : nm.at(c)) : w == 1 ? (FAST ? rv[j] : nv.at(c)) : (FAST ? rp[j] : np_.at(c));
            });
          }
          if (pm)
            mc_st_u16x8(pm + idx, vp[it]);
          else
            st_u16x8(p + idx, vp[it]);
          st_u16x8(m + idx, vm[it]);
          st_u16x8(v + idx, vv[it]);
        } else {
          adamw_tail<NOISE, REC>(a, E, nm, nv, np_, idx, n);
        }
      }
    } else if (pm) {  // an unaligned entry with multicast weights: 4-byte pairs, thread-contiguous
      const int64_t lo = base + static_cast<int64_t>(threadIdx.x) * (ITERS * EW_VEC);
      adamw_tail<NOISE, REC>(a, E, nm, nv, np_, lo, lo + ITERS * EW_VEC < n ? lo + ITERS * EW_VEC : n);
    } else {
      for (int it = 0; it < ITERS * EW_VEC; ++it) {
        const int64_t i = base + it * EW_THREADS + threadIdx.x;
        if (i < n) {
          uint16_t pb = p[i], mb = m[i], vb = v[i];
          adamw_one<NOISE>(pb, g[i], mb, vb, hp_of<REC>(a), ss, bc2s, [&](int w) {
              const uint64_t c = static_cast<uint64_t>(i);
              return w == 0 ? nm.at(c) : w == 1 ? nv.at(c) : np_.at(c);
            });
          p[i] = pb; m[i] = mb; v[i] = vb;
        }
      }
    }
  }
  if (a.any_mc) __threadfence_system();  // multicast stores ordered before the callers' barrier
}

// Gradient centralisation -- muon_sr/triton_adamw.py:179-187: out = bf16(g - c * mean), the
// mean taken in fp32 over all trailing dims of each leading index (over all elements for a
// vector), rounded to nearest-even as the reference's .to(bfloat16). One CTA per row: the
// row is summed in a fixed order (deterministic) and read again, from cache, for the output.
constexpr int CT_THREADS = 256;

__global__ __launch_bounds__(CT_THREADS) void centralize_kernel(const uint16_t* __restrict__ g,
                                                                uint16_t* __restrict__ out, int64_t rows,
                                                                int64_t cols, float c, int vec) {
  __shared__ float red[CT_THREADS / 32];
  __shared__ float mean_s;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t* gr = g + r * cols;
    uint16_t* orow = out + r * cols;
    float s = 0.f;
    if (vec) {
      for (int64_t i = threadIdx.x * 8; i < cols; i += CT_THREADS * 8) {
        const U16x8 w = ld_u16x8(gr + i);
#pragma unroll
        for (int j = 0; j < 8; ++j) s = __fadd_rn(s, bf16_bits_to_f32(w.v[j]));
      }
    } else {
      for (int64_t i = threadIdx.x; i < cols; i += CT_THREADS) s = __fadd_rn(s, bf16_bits_to_f32(gr[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < CT_THREADS / 32; ++w) t = __fadd_rn(t, red[w]);
      mean_s = __fdiv_rn(t, static_cast<float>(cols));
    }
    __syncthreads();
    const float cm = __fmul_rn(mean_s, c);
    if (vec) {
      for (int64_t i = threadIdx.x * 8; i < cols; i += CT_THREADS * 8) {
        U16x8 w = ld_u16x8(gr + i);
#pragma unroll
        for (int j = 0; j < 8; ++j) w.v[j] = rne_bf16_bits(__fsub_rn(bf16_bits_to_f32(w.v[j]), cm));
        st_u16x8(orow + i, w);
      }
    } else {
      for (int64_t i = threadIdx.x; i < cols; i += CT_THREADS)
        orow[i] = rne_bf16_bits(__fsub_rn(bf16_bits_to_f32(gr[i]), cm));
    }
    __syncthreads();  // red / mean_s are reused by the next row
  }
}

inline bool ptr_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int grid_for(int64_t chunks) {
  const int64_t cap = static_cast<int64_t>(sm_count()) * EW_BLOCKS_PER_SM;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(chunks, cap)));
}

inline bool record_ok(const void* rec) { return rec != nullptr && (reinterpret_cast<uintptr_t>(rec) & 15u) == 0; }

// The multi-tensor launchers: entries are packed MAXE at a time (empty ones skipped, each
// group resuming at the first entry the previous one did not take); with a record, the
// kernels take scalars and entries from it (src[] maps packed to record indices).
int prepare_launch(const msr_prepare_entry* entries, int count, float beta, float one_minus_beta, int nesterov,
                   const msr_prepare_record* rec, msr_stream_t stream) {
  if (count < 0 || (count > 0 && entries == nullptr)) return fail(MSR_ERR_INVALID, "msr_muon_prepare: bad entry list");
  int next = 0;
  while (next < count) {
    PrepareArgs a{};
    a.beta = beta;
    a.omb = one_minus_beta;
    a.nesterov = nesterov;
    a.rec = rec;
    int64_t chunks = 0;
    int i = next;
    for (; i < count && a.count < MAXE; ++i) {
      const msr_prepare_entry& e = entries[i];
      if (e.numel < 0 || (e.numel > 0 && (!e.grad || !e.momentum || !e.update)))
        return fail(MSR_ERR_INVALID, "msr_muon_prepare: entry %d has a null pointer or negative numel", i);
      if (e.numel == 0) continue;
      a.e[a.count] = e;
      a.src[a.count] = i;
      a.vec[a.count] = ptr_aligned16(e.grad) && ptr_aligned16(e.momentum) && ptr_aligned16(e.update);
      a.prefix[a.count] = chunks;
      chunks += (e.numel + EW_CHUNK - 1) / EW_CHUNK;
      ++a.count;
    }
    next = i;
    a.prefix[a.count] = chunks;
    if (a.count == 0) continue;
    auto* kern = rec ? pick_noise(muon_prepare_kernel<NOISE_REF, true>, muon_prepare_kernel<NOISE_FAST, true>,
                                  muon_prepare_kernel<NOISE_NONE, true>)
                     : pick_noise(muon_prepare_kernel<NOISE_REF, false>, muon_prepare_kernel<NOISE_FAST, false>,
                                  muon_prepare_kernel<NOISE_NONE, false>);
    kern<<<grid_for(chunks), EW_THREADS, 0, to_stream(stream)>>>(a);
    int st = check_launch("muon_prepare_kernel");
    if (st) return st;
  }
  return MSR_OK;
}

int apply_launch(const msr_apply_entry* entries, int count, float lr, float decay, const msr_apply_record* rec,
                 msr_stream_t stream) {
  if (count < 0 || (count > 0 && entries == nullptr)) return fail(MSR_ERR_INVALID, "msr_muon_apply: bad entry list");
  int next = 0;
  while (next < count) {
    ApplyArgs a{};
    a.lr = lr;
    a.decay = decay;
    a.rec = rec;
    int64_t chunks = 0;
    int i = next;
    for (; i < count && a.count < MAXE; ++i) {
      const msr_apply_entry& e = entries[i];
      if (e.numel < 0 || (e.numel > 0 && (!e.param || !e.update)))
        return fail(MSR_ERR_INVALID, "msr_muon_apply: entry %d has a null pointer or negative numel", i);
      if (e.numel == 0) continue;
      a.e[a.count] = e;
      a.src[a.count] = i;
      if (e.param_mc && (reinterpret_cast<uintptr_t>(e.param_mc) & 15u) != (reinterpret_cast<uintptr_t>(e.param) & 15u))
        return fail(MSR_ERR_INVALID, "msr_muon_apply: entry %d: param_mc must have param's 16-byte alignment", i);
      a.any_mc |= e.param_mc != nullptr;
      a.vec[a.count] = ptr_aligned16(e.param) && ptr_aligned16(e.update);
      a.prefix[a.count] = chunks;
      chunks += (e.numel + APPLY_CHUNK - 1) / APPLY_CHUNK;
      ++a.count;
    }
    next = i;
    a.prefix[a.count] = chunks;
    if (a.count == 0) continue;
    auto* kern = rec ? pick_noise(muon_apply_kernel<NOISE_REF, true>, muon_apply_kernel<NOISE_FAST, true>,
                                  muon_apply_kernel<NOISE_NONE, true>)
                     : pick_noise(muon_apply_kernel<NOISE_REF, false>, muon_apply_kernel<NOISE_FAST, false>,
                                  muon_apply_kernel<NOISE_NONE, false>);
    kern<<<grid_for(chunks), EW_THREADS, 0, to_stream(stream)>>>(a);
    int st = check_launch("muon_apply_kernel");
    if (st) return st;
  }
  return MSR_OK;
}

int adamw_launch(const msr_adamw_entry* entries, int count, const msr_adamw_hparams* hp, const msr_adamw_record* rec,
                 msr_stream_t stream) {
  if (count < 0 || (count > 0 && entries == nullptr))
    return fail(MSR_ERR_INVALID, "msr_adamw_sr: bad entry list or hparams");
  int next = 0;
  while (next < count) {
    AdamWArgs a{};
    if (hp) a.hp = *hp;
    a.rec = rec;
    int64_t chunks = 0;
    int i = next;
    for (; i < count && a.count < MAXE; ++i) {
      const msr_adamw_entry& e = entries[i];
      if (e.numel < 0 || (e.numel > 0 && (!e.param || !e.grad || !e.exp_avg || !e.exp_avg_sq)))
        return fail(MSR_ERR_INVALID, "msr_adamw_sr: entry %d has a null pointer or negative numel", i);
      if (e.numel == 0) continue;
      a.e[a.count] = e;
      a.src[a.count] = i;
      if (e.param_mc && (reinterpret_cast<uintptr_t>(e.param_mc) & 15u) != (reinterpret_cast<uintptr_t>(e.param) & 15u))
        return fail(MSR_ERR_INVALID, "msr_adamw_sr: entry %d: param_mc must have param's 16-byte alignment", i);
      a.any_mc |= e.param_mc != nullptr;
      a.vec[a.count] = ptr_aligned16(e.param) && ptr_aligned16(e.grad) && ptr_aligned16(e.exp_avg) &&
                       ptr_aligned16(e.exp_avg_sq);
      a.prefix[a.count] = chunks;
      chunks += (e.numel + ADAMW_CHUNK - 1) / ADAMW_CHUNK;
      ++a.count;
    }
    next = i;
    a.prefix[a.count] = chunks;
    if (a.count == 0) continue;
    auto* kern = rec ? pick_noise(adamw_kernel<ADAMW_ITERS, ADAMW_MINB, NOISE_REF, true>,
                                  adamw_kernel<ADAMW_ITERS, ADAMW_MINB, NOISE_FAST, true>,
                                  adamw_kernel<ADAMW_ITERS, ADAMW_MINB, NOISE_NONE, true>)
                     : pick_noise(adamw_kernel<ADAMW_ITERS, ADAMW_MINB, NOISE_REF, false>,
                                  adamw_kernel<ADAMW_ITERS, ADAMW_MINB, NOISE_FAST, false>,
                                  adamw_kernel<ADAMW_ITERS, ADAMW_MINB, NOISE_NONE, false>);
    // one wave of resident CTAs (ADAMW_MINB per SM), each walking its chunks
    const int64_t cap = static_cast<int64_t>(sm_count()) * ADAMW_MINB;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(chunks, cap)));
    kern<<<grid, EW_THREADS, 0, to_stream(stream)>>>(a);
    int st = check_launch("adamw_kernel");
    if (st) return st;
  }
  return MSR_OK;
}

}  // namespace
}  // namespace msr

using namespace msr;

extern "C" {

int msr_philox_fill(uint32_t* out, int64_t n, uint64_t ctr_base, uint64_t key, msr_stream_t stream) {
  if (n < 0 || (n > 0 && out == nullptr)) return fail(MSR_ERR_INVALID, "msr_philox_fill: bad arguments");
  if (n == 0) return MSR_OK;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  philox_fill_kernel<<<blocks, 256, 0, to_stream(stream)>>>(out, n, ctr_base, make_key(key));
  return check_launch("philox_fill_kernel");
}

int msr_centralize_bf16(const void* grad, void* out, int64_t rows, int64_t cols, float centralization,
                        msr_stream_t stream) {
  if (!grad || !out || rows <= 0 || cols <= 0)
    return fail(MSR_ERR_INVALID, "msr_centralize_bf16: null pointer or non-positive size");
  if (int st = require_sm100()) return st;
  const int vec = (cols % 8 == 0) && ptr_aligned16(grad) && ptr_aligned16(out);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(rows, 8 * (int64_t)sm_count())));
  centralize_kernel<<<grid, CT_THREADS, 0, to_stream(stream)>>>(static_cast<const uint16_t*>(grad),
                                                                static_cast<uint16_t*>(out), rows, cols,
                                                                centralization, vec);
  return check_launch("centralize_kernel");
}

int msr_grad_accum_bf16(void* acc, const void* grad, int64_t n, uint64_t key, int first, msr_stream_t stream) {
  if (n < 0 || (n > 0 && (acc == nullptr || grad == nullptr)))
    return fail(MSR_ERR_INVALID, "msr_grad_accum_bf16: null pointer or negative size");
  if (n == 0) return MSR_OK;
  const int64_t chunks = (n + EW_CHUNK - 1) / EW_CHUNK;
  const bool vec = ptr_aligned16(acc) && ptr_aligned16(grad);
  if (first) {
    const int grid = grid_for(chunks * 4);
    if (vec)
      grad_accum_first_kernel<true><<<grid, EW_THREADS, 0, to_stream(stream)>>>(
          static_cast<uint16_t*>(acc), static_cast<const uint16_t*>(grad), n);
    else
      grad_accum_first_kernel<false><<<grid, EW_THREADS, 0, to_stream(stream)>>>(
          static_cast<uint16_t*>(acc), static_cast<const uint16_t*>(grad), n);
    return check_launch("grad_accum_first_kernel");
  }
  auto* kern = vec ? pick_noise(grad_accum_kernel<true, NOISE_REF>, grad_accum_kernel<true, NOISE_FAST>,
                                grad_accum_kernel<true, NOISE_NONE>)
                  : pick_noise(grad_accum_kernel<false, NOISE_REF>, grad_accum_kernel<false, NOISE_FAST>,
                               grad_accum_kernel<false, NOISE_NONE>);
  kern<<<grid_for(chunks), EW_THREADS, 0, to_stream(stream)>>>(static_cast<uint16_t*>(acc),
                                                               static_cast<const uint16_t*>(grad), n, make_key(key));
  return check_launch("grad_accum_kernel");
}

int msr_muon_prepare(const msr_prepare_entry* entries, int count, float beta, float one_minus_beta, int nesterov,
                     msr_stream_t stream) {
  return msr::prepare_launch(entries, count, beta, one_minus_beta, nesterov, nullptr, stream);
}

int msr_muon_prepare_rec(const msr_prepare_entry* entries, int count, const void* record, msr_stream_t stream) {
  if (!msr::record_ok(record)) return fail(MSR_ERR_INVALID, "msr_muon_prepare_rec: record must be 16-byte aligned");
  return msr::prepare_launch(entries, count, 0.f, 0.f, 0, static_cast<const msr_prepare_record*>(record), stream);
}

int msr_muon_apply(const msr_apply_entry* entries, int count, float lr, float decay, msr_stream_t stream) {
  return msr::apply_launch(entries, count, lr, decay, nullptr, stream);
}

int msr_muon_apply_rec(const msr_apply_entry* entries, int count, const void* record, msr_stream_t stream) {
  if (!msr::record_ok(record)) return fail(MSR_ERR_INVALID, "msr_muon_apply_rec: record must be 16-byte aligned");
  return msr::apply_launch(entries, count, 0.f, 0.f, static_cast<const msr_apply_record*>(record), stream);
}

int msr_adamw_sr(const msr_adamw_entry* entries, int count, const msr_adamw_hparams* hp, msr_stream_t stream) {
  if (count > 0 && hp == nullptr) return fail(MSR_ERR_INVALID, "msr_adamw_sr: bad entry list or hparams");
  return msr::adamw_launch(entries, count, hp, nullptr, stream);
}

int msr_adamw_sr_rec(const msr_adamw_entry* entries, int count, const void* record, msr_stream_t stream) {
  if (!msr::record_ok(record)) return fail(MSR_ERR_INVALID, "msr_adamw_sr_rec: record must be 16-byte aligned");
  return msr::adamw_launch(entries, count, nullptr, static_cast<const msr_adamw_record*>(record), stream);
}

}  // extern "C"
