// Fused elementwise kernels of the optimizer step: SR gradient accumulation, Muon
// prepare (momentum + Nesterov), Muon apply (decay + scaled update) and AdamW-SR.
//
// Design (B200): multi-tensor launches. Each launch carries up to MAXE tensors in its
// kernel parameters; the work is cut into tiles of 2048 elements that never cross a tensor,
// and a persistent grid (a multiple of the SM count) walks the tiles. Inside each CTA a
// producer warp streams the tiles' inputs into a shared-memory ring with bulk asynchronous
// copies while eight consumer warps compute (stream.cuh): the kernels are bound by the
// FMA-heavy pipe that runs the reference's Philox multiplies, and the ring keeps HBM busy
// underneath that work. Each consumer thread handles 8 bf16 per tile with 16-byte shared
// loads and 16-byte global stores. All fp32 arithmetic uses explicit round-to-nearest
// intrinsics (no contraction into FMA), in the reference's op order, so results are
// bit-identical to the reference kernels' fp32 evaluation. Every kernel is instantiated per
// noise mode (msr_set_sr_noise), and prepare / apply / AdamW once more (REC) for the
// replayable launches that read their scalars and entries from a device record (msr_*_rec,
// used inside captured CUDA graphs).
#include "common.cuh"
#include "host_common.h"
#include "stream.cuh"

#include <algorithm>

namespace msr {
namespace {

constexpr int EW_THREADS = 256;
constexpr int EW_VEC = 8;
constexpr int EW_ITERS = 2;
constexpr int64_t EW_CHUNK = EW_THREADS * EW_VEC * EW_ITERS;  // 8192 elements (first-micro-batch copy)
constexpr int MAXE = 64;
constexpr int EW_BLOCKS_PER_SM = 4;
constexpr int64_t TILE = stream::TILE;
// Streamed kernels: ring stages and CTAs per SM. Prepare, apply and SR accumulation stream
// two bf16 arrays (8 KB per stage); AdamW streams four (16 KB per stage) and keeps three
// Philox chains per element, so it runs two CTAs per SM with more registers each.
constexpr int EW_STAGES = 4, EW_MINB = 3;
constexpr int ADAMW_STAGES = 4, ADAMW_MINB = 2;

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

// 8 bf16 from shared memory (16 bytes).
__device__ __forceinline__ U16x8 lds_u16x8(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(tc::smem_addr(p)));
  U16x8 o;
  *reinterpret_cast<uint4*>(o.v) = r;
  return o;
}

// Dynamic shared memory of a streamed kernel (the ring of stream::Smem).
template <int NIN, int S>
__device__ __forceinline__ stream::Smem<NIN, S>& ring() {
  extern __shared__ __align__(128) uint8_t dsm[];
  return *reinterpret_cast<stream::Smem<NIN, S>*>(dsm);
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

// One tensor per launch (the accumulator hook runs per parameter).
struct AccumArgs {
  uint16_t* acc;
  const uint16_t* g;
  int64_t n;
  int64_t prefix[2];
  PhiloxKey key;
  int vec;
};

template <int NOISE>
struct AccumPolicy {
  static constexpr int NIN = 2;  // acc, g
  const AccumArgs& a;
  __device__ int count() const { return 1; }
  __device__ const int64_t* prefix() const { return a.prefix; }
  __device__ bool vec(int) const { return a.vec != 0; }
  __device__ int64_t numel(int) const { return a.n; }
  __device__ const void* input(int, int i) const { return i == 0 ? static_cast<const void*>(a.acc) : a.g; }
  __device__ void vector8(int, int64_t idx, const uint16_t* const (&in)[2]) const {
    constexpr bool FAST = NOISE == NOISE_FAST;
    const SrNoise<NOISE> nz{a.key};
    const U16x8 va = lds_u16x8(in[0]), vg = lds_u16x8(in[1]);
    uint32_t r[EW_VEC];
    if (FAST) nz.eight(static_cast<uint64_t>(idx), r);
    U16x8 o;
#pragma unroll
    for (int j = 0; j < EW_VEC; ++j)
      o.v[j] = accum_one<NOISE>(va.v[j], vg.v[j], FAST ? r[j] : nz.at(static_cast<uint64_t>(idx + j)));
    st_u16x8(a.acc + idx, o);
  }
  __device__ void scalar_range(int, int64_t lo, int64_t hi) const {
    const SrNoise<NOISE> nz{a.key};
    for (int64_t i = lo; i < hi; ++i) a.acc[i] = accum_one<NOISE>(a.acc[i], a.g[i], nz.at(static_cast<uint64_t>(i)));
  }
  __device__ bool multicast() const { return false; }
};

template <int NOISE>
__global__ __launch_bounds__(stream::THREADS, EW_MINB) void grad_accum_kernel(const __grid_constant__ AccumArgs a,
                                                                           int* err) {
  stream::run(AccumPolicy<NOISE>{a}, ring<2, EW_STAGES>(), err);
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
struct PreparePolicy {
  static constexpr int NIN = 2;  // grad, momentum
  const PrepareArgs& a;
  __device__ int count() const { return a.count; }
  __device__ const int64_t* prefix() const { return a.prefix; }
  __device__ bool vec(int e) const { return a.vec[e] != 0; }
  __device__ int64_t numel(int e) const { return entry_of<REC>(a, e).numel; }
  __device__ const void* input(int e, int i) const {
    const msr_prepare_entry& E = entry_of<REC>(a, e);
    return i == 0 ? E.grad : static_cast<const void*>(E.momentum);
  }
  __device__ void vector8(int e, int64_t idx, const uint16_t* const (&in)[2]) const {
    constexpr bool FAST = NOISE == NOISE_FAST;
    const msr_prepare_entry& E = entry_of<REC>(a, e);
    const SrNoise<NOISE> nz{make_key(E.key)};
    const uint64_t c0 = E.ctr_base + static_cast<uint64_t>(idx);
    const bool nesterov = (REC ? a.rec->nesterov : a.nesterov) != 0;
    const float beta = beta_of<REC>(a), omb = omb_of<REC>(a);
    const U16x8 vg = lds_u16x8(in[0]), vb = lds_u16x8(in[1]);
    uint32_t r[EW_VEC];
    if (FAST) nz.eight(c0, r);
    U16x8 ob, ou;
#pragma unroll
    for (int j = 0; j < EW_VEC; ++j)
      prepare_one<NOISE>(vg.v[j], vb.v[j], beta, omb, nesterov, [&] { return FAST ? r[j] : nz.at(c0 + j); }, ob.v[j],
                         ou.v[j]);
    st_u16x8(static_cast<uint16_t*>(E.momentum) + idx, ob);
    st_u16x8(static_cast<uint16_t*>(E.update) + idx, ou);
  }
  __device__ void scalar_range(int e, int64_t lo, int64_t hi) const {
    const msr_prepare_entry& E = entry_of<REC>(a, e);
    const SrNoise<NOISE> nz{make_key(E.key)};
    const uint16_t* g = static_cast<const uint16_t*>(E.grad);
    uint16_t* mb = static_cast<uint16_t*>(E.momentum);
    uint16_t* up = static_cast<uint16_t*>(E.update);
    const bool nesterov = (REC ? a.rec->nesterov : a.nesterov) != 0;
    for (int64_t i = lo; i < hi; ++i) {
      uint16_t ob, ou;
      prepare_one<NOISE>(g[i], mb[i], beta_of<REC>(a), omb_of<REC>(a), nesterov,
                         [&] { return nz.at(E.ctr_base + static_cast<uint64_t>(i)); }, ob, ou);
      mb[i] = ob;
      up[i] = ou;
    }
  }
  __device__ bool multicast() const { return false; }
};

template <int NOISE, bool REC>
__global__ __launch_bounds__(stream::THREADS, EW_MINB) void muon_prepare_kernel(
    const __grid_constant__ PrepareArgs a, int* err) {
  stream::run(PreparePolicy<NOISE, REC>{a}, ring<2, EW_STAGES>(), err);
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
  int any_mc;  // some entry stores through a multicast address
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

template <int NOISE, bool REC>
struct ApplyPolicy {
  static constexpr int NIN = 2;  // param, update
  const ApplyArgs& a;
  __device__ int count() const { return a.count; }
  __device__ const int64_t* prefix() const { return a.prefix; }
  __device__ bool vec(int e) const { return a.vec[e] != 0; }
  __device__ int64_t numel(int e) const { return entry_of<REC>(a, e).numel; }
  __device__ const void* input(int e, int i) const {
    const msr_apply_entry& E = entry_of<REC>(a, e);
    return i == 0 ? static_cast<const void*>(E.param) : E.update;
  }
  __device__ void vector8(int e, int64_t idx, const uint16_t* const (&in)[2]) const {
    constexpr bool FAST = NOISE == NOISE_FAST;
    const msr_apply_entry& E = entry_of<REC>(a, e);
    const SrNoise<NOISE> nz{make_key(E.key)};
    const float scale = E.scale, lr = lr_of<REC>(a), decay = decay_of<REC>(a);
    const U16x8 vp = lds_u16x8(in[0]), vu = lds_u16x8(in[1]);
    uint32_t r[EW_VEC];
    if (FAST) nz.eight(static_cast<uint64_t>(idx), r);
    U16x8 o;
#pragma unroll
    for (int j = 0; j < EW_VEC; ++j)
      o.v[j] = apply_one<NOISE>(vp.v[j], vu.v[j], scale, lr, decay,
                                FAST ? r[j] : nz.at(static_cast<uint64_t>(idx + j)));
    if (E.param_mc)
      mc_st_u16x8(static_cast<uint16_t*>(E.param_mc) + idx, o);
    else
      st_u16x8(static_cast<uint16_t*>(E.param) + idx, o);
  }
  __device__ void scalar_range(int e, int64_t lo, int64_t hi) const {
    const msr_apply_entry& E = entry_of<REC>(a, e);
    const SrNoise<NOISE> nz{make_key(E.key)};
    uint16_t* p = static_cast<uint16_t*>(E.param);
    const uint16_t* u = static_cast<const uint16_t*>(E.update);
    auto one = [&](int64_t i) {
      return apply_one<NOISE>(p[i], u[i], E.scale, lr_of<REC>(a), decay_of<REC>(a), nz.at(static_cast<uint64_t>(i)));
    };
    if (!E.param_mc) {
      for (int64_t i = lo; i < hi; ++i) p[i] = one(i);
      return;
    }
    // multicast: 4-byte pairs from an even index (lo is a multiple of 8); a pair past the
    // last element writes 0 into the slot's padding
    uint16_t* mc = static_cast<uint16_t*>(E.param_mc);
    for (int64_t i = lo; i < hi; i += 2) {
      const uint32_t v0 = one(i), v1 = i + 1 < hi ? one(i + 1) : 0u;
      mc_st_u32(mc + i, v0 | (v1 << 16));
    }
  }
  __device__ bool multicast() const { return a.any_mc != 0; }
};

template <int NOISE, bool REC>
__global__ __launch_bounds__(stream::THREADS, EW_MINB) void muon_apply_kernel(const __grid_constant__ ApplyArgs a,
                                                                           int* err) {
  stream::run(ApplyPolicy<NOISE, REC>{a}, ring<2, EW_STAGES>(), err);
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
  int any_mc;  // some entry stores through a multicast address
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

template <int NOISE, bool REC>
struct AdamWPolicy {
  static constexpr int NIN = 4;  // param, grad, exp_avg, exp_avg_sq
  const AdamWArgs& a;
  __device__ int count() const { return a.count; }
  __device__ const int64_t* prefix() const { return a.prefix; }
  __device__ bool vec(int e) const { return a.vec[e] != 0; }
  __device__ int64_t numel(int e) const { return entry_of<REC>(a, e).numel; }
  __device__ const void* input(int e, int i) const {
    const msr_adamw_entry& E = entry_of<REC>(a, e);
    return i == 0 ? static_cast<const void*>(E.param) : i == 1 ? E.grad : i == 2 ? E.exp_avg : E.exp_avg_sq;
  }
  __device__ void vector8(int e, int64_t idx, const uint16_t* const (&in)[4]) const {
    constexpr bool FAST = NOISE == NOISE_FAST;
    const msr_adamw_entry& E = entry_of<REC>(a, e);
    SrNoise<NOISE> nm{make_key(E.key_m)}, nv{make_key(E.key_v)}, np_{make_key(E.key_p)};
    const float ss = E.step_size, bc2s = E.bc2_sqrt;
    const msr_adamw_hparams& hp = hp_of<REC>(a);
    U16x8 vp = lds_u16x8(in[0]), vm = lds_u16x8(in[2]), vv = lds_u16x8(in[3]);
    const U16x8 vg = lds_u16x8(in[1]);
    if constexpr (FAST) {
      uint32_t rm[EW_VEC], rv[EW_VEC], rp[EW_VEC];
      nm.eight(static_cast<uint64_t>(idx), rm);
      nv.eight(static_cast<uint64_t>(idx), rv);
      np_.eight(static_cast<uint64_t>(idx), rp);
#pragma unroll
      for (int j = 0; j < EW_VEC; ++j)
        adamw_one<NOISE>(vp.v[j], vg.v[j], vm.v[j], vv.v[j], hp, ss, bc2s,
                         [&](int w) { return w == 0 ? rm[j] : w == 1 ? rv[j] : rp[j]; });
    } else {
      // One Philox word per stream and element (m, v, p: three independent chains). The
      // elements run one after another: an empty asm takes each element's outputs and
      // "rewrites" the counter base the next element's chains start from, so the compiler
      // cannot interleave all 24 chains of the vector (which spills); three chains per
      // thread and two CTAs per SM still keep the FMA-heavy pipe fed.
      uint32_t cb = static_cast<uint32_t>(idx);
#pragma unroll
      for (int j = 0; j < EW_VEC; ++j) {
        const uint32_t c = cb + static_cast<uint32_t>(j);
        adamw_one<NOISE>(vp.v[j], vg.v[j], vm.v[j], vv.v[j], hp, ss, bc2s,
                         [&](int w) { return w == 0 ? nm.at(c) : w == 1 ? nv.at(c) : np_.at(c); });
        const uint32_t om = vm.v[j], ov = vv.v[j], op = vp.v[j];
        asm volatile("" : "+r"(cb), "+r"(nm.key.k0), "+r"(nm.key.k1), "+r"(nv.key.k0), "+r"(nv.key.k1),
                     "+r"(np_.key.k0), "+r"(np_.key.k1) : "r"(om), "r"(ov), "r"(op));
      }
    }
    if (E.param_mc)
      mc_st_u16x8(static_cast<uint16_t*>(E.param_mc) + idx, vp);
    else
      st_u16x8(static_cast<uint16_t*>(E.param) + idx, vp);
    st_u16x8(static_cast<uint16_t*>(E.exp_avg) + idx, vm);
    st_u16x8(static_cast<uint16_t*>(E.exp_avg_sq) + idx, vv);
  }
  __device__ void scalar_range(int e, int64_t lo, int64_t hi) const {
    const msr_adamw_entry& E = entry_of<REC>(a, e);
    const SrNoise<NOISE> nm{make_key(E.key_m)}, nv{make_key(E.key_v)}, np_{make_key(E.key_p)};
    uint16_t* p = static_cast<uint16_t*>(E.param);
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
    if (!E.param_mc) {
      for (int64_t i = lo; i < hi; ++i) p[i] = one(i);
      return;
    }
    uint16_t* mc = static_cast<uint16_t*>(E.param_mc);  // pairs, as in ApplyPolicy
    for (int64_t i = lo; i < hi; i += 2) {
      const uint32_t v0 = one(i), v1 = i + 1 < hi ? one(i + 1) : 0u;
      mc_st_u32(mc + i, v0 | (v1 << 16));
    }
  }
  __device__ bool multicast() const { return a.any_mc != 0; }
};

template <int NOISE, bool REC>
__global__ __launch_bounds__(stream::THREADS, ADAMW_MINB) void adamw_kernel(const __grid_constant__ AdamWArgs a,
                                                                         int* err) {
  stream::run(AdamWPolicy<NOISE, REC>{a}, ring<4, ADAMW_STAGES>(), err);
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

// Launch of one streamed kernel instance: persistent grid of MINB CTAs per SM (at most one
// CTA per tile), the ring in dynamic shared memory (the size attribute is set once per
// device for each kernel function, see set_smem_attr).
template <int NIN, int S, int MINB, class Args>
int launch_streamed(void (*kern)(Args, int*), const Args& a, int64_t tiles, cudaStream_t st, const char* name) {
  constexpr size_t smem = stream::smem_bytes<NIN, S>();
  if (int status = set_smem_attr(reinterpret_cast<const void*>(kern), smem, name)) return status;
  const int64_t cap = static_cast<int64_t>(sm_count()) * MINB;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, cap)));
  kern<<<grid, stream::THREADS, smem, st>>>(a, device_error_word());
  return check_launch(name);
}

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
    int64_t tiles = 0;
    int i = next;
    for (; i < count && a.count < MAXE; ++i) {
      const msr_prepare_entry& e = entries[i];
      if (e.numel < 0 || (e.numel > 0 && (!e.grad || !e.momentum || !e.update)))
        return fail(MSR_ERR_INVALID, "msr_muon_prepare: entry %d has a null pointer or negative numel", i);
      if (e.numel == 0) continue;
      a.e[a.count] = e;
      a.src[a.count] = i;
      a.vec[a.count] = ptr_aligned16(e.grad) && ptr_aligned16(e.momentum) && ptr_aligned16(e.update);
      a.prefix[a.count] = tiles;
      tiles += (e.numel + TILE - 1) / TILE;
      ++a.count;
    }
    next = i;
    a.prefix[a.count] = tiles;
    if (a.count == 0) continue;
    auto* kern = rec ? pick_noise(muon_prepare_kernel<NOISE_REF, true>, muon_prepare_kernel<NOISE_FAST, true>,
                                  muon_prepare_kernel<NOISE_NONE, true>)
                     : pick_noise(muon_prepare_kernel<NOISE_REF, false>, muon_prepare_kernel<NOISE_FAST, false>,
                                  muon_prepare_kernel<NOISE_NONE, false>);
    int st = launch_streamed<2, EW_STAGES, EW_MINB>(kern, a, tiles, to_stream(stream), "muon_prepare_kernel");
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
    int64_t tiles = 0;
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
      a.prefix[a.count] = tiles;
      tiles += (e.numel + TILE - 1) / TILE;
      ++a.count;
    }
    next = i;
    a.prefix[a.count] = tiles;
    if (a.count == 0) continue;
    auto* kern = rec ? pick_noise(muon_apply_kernel<NOISE_REF, true>, muon_apply_kernel<NOISE_FAST, true>,
                                  muon_apply_kernel<NOISE_NONE, true>)
                     : pick_noise(muon_apply_kernel<NOISE_REF, false>, muon_apply_kernel<NOISE_FAST, false>,
                                  muon_apply_kernel<NOISE_NONE, false>);
    int st = launch_streamed<2, EW_STAGES, EW_MINB>(kern, a, tiles, to_stream(stream), "muon_apply_kernel");
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
    int64_t tiles = 0;
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
      a.prefix[a.count] = tiles;
      tiles += (e.numel + TILE - 1) / TILE;
      ++a.count;
    }
    next = i;
    a.prefix[a.count] = tiles;
    if (a.count == 0) continue;
    auto* kern = rec ? pick_noise(adamw_kernel<NOISE_REF, true>, adamw_kernel<NOISE_FAST, true>,
                                  adamw_kernel<NOISE_NONE, true>)
                     : pick_noise(adamw_kernel<NOISE_REF, false>, adamw_kernel<NOISE_FAST, false>,
                                  adamw_kernel<NOISE_NONE, false>);
    int st = launch_streamed<4, ADAMW_STAGES, ADAMW_MINB>(kern, a, tiles, to_stream(stream), "adamw_kernel");
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
  const bool vec = ptr_aligned16(acc) && ptr_aligned16(grad);
  if (first) {
    const int grid = grid_for(((n + EW_CHUNK - 1) / EW_CHUNK) * 4);
    if (vec)
      grad_accum_first_kernel<true><<<grid, EW_THREADS, 0, to_stream(stream)>>>(
          static_cast<uint16_t*>(acc), static_cast<const uint16_t*>(grad), n);
    else
      grad_accum_first_kernel<false><<<grid, EW_THREADS, 0, to_stream(stream)>>>(
          static_cast<uint16_t*>(acc), static_cast<const uint16_t*>(grad), n);
    return check_launch("grad_accum_first_kernel");
  }
  AccumArgs a{};
  a.acc = static_cast<uint16_t*>(acc);
  a.g = static_cast<const uint16_t*>(grad);
  a.n = n;
  a.prefix[0] = 0;
  a.prefix[1] = (n + TILE - 1) / TILE;
  a.key = make_key(key);
  a.vec = vec ? 1 : 0;
  auto* kern = pick_noise(grad_accum_kernel<NOISE_REF>, grad_accum_kernel<NOISE_FAST>, grad_accum_kernel<NOISE_NONE>);
  return launch_streamed<2, EW_STAGES, EW_MINB>(kern, a, a.prefix[1], to_stream(stream), "grad_accum_kernel");
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
