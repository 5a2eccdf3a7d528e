// 8-bit blockwise AdamW with BF16 stochastic rounding of the weights, one HBM pass.
//
// Follows muon_sr/triton_adamw_8bit.py:27-99 (its _quantize and _adamw_8bit_kernel):
// dequantise both moments with the dynamic codebooks and the per-block absmax, run the
// Adam update with the non-finite-gradient mask, write the SR'd weight, then take the
// block absmax of the new moments and requantise them with the reference's 7-step pivot
// walk (bitsandbytes quantize_2D rules). Tensors below the 8-bit threshold keep bf16
// moments with SR instead.
//
// Design (B200): each thread owns 8 consecutive elements (16-byte weight/gradient loads,
// 8-byte code loads); a quantisation block of BS elements is BS/8 consecutive threads, so
// the block absmax is a warp reduction (one redux.sync for a whole warp, shuffles for
// smaller blocks, plus shared memory when a block spans warps). Both codebooks live in shared memory. A persistent grid walks tiles of
// 256 threads x 8 (or x16 for BS = 4096) elements across all tensors of the launch.
#include "common.cuh"
#include "host_common.h"

#include <algorithm>

namespace msr {
namespace {

constexpr int Q_THREADS = 256;
constexpr int Q_MAXE = 64;
constexpr int Q_BLOCKS_PER_SM = 4;

struct Adam8Args {
  msr_adamw8bit_entry e[Q_MAXE];
  int64_t prefix[Q_MAXE + 1];
  uint8_t vec[Q_MAXE];
  int count;
  msr_adamw8bit_hparams hp;
  const float* qmap1;
  const float* qmap2;
  int any_mc;  // some entry stores its weights through a multicast address
};

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }

// _quantize -- muon_sr/triton_adamw_8bit.py:27-53
template <bool SIGNED>
__device__ __forceinline__ uint32_t quantize(float x, const float* __restrict__ Q) {
  int pivot = 127, lower_pivot = 0, upper_pivot = 255;
  float lower = SIGNED ? -1.f : 0.f, upper = 1.f;
  float val = Q[127];
#pragma unroll
  for (int s = 0; s < 7; ++s) {
    const int delta = 64 >> s;
    const bool right = x > val;
    lower_pivot = right ? pivot : lower_pivot;
    upper_pivot = right ? upper_pivot : pivot;
    lower = right ? val : lower;
    upper = right ? upper : val;
    pivot += right ? delta : -delta;
    val = Q[pivot];
  }
  int r;
  if (x > val)
    r = (x > fmul(fadd(upper, val), 0.5f)) ? upper_pivot : pivot;
  else
    r = (x < fmul(fadd(lower, val), 0.5f)) ? lower_pivot : pivot;
  if (SIGNED) {
    const float dec = Q[r];
    if ((dec < 0.f) != (x < 0.f)) r += (x > 0.f) ? 1 : -1;
  }
  return static_cast<uint32_t>(r) & 0xFFu;
}

// The same quantiser through the lookup tables (layout in muon_sr_b200.h): the code at
// the start of |x|'s bucket, moved by one if |x| has reached that code's threshold.
// codes/T point at one side of one codebook (x >= 0) and, for the signed map, the other.
template <bool SIGNED>
__device__ __forceinline__ uint32_t quantize_table(float x, const uint8_t* __restrict__ codes_pos,
                                                   const float* __restrict__ T_pos,
                                                   const uint8_t* __restrict__ codes_neg,
                                                   const float* __restrict__ T_neg) {
  const uint32_t ab = __float_as_uint(x) & 0x7FFFFFFFu;
  const int b = min(max(static_cast<int>(ab >> 15) - MSR_QT_BASE, 0), MSR_QT_NB - 1);
  const float ax = __uint_as_float(ab);
  if (SIGNED) {  // one lookup per table, its side picked by the index
    const bool neg = x < 0.f;
    const int c = codes_pos[b + (neg ? static_cast<int>(codes_neg - codes_pos) : 0)];
    const int hit = ax >= T_pos[c + (neg ? static_cast<int>(T_neg - T_pos) : 0)] ? 1 : 0;
    return static_cast<uint32_t>(neg ? c - hit : c + hit);
  }
  const int c = codes_pos[b];
  return static_cast<uint32_t>(c + (ax >= T_pos[c] ? 1 : 0));
}

// x / d correctly rounded from r = RN(1/d): q = RN(x r), then one residual correction
// (Markstein's theorem: exact FMA residual + RN(q + rem r) gives RN(x / d)).
__device__ __forceinline__ float div_by_recip(float x, float d, float r) {
  const float q = __fmul_rn(x, r);
  const float rem = __fmaf_rn(-q, d, x);
  return __fmaf_rn(rem, r, q);
}

__device__ __forceinline__ bool finite_f(float g) { return fabsf(g) < __int_as_float(0x7f800000); }

// Max-reduce over groups of G consecutive threads (G a power of two, <= Q_THREADS).
// v >= 0 and not NaN (a thread's fmaxf over |values| starting from 0), so the order of the
// bit patterns as unsigned integers is the order of the values.
template <int G>
__device__ __forceinline__ float group_max(float v, float* red) {
  if constexpr (G == 32) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
  } else if constexpr (G < 32) {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
  } else {
    v = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    constexpr int WPG = G / 32;  // warps per group
    const int g0 = (w / WPG) * WPG;
    float r = red[g0];
#pragma unroll
    for (int i = 1; i < WPG; ++i) r = fmaxf(r, red[g0 + i]);
    return r;
  }
}

// Dynamic shared memory: both codebooks, then (TABLES) the lookup tables.
constexpr size_t smem_for(bool tables) { return 2 * 256 * 4 + (tables ? MSR_QT_BYTES : 0); }

// EPT elements per thread, BS elements per quantisation block.
template <int BS, bool TABLES, int NOISE>
__global__ __launch_bounds__(Q_THREADS, 4) void adamw8bit_kernel(const __grid_constant__ Adam8Args a) {
  constexpr bool FAST = NOISE == NOISE_FAST;
  constexpr int EPT = BS > 2048 ? 16 : 8;
  constexpr int TILE = Q_THREADS * EPT;
  constexpr int G = BS / EPT;  // threads per quantisation block
  extern __shared__ __align__(16) uint8_t dsm[];
  float* q1 = reinterpret_cast<float*>(dsm);
  float* q2 = q1 + 256;
  uint8_t* qt = dsm + 2 * 256 * 4;
  __shared__ float red[Q_THREADS / 32];
  for (int i = threadIdx.x; i < 256; i += Q_THREADS) {
    q1[i] = a.qmap1 ? a.qmap1[i] : 0.f;
    q2[i] = a.qmap2 ? a.qmap2[i] : 0.f;
  }
  if (TABLES) {
    const uint4* src = static_cast<const uint4*>(a.hp.qtables);
    for (int i = threadIdx.x; i < MSR_QT_BYTES / 16; i += Q_THREADS) reinterpret_cast<uint4*>(qt)[i] = src[i];
  }
  const uint8_t* c_pos1 = qt;
  const uint8_t* c_neg1 = qt + MSR_QT_NB;
  const uint8_t* c_pos2 = qt + 2 * MSR_QT_NB;
  const float* t_pos1 = reinterpret_cast<const float*>(qt + MSR_QT_T_OFFSET);
  const float* t_neg1 = t_pos1 + 256;
  const float* t_pos2 = t_pos1 + 512;
  __syncthreads();
  const msr_adamw8bit_hparams hp = a.hp;
  const int64_t total = a.prefix[a.count];
  int ei = blockIdx.x < total ? find_entry<Q_MAXE>(a.prefix, a.count, blockIdx.x) : 0;
  for (int64_t tile = blockIdx.x; tile < total; tile += gridDim.x) {
    while (a.prefix[ei + 1] <= tile) ++ei;  // tiles only move forward; prefix[count] = total
    const msr_adamw8bit_entry& E = a.e[ei];
    const int64_t n = E.numel;
    const int64_t base = (tile - a.prefix[ei]) * TILE + static_cast<int64_t>(threadIdx.x) * EPT;
    uint16_t* P = static_cast<uint16_t*>(E.param);
    const uint16_t* Gp = static_cast<const uint16_t*>(E.grad);
    const bool vec = a.vec[ei] && base + EPT <= n;
    const int nvalid = vec ? EPT : (n - base >= EPT ? EPT : (n > base ? static_cast<int>(n - base) : 0));
    const SrNoise<NOISE> np_{make_key(E.key_p)};

    uint16_t pb[EPT], gb[EPT];
    if (vec) {
#pragma unroll
      for (int h = 0; h < EPT; h += 8) {
        U16x8 t = ld_u16x8(P + base + h);
        U16x8 u = ld_u16x8_stream(Gp + base + h);
#pragma unroll
        for (int j = 0; j < 8; ++j) { pb[h + j] = t.v[j]; gb[h + j] = u.v[j]; }
      }
    } else {
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        const bool ok = base + j < n;
        pb[j] = ok ? P[base + j] : 0;
        gb[j] = ok ? Gp[base + j] : 0;
      }
    }

    float m[EPT], v[EPT];
    if (E.quantized) {
      const uint8_t* S1 = static_cast<const uint8_t*>(E.state1);
      const uint8_t* S2 = static_cast<const uint8_t*>(E.state2);
      const int64_t blk = base / BS;
      const bool blk_ok = base < n;
      const float am1 = blk_ok ? E.absmax1[blk] : 0.f;
      const float am2 = blk_ok ? E.absmax2[blk] : 0.f;
      uint8_t c1[EPT], c2[EPT];
      if (vec) {
#pragma unroll
        for (int h = 0; h < EPT; h += 8) {
          uint2 t = *reinterpret_cast<const uint2*>(S1 + base + h);
          uint2 u = *reinterpret_cast<const uint2*>(S2 + base + h);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            c1[h + j] = (t.x >> (8 * j)) & 0xFF; c1[h + 4 + j] = (t.y >> (8 * j)) & 0xFF;
            c2[h + j] = (u.x >> (8 * j)) & 0xFF; c2[h + 4 + j] = (u.y >> (8 * j)) & 0xFF;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
          const bool ok = base + j < n;
          c1[j] = ok ? S1[base + j] : 127;
          c2[j] = ok ? S2[base + j] : 0;
        }
      }
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        m[j] = fmul(q1[c1[j]], am1);
        v[j] = fmul(q2[c2[j]], am2);
      }
    } else {
      const uint16_t* S1 = static_cast<const uint16_t*>(E.state1);
      const uint16_t* S2 = static_cast<const uint16_t*>(E.state2);
      if (vec) {
#pragma unroll
        for (int h = 0; h < EPT; h += 8) {
          U16x8 t = ld_u16x8(S1 + base + h), u = ld_u16x8(S2 + base + h);
#pragma unroll
          for (int j = 0; j < 8; ++j) { m[h + j] = bf16_bits_to_f32(t.v[j]); v[h + j] = bf16_bits_to_f32(u.v[j]); }
        }
      } else {
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
          const bool ok = base + j < n;
          m[j] = ok ? bf16_bits_to_f32(S1[base + j]) : 0.f;
          v[j] = ok ? bf16_bits_to_f32(S2[base + j]) : 0.f;
        }
      }
    }

    // Adam update (decay after the step, bitsandbytes order) -- :72-80
    uint32_t rp[EPT];
    if (FAST) {
#pragma unroll
      for (int h = 0; h < EPT; h += 8) np_.eight(static_cast<uint64_t>(base + h), rp + h);
    }
    float mmax = 0.f, vmax = 0.f;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const float g = bf16_bits_to_f32(gb[j]);
      const bool fin = finite_f(g);
      m[j] = fin ? fadd(fmul(hp.beta1, m[j]), fmul(hp.one_minus_beta1, g)) : 0.f;
      v[j] = fin ? fadd(fmul(hp.beta2, v[j]), fmul(fmul(hp.one_minus_beta2, g), g)) : 0.f;
      const float p = bf16_bits_to_f32(pb[j]);
      const float upd = fsub(p, __fdiv_rn(fmul(E.coef, m[j]), fadd(__fsqrt_rn(v[j]), E.sqrt_bc2_eps)));
      const float updated = fmul(upd, hp.decay);
      if (fin) pb[j] = round_bf16<NOISE>(updated, FAST ? rp[j] : np_.at(static_cast<uint64_t>(base + j)));
      if (j < nvalid) {
        mmax = fmaxf(mmax, fabsf(m[j]));
        vmax = fmaxf(vmax, fabsf(v[j]));
      }
    }

    uint16_t* PM = static_cast<uint16_t*>(E.param_mc);  // multicast weights (sharded steps)
    if (vec) {
#pragma unroll
      for (int h = 0; h < EPT; h += 8) {
        U16x8 t;
#pragma unroll
        for (int j = 0; j < 8; ++j) t.v[j] = pb[h + j];
        if (PM)
          mc_st_u16x8(PM + base + h, t);
        else
          st_u16x8(P + base + h, t);
      }
    } else if (PM) {  // 4-byte pairs from an even index; past the end: 0 into the slot's padding
#pragma unroll
      for (int j = 0; j < EPT; j += 2)
        if (base + j < n)
          mc_st_u32(PM + base + j, pb[j] | (static_cast<uint32_t>(base + j + 1 < n ? pb[j + 1] : 0) << 16));
    } else {
#pragma unroll
      for (int j = 0; j < EPT; ++j)
        if (base + j < n) P[base + j] = pb[j];
    }

    if (E.quantized) {
      mmax = group_max<G>(mmax, red);
      vmax = group_max<G>(vmax, red);
      const float dm = mmax > 0.f ? mmax : 1.f;
      const float dv = vmax > 0.f ? vmax : 1.f;
      uint8_t* S1 = static_cast<uint8_t*>(E.state1);
      uint8_t* S2 = static_cast<uint8_t*>(E.state2);
      uint32_t c1w[EPT / 4], c2w[EPT / 4];
#pragma unroll
      for (int j = 0; j < EPT / 4; ++j) { c1w[j] = 0u; c2w[j] = 0u; }
      const float rm = __frcp_rn(dm), rv = __frcp_rn(dv);
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        const float xm = div_by_recip(m[j], dm, rm);
        const float xv = div_by_recip(v[j], dv, rv);
        uint32_t cm, cv;
        if (TABLES) {
          cm = quantize_table<true>(xm, c_pos1, t_pos1, c_neg1, t_neg1);
          cv = quantize_table<false>(xv, c_pos2, t_pos2, nullptr, nullptr);
        } else {
          cm = quantize<true>(xm, q1);
          cv = quantize<false>(xv, q2);
        }
        c1w[j / 4] |= cm << (8 * (j % 4));
        c2w[j / 4] |= cv << (8 * (j % 4));
      }
      if (vec) {
#pragma unroll
        for (int h = 0; h < EPT / 8; ++h) {
          *reinterpret_cast<uint2*>(S1 + base + 8 * h) = make_uint2(c1w[2 * h], c1w[2 * h + 1]);
          *reinterpret_cast<uint2*>(S2 + base + 8 * h) = make_uint2(c2w[2 * h], c2w[2 * h + 1]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < EPT; ++j)
          if (base + j < n) {
            S1[base + j] = (c1w[j / 4] >> (8 * (j % 4))) & 0xFF;
            S2[base + j] = (c2w[j / 4] >> (8 * (j % 4))) & 0xFF;
          }
      }
      if ((threadIdx.x % G) == 0 && base < n) {
        E.absmax1[base / BS] = mmax;
        E.absmax2[base / BS] = vmax;
      }
    } else {
      const SrNoise<NOISE> nm{make_key(E.key_m)}, nv{make_key(E.key_v)};
      uint16_t* S1 = static_cast<uint16_t*>(E.state1);
      uint16_t* S2 = static_cast<uint16_t*>(E.state2);
      uint16_t mb[EPT], vb[EPT];
      uint32_t rm[EPT], rv[EPT];
      if (FAST) {
#pragma unroll
        for (int h = 0; h < EPT; h += 8) {
          nm.eight(static_cast<uint64_t>(base + h), rm + h);
          nv.eight(static_cast<uint64_t>(base + h), rv + h);
        }
      }
#pragma unroll
      for (int j = 0; j < EPT; ++j) {
        const uint64_t ctr = static_cast<uint64_t>(base + j);
        mb[j] = round_bf16<NOISE>(m[j], FAST ? rm[j] : nm.at(ctr));
        vb[j] = round_bf16<NOISE>(v[j], FAST ? rv[j] : nv.at(ctr));
      }
      if (vec) {
#pragma unroll
        for (int h = 0; h < EPT; h += 8) {
          U16x8 t, u;
#pragma unroll
          for (int j = 0; j < 8; ++j) { t.v[j] = mb[h + j]; u.v[j] = vb[h + j]; }
          st_u16x8(S1 + base + h, t);
          st_u16x8(S2 + base + h, u);
        }
      } else {
#pragma unroll
        for (int j = 0; j < EPT; ++j)
          if (base + j < n) { S1[base + j] = mb[j]; S2[base + j] = vb[j]; }
      }
    }
  }
  // multicast stores are ordered before anything after the kernel (the callers' barrier)
  if (a.any_mc) __threadfence_system();
}

template <int BS, bool TABLES, int NOISE>
int launch_variant(const Adam8Args& a, int64_t tiles, cudaStream_t s) {
  const int64_t cap = static_cast<int64_t>(sm_count()) * Q_BLOCKS_PER_SM;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, cap)));
  constexpr size_t smem = smem_for(TABLES);
  if (smem > 48 * 1024) {
    if (int st = set_smem_attr(reinterpret_cast<const void*>(adamw8bit_kernel<BS, TABLES, NOISE>), smem,
                               "adamw8bit_kernel"))
      return st;
  }
  adamw8bit_kernel<BS, TABLES, NOISE><<<grid, Q_THREADS, smem, s>>>(a);
  return check_launch("adamw8bit_kernel");
}

template <int BS, int NOISE>
int launch_noise(const Adam8Args& a, int64_t tiles, cudaStream_t s) {
  return a.hp.qtables ? launch_variant<BS, true, NOISE>(a, tiles, s) : launch_variant<BS, false, NOISE>(a, tiles, s);
}

template <int BS>
int launch_bs(const Adam8Args& a, int64_t tiles, cudaStream_t s) {
  return pick_noise(launch_noise<BS, NOISE_REF>, launch_noise<BS, NOISE_FAST>, launch_noise<BS, NOISE_NONE>)(a, tiles, s);
}

inline bool al(const void* p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace msr

using namespace msr;

extern "C" int msr_adamw8bit(const msr_adamw8bit_entry* entries, int count, const float* qmap1, const float* qmap2,
                             const msr_adamw8bit_hparams* hp, msr_stream_t stream) {
  if (count < 0 || (count > 0 && (entries == nullptr || hp == nullptr)))
    return fail(MSR_ERR_INVALID, "msr_adamw8bit: bad entry list or hparams");
  const int bs = hp->block_size;
  if (bs < 32 || bs > 4096 || (bs & (bs - 1)))
    return fail(MSR_ERR_INVALID, "msr_adamw8bit: block_size %d is not a power of two in [32, 4096]", bs);
  const int ept = bs > 2048 ? 16 : 8;
  const int64_t tile = static_cast<int64_t>(Q_THREADS) * ept;
  int next = 0;  // each group resumes at the first entry the previous one did not take
  while (next < count) {
    Adam8Args a{};
    a.hp = *hp;
    a.qmap1 = qmap1;
    a.qmap2 = qmap2;
    int64_t tiles = 0;
    bool any_quant = false;
    int i = next;
    for (; i < count && a.count < Q_MAXE; ++i) {
      const msr_adamw8bit_entry& e = entries[i];
      if (e.numel < 0 || (e.numel > 0 && (!e.param || !e.grad || !e.state1 || !e.state2)))
        return fail(MSR_ERR_INVALID, "msr_adamw8bit: entry %d has a null pointer or negative numel", i);
      if (e.numel > 0 && e.quantized && (!e.absmax1 || !e.absmax2))
        return fail(MSR_ERR_INVALID, "msr_adamw8bit: entry %d is quantized but has no absmax buffers", i);
      if (e.numel == 0) continue;
      any_quant |= e.quantized != 0;
      a.e[a.count] = e;
      if (e.param_mc && (reinterpret_cast<uintptr_t>(e.param_mc) & 15u) != (reinterpret_cast<uintptr_t>(e.param) & 15u))
        return fail(MSR_ERR_INVALID, "msr_adamw8bit: entry %d: param_mc must have param's 16-byte alignment", i);
      a.any_mc |= e.param_mc != nullptr;
      const unsigned sa = e.quantized ? 8u : 16u;
      a.vec[a.count] = al(e.param, 16) && al(e.grad, 16) && al(e.state1, sa) && al(e.state2, sa);
      a.prefix[a.count] = tiles;
      tiles += (e.numel + tile - 1) / tile;
      ++a.count;
    }
    next = i;
    a.prefix[a.count] = tiles;
    if (a.count == 0) continue;
    if (any_quant && (qmap1 == nullptr || qmap2 == nullptr))
      return fail(MSR_ERR_INVALID, "msr_adamw8bit: quantized entries need both codebooks");
    if (hp->qtables != nullptr && (reinterpret_cast<uintptr_t>(hp->qtables) & 15))
      return fail(MSR_ERR_INVALID, "msr_adamw8bit: qtables must be 16-byte aligned");
    cudaStream_t s = to_stream(stream);
    int st;
    switch (bs) {
      case 32: st = launch_bs<32>(a, tiles, s); break;
      case 64: st = launch_bs<64>(a, tiles, s); break;
      case 128: st = launch_bs<128>(a, tiles, s); break;
      case 256: st = launch_bs<256>(a, tiles, s); break;
      case 512: st = launch_bs<512>(a, tiles, s); break;
      case 1024: st = launch_bs<1024>(a, tiles, s); break;
      case 2048: st = launch_bs<2048>(a, tiles, s); break;
      default: st = launch_bs<4096>(a, tiles, s); break;
    }
    if (st) return st;
  }
  return MSR_OK;
}
