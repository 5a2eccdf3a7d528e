// Newton-Schulz on the B200 tensor cores: a persistent, warp-specialised tcgen05 GEMM with
// TMA-fed shared-memory stages, fp32 accumulators in TMEM and the Newton-Schulz epilogue
// (alpha * acc + beta * C, per-matrix scale) fused into the TMEM read-back.
//
// Replaces _newton_schulz (muon_sr/muon_sr.py:82-98), which the reference runs as torch
// bf16 matmuls (cuBLAS on the GPU) with a separate elementwise op for every term.
//
// Kernel layout (one CTA per SM, 384 threads):
//   warp 0       TMA producer: streams A and B k-blocks (64 deep) into a 4-stage ring
//   warp 1       TMEM allocator and MMA issuer (one thread issues tcgen05.mma 128x256x16)
//   warps 4..11  epilogue: tcgen05.ld of the accumulator (lane quarter = warp % 4, column
//                half = (warp - 4) / 4), alpha/beta/scale, bf16 rounding, 16-byte stores
// Two 256-column fp32 accumulators (all 512 TMEM columns) let the epilogue of one tile run
// under the main loop of the next. Operands are either K-major or MN-major (descriptor bit),
// which covers X X^T, A A and B X for both orientations of X without any transposes.
// The default variant (gemm_pair_kernel) runs the same roles on clusters of two SMs with
// tcgen05.mma.cta_group::2 and 256 x 256 tiles, each SM loading half of the B tile; both
// variants produce identical bits.
// Every barrier wait has a time limit; on expiry the CTA records an error, drains what it
// has in flight, frees TMEM and returns.
#include "common.cuh"
#include "host_common.h"
#include "tc.cuh"

#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <mutex>

namespace msr {

__device__ int g_msr_device_error = 0;

namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, UMMA_K = 16;
constexpr int NUM_THREADS = 384;  // warps 0-1 TMA/MMA, 4-11 epilogue
constexpr int EPI_THREADS = 256;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t TMEM_COLS = 512;
// Epilogue chunking and staging (see the epilogue helpers below).
constexpr int EPI_CW = 32;                    // columns per epilogue chunk
constexpr int EPI_G = EPI_CW / 8;             // 16-byte groups per chunk row
constexpr int EPI_ROW_BYTES = EPI_CW * 2;     // 64
constexpr int EPI_STAGE_BYTES = 32 * EPI_ROW_BYTES;  // one warp's buffer: 2 KB
constexpr int EPI_WARPS = EPI_THREADS / 32;
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // 1 s: far above any legitimate wait

// Error codes recorded in g_msr_device_error (role of the wait that expired).
constexpr int ERR_TMA_WAIT = 0x101, ERR_MMA_WAIT = 0x102, ERR_EPI_WAIT = 0x103;

struct SharedStorage {
  alignas(1024) uint8_t stage[STAGES][STAGE_BYTES];
  alignas(16) uint8_t epi[EPI_WARPS][EPI_STAGE_BYTES];  // epilogue staging, one buffer per warp
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct Params {
  int64_t M, N, K, batch;
  int64_t tiles_m, tiles_n, num_tiles;
  int64_t tiles_per_batch;  // tiles_m * tiles_n, or the upper-triangle count when sym
  int sym;                  // output is symmetric (M == N): compute tiles touching the upper
                            // triangle only and mirror-write their strictly-upper part
  uint16_t* d;
  const uint16_t* c;
  int64_t ldd, ldc, d_bstride, c_bstride;
  float alpha, beta;
  const float* scale;      // per matrix; interpreted as ||x||_F^2 when scale_is_norm_sq
  int alpha_pow, beta_pow, scale_is_norm_sq;
  int ref_round;           // 1: bf16(bf16(beta*C) + bf16(alpha*bf16(acc))), the torch-op rounding
};

__device__ __forceinline__ float bf16r(float x) { return bf16_bits_to_f32(rne_bf16_bits(x)); }

// Tile rasterisation: row-blocks are taken in bands of GROUP_M; inside a band the tiles run
// column by column, rows fastest, so the tiles of one wave touch about GROUP_M A-panels and
// (wave / GROUP_M) B-panels and both stay in L2. Tiles are TILE_M x BN: 128 x 256 for one
// CTA, 256 x 256 for a CTA pair; RHO = BN / TILE_M row-blocks span one column-block.
constexpr int64_t GROUP_M = 8;

// Symmetric mode keeps, in row-block i, the column-blocks k >= i / RHO (every tile holding
// an element on or above the diagonal). In a band starting at row-block g0 (a multiple of
// RHO), column k = g0 / RHO + d holds the band's first min(R, RHO (d + 1)) row-blocks.
template <int RHO>
__host__ __device__ __forceinline__ int64_t sym_band_tiles(int64_t R, int64_t D) {
  // sum_{d < D} min(R, RHO (d + 1)): a ramp of dr columns, then full columns of R
  const int64_t ramp = R / RHO;
  const int64_t dr = D < ramp ? D : ramp;
  int64_t s = RHO * dr * (dr + 1) / 2;
  if (D > dr) s += (D - dr) * R;
  return s;
}

__host__ __device__ __forceinline__ int64_t imin(int64_t a, int64_t b) { return a < b ? a : b; }

// Linear tile index -> (matrix, first row, first column). Host-callable, so that the tile
// map can be checked without a GPU (msr_gemm_tile_map).
template <int TILE_M>
__host__ __device__ __forceinline__ void decode_tile(const Params& p, int64_t t, int64_t& b, int64_t& m0,
                                                     int64_t& n0) {
  constexpr int RHO = BN / TILE_M;
  b = t / p.tiles_per_batch;
  int64_t r = t % p.tiles_per_batch;
  if (!p.sym) {
    const int64_t band_tiles = GROUP_M * p.tiles_n;
    const int64_t g0 = (r / band_tiles) * GROUP_M;
    const int64_t R = imin(GROUP_M, p.tiles_m - g0);
    const int64_t w = r % band_tiles;
    m0 = (g0 + w % R) * TILE_M;
    n0 = (w / R) * BN;
    return;
  }
  int64_t g0 = 0;
  for (;;) {
    const int64_t R = imin(GROUP_M, p.tiles_m - g0);
    const int64_t cnt = sym_band_tiles<RHO>(R, p.tiles_n - g0 / RHO);
    if (r < cnt) break;
    r -= cnt;
    g0 += GROUP_M;
  }
  const int64_t R = imin(GROUP_M, p.tiles_m - g0);
  // column offset d: the ramp columns hold RHO (d + 1) rows each, later ones R
  int64_t d = 0, rows_d = 0;
  for (;;) {
    rows_d = imin(R, RHO * (d + 1));
    if (r < rows_d) break;
    r -= rows_d;
    ++d;
    if (rows_d == R) {  // past the ramp: every further column holds all R rows
      d += r / R;
      r %= R;
      break;
    }
  }
  m0 = (g0 + r) * TILE_M;
  n0 = (g0 / RHO + d) * BN;
}

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_msr_device_error, 0, code); }

// Epilogue data movement. A warp owns 32 rows of the tile (its TMEM lane quarter) and walks
// its 128 columns in chunks of 32. The accumulator arrives one row per thread (tcgen05.ld
// 32x32b), which would make every global access of a warp touch 32 rows; instead the C
// operand and the output pass through a 2 KB staging buffer per warp in shared memory, so
// that each global access instruction covers 8 rows x 64 contiguous bytes (lane l moves the
// 16-byte group l % 4 of row l / 4 + 8 i in pass i). The buffer holds 32 rows of 64 bytes;
// group g of row r sits at slot g ^ ((r >> 1) & 3), which gives 8 consecutive lanes 8
// distinct 16-byte bank groups in both access patterns (8 lanes at one group of 8 rows; 8
// lanes at 4 groups of 2 rows).

// Shared-memory address of group g of row r in a warp's buffer (stage: its shared address).
// The accesses are explicit 16-byte shared loads and stores (the buffer is reached through a
// generic pointer, which would otherwise leave the access width to the compiler).
__device__ __forceinline__ uint32_t epi_slot(uint32_t stage, int r, int g) {
  return stage + static_cast<uint32_t>(r * EPI_ROW_BYTES + ((g ^ ((r >> 1) & 3)) << 4));
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// The warp's view of one output tile: rows [rbase, rbase + 32) of matrix b, and this lane's
// own row (used by the math and by the mirror stores of symmetric tiles).
struct EpiRows {
  uint16_t* d;           // output matrix b
  const uint16_t* c;     // C operand matrix b, or null when beta * C is not used
  int64_t rbase;         // first row of the warp
  int64_t row;           // this lane's row, rbase + lane
};

// C operand for columns [col0, col0 + EPI_CW) of the warp's 32 rows, coalesced pattern:
// creg[i] = row rbase + 8 i + lane / 4, columns col0 + 8 (lane % 4) .. + 7 (zeros outside).
__device__ __forceinline__ void load_c_coalesced(const Params& p, const EpiRows& er, int64_t col0, int lane,
                                                 uint4 (&creg)[4]) {
  const int64_t col = col0 + (lane & 3) * 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = er.rbase + i * 8 + (lane >> 2);
    if (row < p.M && col + 8 <= p.N) {
      creg[i] = *reinterpret_cast<const uint4*>(er.c + row * p.ldc + col);
    } else {
      U16x8 t;
#pragma unroll
      for (int j = 0; j < 8; ++j) t.v[j] = (row < p.M && col + j < p.N) ? er.c[row * p.ldc + col + j] : uint16_t(0);
      creg[i] = *reinterpret_cast<const uint4*>(t.v);
    }
  }
}

// Coalesced C registers -> staging buffer (row r of the warp at row r of the buffer).
__device__ __forceinline__ void c_to_stage(uint32_t stage, const uint4 (&creg)[4], int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i) sts128(epi_slot(stage, i * 8 + (lane >> 2), lane & 3), creg[i]);
}

// Epilogue math for this lane's row, columns [col0, col0 + EPI_CW), in place in the staging
// buffer: each 16-byte group of the row is read (the C operand, when used) and overwritten
// with the output by this lane alone.
__device__ __forceinline__ void chunk_math(const Params& p, bool use_c, const uint32_t (&v)[EPI_CW], float alpha,
                                           float beta, uint32_t stage, int lane) {
#pragma unroll
  for (int g = 0; g < EPI_G; ++g) {
    const uint32_t slot = epi_slot(stage, lane, g);
    U16x8 cv, o;
    if (use_c) *reinterpret_cast<uint4*>(cv.v) = lds128(slot);
    if (p.ref_round) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float t = bf16r(__fmul_rn(alpha, bf16r(__uint_as_float(v[g * 8 + j]))));
        o.v[j] = use_c ? rne_bf16_bits(__fadd_rn(bf16r(__fmul_rn(beta, bf16_bits_to_f32(cv.v[j]))), t))
                       : rne_bf16_bits(t);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o.v[j] = rne_bf16_bits(
            fmaf(alpha, __uint_as_float(v[g * 8 + j]), beta * (use_c ? bf16_bits_to_f32(cv.v[j]) : 0.f)));
    }
    sts128(slot, *reinterpret_cast<const uint4*>(o.v));
  }
}

// The chunk's output rows in the staging buffer -> coalesced stores of the warp's 32 rows;
// then, in symmetric mode, the mirror of the strictly-upper elements: (row, c) -> (c, row).
// Lanes hold consecutive rows, so each mirrored column's stores form one 64-byte segment.
__device__ __forceinline__ void store_chunk(const Params& p, const EpiRows& er, uint32_t stage, int64_t col0,
                                            int lane) {
  const int64_t col = col0 + (lane & 3) * 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2);
    const int64_t row = er.rbase + r;
    const uint4 w = lds128(epi_slot(stage, r, lane & 3));
    if (row < p.M && col + 8 <= p.N) {
      *reinterpret_cast<uint4*>(er.d + row * p.ldd + col) = w;
    } else if (row < p.M) {
      const uint16_t* wv = reinterpret_cast<const uint16_t*>(&w);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (col + j < p.N) er.d[row * p.ldd + col + j] = wv[j];
    }
  }
  if (p.sym && er.row < p.M && col0 + EPI_CW - 1 > er.row) {
    uint16_t* dcol = er.d + er.row;
#pragma unroll
    for (int g = 0; g < EPI_G; ++g) {
      U16x8 o;
      *reinterpret_cast<uint4*>(o.v) = lds128(epi_slot(stage, lane, g));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t c = col0 + g * 8 + j;
        if (c > er.row && c < p.N) dcol[c * p.ldd] = o.v[j];
      }
    }
  }
}

// One epilogue warp's share of a finished tile: TMEM lane quarter q (rows row0 + 32 q +
// lane) and column half h of the 256-column accumulator at tmem_acc, with the next chunk's
// TMEM read and C-operand loads in flight under the current chunk's math and stores.
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tmem_acc, int64_t b, int64_t row0, int64_t n0,
                                              int q, int h, int lane, uint8_t* stage_ptr) {
  const uint32_t stage = tc::smem_addr(stage_ptr);
  constexpr int CHUNKS = BN / 2 / EPI_CW;
  float alpha = p.alpha, beta = p.beta;
  if (p.scale != nullptr) {
    float s = p.scale[b];
    if (p.scale_is_norm_sq) s = 1.0f / (sqrtf(s) + 1e-7f);
    if (p.alpha_pow == 1) alpha *= s; else if (p.alpha_pow == 2) alpha *= s * s;
    if (p.beta_pow == 1) beta *= s;
  }
  const bool use_c = p.c != nullptr && beta != 0.f;
  EpiRows er;
  er.d = p.d + b * p.d_bstride;
  er.c = use_c ? p.c + b * p.c_bstride : nullptr;
  er.rbase = row0 + q * 32;
  er.row = er.rbase + lane;
  const int64_t cbase = n0 + h * (BN / 2);
  const uint32_t tbase = tmem_acc + static_cast<uint32_t>(h * (BN / 2)) + (static_cast<uint32_t>(q * 32) << 16);
  uint32_t v[EPI_CW], vn[EPI_CW];
  uint4 creg[4];
  __syncwarp();
  tc::tmem_ld_32x32b_x32(tbase, v);
  if (use_c) load_c_coalesced(p, er, cbase, lane, creg);
  tc::tmem_ld_wait();
#pragma unroll 1
  for (int cc = 0; cc < CHUNKS; ++cc) {
    const int64_t col0 = cbase + cc * EPI_CW;
    if (use_c) {
      c_to_stage(stage, creg, lane);
      __syncwarp();
    }
    if (cc + 1 < CHUNKS) {
      tc::tmem_ld_32x32b_x32(tbase + (cc + 1) * EPI_CW, vn);
      if (use_c) load_c_coalesced(p, er, col0 + EPI_CW, lane, creg);
    }
    chunk_math(p, use_c, v, alpha, beta, stage, lane);
    __syncwarp();
    if (col0 < p.N) store_chunk(p, er, stage, col0, lane);
    __syncwarp();
    if (cc + 1 < CHUNKS) {
      tc::tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < EPI_CW; ++j) v[j] = vn[j];
    }
  }
}

template <int A_MN, int B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  SharedStorage& S = *reinterpret_cast<SharedStorage*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort = &S.abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&S.full[s], 1);
      tc::mbar_init(&S.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&S.tmem_full[a], 1);
      tc::mbar_init(&S.tmem_empty[a], EPI_THREADS);
    }
    tc::mbar_init(&S.drain, 1);
    S.abort = 0;
    tc::fence_mbar_init();
    tc::tma_prefetch_desc(&tmA);
    tc::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc(&S.tmem_base, TMEM_COLS);
    tc::tmem_relinquish();
    tc::fence_before_sync();
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = S.tmem_base;
  const int64_t num_kb = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_parity = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int64_t b64, m64, n64;
        decode_tile<BM>(p, t, b64, m64, n64);
        const int32_t b = static_cast<int32_t>(b64);
        const int32_t m0 = static_cast<int32_t>(m64);
        const int32_t n0 = static_cast<int32_t>(n64);
        for (int64_t kb = 0; kb < num_kb; ++kb) {
          if (!tc::mbar_wait(&S.empty[stage], phase ^ 1u, abort, WAIT_LIMIT_NS)) {
            record_error(ERR_TMA_WAIT);
            ok = false;
            break;
          }
          uint8_t* sa = S.stage[stage];
          uint8_t* sb = S.stage[stage] + A_BYTES;
          const int32_t k0 = static_cast<int32_t>(kb * BK);
          tc::mbar_arrive_expect_tx(&S.full[stage], STAGE_BYTES);
          if (A_MN) {
            tc::tma_load_3d(sa, &tmA, &S.full[stage], m0, k0, b);
            tc::tma_load_3d(sa + 8192, &tmA, &S.full[stage], m0 + 64, k0, b);
          } else {
            tc::tma_load_3d(sa, &tmA, &S.full[stage], k0, m0, b);
          }
          if (B_MN) {
#pragma unroll
            for (int i = 0; i < 4; ++i) tc::tma_load_3d(sb + 8192 * i, &tmB, &S.full[stage], n0 + 64 * i, k0, b);
          } else {
            tc::tma_load_3d(sb, &tmB, &S.full[stage], k0, n0, b);
          }
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Give up: let every copy already issued land before the CTA's shared memory goes.
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s)) {
            volatile int no_abort = 0;
            tc::mbar_wait(&S.full[s], (last_parity >> s) & 1u, &no_abort, WAIT_LIMIT_NS);
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t a_lbo = A_MN ? 8192u : 16u, b_lbo = B_MN ? 8192u : 16u;
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        if (!tc::mbar_wait(&S.tmem_empty[acc], acc_phase ^ 1u, abort, WAIT_LIMIT_NS)) {
          record_error(ERR_MMA_WAIT);
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int64_t kb = 0; kb < num_kb; ++kb) {
          if (!tc::mbar_wait(&S.full[stage], phase, abort, WAIT_LIMIT_NS)) {
            record_error(ERR_MMA_WAIT);
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sa = tc::smem_addr(S.stage[stage]);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint32_t aoff = A_MN ? static_cast<uint32_t>(k * UMMA_K * 128) : static_cast<uint32_t>(k * UMMA_K * 2);
            const uint32_t boff = B_MN ? static_cast<uint32_t>(k * UMMA_K * 128) : static_cast<uint32_t>(k * UMMA_K * 2);
            const uint64_t adesc = tc::smem_desc_sw128(sa + aoff, a_lbo, 1024u);
            const uint64_t bdesc = tc::smem_desc_sw128(sb + boff, b_lbo, 1024u);
            tc::mma_bf16(d_tmem, adesc, bdesc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc::mma_commit(&S.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc::mma_commit(&S.tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued above has finished before TMEM can be released.
      tc::mma_commit(&S.drain);
      volatile int no_abort = 0;
      tc::mbar_wait(&S.drain, 0, &no_abort, WAIT_LIMIT_NS);
    }
  } else if (warp >= 4) {
    // ------------------------------ epilogue ------------------------------
    // 8 warps: lane quarter q = warp % 4 (the only TMEM lanes warp q may read) and column
    // half h of the tile; each warp walks its 4 chunks of 32 columns with the next chunk's
    // TMEM read and C-operand loads in flight under the current chunk's math.
    const int q = warp & 3;
    const int h = (warp - 4) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      if (!tc::mbar_wait(&S.tmem_full[acc], acc_phase, abort, WAIT_LIMIT_NS)) {
        record_error(ERR_EPI_WAIT);
        break;
      }
      tc::fence_after_sync();
      int64_t b, m0, n0;
      decode_tile<BM>(p, t, b, m0, n0);
      epilogue_tile(p, tmem_base + static_cast<uint32_t>(acc * BN), b, m0, n0, q, h, lane, S.epi[warp - 4]);
      tc::fence_before_sync();
      tc::mbar_arrive(&S.tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2, issued by the even CTA of the pair. Each CTA loads its own 128
// rows of A and its own 128 rows of B (half of the tile's output columns) and receives its
// 128 rows of the accumulator in its TMEM, so a pair moves 64 KB per 64-deep k-block where
// two single CTAs move 96 KB for the same MMA work: a third less L2 -> shared-memory
// traffic, and a 6-stage ring in the same shared memory.
//
// Barriers: `full` of the leader counts both CTAs' copies of a stage (the leader expects the
// pair's bytes; each CTA's copies complete on it); the MMA commit arrives on `empty` and
// `tmem_full` of both CTAs; both CTAs' epilogue warps arrive on the leader's `tmem_empty`.
// A wait that gives up stops its own CTA and sets the peer's abort flag; copies already in
// flight get a bounded settling time, and a cluster barrier keeps both CTAs resident until
// neither touches the other's shared memory.
// ---------------------------------------------------------------------------------------
namespace pair {
constexpr int TILE_M = 256;
constexpr int HALF = 128;
constexpr int STAGES = 6;
constexpr int A_BYTES = HALF * BK * 2;
constexpr int B_BYTES = HALF * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t EMPTY_ARRIVALS = 2 * (EPI_THREADS / 32);  // one per epilogue warp of each CTA
constexpr uint64_t SETTLE_NS = 200000;  // after giving up: time for copies in flight to land
constexpr uint16_t BOTH = 0x3;

struct SharedStorage {
  alignas(1024) uint8_t stage[STAGES][STAGE_BYTES];
  alignas(16) uint8_t epi[EPI_WARPS][EPI_STAGE_BYTES];  // epilogue staging, one buffer per warp
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
}  // namespace pair

// Failure-detection test hook: one thread waits, through the same bounded wait the GEMM
// roles use, on an mbarrier that nothing arrives on, and records ERR_TEST_WAIT when the
// limit runs out; the kernel then returns normally and the context stays usable.
constexpr int ERR_TEST_WAIT = 0x1FF;

__global__ void wait_timeout_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !tc::mbar_wait(&bar, 0, &abort_flag, limit_ns)) record_error(ERR_TEST_WAIT);
}

// Sleeps for about `ns` nanoseconds of wall time.
__device__ __forceinline__ void settle(uint64_t ns) {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  do {
    __nanosleep(1000);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < ns);
}

template <int A_MN, int B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  using pair::HALF;
  using pair::STAGES;
  using pair::TILE_M;
  extern __shared__ uint8_t smem_raw[];
  pair::SharedStorage& S =
      *reinterpret_cast<pair::SharedStorage*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();  // 0: the leader, which issues the MMAs
  const int64_t pair_id = blockIdx.x >> 1;
  const int64_t num_pairs = gridDim.x >> 1;
  volatile int* abort = &S.abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&S.full[s], 1);
      tc::mbar_init(&S.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&S.tmem_full[a], 1);
      tc::mbar_init(&S.tmem_empty[a], pair::EMPTY_ARRIVALS);
    }
    tc::mbar_init(&S.drain, 1);
    S.abort = 0;
    tc::fence_mbar_init();
    tc::tma_prefetch_desc(&tmA);
    tc::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(&S.tmem_base, TMEM_COLS);
    tc::tmem_relinquish_pair();
    tc::fence_before_sync();
  }
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers exist before any remote arrive or copy
  tc::fence_after_sync();
  const uint32_t tmem_base = S.tmem_base;
  const int64_t num_kb = (p.K + BK - 1) / BK;
  const uint32_t peer_abort = tc::cluster_addr(&S.abort, rank ^ 1u);
  auto give_up = [&](int code) {
    record_error(code);
    *abort = 1;
    tc::st_cluster_u32(peer_abort, 1u);
  };

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t t = pair_id; t < p.num_tiles && ok; t += num_pairs) {
        int64_t b64, m64, n64;
        decode_tile<TILE_M>(p, t, b64, m64, n64);
        const int32_t b = static_cast<int32_t>(b64);
        const int32_t ma = static_cast<int32_t>(m64 + HALF * rank);
        const int32_t nb = static_cast<int32_t>(n64 + HALF * rank);
        for (int64_t kb = 0; kb < num_kb; ++kb) {
          if (!tc::mbar_wait(&S.empty[stage], phase ^ 1u, abort, WAIT_LIMIT_NS)) {
            give_up(ERR_TMA_WAIT);
            ok = false;
            break;
          }
          uint8_t* sa = S.stage[stage];
          uint8_t* sb = S.stage[stage] + pair::A_BYTES;
          const int32_t k0 = static_cast<int32_t>(kb * BK);
          if (rank == 0) tc::mbar_arrive_expect_tx(&S.full[stage], 2 * pair::STAGE_BYTES);
          const uint32_t bar = tc::cluster_addr(&S.full[stage], 0);
          if (A_MN) {
            tc::tma_load_3d_pair(sa, &tmA, bar, ma, k0, b);
            tc::tma_load_3d_pair(sa + 8192, &tmA, bar, ma + 64, k0, b);
          } else {
            tc::tma_load_3d_pair(sa, &tmA, bar, k0, ma, b);
          }
          if (B_MN) {
            tc::tma_load_3d_pair(sb, &tmB, bar, nb, k0, b);
            tc::tma_load_3d_pair(sb + 8192, &tmB, bar, nb + 64, k0, b);
          } else {
            tc::tma_load_3d_pair(sb, &tmB, bar, k0, nb, b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) settle(pair::SETTLE_NS);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader only) ------------------------------
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(TILE_M, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t a_lbo = A_MN ? 8192u : 16u, b_lbo = B_MN ? 8192u : 16u;
      for (int64_t t = pair_id; t < p.num_tiles && ok; t += num_pairs) {
        if (!tc::mbar_wait(&S.tmem_empty[acc], acc_phase ^ 1u, abort, WAIT_LIMIT_NS)) {
          give_up(ERR_MMA_WAIT);
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int64_t kb = 0; kb < num_kb; ++kb) {
          if (!tc::mbar_wait(&S.full[stage], phase, abort, WAIT_LIMIT_NS)) {
            give_up(ERR_MMA_WAIT);
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sa = tc::smem_addr(S.stage[stage]);
          const uint32_t sb = sa + pair::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint32_t aoff = A_MN ? static_cast<uint32_t>(k * UMMA_K * 128) : static_cast<uint32_t>(k * UMMA_K * 2);
            const uint32_t boff = B_MN ? static_cast<uint32_t>(k * UMMA_K * 128) : static_cast<uint32_t>(k * UMMA_K * 2);
            const uint64_t adesc = tc::smem_desc_sw128(sa + aoff, a_lbo, 1024u);
            const uint64_t bdesc = tc::smem_desc_sw128(sb + boff, b_lbo, 1024u);
            tc::mma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc::mma_commit_pair(&S.empty[stage], pair::BOTH);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc::mma_commit_pair(&S.tmem_full[acc], pair::BOTH);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued above (they read both CTAs' shared memory) has finished before
      // either CTA may leave.
      tc::mma_commit_pair(&S.drain, 0x1);
      volatile int no_abort = 0;
      tc::mbar_wait(&S.drain, 0, &no_abort, WAIT_LIMIT_NS);
    }
  } else if (warp >= 4) {
    // ------------------------------ epilogue (both CTAs) ------------------------------
    const int q = warp & 3;
    const int h = (warp - 4) >> 2;
    const uint32_t leader_empty[2] = {tc::cluster_addr(&S.tmem_empty[0], 0), tc::cluster_addr(&S.tmem_empty[1], 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t t = pair_id; t < p.num_tiles; t += num_pairs) {
      if (!tc::mbar_wait(&S.tmem_full[acc], acc_phase, abort, WAIT_LIMIT_NS)) {
        give_up(ERR_EPI_WAIT);
        break;
      }
      tc::fence_after_sync();
      int64_t b, m0, n0;
      decode_tile<TILE_M>(p, t, b, m0, n0);
      epilogue_tile(p, tmem_base + static_cast<uint32_t>(acc * BN), b, m0 + HALF * rank, n0, q, h, lane,
                    S.epi[warp - 4]);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(leader_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  tc::cluster_sync();  // neither CTA touches the other's shared memory or TMEM any more
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// Host side: tensor maps and launches
// ---------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 3-D bf16 tensor map over [batch][outer][inner] (inner contiguous), box {64, box_outer, 1},
// 128-byte swizzle, zero fill outside the tensor.
int make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t batch, int64_t batch_stride_elems,
             uint32_t box_outer) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(MSR_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(inner) * 2, static_cast<cuuint64_t>(batch_stride_elems) * 2};
  cuuint32_t box[3] = {64u, box_outer, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MSR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for inner=%lld outer=%lld batch=%lld", (int)r,
                (long long)inner, (long long)outer, (long long)batch);
  return MSR_OK;
}

size_t smem_bytes() { return sizeof(SharedStorage) + 1024; }

std::atomic<int> g_gemm_max_ctas{0};

constexpr int MAX_DEVICES = 64;

// Sets a kernel's dynamic shared memory limit once per device (slot: one per kernel
// variant), so that launches after the first -- e.g. inside a CUDA graph capture -- make
// no attribute call.
template <class K>
int smem_attr_once(K kern, int smem, std::atomic<int>* done_per_device) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>& done = done_per_device[dev % MAX_DEVICES];
  if (done.load(std::memory_order_acquire)) return MSR_OK;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(MSR_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  done.store(1, std::memory_order_release);
  return MSR_OK;
}

std::atomic<int> g_single_attr[4][MAX_DEVICES];
std::atomic<int> g_pair_attr[4][MAX_DEVICES];

template <int A_MN, int B_MN>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t s) {
  auto kern = gemm_kernel<A_MN, B_MN>;
  if (int st = smem_attr_once(kern, (int)smem_bytes(), g_single_attr[A_MN * 2 + B_MN])) return st;
  int ctas = sm_count();
  const int cap = g_gemm_max_ctas.load(std::memory_order_relaxed);
  if (cap > 0 && cap < ctas) ctas = cap;
  const int grid = static_cast<int>(std::min<int64_t>(p.num_tiles, ctas));
  kern<<<grid, NUM_THREADS, smem_bytes(), s>>>(ta, tb, p);
  return check_launch("gemm_kernel");
}

size_t pair_smem_bytes() { return sizeof(pair::SharedStorage) + 1024; }

std::atomic<int> g_gemm_pairs{1};

// Clusters of two that fit on the device at once (a GPC with an odd number of free SMs
// leaves one idle), per kernel variant and device.
std::atomic<int> g_pair_capacity[4][MAX_DEVICES];

template <int A_MN, int B_MN>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t s) {
  auto kern = gemm_pair_kernel<A_MN, B_MN>;
  const int smem = static_cast<int>(pair_smem_bytes());
  if (int st = smem_attr_once(kern, smem, g_pair_attr[A_MN * 2 + B_MN])) return st;
  cudaError_t e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>& cap_slot = g_pair_capacity[A_MN * 2 + B_MN][dev % MAX_DEVICES];
  int pairs = cap_slot.load(std::memory_order_relaxed);
  if (pairs <= 0) {
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n <= 0)
      return fail(MSR_ERR_CUDA, "cudaOccupancyMaxActiveClusters: %s (%d)", cudaGetErrorString(e), n);
    pairs = n;
    cap_slot.store(n, std::memory_order_relaxed);
  }
  const int cap = g_gemm_max_ctas.load(std::memory_order_relaxed);
  if (cap > 0) pairs = std::min(pairs, std::max(1, cap / 2));
  pairs = static_cast<int>(std::min<int64_t>(p.num_tiles, pairs));
  cfg.gridDim = dim3(2 * pairs);
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) return fail(MSR_ERR_CUDA, "gemm_pair_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("gemm_pair_kernel");
}

// The tile grid of a GEMM: tiles of tile_m x BN over [M][N] per matrix; in symmetric mode
// row-block i keeps column-blocks i / RHO .. tiles_n - 1 (see decode_tile).
void set_tiles(Params& p, int64_t M, int64_t N, int64_t batch, int sym, int64_t tile_m) {
  p.M = M; p.N = N; p.batch = batch;
  p.tiles_m = (M + tile_m - 1) / tile_m;
  p.tiles_n = (N + BN - 1) / BN;
  p.sym = sym;
  p.tiles_per_batch = p.tiles_m * p.tiles_n;
  if (sym) {
    const int64_t rho = BN / tile_m;
    p.tiles_per_batch = 0;
    for (int64_t i = 0; i < p.tiles_m; ++i) p.tiles_per_batch += p.tiles_n - i / rho;
  }
  p.num_tiles = p.tiles_per_batch * batch;
}

// D[b] = alpha_b * op(A)[b] x op(B)[b]^T + beta_b * C[b]. A K-major: [batch][M][K]; MN-major:
// [batch][K][M]. B K-major: [batch][N][K]; MN-major: [batch][K][N]. C, D: [batch][M][N] with
// row strides ldc, ldd.
int run_gemm(const void* a, int a_mn, int64_t a_bstride, const void* b, int b_mn, int64_t b_bstride, const void* c,
         int64_t ldc, int64_t c_bstride, void* d, int64_t ldd, int64_t d_bstride, int64_t batch, int64_t M, int64_t N,
         int64_t K, float alpha, float beta, const float* scale, int alpha_pow, int beta_pow, int scale_is_norm_sq,
         int ref_round, int sym, cudaStream_t s) {
  if (sym && M != N) return fail(MSR_ERR_INVALID, "symmetric GEMM needs M == N");
  const bool pairs = g_gemm_pairs.load(std::memory_order_relaxed) != 0;
  const int64_t tile_m = pairs ? pair::TILE_M : BM;
  // K-major boxes: one CTA's rows of A (128) and of B (256 alone, 128 as half of a pair)
  const uint32_t b_rows = pairs ? pair::HALF : BN;
  CUtensorMap ta, tb;
  int st = a_mn ? make_map(&ta, a, M, K, batch, a_bstride, 64) : make_map(&ta, a, K, M, batch, a_bstride, BM);
  if (st) return st;
  st = b_mn ? make_map(&tb, b, N, K, batch, b_bstride, 64) : make_map(&tb, b, K, N, batch, b_bstride, b_rows);
  if (st) return st;
  Params p{};
  p.K = K;
  set_tiles(p, M, N, batch, sym, tile_m);
  p.d = static_cast<uint16_t*>(d);
  p.c = static_cast<const uint16_t*>(c);
  p.ldd = ldd; p.ldc = ldc; p.d_bstride = d_bstride; p.c_bstride = c_bstride;
  p.alpha = alpha; p.beta = beta;
  p.scale = scale; p.alpha_pow = alpha_pow; p.beta_pow = beta_pow; p.scale_is_norm_sq = scale_is_norm_sq;
  p.ref_round = ref_round;
  if (pairs) {
    if (a_mn && b_mn) return launch_pair<1, 1>(ta, tb, p, s);
    if (a_mn) return launch_pair<1, 0>(ta, tb, p, s);
    if (b_mn) return launch_pair<0, 1>(ta, tb, p, s);
    return launch_pair<0, 0>(ta, tb, p, s);
  }
  if (a_mn && b_mn) return launch<1, 1>(ta, tb, p, s);
  if (a_mn) return launch<1, 0>(ta, tb, p, s);
  if (b_mn) return launch<0, 1>(ta, tb, p, s);
  return launch<0, 0>(ta, tb, p, s);
}

// ---------------------------------------------------------------------------------------
// Small helper kernels of the Newton-Schulz driver
// ---------------------------------------------------------------------------------------
// Squared Frobenius norms in two passes with a fixed summation order, so the result is the
// same bits on every run (data-parallel replicas must agree; float atomics would not).
constexpr int NORM_THREADS = 256;
constexpr int NORM_MAX_PARTS = 256;

// Partial sums: parts blocks per matrix (gridDim.x), block i covers a grid-stride share.
__global__ void __launch_bounds__(NORM_THREADS) norm_partial_kernel(const uint16_t* __restrict__ x, int64_t per,
                                                                    float* __restrict__ partials) {
  const int64_t b = blockIdx.y;
  const uint16_t* xb = x + b * per;
  float s = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)NORM_THREADS + threadIdx.x; i < per; i += (int64_t)gridDim.x * NORM_THREADS) {
    const float v = bf16_bits_to_f32(xb[i]);
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[NORM_THREADS / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < NORM_THREADS / 32; ++i) t += red[i];
    partials[b * gridDim.x + blockIdx.x] = t;
  }
}

// norm_sq[b] = sum of the parts partials of matrix b, one block per matrix.
__global__ void __launch_bounds__(NORM_MAX_PARTS) norm_final_kernel(const float* __restrict__ partials, int parts,
                                                                    float* __restrict__ norm_sq) {
  __shared__ float red[NORM_MAX_PARTS];
  const int b = blockIdx.x;
  red[threadIdx.x] = threadIdx.x < parts ? partials[b * parts + threadIdx.x] : 0.f;
  __syncthreads();
  for (int w = NORM_MAX_PARTS / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) norm_sq[b] = red[0];
}

// Blocks per matrix: a function of the shape only (not of the device), so every GPU model
// sums in the same order.
inline int norm_parts(int64_t per) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(NORM_MAX_PARTS, (per + 65535) / 65536)));
}

// dst[b][r][c] (dst dims R2 x C2) = src[b][r][c] for r < R, c < C, else 0 -- or the reverse copy.
__global__ void pad_copy_kernel(const uint16_t* __restrict__ src, int64_t sR, int64_t sC, uint16_t* __restrict__ dst,
                                int64_t dR, int64_t dC, int64_t batch) {
  const int64_t total = batch * dR * dC;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i % dC;
    const int64_t r = (i / dC) % dR;
    const int64_t b = i / (dC * dR);
    dst[i] = (r < sR && c < sC) ? src[(b * sR + r) * sC + c] : uint16_t(0);
  }
}

// Normalisation by the Frobenius norm (may run in place).
//  ref != 0: out = bf16(x / d), d = bf16(bf16(sqrt(norm_sq)) + 1e-7): the reference's bf16 ops
//            X / (X.norm() + 1e-7) on a bf16 tensor (muon_sr/muon_sr.py:91).
//  ref == 0: out = bf16(x * (1 / (sqrt(norm_sq) + 1e-7))) in fp32.
// One matrix per blockIdx.y; 8 elements per thread per step when the matrix stride allows
// 16-byte accesses.
__device__ __forceinline__ uint16_t normalize_one(uint16_t xb, float d, float s, int ref) {
  const float v = bf16_bits_to_f32(xb);
  return ref ? rne_bf16_bits(__fdiv_rn(v, d)) : rne_bf16_bits(v * s);
}

__global__ void __launch_bounds__(256) normalize_kernel(const uint16_t* x, uint16_t* out, int64_t per,
                                                        const float* __restrict__ nsq, int ref) {
  const int64_t b = blockIdx.y;
  const float nrm = sqrtf(nsq[b]);
  const float d = bf16r(__fadd_rn(bf16r(nrm), 1e-7f));
  const float s = 1.0f / (nrm + 1e-7f);
  const uint16_t* xb = x + b * per;
  uint16_t* ob = out + b * per;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if ((per & 7) == 0) {
    for (int64_t v = t0; v < per / 8; v += stride) {
      U16x8 w = ld_u16x8(xb + v * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j) w.v[j] = normalize_one(w.v[j], d, s, ref);
      st_u16x8(ob + v * 8, w);
    }
  } else {
    for (int64_t i = t0; i < per; i += stride) ob[i] = normalize_one(xb[i], d, s, ref);
  }
}

// Launches normalize_kernel over `batch` matrices of `per` elements (x may equal out; both
// 16-byte aligned, which with per % 8 == 0 makes every matrix's vectors aligned).
int launch_normalize(const uint16_t* x, uint16_t* out, int64_t per, int64_t batch, const float* nsq, int ref,
                     cudaStream_t s) {
  const int64_t work = (per & 7) == 0 ? per / 8 : per;
  const int64_t want = std::max<int64_t>(1, (4 * (int64_t)sm_count() + batch - 1) / batch);
  const int gx = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, want)));
  for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, batch - b0);
    normalize_kernel<<<dim3(gx, static_cast<unsigned>(nb)), 256, 0, s>>>(x + b0 * per, out + b0 * per, per, nsq + b0,
                                                                          ref);
    if (int st = check_launch("normalize_kernel")) return st;
  }
  return MSR_OK;
}

inline int64_t round8(int64_t v) { return (v + 7) / 8 * 8; }
inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }

struct NsLayout {
  bool padded, transposed;
  int64_t R8, C8, m, n;
  size_t off_nsq, off_part, off_a, off_b, off_w1, off_w2, off_pin, total;
};

NsLayout ns_layout(int64_t batch, int64_t rows, int64_t cols) {
  NsLayout L{};
  L.transposed = rows > cols;
  L.R8 = round8(rows);
  L.C8 = round8(cols);
  L.padded = (L.R8 != rows) || (L.C8 != cols);
  L.m = L.transposed ? L.C8 : L.R8;
  L.n = L.transposed ? L.R8 : L.C8;
  const size_t xb = static_cast<size_t>(batch) * L.R8 * L.C8 * 2;
  const size_t gb = static_cast<size_t>(batch) * L.m * L.m * 2;
  size_t o = 0;
  L.off_nsq = o; o = align256(o + static_cast<size_t>(batch) * 4);
  L.off_part = o; o = align256(o + static_cast<size_t>(batch) * NORM_MAX_PARTS * 4);
  L.off_a = o;   o = align256(o + gb);
  L.off_b = o;   o = align256(o + gb);
  L.off_w1 = o;  o = align256(o + xb);
  L.off_w2 = o;  if (L.padded) o = align256(o + xb);
  L.off_pin = o; if (L.padded) o = align256(o + xb);
  L.total = o;
  return L;
}


}  // namespace gemm
}  // namespace msr


using namespace msr;
using namespace msr::gemm;

extern "C" {

void msr_set_gemm_max_ctas(int max_ctas) { g_gemm_max_ctas.store(max_ctas > 0 ? max_ctas : 0); }

void msr_set_gemm_pairs(int enable) { g_gemm_pairs.store(enable ? 1 : 0); }

int msr_gemm_tile_map(int64_t M, int64_t N, int64_t batch, int symmetric, int pairs, int64_t* out, int64_t capacity,
                      int64_t* num_tiles) {
  if (M <= 0 || N <= 0 || batch <= 0 || !num_tiles || (symmetric && M != N))
    return fail(MSR_ERR_INVALID, "msr_gemm_tile_map: bad shape");
  Params p{};
  set_tiles(p, M, N, batch, symmetric ? 1 : 0, pairs ? pair::TILE_M : BM);
  *num_tiles = p.num_tiles;
  if (out == nullptr) return MSR_OK;
  if (capacity < 3 * p.num_tiles) return fail(MSR_ERR_INVALID, "msr_gemm_tile_map: out holds fewer than 3 x %lld",
                                              (long long)p.num_tiles);
  for (int64_t t = 0; t < p.num_tiles; ++t) {
    int64_t b, m0, n0;
    if (pairs) decode_tile<pair::TILE_M>(p, t, b, m0, n0);
    else decode_tile<BM>(p, t, b, m0, n0);
    out[3 * t] = b;
    out[3 * t + 1] = m0;
    out[3 * t + 2] = n0;
  }
  return MSR_OK;
}

int msr_get_gemm_pairs(void) { return g_gemm_pairs.load(); }

int msr_test_wait_timeout(uint64_t limit_ns, msr_stream_t stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return fail(MSR_ERR_INVALID, "msr_test_wait_timeout: limit must be in (0, 10 s]");
  if (int st = require_sm100()) return st;
  wait_timeout_kernel<<<1, 32, 0, to_stream(stream)>>>(limit_ns);
  return check_launch("wait_timeout_kernel");
}


int msr_device_error(msr_stream_t stream, int clear) {
  cudaError_t e = cudaStreamSynchronize(to_stream(stream));
  if (e != cudaSuccess) return fail(-1, "cudaStreamSynchronize: %s", cudaGetErrorString(e)), -1;
  int value = 0;
  e = cudaMemcpyFromSymbol(&value, g_msr_device_error, sizeof(int));
  if (e != cudaSuccess) return fail(-1, "read device error: %s", cudaGetErrorString(e)), -1;
  if (clear && value != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_msr_device_error, &zero, sizeof(int));
  }
  return value;
}

int msr_gemm_bf16(const void* a, int a_mn_major, const void* b, int b_mn_major, const void* c, void* d, int64_t batch,
                  int64_t M, int64_t N, int64_t K, float alpha, float beta, const float* scale, int alpha_pow,
                  int beta_pow, int flags, msr_stream_t stream) {
  if (!a || !b || !d || batch <= 0 || M <= 0 || N <= 0 || K <= 0)
    return fail(MSR_ERR_INVALID, "msr_gemm_bf16: null pointer or non-positive size");
  const int64_t a_inner = a_mn_major ? M : K, b_inner = b_mn_major ? N : K;
  if (a_inner % 8 || b_inner % 8 || N % 8)
    return fail(MSR_ERR_INVALID, "msr_gemm_bf16: contiguous dims must be multiples of 8 (got A %lld, B %lld, N %lld)",
                (long long)a_inner, (long long)b_inner, (long long)N);
  if (int st = require_sm100()) return st;
  const int ref = (flags & MSR_GEMM_REFERENCE_ROUNDING) ? 1 : 0;
  const int sym = (flags & MSR_GEMM_SYMMETRIC) ? 1 : 0;
  if (sym && M != N) return fail(MSR_ERR_INVALID, "msr_gemm_bf16: MSR_GEMM_SYMMETRIC needs M == N");
  return run_gemm(a, a_mn_major, M * K, b, b_mn_major, N * K, c, N, M * N, d, N, M * N, batch, M, N, K, alpha, beta,
                  ref ? nullptr : scale, alpha_pow, beta_pow, 0, ref, sym, to_stream(stream));
}

size_t msr_ns_workspace_bytes(int64_t batch, int64_t rows, int64_t cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  return ns_layout(batch, rows, cols).total;
}

int msr_newton_schulz_bf16(const void* x, void* out, int64_t batch, int64_t rows, int64_t cols, int steps, int mode,
                           const float* norm_sq, void* workspace, size_t workspace_bytes, msr_stream_t stream) {
  if (!x || !out || batch <= 0 || rows <= 0 || cols <= 0 || steps < 0)
    return fail(MSR_ERR_INVALID, "msr_newton_schulz_bf16: null pointer or bad size");
  if (mode != MSR_NS_REFERENCE_ROUNDING && mode != MSR_NS_FUSED_ROUNDING)
    return fail(MSR_ERR_INVALID, "msr_newton_schulz_bf16: unknown mode %d", mode);
  const int ref = mode == MSR_NS_REFERENCE_ROUNDING;
  if (x == out) return fail(MSR_ERR_INVALID, "msr_newton_schulz_bf16: out must not alias x");
  const NsLayout L = ns_layout(batch, rows, cols);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(MSR_ERR_WORKSPACE, "msr_newton_schulz_bf16: workspace %zu < %zu bytes", workspace_bytes, L.total);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 || reinterpret_cast<uintptr_t>(x) % 16 ||
      reinterpret_cast<uintptr_t>(out) % 16)
    return fail(MSR_ERR_INVALID, "msr_newton_schulz_bf16: x/out must be 16-byte and workspace 256-byte aligned");
  if (int st = require_sm100()) return st;
  cudaStream_t s = to_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t per = rows * cols;

  const float* nsq = norm_sq;
  if (nsq == nullptr) {
    float* t = reinterpret_cast<float*>(ws + L.off_nsq);
    float* part = reinterpret_cast<float*>(ws + L.off_part);
    const int parts = norm_parts(per);
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {  // gridDim.y limit
      const int64_t nb = std::min<int64_t>(65535, batch - b0);
      norm_partial_kernel<<<dim3(parts, static_cast<unsigned>(nb)), NORM_THREADS, 0, s>>>(
          static_cast<const uint16_t*>(x) + b0 * per, per, part + b0 * parts);
      if (int st = check_launch("norm_partial_kernel")) return st;
    }
    norm_final_kernel<<<static_cast<unsigned>(batch), NORM_MAX_PARTS, 0, s>>>(part, parts, t);
    if (int st = check_launch("norm_final_kernel")) return st;
    nsq = t;
  }
  const int ew_grid = 4 * sm_count();
  if (steps == 0)
    return launch_normalize(static_cast<const uint16_t*>(x), static_cast<uint16_t*>(out), per, batch, nsq, ref, s);

  const int64_t R = L.R8, C = L.C8, m = L.m, n = L.n;
  const int64_t xs = R * C, gs = m * m;
  uint16_t* A = reinterpret_cast<uint16_t*>(ws + L.off_a);
  uint16_t* B = reinterpret_cast<uint16_t*>(ws + L.off_b);
  const uint16_t* src;
  uint16_t* bufs[2];
  if (L.padded) {
    uint16_t* pin = reinterpret_cast<uint16_t*>(ws + L.off_pin);
    pad_copy_kernel<<<ew_grid, 256, 0, s>>>(static_cast<const uint16_t*>(x), rows, cols, pin, R, C, batch);
    if (int st = check_launch("pad_copy_kernel")) return st;
    if (ref)
      if (int st = launch_normalize(pin, pin, xs, batch, nsq, 1, s)) return st;
    src = pin;
    bufs[0] = reinterpret_cast<uint16_t*>(ws + L.off_w1);
    bufs[1] = reinterpret_cast<uint16_t*>(ws + L.off_w2);
  } else {
    src = static_cast<const uint16_t*>(x);
    // Step s writes bufs[(steps - 1 - s) & 1] so that the last step lands in `out`.
    bufs[0] = static_cast<uint16_t*>(out);
    bufs[1] = reinterpret_cast<uint16_t*>(ws + L.off_w1);
    if (ref) {
      // X0 goes to the buffer that step 0 does not write.
      uint16_t* x0 = bufs[steps & 1];
      if (int st = launch_normalize(static_cast<const uint16_t*>(x), x0, per, batch, nsq, 1, s)) return st;
      src = x0;
    }
  }
  const float a_ = 3.4445f, b_ = -4.7750f, c_ = 2.0315f;
  for (int st_i = 0; st_i < steps; ++st_i) {
    uint16_t* dst = L.padded ? bufs[st_i & 1] : bufs[(steps - 1 - st_i) & 1];
    // Fused mode folds 1/(||x|| + 1e-7) into step 0; reference mode normalised X0 above.
    const float* sc = (!ref && st_i == 0) ? nsq : nullptr;
    int st;
    // A = X X^T (wide orientation): K-major X rows, or MN-major columns of a tall X.
    if (!L.transposed)
      st = run_gemm(src, 0, xs, src, 0, xs, nullptr, m, gs, A, m, gs, batch, m, m, n, 1.f, 0.f, sc, 2, 0, 1, ref, 1, s);
    else
      st = run_gemm(src, 1, xs, src, 1, xs, nullptr, m, gs, A, m, gs, batch, m, m, n, 1.f, 0.f, sc, 2, 0, 1, ref, 1, s);
    if (st) return st;
    // B = c (A A) + b A   (A symmetric: A A = A A^T)
    st = run_gemm(A, 0, gs, A, 0, gs, A, m, gs, B, m, gs, batch, m, m, m, c_, b_, nullptr, 0, 0, 0, ref, 1, s);
    if (st) return st;
    // X' = B X + a X  (tall X: X' = X B + a X with B symmetric)
    if (!L.transposed)
      st = run_gemm(B, 0, gs, src, 1, xs, src, C, xs, dst, C, xs, batch, m, n, m, 1.f, a_, sc, 1, 1, 1, ref, 0, s);
    else
      st = run_gemm(src, 0, xs, B, 0, gs, src, C, xs, dst, C, xs, batch, R, C, C, 1.f, a_, sc, 1, 1, 1, ref, 0, s);
    if (st) return st;
    src = dst;
  }
  if (L.padded) {
    pad_copy_kernel<<<ew_grid, 256, 0, s>>>(src, R, C, static_cast<uint16_t*>(out), rows, cols, batch);
    return check_launch("pad_copy_kernel (out)");
  }
  return MSR_OK;
}

}  // extern "C"
