// Streamed multi-tensor elementwise launches (sm_100a).
//
// The optimizer's elementwise kernels are bound by the FMA-heavy pipe (the 32-bit integer
// multiplies of the reference's Philox noise) and by how well loads overlap that work. Here
// the two are decoupled: per CTA one producer warp moves each tile's inputs from HBM into a
// ring of shared-memory stages with bulk asynchronous copies (cp.async.bulk, completion
// counted in bytes on an mbarrier; no multicast), while the consumer warps compute tiles
// already in shared memory and store their results straight to global memory. The producer
// runs up to STAGES tiles ahead, so the consumers find their inputs waiting instead of
// stalling on HBM latency, and no registers are spent holding loads in flight.
//
// Work layout is the multi-tensor one of the plain launches: tiles of TILE elements never
// cross a tensor, a persistent grid walks them (tile = blockIdx.x + k * gridDim.x), and
// producer and consumers walk the same sequence. A tile's bulk copy covers its elements up to
// the last whole 16 bytes (bulk copies need 16-byte aligned addresses and sizes); elements
// past that (a tensor's ragged end) and every element of an entry whose pointers are not
// 16-byte aligned are read by the consumers from global memory directly.
//
// Every mbarrier wait is bounded (WAIT_LIMIT_NS). A role that gives up records a code in the
// library's device error word (passed in by address; read with msr_device_error), raises the
// CTA's abort flag so the other role stops too, and the producer waits (again bounded) for
// the CTA's own copies in flight before the CTA returns.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace msr {
namespace stream {

constexpr int CONS_WARPS = 8;
constexpr int CONS_THREADS = CONS_WARPS * 32;
constexpr int THREADS = CONS_THREADS + 32;  // warp 0 produces, warps 1..8 consume
constexpr int EPT = 8;                       // elements per consumer thread and tile
constexpr int TILE = CONS_THREADS * EPT;     // 2048 elements
constexpr int TILE_BYTES = TILE * 2;         // one bf16 array of a tile
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;
constexpr int ERR_PRODUCER_WAIT = 0x201, ERR_CONSUMER_WAIT = 0x202;

__device__ __forceinline__ void record_error(int* flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

// Entry of tile `t`: binary search over the exclusive prefix of per-entry tile counts.
__device__ __forceinline__ int find_entry_dyn(const int64_t* prefix, int count, int64_t t) {
  int lo = 0, hi = count;  // prefix[lo] <= t < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

// Bulk copy global -> this CTA's shared memory, completion counted on `bar` (the CTA's own
// shared memory window of the cluster address space; a non-cluster launch is a cluster of 1).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          tc::smem_addr(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(tc::smem_addr(bar))
      : "memory");
}

// Shared-memory layout of a streamed kernel with NIN input arrays and S stages.
template <int NIN, int S>
struct Smem {
  alignas(128) uint16_t data[S][NIN][TILE];
  uint64_t full[S];
  uint64_t empty[S];
  int abort;
};

template <int NIN, int S>
constexpr size_t smem_bytes() {
  return sizeof(Smem<NIN, S>);
}

// One tile as the roles see it: the entry it belongs to, its first element, the element
// count and how many of them the bulk copy brought in (a multiple of 8, or 0).
struct TileRef {
  int entry;
  int64_t base;
  int64_t count;
  int64_t bulk;
};

// The multi-tensor streamed kernel body. Policy provides:
//   static constexpr int NIN;
//   int count() const; const int64_t* prefix() const;   (tiles per entry, exclusive prefix)
//   bool vec(int e) const;  int64_t numel(int e) const;  const void* input(int e, int i) const;
//   void vector8(int e, int64_t idx, const uint16_t* const (&in)[NIN]) const;   8 elements from smem
//   void scalar_range(int e, int64_t lo, int64_t hi) const;   elements lo..hi-1 (< 8) from global
//   bool multicast() const;   the launch stores through multicast addresses (a system fence ends it)
template <class Policy, int S>
__device__ __forceinline__ void run(const Policy& P, Smem<Policy::NIN, S>& sm, int* err) {
  constexpr int NIN = Policy::NIN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&sm.full[s], 1);
      tc::mbar_init(&sm.empty[s], CONS_WARPS);
    }
    sm.abort = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  const int64_t total = P.prefix()[P.count()];
  volatile int* abort = &sm.abort;
  auto tile_of = [&](int64_t t) {
    TileRef r;
    r.entry = find_entry_dyn(P.prefix(), P.count(), t);
    const int64_t n = P.numel(r.entry);
    r.base = (t - P.prefix()[r.entry]) * TILE;
    r.count = n - r.base < TILE ? n - r.base : TILE;
    r.bulk = P.vec(r.entry) ? (r.count & ~int64_t(7)) : 0;
    return r;
  };
  if (warp == 0) {
    // ---- producer: one lane issues the copies of every tile, up to S tiles ahead ----
    if (lane == 0) {
      int s = 0;
      uint32_t phase = 0, armed = 0, armed_parity = 0;  // per stage: ever armed, parity of its last arming
      for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        if (!tc::mbar_wait(&sm.empty[s], phase ^ 1u, abort, WAIT_LIMIT_NS)) {
          record_error(err, ERR_PRODUCER_WAIT);
          break;
        }
        const TileRef r = tile_of(t);
        const uint32_t bytes = static_cast<uint32_t>(r.bulk) * 2u;
        tc::mbar_arrive_expect_tx(&sm.full[s], bytes * NIN);
        if (bytes) {
#pragma unroll
          for (int i = 0; i < NIN; ++i)
            bulk_g2s(sm.data[s][i], static_cast<const uint16_t*>(P.input(r.entry, i)) + r.base, bytes, &sm.full[s]);
        }
        armed |= 1u << s;
        armed_parity = (armed_parity & ~(1u << s)) | (phase << s);
        if (++s == S) { s = 0; phase ^= 1u; }
      }
      // After an abort, copies still in flight would land in this CTA's shared memory after
      // it exits: wait (bounded) until the last arming of every stage has completed (a phase
      // the consumers already took has completed too, so the wait returns at once).
      if (*abort) {
        const uint64_t t0 = globaltimer_ns();
        for (int k = 0; k < S; ++k) {
          if (!(armed >> k & 1u)) continue;
          while (!tc::mbar_try_wait(&sm.full[k], armed_parity >> k & 1u))
            if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
        }
      }
    }
    return;
  }
  // ---- consumers: warps 1..8, thread c handles elements base + 8c .. base + 8c + 7 ----
  const int c = threadIdx.x - 32;
  int s = 0;
  uint32_t phase = 0;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    if (!tc::mbar_wait(&sm.full[s], phase, abort, WAIT_LIMIT_NS)) {
      record_error(err, ERR_CONSUMER_WAIT);
      break;
    }
    const TileRef r = tile_of(t);
    const int64_t off = static_cast<int64_t>(c) * EPT;
    if (off + EPT <= r.bulk) {
      const uint16_t* in[NIN];
#pragma unroll
      for (int i = 0; i < NIN; ++i) in[i] = sm.data[s][i] + off;
      P.vector8(r.entry, r.base + off, in);
    } else if (off < r.count) {
      P.scalar_range(r.entry, r.base + off, r.base + (off + EPT < r.count ? off + EPT : r.count));
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&sm.empty[s]);
    if (++s == S) { s = 0; phase ^= 1u; }
  }
  // multicast stores are ordered before anything this thread does after the kernel (the
  // callers' cross-rank barrier)
  if (P.multicast()) __threadfence_system();
}

}  // namespace stream
}  // namespace msr
