// Max of a 4-byte amax over the ranks of a token-/CFG-sharded run, exchanged
// through peer memory instead of an NCCL all-reduce.
//
// Replaces the max all-reduce that keeps one NVFP4 global scale per
// activation across ranks (the CFG batch and token shards of one activation
// tensor; QuantizedActivation's amax, h3_inference/nvfp4.py:92-110).
//
// Every rank owns a slot array of 2 * world 64-bit words in device memory that
// every other rank has mapped (CUDA IPC).  Exchange number e (e >= 1, the same
// count on every rank) uses half e % 2 of every array:
//   lane r of rank q stores (e << 32 | amax bits) to word [e % 2][q] of rank
//   r's array (a plain 64-bit peer store), then lane r polls word [e % 2][r]
//   of its own array until it carries epoch e; the warp takes the max.
// Halves alternate so a fast rank's exchange e + 1 cannot overwrite a value
// a slow rank has not yet read for e: finishing e + 1 needs every rank's
// e + 1 store, which a rank makes only after its own e has completed.  The
// wait is bounded (limit_ns); on expiry the kernel records H3B_ERR_TIMEOUT,
// leaves the local amax in place and returns.  No multicast, no NVLS.
#pragma once

#include "common.cuh"

namespace h3b {
namespace peer {

constexpr int kMaxRanks = 32;

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One warp.  slots[r]: rank r's slot array as mapped in this process.
__global__ void __launch_bounds__(32)
    k_amax_exchange(float* __restrict__ amax, const unsigned long long* const* __restrict__ slots,
                    int rank, int world, uint32_t epoch, uint64_t limit_ns) {
  const int lane = threadIdx.x;
  const float mine = *amax;
  const unsigned long long word =
      ((unsigned long long)epoch << 32) | (unsigned long long)__float_as_uint(mine);
  const int half = (int)(epoch & 1u) * world;
  if (lane < world)
    st_relaxed_sys_u64(const_cast<unsigned long long*>(slots[lane]) + half + rank, word);
  float m = mine;
  // after a recorded failure (an earlier wait expired: a rank is gone) no
  // exchange waits again, so a lost rank costs one bound, not one per call
  bool ok = *(volatile int*)&g_dev_error == 0;
  if (lane < world && ok) {
    const unsigned long long* src = slots[rank] + half + lane;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
      const unsigned long long w = ld_relaxed_sys_u64(src);
      if ((uint32_t)(w >> 32) == epoch) {
        m = fmaxf(m, __uint_as_float((uint32_t)w));
        break;
      }
      if ((i & 15u) == 15u && globaltimer() - t0 > limit_ns) {
        ok = false;
        break;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  ok = __all_sync(0xffffffffu, ok);
  if (lane == 0) {
    if (ok) *amax = m;
    else record_error(H3B_ERR_TIMEOUT);   // no-op when a failure is already recorded
  }
}

}  // namespace peer
}  // namespace h3b
