// Warp-aggregated scatter helpers shared by the backward kernels.
//
// Gradient scatters add many small contributions to a few addresses: neighbouring pixels show the
// same triangle, so they share vertices. Lanes of a warp that target the same address are found
// with __match_any_sync and their values summed with a log-depth segmented reduction over shuffles
// (each lane repeatedly adds the partial sum of its next-higher remaining peer; after round k only
// lanes whose peer rank is a multiple of 2^k remain), so one lane per distinct address issues the
// atomic.
#pragma once

#include <cuda_runtime.h>

namespace dr {

// Sum of `v` over the lanes in `peers` (which must contain the calling lane), returned on the
// lowest lane of `peers`; other lanes get partial sums. All 32 lanes must call it together; lanes
// with nothing to add pass peers = their own bit and any value.
template <int N>
__device__ __forceinline__ void segmented_sum(unsigned peers, float (&v)[N]) {
  const unsigned lane = threadIdx.x & 31u;
  unsigned rank = __popc(peers & ((1u << lane) - 1u));
  unsigned above = peers & ~((2u << lane) - 1u);
  while (__any_sync(0xffffffffu, above != 0u)) {
    const int next = above ? __ffs(above) - 1 : static_cast<int>(lane);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float other = __shfl_sync(0xffffffffu, v[i], next);
      if (above) v[i] += other;
    }
    const unsigned done = rank & 1u;
    above &= __ballot_sync(0xffffffffu, done == 0u);
    rank >>= 1;
  }
}

// Adds a float4 to global memory with one vector reduction (sm_90+ red.global.add.v4.f32).
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ void red_add(float* addr, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(a) : "memory");
}

// Warp-aggregated float4 add of `g` to row `row` (16-byte aligned rows of 4 floats) of `base`.
// Lanes with active == false contribute nothing. All 32 lanes must call it together.
__device__ __forceinline__ void scatter_row4(float* base, long long row, bool active, float (&g)[4]) {
  const unsigned act = __ballot_sync(0xffffffffu, active);
  if (act == 0u) return;
  const unsigned lane = threadIdx.x & 31u;
  unsigned peers = 1u << lane;
  if (active) peers = __match_any_sync(act, static_cast<unsigned long long>(row));
  segmented_sum<4>(peers, g);
  if (active && (peers & ((1u << lane) - 1u)) == 0u) {
    red_add_v4(base + row * 4, g[0], g[1], g[2], g[3]);
  }
}

}  // namespace dr
