// Edge adjacency of an index buffer (diffrast reference.py:768-787) with an open-addressing hash
// table on 64-bit vertex-pair keys: per key a count and the first two edges that carry it. Edge
// 3 t + k (opposite vertex k) gets the other edge of its key when exactly two edges share it, -1
// otherwise. No sort is needed and the result is deterministic. Included by the translation
// units that build the table.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace dr {
namespace {

constexpr unsigned long long kNoKey = ~0ull;

__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

__device__ __forceinline__ unsigned long long edge_key(const int* __restrict__ tri, long long e) {
  const long long t = e / 3;
  const int k = static_cast<int>(e - 3 * t);
  const unsigned a = static_cast<unsigned>(__ldg(tri + 3 * t + (k + 1) % 3));
  const unsigned b = static_cast<unsigned>(__ldg(tri + 3 * t + (k + 2) % 3));
  const unsigned lo = min(a, b), hi = max(a, b);
  return (static_cast<unsigned long long>(lo) << 32) | hi;
}

__global__ void __launch_bounds__(256) edge_insert_kernel(const int* __restrict__ tri,
                                                          long long num_edges,
                                                          unsigned long long* __restrict__ keys,
                                                          int* __restrict__ count,
                                                          int* __restrict__ first,
                                                          int* __restrict__ second,
                                                          unsigned long long mask) {
  const long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (e >= num_edges) return;
  const unsigned long long key = edge_key(tri, e);
  unsigned long long h = mix64(key) & mask;
  // The table holds at least twice as many slots as edges, so a free or matching slot is found
  // within `mask + 1` probes.
  for (unsigned long long probe = 0; probe <= mask; ++probe) {
    const unsigned long long prev = atomicCAS(keys + h, kNoKey, key);
    if (prev == kNoKey || prev == key) {
      const int c = atomicAdd(count + h, 1);
      if (c == 0) first[h] = static_cast<int>(e);
      else if (c == 1) second[h] = static_cast<int>(e);
      return;
    }
    h = (h + 1) & mask;
  }
}

__global__ void __launch_bounds__(256) edge_lookup_kernel(const int* __restrict__ tri,
                                                          long long num_edges,
                                                          const unsigned long long* __restrict__ keys,
                                                          const int* __restrict__ count,
                                                          const int* __restrict__ first,
                                                          const int* __restrict__ second,
                                                          unsigned long long mask,
                                                          long long* __restrict__ out) {
  const long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (e >= num_edges) return;
  const unsigned long long key = edge_key(tri, e);
  unsigned long long h = mix64(key) & mask;
  long long result = -1;
  for (unsigned long long probe = 0; probe <= mask; ++probe) {
    const unsigned long long k = keys[h];
    if (k == key) {
      if (count[h] == 2) result = first[h] == e ? second[h] : first[h];
      break;
    }
    if (k == kNoKey) break;
    h = (h + 1) & mask;
  }
  out[e] = result;
}

unsigned long long table_slots(int64_t num_tri) {
  unsigned long long slots = 64;
  while (slots < 2ull * 3ull * static_cast<unsigned long long>(num_tri)) slots <<= 1;
  return slots;
}

}  // namespace
}  // namespace dr
