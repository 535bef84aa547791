// Shared device helpers of the diffrast_b200 CUDA library (sm_100a).
//
// Visibility decisions (coverage, tie rules, area tolerance, antialias edge tests) are made with
// explicitly rounded float32 operations (__fmul_rn / __fadd_rn / __fsub_rn / __fdiv_rn), which the
// compiler never contracts into fused multiply-adds. They reproduce, operation for operation, the
// float32 arithmetic of diffrast's reference backend (src/diffrast/backends/reference.py:293-365,
// :675-765), so triangle ids and the antialias edge set agree bit for bit. Everything else (the
// barycentric resolve, interpolation, texturing, gradients) uses ordinary float arithmetic.
//
// Cache policy: per-pixel streams that a kernel reads or writes once (rast, rast_db, keys, uv,
// uv_da, upstream gradients, outputs) use the evict-first hints (__ldcs / __stcs), so that they do
// not push the data the kernels gather many times (vertices, attribute rows, texels) out of L2.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/diffrast_b200.h"

// Checked build (nvcc -DDR_CHECKED=1, loaded with DIFFRAST_B200_CHECK=1): every index that comes
// from the data (vertex indices read from tri, triangle ids read from rast or the visibility keys,
// opposite vertices, attribute rows, texel offsets, key offsets) is checked against the size of
// the buffer it addresses before the access. A failed check does not trap: it records
// (site << 48) | index in this translation unit's fault word (the first one wins) and the access
// goes to element 0 instead, so the kernel finishes and the host reports the fault
// (dr_check_faults). Ordinary builds compile the checks away.
#ifndef DR_CHECKED
#define DR_CHECKED 0
#endif

namespace dr {

// Sites of the checked build's bounds checks (the high 16 bits of a fault record).
enum CheckSite : int {
  kSiteTriangle = 1,    // triangle index into tri (from rast, keys or a work list)
  kSiteVertex = 2,      // vertex index read from tri, into pos or attr rows
  kSiteOpposite = 3,    // vertex index read from the opposite-vertex table
  kSiteTexel = 4,       // texel offset into a texture level (or its gradient)
  kSitePixel = 5,       // pixel offset into the visibility keys
  kSiteAttrRow = 6,     // attribute row (view * vertices + vertex)
};

#if DR_CHECKED
static __device__ unsigned long long g_fault;

__device__ __forceinline__ long long checked_index(long long index, long long bound, int site) {
  if (index >= 0 && index < bound) return index;
  atomicCAS(&g_fault, 0ull,
            (static_cast<unsigned long long>(site) << 48) |
                (static_cast<unsigned long long>(index) & 0xFFFFFFFFFFFFull));
  return 0;
}

// Reads and clears this translation unit's fault word (after the device has finished).
#define DR_DEFINE_FAULT_QUERY(unit)                                                        \
  extern "C" int dr_fault_##unit(uint64_t* fault) {                                       \
    unsigned long long value = 0, zero = 0;                                                \
    cudaError_t err = cudaMemcpyFromSymbol(&value, ::dr::g_fault, sizeof(value));         \
    if (err == cudaSuccess) err = cudaMemcpyToSymbol(::dr::g_fault, &zero, sizeof(zero)); \
    *fault = value;                                                                        \
    return static_cast<int>(err);                                                          \
  }
#else
__device__ __forceinline__ long long checked_index(long long index, long long, int) {
  return index;
}
#define DR_DEFINE_FAULT_QUERY(unit)                    \
  extern "C" int dr_fault_##unit(uint64_t* fault) {   \
    *fault = 0;                                        \
    return 0;                                          \
  }
#endif

// Empty visibility key: no triangle covers the pixel (INT64_MAX, as a signed 64-bit key).
constexpr long long kEmptyKey = 0x7FFFFFFFFFFFFFFFLL;
// Depth field (upper 32 bits) of a poisoned key: the ordered bits of a quiet NaN, which no
// covered pixel can have (its depth lies in [-1, 1]) and which sorts below the empty key. Keys
// of a graph-captured pass that outgrew its binning capacity carry it, and the resolve pass
// turns it into NaN barycentrics, depth and derivatives.
constexpr int kPoisonDepth = 0x7FC00000;
// Two float32 epsilons: the area tolerance of the reference (reference.py:27).
constexpr float kAreaTolerance = 2.0f * 1.1920928955078125e-07f;
// Four float32 epsilons: the edge-tie slack of antialiasing (reference.py:35, :746).
constexpr float kEdgeTie = 4.0f * 1.1920928955078125e-07f;
// Slope margin deciding which axis handles a 45 degree edge (reference.py:32).
constexpr float kAxisTie = 1.0001f;
// Footprint and direction-derivative saturation (reference.py:402, _cube.py:36).
constexpr float kLimit = 1e18f;
// Screen tiles of the binned visibility pass.
constexpr int kTile = 16;
// Triangles per tile work item (one per thread of a 16x16 tile block).
constexpr int kChunk = 256;
// Triangles whose pixel box holds at most kWarpPixels pixels are rasterized directly by the setup
// warp (its lanes share the (triangle, pixel) items of all such triangles of the warp); larger
// ones are binned into screen tiles.
constexpr int kWarpPixels = 512;

__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float dvd(float a, float b) { return __fdiv_rn(a, b); }
// a * b - c * d with every product and difference rounded separately.
__device__ __forceinline__ float cross2(float a, float b, float c, float d) {
  return sub(mul(a, b), mul(c, d));
}
// torch.maximum semantics: NaN propagates.
__device__ __forceinline__ float nanmax(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}

// NDC centre of pixel i of a row or column of n pixels: (2 i + 1) / n - 1, as in
// reference.py:268-271 (float32 arange * 2 + 1, IEEE division, then minus one).
__device__ __forceinline__ float pixel_centre(int i, int n) {
  float v = add(mul(static_cast<float>(i), 2.0f), 1.0f);
  return sub(dvd(v, static_cast<float>(n)), 1.0f);
}

struct Vert {
  float x, y, z, w;
};

__device__ __forceinline__ Vert load_vert(const float* __restrict__ pos, long long index) {
  float4 v = __ldg(reinterpret_cast<const float4*>(pos) + index);
  return {v.x, v.y, v.z, v.w};
}

__device__ __forceinline__ bool finite4(const Vert& v) {
  return isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
}

// Packed key of a covered pixel: order-preserving integer of the float32 depth in the high word
// (negative floats have their magnitude bits flipped, -0 maps to 0) and the triangle index in
// the low word. A signed 64-bit minimum then keeps the nearest triangle and, at equal depth,
// the lowest index, which is the reference's rule (reference.py:368-397).
__device__ __forceinline__ long long pack_key(float depth, int tri) {
  int bits = __float_as_int(depth);
  int ordered = bits >= 0 ? bits : (bits ^ 0x7FFFFFFF);
  if (depth == 0.0f) ordered = 0;
  return (static_cast<long long>(ordered) << 32) | static_cast<unsigned int>(tri);
}

// Coverage and depth of one triangle at one pixel centre, returning the packed key or the empty
// key. The float32 operations and their order are those of the reference's coverage test
// (reference.py:293-365): edge functions e = a x c with a = x - px w and c = y - py w, the
// top-left rule for exact zeros from the sign of the edge's screen gradient, the area tolerance
// against the magnitude of the terms, the sign of the interpolated w and -1 <= z/w <= 1.
// Non-finite vertices are rejected by the caller. All conditions are conjunctions of pure
// functions of the same rounded values, so testing the cheap edge signs first and returning early
// changes no result; it only skips the tolerance and depth arithmetic for pixels outside.
//
// reach_x and reach_y are the per-triangle maxima of |x| + |w| and |y| + |w| over the vertices
// (coverage_reach), which callers testing many pixels of one triangle compute once.
__device__ __forceinline__ long long coverage_key(const Vert& v0, const Vert& v1, const Vert& v2,
                                                  float px, float py, int tri, float reach_x,
                                                  float reach_y) {
  const float a0 = sub(v0.x, mul(px, v0.w)), a1 = sub(v1.x, mul(px, v1.w)),
              a2 = sub(v2.x, mul(px, v2.w));
  const float c0 = sub(v0.y, mul(py, v0.w)), c1 = sub(v1.y, mul(py, v1.w)),
              c2 = sub(v2.y, mul(py, v2.w));
  const float e0 = cross2(a1, c2, a2, c1);
  const float e1 = cross2(a2, c0, a0, c2);
  const float e2 = cross2(a0, c1, a1, c0);
  const float s = add(add(e0, e1), e2);
  const bool positive = s > 0.0f;
  // A nonzero edge function must have the sign of the area (NaN fails both tests).
  if (positive ? !(e0 >= 0.0f && e1 >= 0.0f && e2 >= 0.0f)
               : !(e0 <= 0.0f && e1 <= 0.0f && e2 <= 0.0f))
    return kEmptyKey;
  // Edge k runs from vertex i = k + 1 to j = k + 2; a pixel exactly on it is decided by the
  // direction of its screen gradient.
  auto on_edge_inside = [&](float ai, float ci, float wi, float aj, float cj, float wj) {
    const float gx = cross2(ci, wj, cj, wi);
    const float gy = cross2(aj, wi, ai, wj);
    const float q = (gx == 0.0f) ? gy : gx;
    return positive ? (q > 0.0f) : (q < 0.0f);
  };
  if (e0 == 0.0f && !on_edge_inside(a1, c1, v1.w, a2, c2, v2.w)) return kEmptyKey;
  if (e1 == 0.0f && !on_edge_inside(a2, c2, v2.w, a0, c0, v0.w)) return kEmptyKey;
  if (e2 == 0.0f && !on_edge_inside(a0, c0, v0.w, a1, c1, v1.w)) return kEmptyKey;

  const float span_x = add(add(fabsf(a0), fabsf(a1)), fabsf(a2));
  const float span_y = add(add(fabsf(c0), fabsf(c1)), fabsf(c2));
  const float bound = mul(add(mul(reach_x, span_y), mul(span_x, add(reach_y, span_y))), kAreaTolerance);
  if (!(fabsf(s) > bound)) return kEmptyKey;
  const float ew = add(add(mul(e0, v0.w), mul(e1, v1.w)), mul(e2, v2.w));
  if (positive ? !(ew > 0.0f) : !(ew < 0.0f)) return kEmptyKey;
  const float ez = add(add(mul(e0, v0.z), mul(e1, v1.z)), mul(e2, v2.z));
  const float depth = dvd(ez, ew);
  if (!(depth >= -1.0f && depth <= 1.0f)) return kEmptyKey;
  return pack_key(depth, tri);
}

// Largest |x| + |w| and |y| + |w| over the three vertices, the magnitude terms of the area
// tolerance (reference.py:321-327).
__device__ __forceinline__ float2 coverage_reach(const Vert& v0, const Vert& v1, const Vert& v2) {
  return make_float2(
      nanmax(nanmax(add(fabsf(v0.x), fabsf(v0.w)), add(fabsf(v1.x), fabsf(v1.w))),
             add(fabsf(v2.x), fabsf(v2.w))),
      nanmax(nanmax(add(fabsf(v0.y), fabsf(v0.w)), add(fabsf(v1.y), fabsf(v1.w))),
             add(fabsf(v2.y), fabsf(v2.w))));
}

__device__ __forceinline__ long long coverage_key(const Vert& v0, const Vert& v1, const Vert& v2,
                                                  float px, float py, int tri) {
  const float2 r = coverage_reach(v0, v1, v2);
  return coverage_key(v0, v1, v2, px, py, tri, r.x, r.y);
}

// Triangle index of a rast pixel: round(id + 1) - 1 (round half to even, like torch.round), or
// -1 for background, negative values and ids past the end of tri (reference.py:127-129).
__device__ __forceinline__ int rast_triangle(float id_plus_one, int num_tri) {
  const float r = rintf(id_plus_one);
  if (!(r >= 1.0f) || r > static_cast<float>(num_tri)) return -1;
  return static_cast<int>(r) - 1;
}

// Status of the launches just made on this thread.
inline int launch_status() {
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? DR_OK : static_cast<int>(err);
}

inline cudaStream_t as_stream(void* stream) { return reinterpret_cast<cudaStream_t>(stream); }

inline unsigned int blocks_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  return static_cast<unsigned int>(b < 1 ? 1 : b);
}

// Blocks of `kernel` that fit on the current device at once (all SMs, `threads` per block): the
// grid of a persistent kernel.
template <typename Kernel>
unsigned int resident_blocks(Kernel kernel, int threads, size_t shared_bytes = 0) {
  int device = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, shared_bytes) !=
          cudaSuccess)
    return 148u;
  return static_cast<unsigned int>(max(sms, 1) * max(per_sm, 1));
}

// Bytes rounded up to the 256-byte alignment of every workspace sub-buffer.
inline size_t align256(size_t bytes) { return (bytes + 255) & ~static_cast<size_t>(255); }

}  // namespace dr
