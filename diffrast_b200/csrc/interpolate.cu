// Attribute interpolation on B200 (diffrast reference.py:117-146).
//
// One thread per pixel: the triangle id from rast selects three attribute rows, which are blended
// with the barycentrics; the selected channels also get their screen-space derivatives from
// rast_db. The forward weighted sums use explicitly rounded operations in the reference's order,
// (u a0 + v a1) + ((1 - u) - v) a2, so they round as the reference does for the same rast.
// The backward pass writes the gradients of rast and rast_db per pixel and, when attr needs them,
// scatters attribute gradients with warp-aggregated atomics (lanes showing the same vertex sum
// their contributions first).
#include <cstdint>

#include "common.cuh"
#include "warp_reduce.cuh"

namespace dr {
namespace {

struct Corners {
  bool covered;
  long long row0, row1, row2;  // attribute rows (view * num_vert + vertex)
};

__device__ __forceinline__ Corners corners(const int* __restrict__ tri, int t, long long pixel,
                                           long long pixels_per_image, long long attr_batch,
                                           long long num_vert) {
  Corners k;
  k.covered = t >= 0;
  k.row0 = k.row1 = k.row2 = 0;
  if (k.covered) {
    const long long view = attr_batch == 1 ? 0 : pixel / pixels_per_image;
    const long long base = view * num_vert;
    const int* vt = tri + 3 * static_cast<long long>(t);
    k.row0 = base + checked_index(__ldg(vt), num_vert, kSiteVertex);
    k.row1 = base + checked_index(__ldg(vt + 1), num_vert, kSiteVertex);
    k.row2 = base + checked_index(__ldg(vt + 2), num_vert, kSiteVertex);
  }
  return k;
}

// Up to kRowCache channels of an attribute row held in registers: read once per pixel (with
// 16-byte loads when rows are 16-byte aligned) and reused by the value and derivative outputs.
constexpr int kRowCache = 8;

struct AttrRow {
  float v[kRowCache];
};

__device__ __forceinline__ AttrRow load_row(const float* __restrict__ attr, long long row,
                                            int stride, int channels, bool vec4) {
  AttrRow r;
  const float* p = attr + row * stride;
  if (vec4) {
    const float4 lo = __ldg(reinterpret_cast<const float4*>(p));
    const float4 hi = channels > 4 ? __ldg(reinterpret_cast<const float4*>(p) + 1)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    r.v[0] = lo.x; r.v[1] = lo.y; r.v[2] = lo.z; r.v[3] = lo.w;
    r.v[4] = hi.x; r.v[5] = hi.y; r.v[6] = hi.z; r.v[7] = hi.w;
  } else {
#pragma unroll
    for (int c = 0; c < kRowCache; ++c) r.v[c] = c < channels ? __ldg(p + c) : 0.0f;
  }
  return r;
}

// r.v[c] for a channel index known only at run time, without local memory.
__device__ __forceinline__ float pick(const AttrRow& r, int c) {
  float x = r.v[0];
#pragma unroll
  for (int i = 1; i < kRowCache; ++i)
    if (c == i) x = r.v[i];
  return x;
}

// Copies `count` floats of a block's pixel outputs from shared memory to `dst` (contiguous),
// with 16-byte stores where the addresses allow it.
__device__ __forceinline__ void store_block(float* __restrict__ dst, const float* __restrict__ src,
                                            int count) {
  const bool aligned = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  if (aligned) {
    const int vec = count / 4;
    for (int i = threadIdx.x; i < vec; i += blockDim.x)
      __stcs(reinterpret_cast<float4*>(dst) + i, reinterpret_cast<const float4*>(src)[i]);
    for (int i = vec * 4 + threadIdx.x; i < count; i += blockDim.x) __stcs(dst + i, src[i]);
  } else {
    for (int i = threadIdx.x; i < count; i += blockDim.x) __stcs(dst + i, src[i]);
  }
}

// Each block covers kInterpBlockPixels consecutive pixels with kInterpThreads threads, a thread
// taking kInterpPix of them 128 apart, one load phase at a time (rast and rast_db, then the vertex
// indices, then the attributes), so that the loads of all its pixels are in flight together. With
// `staged`, the block's outputs (out and out_da of its pixels are each one contiguous range) go
// through shared memory so that global stores are coalesced float4s; otherwise each thread
// stores its own channels.
constexpr int kInterpThreads = 128;
constexpr int kInterpPix = 2;
constexpr int kInterpBlockPixels = kInterpThreads * kInterpPix;

__global__ void __launch_bounds__(kInterpThreads) interp_fwd_kernel(
    const float* __restrict__ attr, long long attr_batch, long long num_vert, int channels,
    int attr_stride, bool vec4,
    const float4* __restrict__ rast, const float4* __restrict__ rast_db, const int* __restrict__ tri,
    int num_tri, const int* __restrict__ diff, int num_diff, long long total,
    long long pixels_per_image, float* __restrict__ out, float* __restrict__ out_da, bool staged) {
  extern __shared__ float stage[];
  const long long first = blockIdx.x * static_cast<long long>(kInterpBlockPixels);
  const int nd = 2 * num_diff;
  float* so = stage;                                  // [block pixels][channels]
  float* sd = stage + kInterpBlockPixels * channels;  // [block pixels][2 * num_diff]
  float4 r[kInterpPix], d[kInterpPix];
#pragma unroll
  for (int i = 0; i < kInterpPix; ++i) {
    const long long p = first + i * kInterpThreads + threadIdx.x;
    r[i] = p < total ? __ldcs(rast + p) : make_float4(0.f, 0.f, 0.f, 0.f);
    d[i] = p < total && num_diff > 0 ? __ldcs(rast_db + p) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  Corners k[kInterpPix];
#pragma unroll
  for (int i = 0; i < kInterpPix; ++i) {
    const long long p = first + i * kInterpThreads + threadIdx.x;
    k[i] = corners(tri, p < total ? rast_triangle(r[i].w, num_tri) : -1, p, pixels_per_image,
                   attr_batch, num_vert);
  }
#pragma unroll
  for (int i = 0; i < kInterpPix; ++i) {
    const int slot = i * kInterpThreads + threadIdx.x;
    const long long p = first + slot;
    if (p >= total) continue;
    float* o = staged ? so + slot * channels : out + p * channels;
    float* od = staged ? sd + slot * nd : out_da + p * nd;
    if (!k[i].covered) {
      for (int c = 0; c < channels; ++c) o[c] = 0.0f;
      for (int c = 0; c < nd; ++c) od[c] = 0.0f;
      continue;
    }
    const float u = r[i].x, v = r[i].y;
    const float w2 = sub(sub(1.0f, u), v);
    if (channels <= kRowCache) {
      const AttrRow x0 = load_row(attr, k[i].row0, attr_stride, channels, vec4);
      const AttrRow x1 = load_row(attr, k[i].row1, attr_stride, channels, vec4);
      const AttrRow x2 = load_row(attr, k[i].row2, attr_stride, channels, vec4);
#pragma unroll
      for (int c = 0; c < kRowCache; ++c)
        if (c < channels) o[c] = add(add(mul(u, x0.v[c]), mul(v, x1.v[c])), mul(w2, x2.v[c]));
      for (int j = 0; j < num_diff; ++j) {
        const int c = __ldg(diff + j);
        const float b2 = pick(x2, c);
        const float du = sub(pick(x0, c), b2), dv = sub(pick(x1, c), b2);
        od[2 * j] = add(mul(d[i].x, du), mul(d[i].z, dv));
        od[2 * j + 1] = add(mul(d[i].y, du), mul(d[i].w, dv));
      }
      continue;
    }
    const float* a0 = attr + k[i].row0 * attr_stride;
    const float* a1 = attr + k[i].row1 * attr_stride;
    const float* a2 = attr + k[i].row2 * attr_stride;
    for (int c = 0; c < channels; ++c) {
      o[c] = add(add(mul(u, __ldg(a0 + c)), mul(v, __ldg(a1 + c))), mul(w2, __ldg(a2 + c)));
    }
    for (int j = 0; j < num_diff; ++j) {
      const int c = __ldg(diff + j);
      const float x2 = __ldg(a2 + c);
      const float du = sub(__ldg(a0 + c), x2), dv = sub(__ldg(a1 + c), x2);
      od[2 * j] = add(mul(d[i].x, du), mul(d[i].z, dv));
      od[2 * j + 1] = add(mul(d[i].y, du), mul(d[i].w, dv));
    }
  }
  if (!staged) return;
  __syncthreads();
  const int pixels = static_cast<int>(min(static_cast<long long>(kInterpBlockPixels), total - first));
  store_block(out + first * channels, so, pixels * channels);
  if (nd > 0) store_block(out_da + first * nd, sd, pixels * nd);
}

// Adds value to grad_attr[row * channels + c] with the lanes of the warp that share `row` summed
// first. All lanes must call it together with the same c.
__device__ __forceinline__ void scatter_attr(float* __restrict__ grad_attr, long long row,
                                             unsigned peers, bool active, int channels, int c,
                                             float value) {
  float v[1] = {value};
  segmented_sum<1>(peers, v);
  const unsigned lane = threadIdx.x & 31u;
  if (active && (peers & ((1u << lane) - 1u)) == 0u) red_add(grad_attr + row * channels + c, v[0]);
}

// The gradients of interpolate's outputs, given in pieces: whole pixel records of out
// ([P, channels]) and out_da ([P, 2 num_diff]), either of which may be missing, plus compact
// channel ranges handed over by a consumer that read a channel slice of an output (part:
// [P, part_count] for out channels part_first ..; part_da: [P, da_count] for out_da channels
// da_first ..), as texture does with interpolated uv and uv_da. Missing pieces are zero, and
// channels no piece covers are not visited when no whole record is given.
struct GradParts {
  const float* out;
  const float* out_da;
  const float* part;
  int part_first, part_count;
  const float* part_da;
  int da_first, da_count;
};

__device__ __forceinline__ float part_value(const float* __restrict__ part, int first, int count,
                                            long long p, int c) {
  const int i = c - first;
  return (part != nullptr && i >= 0 && i < count) ? part[p * count + i] : 0.0f;
}

__global__ void __launch_bounds__(256, 6) interp_bwd_kernel(
    const float* __restrict__ attr, long long attr_batch, long long num_vert, int channels,
    const float4* __restrict__ rast, const float4* __restrict__ rast_db, const int* __restrict__ tri,
    int num_tri, const int* __restrict__ diff, int num_diff, long long total,
    long long pixels_per_image, const GradParts gp, float* __restrict__ grad_attr,
    float4* __restrict__ grad_rast, float4* __restrict__ grad_db) {
  const long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const bool in_range = p < total;
  const float4 r = in_range ? __ldcs(rast + p) : make_float4(0.f, 0.f, 0.f, 0.f);
  const int t = in_range ? rast_triangle(r.w, num_tri) : -1;
  const Corners k = corners(tri, t, p, pixels_per_image, attr_batch, num_vert);
  const float u = r.x, v = r.y, w2 = 1.0f - u - v;
  const float* a0 = attr + k.row0 * channels;
  const float* a1 = attr + k.row1 * channels;
  const float* a2 = attr + k.row2 * channels;

  // Lanes that share a vertex row; computed once, reused for every channel.
  const unsigned lane = threadIdx.x & 31u;
  unsigned peers[3] = {1u << lane, 1u << lane, 1u << lane};
  if (grad_attr != nullptr) {
    const unsigned act = __ballot_sync(0xffffffffu, k.covered);
    if (k.covered) {
      peers[0] = __match_any_sync(act, static_cast<unsigned long long>(k.row0));
      peers[1] = __match_any_sync(act, static_cast<unsigned long long>(k.row1));
      peers[2] = __match_any_sync(act, static_cast<unsigned long long>(k.row2));
    }
  }

  // Channels that can carry a gradient (uniform over the grid).
  const int c_lo = gp.out != nullptr ? 0 : max(0, gp.part_first);
  const int c_hi = gp.out != nullptr ? channels
                                     : (gp.part != nullptr ? min(channels, gp.part_first + gp.part_count) : 0);
  float gu = 0.0f, gv = 0.0f;
  for (int c = c_lo; c < c_hi; ++c) {
    float g = 0.0f, x0 = 0.0f, x1 = 0.0f, x2 = 0.0f;
    if (k.covered) {
      if (gp.out != nullptr) g = gp.out[p * channels + c];
      g += part_value(gp.part, gp.part_first, gp.part_count, p, c);
      x0 = __ldg(a0 + c);
      x1 = __ldg(a1 + c);
      x2 = __ldg(a2 + c);
      gu += g * (x0 - x2);
      gv += g * (x1 - x2);
    }
    if (grad_attr != nullptr) {
      scatter_attr(grad_attr, k.row0, peers[0], k.covered, channels, c, g * u);
      scatter_attr(grad_attr, k.row1, peers[1], k.covered, channels, c, g * v);
      scatter_attr(grad_attr, k.row2, peers[2], k.covered, channels, c, g * w2);
    }
  }
  if (in_range) __stcs(grad_rast + p, make_float4(gu, gv, 0.0f, 0.0f));

  if (gp.out_da == nullptr && gp.part_da == nullptr) return;
  // Differentiated channel pairs (2 j, 2 j + 1) that can carry a gradient.
  const int j_lo = gp.out_da != nullptr ? 0 : max(0, gp.da_first) / 2;
  const int j_hi = gp.out_da != nullptr ? num_diff
                                        : min(num_diff, (gp.da_first + gp.da_count + 1) / 2);
  const float4 d = k.covered ? __ldcs(rast_db + p) : make_float4(0.f, 0.f, 0.f, 0.f);
  float g_dudx = 0.0f, g_dudy = 0.0f, g_dvdx = 0.0f, g_dvdy = 0.0f;
  for (int j = j_lo; j < j_hi; ++j) {
    float gx = 0.0f, gy = 0.0f, du = 0.0f, dv = 0.0f;
    int c = 0;
    if (k.covered) {
      c = __ldg(diff + j);
      if (gp.out_da != nullptr) {
        gx = gp.out_da[(p * num_diff + j) * 2];
        gy = gp.out_da[(p * num_diff + j) * 2 + 1];
      }
      gx += part_value(gp.part_da, gp.da_first, gp.da_count, p, 2 * j);
      gy += part_value(gp.part_da, gp.da_first, gp.da_count, p, 2 * j + 1);
      const float x2 = __ldg(a2 + c);
      du = __ldg(a0 + c) - x2;
      dv = __ldg(a1 + c) - x2;
      g_dudx += gx * du;
      g_dudy += gy * du;
      g_dvdx += gx * dv;
      g_dvdy += gy * dv;
    }
    if (grad_attr != nullptr) {
      // All lanes agree on j; c differs only between covered and uncovered lanes, and an
      // uncovered lane adds nothing, so a shared c per group holds.
      const float g0 = gx * d.x + gy * d.y;
      const float g1 = gx * d.z + gy * d.w;
      scatter_attr(grad_attr, k.row0, peers[0], k.covered, channels, c, g0);
      scatter_attr(grad_attr, k.row1, peers[1], k.covered, channels, c, g1);
      scatter_attr(grad_attr, k.row2, peers[2], k.covered, channels, c, -(g0 + g1));
    }
  }
  if (in_range) __stcs(grad_db + p, make_float4(g_dudx, g_dudy, g_dvdx, g_dvdy));
}

bool bad_interp_args(const float* attr, int64_t attr_batch, int64_t num_vert, int32_t channels,
                     const float* rast, const float* rast_db, const int32_t* tri, int64_t num_tri,
                     const int32_t* diff, int32_t num_diff, int64_t batch, int32_t height,
                     int32_t width) {
  if (attr_batch < 1 || num_vert < 0 || channels < 0 || num_tri < 0 || num_diff < 0 || batch < 0 ||
      height < 0 || width < 0)
    return true;
  if (attr_batch != 1 && attr_batch != batch) return true;
  if (num_tri >= (1LL << 31)) return true;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total > 0 && (rast == nullptr || (reinterpret_cast<uintptr_t>(rast) & 15u) != 0)) return true;
  if (num_diff > 0 && (diff == nullptr || rast_db == nullptr ||
                       (reinterpret_cast<uintptr_t>(rast_db) & 15u) != 0))
    return true;
  if (num_tri > 0 && tri == nullptr) return true;
  if (channels > 0 && num_vert > 0 && attr == nullptr) return true;
  return false;
}

}  // namespace
}  // namespace dr

using namespace dr;

extern "C" int dr_interpolate_fwd(const float* attr, int64_t attr_batch, int64_t num_vert,
                                  int32_t channels, int32_t attr_stride, const float* rast,
                                  const float* rast_db,
                                  const int32_t* tri, int64_t num_tri, const int32_t* diff,
                                  int32_t num_diff, int64_t batch, int32_t height, int32_t width,
                                  float* out, float* out_da, void* stream) {
  if (bad_interp_args(attr, attr_batch, num_vert, channels, rast, rast_db, tri, num_tri, diff,
                      num_diff, batch, height, width) ||
      out == nullptr || (num_diff > 0 && out_da == nullptr))
    return DR_ERR_INVALID_ARGUMENT;
  if (attr_stride == 0) attr_stride = channels;
  if (attr_stride < channels) return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0) return DR_OK;
  const bool vec4 = attr_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(attr) & 15u) == 0;
  const size_t stage_bytes =
      sizeof(float) * kInterpBlockPixels * (static_cast<size_t>(channels) + 2 * num_diff);
  const bool staged = stage_bytes <= 48 * 1024;
  interp_fwd_kernel<<<blocks_for(total, kInterpBlockPixels), kInterpThreads,
                      staged ? stage_bytes : 0, as_stream(stream)>>>(
      attr, attr_batch, num_vert, channels, attr_stride, vec4, reinterpret_cast<const float4*>(rast),
      reinterpret_cast<const float4*>(rast_db), tri, static_cast<int>(num_tri), diff, num_diff,
      total, static_cast<long long>(height) * width, out, out_da, staged);
  return launch_status();
}

namespace dr {
namespace {

int launch_interp_bwd(const float* attr, int64_t attr_batch, int64_t num_vert, int32_t channels,
                      const float* rast, const float* rast_db, const int32_t* tri,
                      int64_t num_tri, const int32_t* diff, int32_t num_diff, int64_t batch,
                      int32_t height, int32_t width, const GradParts& gp, float* grad_attr,
                      float* grad_rast, float* grad_db, cudaStream_t s) {
  const bool any_da = gp.out_da != nullptr || gp.part_da != nullptr;
  if (bad_interp_args(attr, attr_batch, num_vert, channels, rast, rast_db, tri, num_tri, diff,
                      any_da ? num_diff : 0, batch, height, width) ||
      grad_rast == nullptr || (any_da && (grad_db == nullptr || num_diff == 0)) ||
      (gp.part != nullptr && (gp.part_first < 0 || gp.part_count < 1 ||
                              gp.part_first + gp.part_count > channels)) ||
      (gp.part_da != nullptr && (gp.da_first < 0 || gp.da_count < 1 ||
                                 gp.da_first + gp.da_count > 2 * num_diff)))
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0) return DR_OK;
  interp_bwd_kernel<<<blocks_for(total, 256), 256, 0, s>>>(
      attr, attr_batch, num_vert, channels, reinterpret_cast<const float4*>(rast),
      reinterpret_cast<const float4*>(rast_db), tri, static_cast<int>(num_tri), diff,
      any_da ? num_diff : 0, total, static_cast<long long>(height) * width, gp, grad_attr,
      reinterpret_cast<float4*>(grad_rast), reinterpret_cast<float4*>(grad_db));
  return launch_status();
}

}  // namespace
}  // namespace dr

extern "C" int dr_interpolate_bwd(const float* attr, int64_t attr_batch, int64_t num_vert,
                                  int32_t channels, const float* rast, const float* rast_db,
                                  const int32_t* tri, int64_t num_tri, const int32_t* diff,
                                  int32_t num_diff, int64_t batch, int32_t height, int32_t width,
                                  const float* grad_out, const float* grad_out_da,
                                  float* grad_attr, float* grad_rast, float* grad_db,
                                  void* stream) {
  if (grad_out == nullptr) return DR_ERR_INVALID_ARGUMENT;
  const GradParts gp{grad_out, grad_out_da, nullptr, 0, 0, nullptr, 0, 0};
  return launch_interp_bwd(attr, attr_batch, num_vert, channels, rast, rast_db, tri, num_tri,
                           diff, num_diff, batch, height, width, gp, grad_attr, grad_rast,
                           grad_db, as_stream(stream));
}

extern "C" int dr_interpolate_bwd_parts(const float* attr, int64_t attr_batch, int64_t num_vert,
                                        int32_t channels, const float* rast, const float* rast_db,
                                        const int32_t* tri, int64_t num_tri, const int32_t* diff,
                                        int32_t num_diff, int64_t batch, int32_t height,
                                        int32_t width, const float* grad_out,
                                        const float* grad_out_da, const float* part,
                                        int32_t part_first, int32_t part_count,
                                        const float* part_da, int32_t da_first, int32_t da_count,
                                        float* grad_attr, float* grad_rast, float* grad_db,
                                        void* stream) {
  const GradParts gp{grad_out, grad_out_da, part, part_first, part_count,
                     part_da, da_first, da_count};
  return launch_interp_bwd(attr, attr_batch, num_vert, channels, rast, rast_db, tri, num_tri,
                           diff, num_diff, batch, height, width, gp, grad_attr, grad_rast,
                           grad_db, as_stream(stream));
}
DR_DEFINE_FAULT_QUERY(interpolate)
