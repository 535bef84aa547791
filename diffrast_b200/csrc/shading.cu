// Lambert shading from interpolated normals, forward and backward: the optional shading step of a
// fused render-and-fit loop (one pass over the pixels instead of the half-dozen elementwise torch
// kernels of normalise, dot, clamp and multiply, and their backward passes).
//
//   n = normal / |normal|, l = light / |light| (one light per view, or one for all)
//   d = max(0, n . l),  out = color * (ambient + d)
//   grad_color = g * (ambient + d)
//   grad_normal = (s l - (s l . n) n) / |normal|,  s = sum_c g_c color_c where n . l > 0, else 0
//
// A zero normal (a background pixel of the interpolation) shades with the ambient term alone and
// gets no normal gradient. The light is a constant (it gets no gradient). Normals are read with a
// pixel stride, so a channel slice of interpolate's output (out[..., 2:5]) is used in place.
#include <cstdint>

#include "common.cuh"

namespace dr {
namespace {

struct Shade {
  float n[3];    // unit normal (zero for a zero normal)
  float inv;     // 1 / |normal| (zero for a zero normal)
  float l[3];    // unit light direction
  float d;       // max(0, n . l)
};

__device__ __forceinline__ Shade shade(const float* __restrict__ normal, long long stride,
                                       const float* __restrict__ light, long long p,
                                       long long view) {
  Shade s;
  const float* q = normal + p * stride;
  const float nx = __ldcs(q), ny = __ldcs(q + 1), nz = __ldcs(q + 2);
  const float len2 = nx * nx + ny * ny + nz * nz;
  s.inv = len2 > 0.0f ? rsqrtf(len2) : 0.0f;
  s.n[0] = nx * s.inv;
  s.n[1] = ny * s.inv;
  s.n[2] = nz * s.inv;
  const float* lv = light + 3 * view;
  const float lx = __ldg(lv), ly = __ldg(lv + 1), lz = __ldg(lv + 2);
  const float l2 = lx * lx + ly * ly + lz * lz;
  const float il = l2 > 0.0f ? rsqrtf(l2) : 0.0f;
  s.l[0] = lx * il;
  s.l[1] = ly * il;
  s.l[2] = lz * il;
  s.d = fmaxf(0.0f, s.n[0] * s.l[0] + s.n[1] * s.l[1] + s.n[2] * s.l[2]);
  return s;
}

// Grid: x over the pixels of an image, y over the views (no division to find the view).
__global__ void __launch_bounds__(256) lambert_fwd_kernel(
    const float* __restrict__ color, const float* __restrict__ normal, long long normal_stride,
    const float* __restrict__ light, bool light_per_view, float ambient, long long ppi,
    int channels, float* __restrict__ out) {
  const long long view = blockIdx.y;
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= ppi) return;
  const long long p = view * ppi + i;
  const Shade s = shade(normal, normal_stride, light, p, light_per_view ? view : 0);
  const float k = ambient + s.d;
  for (int c = 0; c < channels; ++c)
    __stcs(out + p * channels + c, __ldcs(color + p * channels + c) * k);
}

__global__ void __launch_bounds__(256) lambert_bwd_kernel(
    const float* __restrict__ color, const float* __restrict__ normal, long long normal_stride,
    const float* __restrict__ light, bool light_per_view, float ambient, long long ppi,
    int channels, const float* __restrict__ grad_out, float* __restrict__ grad_color,
    float* __restrict__ grad_normal) {
  const long long view = blockIdx.y;
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= ppi) return;
  const long long p = view * ppi + i;
  const Shade s = shade(normal, normal_stride, light, p, light_per_view ? view : 0);
  const float k = ambient + s.d;
  float sum = 0.0f;
  for (int c = 0; c < channels; ++c) {
    const float g = __ldcs(grad_out + p * channels + c);
    if (grad_color != nullptr) __stcs(grad_color + p * channels + c, g * k);
    sum += g * __ldcs(color + p * channels + c);
  }
  if (grad_normal == nullptr) return;
  // d n / d normal = (I - n n^T) / |normal|, applied to sum * l where the clamp is open.
  const float s_l = s.d > 0.0f ? sum : 0.0f;
  const float gx = s_l * s.l[0], gy = s_l * s.l[1], gz = s_l * s.l[2];
  const float along = gx * s.n[0] + gy * s.n[1] + gz * s.n[2];
  float* gn = grad_normal + 3 * p;
  __stcs(gn, (gx - along * s.n[0]) * s.inv);
  __stcs(gn + 1, (gy - along * s.n[1]) * s.inv);
  __stcs(gn + 2, (gz - along * s.n[2]) * s.inv);
}

bool bad_lambert_args(const float* color, const float* normal, int64_t normal_stride,
                      const float* light, int64_t light_batch, int64_t batch, int32_t height,
                      int32_t width, int32_t channels) {
  if (batch < 0 || height < 0 || width < 0 || channels < 1) return true;
  if (light_batch != 1 && light_batch != batch) return true;
  if (batch > 65535) return true;
  if (batch * static_cast<long long>(height) * width == 0) return false;
  return color == nullptr || normal == nullptr || light == nullptr || normal_stride < 3;
}

}  // namespace
}  // namespace dr

using namespace dr;

extern "C" int dr_lambert_fwd(const float* color, const float* normal, int64_t normal_stride,
                              const float* light, int64_t light_batch, float ambient,
                              int64_t batch, int32_t height, int32_t width, int32_t channels,
                              float* out, void* stream) {
  if (bad_lambert_args(color, normal, normal_stride, light, light_batch, batch, height, width,
                       channels))
    return DR_ERR_INVALID_ARGUMENT;
  const long long ppi = static_cast<long long>(height) * width;
  if (batch * ppi == 0) return DR_OK;
  if (out == nullptr) return DR_ERR_INVALID_ARGUMENT;
  const dim3 grid(blocks_for(ppi, 256), static_cast<unsigned>(batch));
  lambert_fwd_kernel<<<grid, 256, 0, as_stream(stream)>>>(color, normal, normal_stride, light,
                                                          light_batch > 1, ambient, ppi, channels,
                                                          out);
  return launch_status();
}

extern "C" int dr_lambert_bwd(const float* color, const float* normal, int64_t normal_stride,
                              const float* light, int64_t light_batch, float ambient,
                              int64_t batch, int32_t height, int32_t width, int32_t channels,
                              const float* grad_out, float* grad_color, float* grad_normal,
                              void* stream) {
  if (bad_lambert_args(color, normal, normal_stride, light, light_batch, batch, height, width,
                       channels))
    return DR_ERR_INVALID_ARGUMENT;
  const long long ppi = static_cast<long long>(height) * width;
  if (batch * ppi == 0) return DR_OK;
  if (grad_out == nullptr) return DR_ERR_INVALID_ARGUMENT;
  const dim3 grid(blocks_for(ppi, 256), static_cast<unsigned>(batch));
  lambert_bwd_kernel<<<grid, 256, 0, as_stream(stream)>>>(color, normal, normal_stride, light,
                                                          light_batch > 1, ambient, ppi, channels,
                                                          grad_out, grad_color, grad_normal);
  return launch_status();
}

DR_DEFINE_FAULT_QUERY(shading)
