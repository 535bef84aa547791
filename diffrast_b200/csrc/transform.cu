// World-to-clip transform of one shared vertex buffer by per-view 4x4 matrices, forward and
// backward: the step ahead of the rasterizer in a multi-view fit (diffrast examples/common.py:
// 320-323, `to_clip`: homogeneous positions times the transposed matrices).
//
//   forward   clip[b, v] = M[b] (p[v], 1)                       row-major M, float4 rows out
//   backward  grad_p[v] = sum_b (M[b]^T grad_clip[b, v])[0:3]   one thread per vertex, all views
//             grad_M[b] = sum_v grad_clip[b, v] (p[v], 1)^T     block partial sums, then reductions
//
// Every kernel streams the [batch, vertices, 4] clip buffer (or its gradient) once with coalesced
// 16-byte accesses; the positions (12 bytes per vertex) and the matrices stay in L2 / shared memory.
#include <cstdint>

#include "common.cuh"

namespace dr {
namespace {

constexpr int kViewsPerPass = 64;  // matrices staged in shared memory at a time

__global__ void __launch_bounds__(256) to_clip_fwd_kernel(const float* __restrict__ p, int num_vert,
                                                          const float* __restrict__ m,
                                                          float4* __restrict__ out) {
  __shared__ float mat[16];
  const long long b = blockIdx.y;
  if (threadIdx.x < 16) mat[threadIdx.x] = __ldg(m + b * 16 + threadIdx.x);
  __syncthreads();
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < num_vert; v += gridDim.x * blockDim.x) {
    const float x = __ldg(p + 3LL * v), y = __ldg(p + 3LL * v + 1), z = __ldg(p + 3LL * v + 2);
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      r[i] = fmaf(mat[4 * i + 2], z, fmaf(mat[4 * i + 1], y, mat[4 * i] * x)) + mat[4 * i + 3];
    out[b * num_vert + v] = make_float4(r[0], r[1], r[2], r[3]);
  }
}

__global__ void __launch_bounds__(256) to_clip_bwd_pos_kernel(const float4* __restrict__ g,
                                                              int num_vert,
                                                              const float* __restrict__ m,
                                                              int batch, float* __restrict__ grad_p) {
  __shared__ float mat[kViewsPerPass][16];
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  float gx = 0.0f, gy = 0.0f, gz = 0.0f;
  for (int b0 = 0; b0 < batch; b0 += kViewsPerPass) {
    const int nb = min(kViewsPerPass, batch - b0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * 16; i += blockDim.x)
      mat[i >> 4][i & 15] = __ldg(m + static_cast<long long>(b0) * 16 + i);
    __syncthreads();
    if (v >= num_vert) continue;
#pragma unroll 8
    for (int j = 0; j < nb; ++j) {
      const float4 q = __ldcs(g + static_cast<long long>(b0 + j) * num_vert + v);
      const float* M = mat[j];
      gx = fmaf(q.x, M[0], fmaf(q.y, M[4], fmaf(q.z, M[8], fmaf(q.w, M[12], gx))));
      gy = fmaf(q.x, M[1], fmaf(q.y, M[5], fmaf(q.z, M[9], fmaf(q.w, M[13], gy))));
      gz = fmaf(q.x, M[2], fmaf(q.y, M[6], fmaf(q.z, M[10], fmaf(q.w, M[14], gz))));
    }
  }
  if (v >= num_vert) return;
  grad_p[3LL * v] = gx;
  grad_p[3LL * v + 1] = gy;
  grad_p[3LL * v + 2] = gz;
}

// grad_M[b] (zeroed by the caller) += the block's partial sum over its vertices.
__global__ void __launch_bounds__(256) to_clip_bwd_mat_kernel(const float4* __restrict__ g,
                                                              const float* __restrict__ p,
                                                              int num_vert,
                                                              float* __restrict__ grad_m) {
  __shared__ float part[8][16];
  const long long b = blockIdx.y;
  float acc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) acc[k] = 0.0f;
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < num_vert; v += gridDim.x * blockDim.x) {
    const float4 q = __ldg(g + b * num_vert + v);
    const float h[4] = {__ldg(p + 3LL * v), __ldg(p + 3LL * v + 1), __ldg(p + 3LL * v + 2), 1.0f};
    const float gq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[4 * i + j] = fmaf(gq[i], h[j], acc[4 * i + j]);
  }
#pragma unroll
  for (int k = 0; k < 16; ++k)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int k = 0; k < 16; ++k) part[warp][k] = acc[k];
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    float s = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += part[w][threadIdx.x];
    atomicAdd(grad_m + b * 16 + threadIdx.x, s);
  }
}

bool bad_transform_args(const float* p, int64_t num_vert, const float* m, int64_t batch) {
  if (num_vert < 0 || batch < 0 || num_vert >= (1LL << 31) || batch >= 65536) return true;
  if (num_vert > 0 && batch > 0 && (p == nullptr || m == nullptr)) return true;
  return false;
}

}  // namespace
}  // namespace dr

using namespace dr;

extern "C" int dr_to_clip_fwd(const float* positions, int64_t num_vert, const float* matrices,
                              int64_t batch, float* out, void* stream) {
  if (bad_transform_args(positions, num_vert, matrices, batch)) return DR_ERR_INVALID_ARGUMENT;
  if (num_vert == 0 || batch == 0) return DR_OK;
  if (out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15u) != 0) return DR_ERR_INVALID_ARGUMENT;
  const unsigned bx = min(blocks_for(num_vert, 256), 1024u);
  to_clip_fwd_kernel<<<dim3(bx, static_cast<unsigned>(batch)), 256, 0, as_stream(stream)>>>(
      positions, static_cast<int>(num_vert), matrices, reinterpret_cast<float4*>(out));
  return launch_status();
}

extern "C" int dr_to_clip_bwd(const float* grad_out, const float* positions, int64_t num_vert,
                              const float* matrices, int64_t batch, float* grad_positions,
                              float* grad_matrices, void* stream) {
  if (bad_transform_args(positions, num_vert, matrices, batch)) return DR_ERR_INVALID_ARGUMENT;
  if (num_vert > 0 && batch > 0 &&
      (grad_out == nullptr || (reinterpret_cast<uintptr_t>(grad_out) & 15u) != 0))
    return DR_ERR_INVALID_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  const int nv = static_cast<int>(num_vert);
  if (grad_positions != nullptr && num_vert > 0) {
    if (batch == 0) {
      cudaError_t err = cudaMemsetAsync(grad_positions, 0, 12 * num_vert, s);
      if (err != cudaSuccess) return static_cast<int>(err);
    } else {
      to_clip_bwd_pos_kernel<<<blocks_for(num_vert, 256), 256, 0, s>>>(
          reinterpret_cast<const float4*>(grad_out), nv, matrices, static_cast<int>(batch),
          grad_positions);
    }
  }
  if (grad_matrices != nullptr && batch > 0) {
    cudaError_t err = cudaMemsetAsync(grad_matrices, 0, 64 * batch, s);
    if (err != cudaSuccess) return static_cast<int>(err);
    if (num_vert > 0) {
      const unsigned bx = min(blocks_for(num_vert, 256 * 16), 148u);
      to_clip_bwd_mat_kernel<<<dim3(bx, static_cast<unsigned>(batch)), 256, 0, s>>>(
          reinterpret_cast<const float4*>(grad_out), positions, nv, grad_matrices);
    }
  }
  return launch_status();
}
DR_DEFINE_FAULT_QUERY(transform)
