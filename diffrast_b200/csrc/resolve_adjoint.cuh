// The rasterizer's backward pass for one covered pixel (reference.py:69-114, the adjoint of
// rasterize_from_ids; backends/_triton_resolve.py:120-244): gradients of the clip-space vertices
// of the pixel's triangle from the gradients of its rast (gr: barycentrics u, v and depth z / w)
// and, with has_db, of its rast_db (gd), analytic adjoints of e = a x c, b = e / s, z / w =
// (e . z) / (e . w) and of the screen derivatives de/dx = c x w, de/dy = w x a. Shared by the
// rasterizer's backward kernel and the texture backward kernel that runs it in its epilogue.
#pragma once

#include "common.cuh"

namespace dr {

__device__ __forceinline__ void cross3(const float u[3], const float v[3], float out[3]) {
  out[0] = u[1] * v[2] - u[2] * v[1];
  out[1] = u[2] * v[0] - u[0] * v[2];
  out[2] = u[0] * v[1] - u[1] * v[0];
}

// gv[k] = d loss / d (x, y, z, w) of vertex k; (px, py) is the pixel centre in NDC.
__device__ __forceinline__ void resolve_adjoint(const Vert& v0, const Vert& v1, const Vert& v2,
                                                float px, float py, float4 gr, bool has_db,
                                                float4 gd, int width, int height,
                                                float (&gv)[3][4]) {
  const float w[3] = {v0.w, v1.w, v2.w};
  const float z[3] = {v0.z, v1.z, v2.z};
  const float a[3] = {v0.x - px * w[0], v1.x - px * w[1], v2.x - px * w[2]};
  const float c[3] = {v0.y - py * w[0], v1.y - py * w[1], v2.y - py * w[2]};
  float e[3];
  cross3(a, c, e);
  const float s = e[0] + e[1] + e[2];
  const float inv_s = 1.0f / s;
  const float b[3] = {e[0] * inv_s, e[1] * inv_s, e[2] * inv_s};
  const float ew = e[0] * w[0] + e[1] * w[1] + e[2] * w[2];
  const float inv_ew = 1.0f / ew;
  const float depth = (e[0] * z[0] + e[1] * z[1] + e[2] * z[2]) * inv_ew;
  float gb[3] = {gr.x, gr.y, 0.0f};
  float gs = 0.0f;
  float ga[3] = {0.f, 0.f, 0.f}, gc[3] = {0.f, 0.f, 0.f}, gw[3] = {0.f, 0.f, 0.f};
  if (has_db) {
    float dx[3], dy[3];
    cross3(c, w, dx);
    cross3(w, a, dy);
    const float sx = dx[0] + dx[1] + dx[2], sy = dy[0] + dy[1] + dy[2];
    const float scale_x = 2.0f / static_cast<float>(width), scale_y = 2.0f / static_cast<float>(height);
    // Gradients of db_dx_k = (dx_k - b_k sx) / s and db_dy_k, k = 0, 1.
    const float gbx[3] = {gd.x * scale_x, gd.z * scale_x, 0.0f};
    const float gby[3] = {gd.y * scale_y, gd.w * scale_y, 0.0f};
    const float dbx0 = (dx[0] - b[0] * sx) * inv_s, dbx1 = (dx[1] - b[1] * sx) * inv_s;
    const float dby0 = (dy[0] - b[0] * sy) * inv_s, dby1 = (dy[1] - b[1] * sy) * inv_s;
    const float shared_x = (gbx[0] * b[0] + gbx[1] * b[1]) * inv_s;
    const float shared_y = (gby[0] * b[0] + gby[1] * b[1]) * inv_s;
    float gdx[3], gdy[3];
    for (int k = 0; k < 3; ++k) {
      gdx[k] = gbx[k] * inv_s - shared_x;
      gdy[k] = gby[k] * inv_s - shared_y;
    }
    gb[0] -= (gbx[0] * sx + gby[0] * sy) * inv_s;
    gb[1] -= (gbx[1] * sx + gby[1] * sy) * inv_s;
    gs -= (gbx[0] * dbx0 + gbx[1] * dbx1 + gby[0] * dby0 + gby[1] * dby1) * inv_s;
    // dx = c x w: dL/dc += w x gdx, dL/dw += gdx x c. dy = w x a: dL/dw += a x gdy,
    // dL/da += gdy x w.
    float t[3];
    cross3(w, gdx, t);
    for (int k = 0; k < 3; ++k) gc[k] += t[k];
    cross3(gdx, c, t);
    for (int k = 0; k < 3; ++k) gw[k] += t[k];
    cross3(a, gdy, t);
    for (int k = 0; k < 3; ++k) gw[k] += t[k];
    cross3(gdy, w, t);
    for (int k = 0; k < 3; ++k) ga[k] += t[k];
  }
  // b = e / s with s = sum(e).
  gs -= (gb[0] * b[0] + gb[1] * b[1] + gb[2] * b[2]) * inv_s;
  float ge[3];
  for (int k = 0; k < 3; ++k) ge[k] = gb[k] * inv_s + gs;
  // depth = (e . z) / (e . w).
  const float g_ew = gr.z * inv_ew;
  float gz[3];
  for (int k = 0; k < 3; ++k) {
    ge[k] += g_ew * (z[k] - depth * w[k]);
    gz[k] = g_ew * e[k];
    gw[k] -= g_ew * depth * e[k];
  }
  // e = a x c.
  float t[3];
  cross3(c, ge, t);
  for (int k = 0; k < 3; ++k) ga[k] += t[k];
  cross3(ge, a, t);
  for (int k = 0; k < 3; ++k) gc[k] += t[k];
  // a = x - px w, c = y - py w.
  for (int k = 0; k < 3; ++k) {
    gw[k] -= px * ga[k] + py * gc[k];
    gv[k][0] = ga[k];
    gv[k][1] = gc[k];
    gv[k][2] = gz[k];
    gv[k][3] = gw[k];
  }
}

}  // namespace dr
