// Texture sampling on B200: 2D and cube maps, nearest / bilinear / mipmapped / trilinear,
// forward and backward, plus the area-weighted mip build and its adjoint.
//
// Semantics follow diffrast's reference backend (reference.py:149-194, :491-672; _cube.py):
//   - texel [row, col] is centred at ((col + 0.5) / w, (row + 0.5) / h); wrap keeps the fractional
//     part of a coordinate first; clamp and zero saturate the texel coordinate to [-1, size];
//   - the level of detail is 0.5 log2 of the longer squared footprint axis in base-level texels,
//     footprints saturating at 1e18, plus an optional per-pixel bias, clamped to the levels;
//   - a pixel whose coordinates or level are NaN (or infinite under wrap) is NaN and passes no
//     gradient; cube directions that select no point read zero;
//   - cube lookups fold taps across face edges onto the neighbouring face and fill a tap beyond a
//     cube corner with the mean of the other three.
// Levels are addressed through a table of per-level pointers passed by value, so the base level is
// the caller's texture tensor itself and no packed copy of the mip stack is ever made. The
// coordinate arithmetic that decides which texels are read uses explicitly rounded operations in
// the reference's order. Texel gradients are summed per warp and scattered with one reduction per
// distinct texel.
#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "resolve_adjoint.cuh"
#include "warp_reduce.cuh"

namespace dr {
namespace {

struct Levels {
  const float* ptr[DR_MAX_LEVELS];
  float* grad[DR_MAX_LEVELS];
  long long bstride[DR_MAX_LEVELS];  // batch stride in texels (0 when shared by all views)
  long long texels[DR_MAX_LEVELS];   // texels of the whole level buffer (bounds checks only)
  int h[DR_MAX_LEVELS];
  int w[DR_MAX_LEVELS];
  int num_levels;
};

constexpr float kNaN = __builtin_nanf("");

// torch.clamp(x, -1e18, 1e18) with NaN kept.
__device__ __forceinline__ float saturate(float x) {
  return x != x ? x : fminf(fmaxf(x, -kLimit), kLimit);
}

// ---------------------------------------------------------------------------------------------
// Cube-map projection (_cube.py:44-102).
// ---------------------------------------------------------------------------------------------

// Per face: axis and sign of the major direction, and of the directions of s and t.
__device__ __forceinline__ void face_axes(int face, int& am, float& sm, int& as, float& ss, int& at,
                                          float& st) {
  switch (face) {
    case 0: am = 0; sm = 1.f; as = 2; ss = -1.f; at = 1; st = -1.f; break;
    case 1: am = 0; sm = -1.f; as = 2; ss = 1.f; at = 1; st = -1.f; break;
    case 2: am = 1; sm = 1.f; as = 0; ss = 1.f; at = 2; st = 1.f; break;
    case 3: am = 1; sm = -1.f; as = 0; ss = 1.f; at = 2; st = -1.f; break;
    case 4: am = 2; sm = 1.f; as = 0; ss = 1.f; at = 1; st = -1.f; break;
    default: am = 2; sm = -1.f; as = 0; ss = -1.f; at = 1; st = -1.f; break;
  }
}

struct CubeProj {
  bool valid, undefined;
  int face, am, as, at;
  float sm, ss, st;
  float length, ma, rs, rt;
  float s, t;
  float dmask[3][2];
  float dma[2], dsc[2], dtc[2];
  float st_da[4];
};

__device__ __forceinline__ CubeProj cube_project(const float* dir, const float* dir_da) {
  CubeProj c;
  float d[3] = {dir[0], dir[1], dir[2]};
  const float big = fmaxf(fmaxf(fabsf(d[0]), fabsf(d[1])), fabsf(d[2]));
  c.valid = isfinite(d[0]) && isfinite(d[1]) && isfinite(d[2]) && big >= 1.17549435e-38f;
  if (!c.valid) {
    d[0] = 0.f;
    d[1] = 0.f;
    d[2] = 1.f;
  }
  const float ax = fabsf(d[0]), ay = fabsf(d[1]), az = fabsf(d[2]);
  const bool x_major = (ax >= ay) && (ax >= az);
  const bool y_major = !x_major && (ay >= az);
  const int axis = x_major ? 0 : (y_major ? 1 : 2);
  c.face = 2 * axis + (d[axis] < 0.f ? 1 : 0);
  face_axes(c.face, c.am, c.sm, c.as, c.ss, c.at, c.st);
  c.length = fmaxf(fmaxf(ax, ay), az);
  const float unit[3] = {dvd(d[0], c.length), dvd(d[1], c.length), dvd(d[2], c.length)};
  c.ma = mul(c.sm, unit[c.am]);
  c.rs = dvd(mul(c.ss, unit[c.as]), c.ma);
  c.rt = dvd(mul(c.st, unit[c.at]), c.ma);
  c.s = mul(0.5f, add(c.rs, 1.0f));
  c.t = mul(0.5f, add(c.rt, 1.0f));
  c.undefined = false;
  for (int k = 0; k < 3; ++k) c.dmask[k][0] = c.dmask[k][1] = 0.0f;
  for (int xy = 0; xy < 2; ++xy) c.dma[xy] = c.dsc[xy] = c.dtc[xy] = 0.0f;
  for (int i = 0; i < 4; ++i) c.st_da[i] = 0.0f;
  if (dir_da != nullptr) {
    float raw[6];
    bool nan = false;
    for (int i = 0; i < 6; ++i) {
      raw[i] = dir_da[i];
      nan |= raw[i] != raw[i];
    }
    c.undefined = c.valid && nan;
    const bool use = c.valid && !c.undefined;
    float da[3][2];
    for (int k = 0; k < 3; ++k) {
      for (int xy = 0; xy < 2; ++xy) {
        const float v = dvd(use ? raw[2 * k + xy] : 0.0f, c.length);
        c.dmask[k][xy] = (v >= -kLimit && v <= kLimit) ? 1.f : 0.f;
        da[k][xy] = fminf(fmaxf(v, -kLimit), kLimit);
      }
    }
    for (int xy = 0; xy < 2; ++xy) {
      c.dma[xy] = mul(c.sm, da[c.am][xy]);
      c.dsc[xy] = mul(c.ss, da[c.as][xy]);
      c.dtc[xy] = mul(c.st, da[c.at][xy]);
      const float ds = dvd(mul(0.5f, sub(c.dsc[xy], mul(c.rs, c.dma[xy]))), c.ma);
      const float dt = dvd(mul(0.5f, sub(c.dtc[xy], mul(c.rt, c.dma[xy]))), c.ma);
      c.st_da[xy] = c.undefined ? kNaN : ds;
      c.st_da[2 + xy] = c.undefined ? kNaN : dt;
    }
  }
  return c;
}

// Gradients of the directions (and their derivatives) from those of st and st_da.
__device__ __forceinline__ void cube_project_bwd(const CubeProj& c, float g_s, float g_t,
                                                 const float g_st_da[4], float g_dir[3],
                                                 float g_dir_da[6]) {
  float g_rs = 0.5f * g_s, g_rt = 0.5f * g_t, g_ma = 0.0f;
  float g_da[3][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
  if (g_st_da != nullptr) {
    for (int xy = 0; xy < 2; ++xy) {
      const float g_ds = g_st_da[xy], g_dt = g_st_da[2 + xy];
      const float ds = 0.5f * (c.dsc[xy] - c.rs * c.dma[xy]) / c.ma;
      const float dt = 0.5f * (c.dtc[xy] - c.rt * c.dma[xy]) / c.ma;
      const float g_dsc = 0.5f * g_ds / c.ma;
      const float g_dtc = 0.5f * g_dt / c.ma;
      const float g_dma = -0.5f * (g_ds * c.rs + g_dt * c.rt) / c.ma;
      g_rs -= 0.5f * g_ds * c.dma[xy] / c.ma;
      g_rt -= 0.5f * g_dt * c.dma[xy] / c.ma;
      g_ma -= (g_ds * ds + g_dt * dt) / c.ma;
      g_da[c.am][xy] += c.sm * g_dma;
      g_da[c.as][xy] += c.ss * g_dsc;
      g_da[c.at][xy] += c.st * g_dtc;
    }
  }
  float g_unit[3] = {0.f, 0.f, 0.f};
  g_unit[c.as] += c.ss * g_rs / c.ma;
  g_unit[c.at] += c.st * g_rt / c.ma;
  g_ma -= (g_rs * c.rs + g_rt * c.rt) / c.ma;
  g_unit[c.am] += c.sm * g_ma;
  for (int k = 0; k < 3; ++k) g_dir[k] = g_unit[k] / c.length;
  for (int k = 0; k < 3; ++k)
    for (int xy = 0; xy < 2; ++xy) g_dir_da[2 * k + xy] = g_da[k][xy] * c.dmask[k][xy] / c.length;
}

// Texel one step outside its face moved onto the neighbouring face, in half-texel integer units
// (_cube.py:105-143). `exists` is false beyond a cube corner.
__device__ __forceinline__ void cube_fold(int face, int row, int col, int size, int& out_face,
                                          int& out_row, int& out_col, bool& exists) {
  const bool over_col = col < 0 || col >= size;
  const bool over_row = row < 0 || row >= size;
  exists = !(over_col && over_row);
  if (!over_col && !over_row) {
    out_face = face;
    out_row = row;
    out_col = col;
    return;
  }
  int am, as, at;
  float sm, ss, st;
  face_axes(face, am, sm, as, ss, at, st);
  int p[3] = {0, 0, 0};
  p[am] += size * static_cast<int>(sm);
  p[as] += (2 * col + 1 - size) * static_cast<int>(ss);
  p[at] += (2 * row + 1 - size) * static_cast<int>(st);
  for (int k = 0; k < 3; ++k) p[k] = min(max(p[k], -size), size);
  p[am] -= static_cast<int>(sm);
  int axis = 0;
  if (abs(p[1]) > abs(p[axis])) axis = 1;
  if (abs(p[2]) > abs(p[axis])) axis = 2;
  out_face = 2 * axis + (p[axis] < 0 ? 1 : 0);
  face_axes(out_face, am, sm, as, ss, at, st);
  const int sc = p[as] * static_cast<int>(ss) + size - 1;
  const int tc = p[at] * static_cast<int>(st) + size - 1;
  // Floor division by 2 of possibly negative values.
  out_col = max((sc >= 0 ? sc : sc - 1) / 2, 0);
  out_row = max((tc >= 0 ? tc : tc - 1) / 2, 0);
}

// ---------------------------------------------------------------------------------------------
// Texel coordinates and footprints.
// ---------------------------------------------------------------------------------------------

// Continuous texel coordinate coord * size - shift under the boundary mode (reference.py:615-633),
// with its derivative with respect to coord * size (0 where clamped) and whether it is unusable.
template <int B>
__device__ __forceinline__ float texel_coord(float coord, int size, float shift, bool& bad,
                                             float& slope) {
  const float s = static_cast<float>(size);
  float x;
  slope = 1.0f;
  if (B == DR_BOUNDARY_WRAP) {
    x = sub(mul(sub(coord, floorf(coord)), s), shift);
    bad = !isfinite(x);
  } else if (B == DR_BOUNDARY_CUBE) {
    x = sub(mul(coord, s), shift);
    bad = !isfinite(x);
  } else {
    x = sub(mul(coord, s), shift);
    bad = x != x;
    slope = (x >= -1.0f && x <= s) ? 1.0f : 0.0f;
    x = fminf(fmaxf(x, -1.0f), s);
  }
  if (bad) {
    x = 0.0f;
    slope = 0.0f;
  }
  return x;
}

// Element offset (without channel) of texel (row, col) of level l for this view, or ok = false
// for a texel that does not exist (zero boundary, beyond a cube corner).
template <int B>
__device__ __forceinline__ long long texel_offset(const Levels& L, int l, long long view, int face,
                                                  int row, int col, int channels, bool& ok) {
  const int h = L.h[l], w = L.w[l];
  ok = true;
  if (B == DR_BOUNDARY_WRAP) {
    row %= h;
    row += row < 0 ? h : 0;
    col %= w;
    col += col < 0 ? w : 0;
  } else if (B == DR_BOUNDARY_CUBE) {
    int f2, r2, c2;
    cube_fold(face, row, col, w, f2, r2, c2, ok);
    face = f2;
    row = r2;
    col = c2;
  } else {
    if (B == DR_BOUNDARY_ZERO) ok = row >= 0 && row < h && col >= 0 && col < w;
    row = min(max(row, 0), h - 1);
    col = min(max(col, 0), w - 1);
  }
  long long texel = static_cast<long long>(row) * w + col;
  if (B == DR_BOUNDARY_CUBE) texel += static_cast<long long>(face) * h * w;
  return checked_index(view * L.bstride[l] + texel, L.texels[l], kSiteTexel);
}

struct Footprint {
  long long off[4];
  bool ok[4];
  float fx, fy;
  float slope_x, slope_y;  // d(texel coordinate) / d(coord * size)
  float missing;           // weight of the taps that do not exist beyond a cube corner
  float dmiss_dx, dmiss_dy;
  bool bad;
};

// Bilinear footprint of (u, v) in level l (reference.py:576-612).
template <int B>
__device__ __forceinline__ Footprint bilinear_footprint(const Levels& L, int l, long long view,
                                                        int face, float u, float v, int channels) {
  Footprint f;
  bool bad_x, bad_y;
  const float x = texel_coord<B>(u, L.w[l], 0.5f, bad_x, f.slope_x);
  const float y = texel_coord<B>(v, L.h[l], 0.5f, bad_y, f.slope_y);
  f.bad = bad_x || bad_y;
  const float x0 = floorf(x), y0 = floorf(y);
  f.fx = sub(x, x0);
  f.fy = sub(y, y0);
  const int col = static_cast<int>(x0), row = static_cast<int>(y0);
  if (B == DR_BOUNDARY_CUBE) {
    f.off[0] = texel_offset<B>(L, l, view, face, row, col, channels, f.ok[0]);
    f.off[1] = texel_offset<B>(L, l, view, face, row, col + 1, channels, f.ok[1]);
    f.off[2] = texel_offset<B>(L, l, view, face, row + 1, col, channels, f.ok[2]);
    f.off[3] = texel_offset<B>(L, l, view, face, row + 1, col + 1, channels, f.ok[3]);
  } else {
    // The two columns and two rows are resolved once each (one modulo per axis when wrapping).
    const int w = L.w[l], h = L.h[l];
    int c0, c1, r0, r1;
    bool okc0 = true, okc1 = true, okr0 = true, okr1 = true;
    if (B == DR_BOUNDARY_WRAP) {
      // Positive remainders; a mask for power-of-two sizes (two's complement makes it exact for
      // negative coordinates too).
      if ((w & (w - 1)) == 0) {
        c0 = col & (w - 1);
      } else {
        c0 = col % w;
        c0 += c0 < 0 ? w : 0;
      }
      c1 = c0 + 1 == w ? 0 : c0 + 1;
      if ((h & (h - 1)) == 0) {
        r0 = row & (h - 1);
      } else {
        r0 = row % h;
        r0 += r0 < 0 ? h : 0;
      }
      r1 = r0 + 1 == h ? 0 : r0 + 1;
    } else {
      if (B == DR_BOUNDARY_ZERO) {
        okc0 = col >= 0 && col < w;
        okc1 = col + 1 >= 0 && col + 1 < w;
        okr0 = row >= 0 && row < h;
        okr1 = row + 1 >= 0 && row + 1 < h;
      }
      c0 = min(max(col, 0), w - 1);
      c1 = min(max(col + 1, 0), w - 1);
      r0 = min(max(row, 0), h - 1);
      r1 = min(max(row + 1, 0), h - 1);
    }
    const long long base = view * L.bstride[l];
    const long long row0 = base + static_cast<long long>(r0) * w;
    const long long row1 = base + static_cast<long long>(r1) * w;
    f.off[0] = checked_index(row0 + c0, L.texels[l], kSiteTexel);
    f.off[1] = checked_index(row0 + c1, L.texels[l], kSiteTexel);
    f.off[2] = checked_index(row1 + c0, L.texels[l], kSiteTexel);
    f.off[3] = checked_index(row1 + c1, L.texels[l], kSiteTexel);
    f.ok[0] = okr0 && okc0;
    f.ok[1] = okr0 && okc1;
    f.ok[2] = okr1 && okc0;
    f.ok[3] = okr1 && okc1;
  }
  f.missing = f.dmiss_dx = f.dmiss_dy = 0.0f;
  if (B == DR_BOUNDARY_CUBE) {
    const int w = L.w[l], h = L.h[l];
    const float left = col < 0, right = col + 1 >= w, above = row < 0, below = row + 1 >= h;
    const float m00 = left * above, m01 = right * above, m10 = left * below, m11 = right * below;
    const float fx = f.fx, fy = f.fy;
    f.missing = add(mul(sub(1.0f, fy), add(mul(sub(1.0f, fx), m00), mul(fx, m01))),
                    mul(fy, add(mul(sub(1.0f, fx), m10), mul(fx, m11))));
    f.dmiss_dx = (1.0f - fy) * (m01 - m00) + fy * (m11 - m10);
    f.dmiss_dy = ((1.0f - fx) * m10 + fx * m11) - ((1.0f - fx) * m00 + fx * m01);
  }
  return f;
}

// Bilinear value of channel c with the reference's rounding order.
template <int B>
__device__ __forceinline__ float bilinear_value(const float* __restrict__ level, const Footprint& f,
                                                int channels, int c, float t[4]) {
  for (int k = 0; k < 4; ++k) t[k] = f.ok[k] ? __ldg(level + f.off[k] * channels + c) : 0.0f;
  const float gx = sub(1.0f, f.fx), gy = sub(1.0f, f.fy);
  float out = add(mul(gy, add(mul(gx, t[0]), mul(f.fx, t[1]))),
                  mul(f.fy, add(mul(gx, t[2]), mul(f.fx, t[3]))));
  if (B == DR_BOUNDARY_CUBE) {
    out = add(out, dvd(mul(f.missing, add(add(add(t[0], t[1]), t[2]), t[3])), 3.0f));
  }
  return out;
}

// Level of detail from the footprint (reference.py:491-501), NaN propagated, with the squared
// axis lengths kept for the backward pass.
__device__ __forceinline__ float level_of_detail(const float da[4], int h, int w, float& len_x,
                                                 float& len_y) {
  const float fw = static_cast<float>(w), fh = static_cast<float>(h);
  const float ux = saturate(mul(da[0], fw)), uy = saturate(mul(da[1], fw));
  const float vx = saturate(mul(da[2], fh)), vy = saturate(mul(da[3], fh));
  len_x = add(mul(ux, ux), mul(vx, vx));
  len_y = add(mul(uy, uy), mul(vy, vy));
  float m = nanmax(len_x, len_y);
  m = m != m ? m : fmaxf(m, 1e-30f);
  return mul(0.5f, log2f(m));
}

__device__ __forceinline__ void level_of_detail_bwd(const float da[4], int h, int w, float g_lod,
                                                    float g_da[4]) {
  const float fw = static_cast<float>(w), fh = static_cast<float>(h);
  const float raw[4] = {da[0] * fw, da[1] * fw, da[2] * fh, da[3] * fh};
  const float scale[4] = {fw, fw, fh, fh};
  float cl[4], mask[4];
  for (int i = 0; i < 4; ++i) {
    cl[i] = fminf(fmaxf(raw[i], -kLimit), kLimit);
    mask[i] = (raw[i] >= -kLimit && raw[i] <= kLimit) ? 1.0f : 0.0f;
  }
  const float len_x = cl[0] * cl[0] + cl[2] * cl[2];
  const float len_y = cl[1] * cl[1] + cl[3] * cl[3];
  const float m = fmaxf(len_x, len_y);
  const float g_m = m >= 1e-30f ? g_lod * 0.5f / (m * 0.6931471805599453f) : 0.0f;
  const float share_x = len_x > len_y ? 1.0f : (len_x == len_y ? 0.5f : 0.0f);
  const float g_lx = g_m * share_x, g_ly = g_m * (1.0f - share_x);
  g_da[0] = g_lx * 2.0f * cl[0] * scale[0] * mask[0];
  g_da[1] = g_ly * 2.0f * cl[1] * scale[1] * mask[1];
  g_da[2] = g_lx * 2.0f * cl[2] * scale[2] * mask[2];
  g_da[3] = g_ly * 2.0f * cl[3] * scale[3] * mask[3];
}

// Everything a pixel's lookup needs before the channel loop.
template <int MODE, int B>
struct Lookup {
  bool bad, valid;
  CubeProj cube;
  float u, v;
  int face;
  float da[4];
  bool has_da;
  float lod_raw;  // level of detail before clamping (NaN replaced by 0)
  int lo, hi;
  float frac;
  Footprint f_lo, f_hi;
  long long near_off;
  bool near_ok;
};

// Pixel strides (floats between consecutive pixels) of uv and uv_da, which may be channel slices
// of a wider tensor.
struct Strides {
  long long uv, uv_da;
};

template <int MODE, int B>
__device__ __forceinline__ void prepare(const Levels& L, int channels, const float* __restrict__ uv,
                                        const float* __restrict__ uv_da,
                                        const float* __restrict__ bias, const Strides st,
                                        long long p, long long view, Lookup<MODE, B>& k) {
  constexpr bool kMip = MODE >= DR_FILTER_LINEAR_MIPMAP_NEAREST;
  k.valid = true;
  k.face = 0;
  k.has_da = kMip && uv_da != nullptr;
  if (B == DR_BOUNDARY_CUBE) {
    k.cube = cube_project(uv + p * st.uv, k.has_da ? uv_da + p * st.uv_da : nullptr);
    k.valid = k.cube.valid;
    k.face = k.cube.face;
    k.u = k.cube.s;
    k.v = k.cube.t;
    for (int i = 0; i < 4; ++i) k.da[i] = k.has_da ? k.cube.st_da[i] : 0.0f;
  } else {
    k.u = __ldcs(uv + p * st.uv);
    k.v = __ldcs(uv + p * st.uv + 1);
    for (int i = 0; i < 4; ++i) k.da[i] = k.has_da ? __ldcs(uv_da + p * st.uv_da + i) : 0.0f;
  }
  k.bad = false;
  k.lo = k.hi = 0;
  k.frac = 0.0f;
  k.lod_raw = 0.0f;
  if (kMip) {
    float lod = 0.0f;
    if (k.has_da) {
      float lx, ly;
      lod = add(lod, level_of_detail(k.da, L.h[0], L.w[0], lx, ly));
    }
    if (bias != nullptr) lod = add(lod, __ldcs(bias + p));
    k.bad = lod != lod;
    if (k.bad) lod = 0.0f;
    k.lod_raw = lod;
    const float top = static_cast<float>(L.num_levels - 1);
    lod = fminf(fmaxf(lod, 0.0f), top);
    const bool blend = MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR;
    const float lower = floorf(blend ? lod : add(lod, 0.5f));
    k.lo = static_cast<int>(lower);
    k.hi = min(k.lo + 1, L.num_levels - 1);
    k.frac = blend ? sub(lod, lower) : 0.0f;
  }
  if (MODE == DR_FILTER_NEAREST) {
    bool bx, by;
    float sx, sy;
    const float x = texel_coord<B>(k.u, L.w[0], 0.0f, bx, sx);
    const float y = texel_coord<B>(k.v, L.h[0], 0.0f, by, sy);
    k.bad = k.bad || bx || by;
    // A direction exactly on the far edge of a cube face stays on that face.
    if (B == DR_BOUNDARY_CUBE) {
      const int h = L.h[0], w = L.w[0];
      const int row = min(max(static_cast<int>(floorf(y)), 0), h - 1);
      const int col = min(max(static_cast<int>(floorf(x)), 0), w - 1);
      k.near_ok = true;
      k.near_off = checked_index(
          view * L.bstride[0] + (static_cast<long long>(k.face) * h + row) * w + col, L.texels[0],
          kSiteTexel);
    } else {
      k.near_off = texel_offset<B>(L, 0, view, 0, static_cast<int>(floorf(y)),
                                   static_cast<int>(floorf(x)), channels, k.near_ok);
    }
  } else {
    k.f_lo = bilinear_footprint<B>(L, k.lo, view, k.face, k.u, k.v, channels);
    k.bad = k.bad || k.f_lo.bad;
    if (MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR) {
      k.f_hi = bilinear_footprint<B>(L, k.hi, view, k.face, k.u, k.v, channels);
      k.bad = k.bad || k.f_hi.bad;
    }
  }
}

// Copies `count` floats from shared memory to contiguous `dst`, with 16-byte stores where the
// address allows.
__device__ __forceinline__ void store_block(float* __restrict__ dst, const float* __restrict__ src,
                                            int count) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    const int vec = count / 4;
    for (int i = threadIdx.x; i < vec; i += blockDim.x)
      reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
    for (int i = vec * 4 + threadIdx.x; i < count; i += blockDim.x) dst[i] = src[i];
  } else {
    for (int i = threadIdx.x; i < count; i += blockDim.x) dst[i] = src[i];
  }
}

// One thread per pixel; with `staged` the block's 256 output pixels (one contiguous range) go
// through shared memory so that the global stores are coalesced float4s. NC > 0: exactly NC
// channels, known at compile time, so that the channel loop unrolls and every channel's texel
// gathers are in flight together (a runtime loop waits for each channel's gathers in turn); the
// arithmetic of each channel is the same either way.
template <int MODE, int B, int NC>
__global__ void __launch_bounds__(256) texture_fwd_kernel(
    const Levels L, int channels, const float* __restrict__ uv, const float* __restrict__ uv_da,
    const float* __restrict__ bias, const Strides st, long long total, long long pixels_per_image,
    float* __restrict__ out, bool staged) {
  extern __shared__ float stage[];
  __shared__ long long block_view;
  const long long first = blockIdx.x * static_cast<long long>(blockDim.x);
  const long long p = first + threadIdx.x;
  float* o = staged ? stage + threadIdx.x * channels : out + p * channels;
  // One 64-bit division per block: a block spans at most two views when an image has at least
  // blockDim.x pixels.
  if (threadIdx.x == 0) block_view = first / pixels_per_image;
  __syncthreads();
  if (p < total) {
    long long view = block_view;
    if (pixels_per_image >= blockDim.x) {
      if (p >= (view + 1) * pixels_per_image) ++view;
    } else {
      view = p / pixels_per_image;
    }
    Lookup<MODE, B> k;
    prepare<MODE, B>(L, channels, uv, uv_da, bias, st, p, view, k);
    const int nch = NC > 0 ? NC : channels;
    auto channel = [&](int c) {
      float value;
      if (MODE == DR_FILTER_NEAREST) {
        value = k.near_ok ? __ldg(L.ptr[0] + k.near_off * nch + c) : 0.0f;
      } else {
        float t[4];
        value = bilinear_value<B>(L.ptr[k.lo], k.f_lo, nch, c, t);
        if (MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR) {
          const float above = bilinear_value<B>(L.ptr[k.hi], k.f_hi, nch, c, t);
          value = add(mul(value, sub(1.0f, k.frac)), mul(above, k.frac));
        }
      }
      if (k.bad) value = kNaN;
      if (!k.valid) value = 0.0f;
      if (staged) o[c] = value; else __stcs(o + c, value);
    };
    if constexpr (NC > 0) {
#pragma unroll
      for (int c = 0; c < NC; ++c) channel(c);
    } else {
      for (int c = 0; c < channels; ++c) channel(c);
    }
  }
  if (!staged) return;
  __syncthreads();
  const int pixels = static_cast<int>(min(static_cast<long long>(blockDim.x), total - first));
  store_block(out + first * channels, stage, pixels * channels);
}

// Taps of a pixel's lookup with their weights (bilinear weight times level weight, plus the
// cube-corner share): up to 4 per level, 2 levels.
struct Taps {
  int n;
  int level[8];
  long long off[8];
  float w[8];
};

template <int B>
__device__ __forceinline__ void add_footprint_taps(Taps& taps, const Footprint& f, int level,
                                                   float scale) {
  const float gx = 1.0f - f.fx, gy = 1.0f - f.fy;
  const float wgt[4] = {gx * gy, f.fx * gy, gx * f.fy, f.fx * f.fy};
  const float extra = B == DR_BOUNDARY_CUBE ? f.missing / 3.0f : 0.0f;
  for (int t = 0; t < 4; ++t) {
    if (!f.ok[t]) continue;
    taps.level[taps.n] = level;
    taps.off[taps.n] = f.off[t];
    taps.w[taps.n] = scale * (wgt[t] + extra);
    ++taps.n;
  }
}

// Where the coordinate gradients go: pixel strides and, when the gradient is a channel slice of
// wider pixel records whose other channels get zero gradient, the slice's first channel (-1: a
// plain strided output, nothing else written).
struct GradLayout {
  long long uv, uv_da;
  int uv_first, da_first;
};

// The N gradient values of pixel p: into the record's channels [first, first + N) with the rest
// of the record zeroed (whole records, so that stores cover full sectors), or at out + p stride.
template <int N>
__device__ __forceinline__ void write_record(float* __restrict__ out, long long p, long long stride,
                                             int first, const float (&v)[N]) {
  if (first < 0) {
#pragma unroll
    for (int i = 0; i < N; ++i) out[p * stride + i] = v[i];
    return;
  }
  float* rec = out + p * stride;
  for (int i = 0; i < first; ++i) rec[i] = 0.0f;
#pragma unroll
  for (int j = 0; j < N; ++j) rec[first + j] = v[j];
  for (int i = first + N; i < stride; ++i) rec[i] = 0.0f;
}

// The interpolation that produced a 2D lookup's coordinates, for the texture backward pass with
// the interpolation's backward pass for them fused in: uv = attribute channels (cu, cv)
// interpolated with rast's barycentrics, uv_da = the screen derivatives of channels (du, dv)
// from rast_db. The coordinate gradients are chained into gradients of rast (b0, b1; z and the
// id get zero) and of rast_db instead of being written out. grad_rast null: not fused.
struct InterpChain {
  const float4* rast;
  const int* tri;
  const float* attr;            // [views or 1, vertices, attr_channels]
  long long attr_view_stride;   // floats between the views' attribute tables (0: shared)
  long long num_vert;
  int attr_channels, num_tri;
  int cu, cv, du, dv;
  float4* grad_rast;
  float4* grad_db;              // null when uv_da carries no gradient
  // The rasterizer's backward pass as well (grad_pos non-null; grad_rast and grad_db are then
  // null): the pixel's triangle comes from the rasterizer's keys, and the gradients of the
  // triangle's clip-space vertices for this pixel's rast / rast_db gradients are added to
  // grad_pos, warp-aggregated, as the rasterizer's backward kernel would add them.
  const long long* keys;
  const float* pos;             // [views or 1, pos_num_vert, 4]
  long long pos_view_stride;    // vertices between the views' positions (0: shared)
  long long pos_num_vert;
  float* grad_pos;
  bool resolve_db;              // rast_db's gradient reaches the positions
};

// Gradients of rast and rast_db at pixel p from those of the lookup's coordinates, with the
// arithmetic and order of the interpolation backward kernel given the same coordinate
// gradients: d out_c / d b0 = a0_c - a2_c, d out_c / d b1 = a1_c - a2_c, and the derivative
// channels likewise with rast_db's (d b / dX, d b / dY). With RESOLVE they go on through the
// rasterizer's backward pass into the positions (inside = false for pixels past the image: they
// read and write nothing).
template <bool RESOLVE>
__device__ __forceinline__ void chain_interpolation(const InterpChain& c, long long p,
                                                    long long view, int col, int row, int width,
                                                    int height, bool inside,
                                                    const float (&g_uv)[2],
                                                    const float (&g_da)[4]) {
  int t = -1;
  if (inside) {
    if (RESOLVE) {
      const long long key = __ldcs(c.keys + p);
      t = key != kEmptyKey ? static_cast<int>(key & 0xFFFFFFFFLL) : -1;
    } else {
      t = rast_triangle(__ldcs(c.rast + p).w, c.num_tri);
    }
  }
  float gu = 0.0f, gv = 0.0f;
  float g_dudx = 0.0f, g_dudy = 0.0f, g_dvdx = 0.0f, g_dvdy = 0.0f;
  int i0 = 0, i1 = 0, i2 = 0;
  Vert v0 = {0.f, 0.f, 0.f, 1.f}, v1 = v0, v2 = v0;
  const long long pbase = view * c.pos_view_stride;
  if (t >= 0) {
    const int* vt = c.tri + 3 * static_cast<long long>(t);
    i0 = __ldg(vt);
    i1 = __ldg(vt + 1);
    i2 = __ldg(vt + 2);
    const float* base = c.attr + view * c.attr_view_stride;
    const float* a0 = base + checked_index(i0, c.num_vert, kSiteVertex) * c.attr_channels;
    const float* a1 = base + checked_index(i1, c.num_vert, kSiteVertex) * c.attr_channels;
    const float* a2 = base + checked_index(i2, c.num_vert, kSiteVertex) * c.attr_channels;
    // Every gather of the pixel is issued once its triangle's indices are in: the coordinate and
    // (when rast_db's gradient is wanted) derivative channels of the three attribute rows and,
    // with RESOLVE, the three vertices; the arithmetic below is unchanged.
    const bool want_db = c.grad_db != nullptr || c.resolve_db;
    const int ch[2] = {c.cu, c.cv}, dch[2] = {c.du, c.dv};
    float x[2][3], xd[2][3];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      x[i][0] = __ldg(a0 + ch[i]);
      x[i][1] = __ldg(a1 + ch[i]);
      x[i][2] = __ldg(a2 + ch[i]);
      xd[i][0] = want_db ? __ldg(a0 + dch[i]) : 0.0f;
      xd[i][1] = want_db ? __ldg(a1 + dch[i]) : 0.0f;
      xd[i][2] = want_db ? __ldg(a2 + dch[i]) : 0.0f;
    }
    if constexpr (RESOLVE) {
      i0 = static_cast<int>(checked_index(i0, c.pos_num_vert, kSiteVertex));
      i1 = static_cast<int>(checked_index(i1, c.pos_num_vert, kSiteVertex));
      i2 = static_cast<int>(checked_index(i2, c.pos_num_vert, kSiteVertex));
      v0 = load_vert(c.pos, pbase + i0);
      v1 = load_vert(c.pos, pbase + i1);
      v2 = load_vert(c.pos, pbase + i2);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      gu += g_uv[i] * (x[i][0] - x[i][2]);
      gv += g_uv[i] * (x[i][1] - x[i][2]);
    }
    if (want_db) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float gx = g_da[2 * j], gy = g_da[2 * j + 1];
        const float du = xd[j][0] - xd[j][2];
        const float dv = xd[j][1] - xd[j][2];
        g_dudx += gx * du;
        g_dudy += gy * du;
        g_dvdx += gx * dv;
        g_dvdy += gy * dv;
      }
    }
  }
  if constexpr (!RESOLVE) {
    if (!inside) return;
    __stcs(c.grad_rast + p, make_float4(gu, gv, 0.0f, 0.0f));
    if (c.grad_db != nullptr) __stcs(c.grad_db + p, make_float4(g_dudx, g_dudy, g_dvdx, g_dvdy));
    return;
  } else {
  float gvert[3][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  if (t >= 0)
    resolve_adjoint(v0, v1, v2, pixel_centre(col, width), pixel_centre(row, height),
                    make_float4(gu, gv, 0.0f, 0.0f), c.resolve_db,
                    make_float4(g_dudx, g_dudy, g_dvdx, g_dvdy), width, height, gvert);
  // Each pixel adds its own three vector reductions: a warp covers 16 x 2 pixels, where a
  // triangle (about four pixels on config 5) repeats too rarely for a warp-level merge to pay
  // for its shuffles (5.39 ms with it, 5.27 without).
  if (t < 0) return;
  red_add_v4(c.grad_pos + (pbase + i0) * 4, gvert[0][0], gvert[0][1], gvert[0][2], gvert[0][3]);
  red_add_v4(c.grad_pos + (pbase + i1) * 4, gvert[1][0], gvert[1][1], gvert[1][2], gvert[1][3]);
  red_add_v4(c.grad_pos + (pbase + i2) * 4, gvert[2][0], gvert[2][1], gvert[2][2], gvert[2][3]);
  }
}

// The chained position part of a lookup on its own, from its compact coordinate gradients
// (g_uv [pixels, 2], g_da [pixels, 4] or null) written by an earlier texture backward pass: the
// interpolation's and the rasterizer's backward passes for them, into c.grad_pos. One thread per
// pixel; grid: columns in x, rows in y, views in z (short blocks, so that a concurrent all-reduce
// gets SMs as they finish).
__global__ void __launch_bounds__(256) chain_parts_kernel(const InterpChain c,
                                                          const float2* __restrict__ g_uv,
                                                          const float4* __restrict__ g_da,
                                                          int height, int width) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = blockIdx.y;
  const long long view = blockIdx.z;
  const bool inside = col < width;
  const long long p = (view * height + row) * width + col;
  float guv[2] = {0.f, 0.f}, gda[4] = {0.f, 0.f, 0.f, 0.f};
  if (inside) {
    const float2 u = __ldcs(g_uv + p);
    guv[0] = u.x;
    guv[1] = u.y;
    if (g_da != nullptr) {
      const float4 d = __ldcs(g_da + p);
      gda[0] = d.x;
      gda[1] = d.y;
      gda[2] = d.z;
      gda[3] = d.w;
    }
  }
  chain_interpolation<true>(c, p, view, col, row, width, height, inside, guv, gda);
}

// A quad that a whole warp added to (lane 0 keeps it): pixels that all read the same four texels
// (a background that samples one point, a magnified region) accumulate here across the tiles a
// warp visits and reach global memory once, instead of every warp reducing into the same four
// addresses. Each warp has two: the one held and the one that replaces it, flushed between tiles
// (where the tile's registers are free).
struct HotQuad {
  long long off[4];
  float v[16];  // 4 taps x up to 4 channels of group c0
  int level, c0;
};

// Reduces a held quad into the texel gradients and empties it.
template <int NC>
__device__ __forceinline__ void flush_quad(const Levels& L, HotQuad& h, int channels,
                                           int grad_stride) {
  if (h.level < 0) return;
  const int group = min(4, channels - h.c0);
  const bool vector = grad_stride == 4 && channels <= 4;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    bool zero = true;
#pragma unroll
    for (int cc = 0; cc < NC; ++cc) zero = zero && h.v[NC * t + cc] == 0.0f;
    if (zero) continue;
    float* dst = L.grad[h.level] + h.off[t] * grad_stride + h.c0;
    if constexpr (NC == 3) {
      red_add_v4(dst, h.v[3 * t], h.v[3 * t + 1], h.v[3 * t + 2], 0.0f);
    } else if (vector) {
      red_add_v4(dst, h.v[4 * t], h.v[4 * t + 1], h.v[4 * t + 2], h.v[4 * t + 3]);
    } else {
      for (int cc = 0; cc < group; ++cc)
        if (h.v[4 * t + cc] != 0.0f) red_add(dst + cc, h.v[4 * t + cc]);
    }
  }
  h.level = -1;
}

// Texel gradients: a warp covers 16 x 2 pixels of a 16 x 16 tile, whose taps mostly land on the
// same texels (a texel of the chosen levels spans about a pixel; background pixels all read the
// same few). Tap by tap, lanes adding to the same texel sum their contributions with a shuffle
// reduction and one lane issues a single reduction per texel: a 16-byte vector reduction into a
// gradient level padded to 4 channels (grad_stride 4), scalar reductions otherwise. RGB: exactly
// three channels into a padded level, so the lanes reduce 3 values per tap instead of 4.
// CHAIN: 0 coordinate gradients written out, 1 chained through the interpolation (grad_rast /
// grad_db), 2 through the rasterizer as well (grad_pos).
template <int MODE, int B, bool RGB, int CHAIN>
__device__ __forceinline__ void texture_bwd_tile(
    const Levels& L, int channels, int grad_stride, const float* __restrict__ uv,
    const float* __restrict__ uv_da, const float* __restrict__ bias, const Strides& st, int height,
    int width, const float* __restrict__ grad_out, float* __restrict__ grad_uv,
    float* __restrict__ grad_uv_da, float* __restrict__ grad_bias, const GradLayout& gst,
    const InterpChain& chain, int col, int row, long long view, HotQuad& hot, HotQuad& incoming,
    bool& pending) {
  const bool inside = row < height && col < width;
  const long long p = (view * height + row) * width + col;
  Lookup<MODE, B> k;
  bool live = false;
  Taps taps;
  taps.n = 0;
  if (inside) {
    prepare<MODE, B>(L, channels, uv, uv_da, bias, st, p, view, k);
    live = !k.bad && k.valid;
    if (live) {
      if (MODE == DR_FILTER_NEAREST) {
        if (k.near_ok) {
          taps.level[0] = 0;
          taps.off[0] = k.near_off;
          taps.w[0] = 1.0f;
          taps.n = 1;
        }
      } else if (MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR) {
        add_footprint_taps<B>(taps, k.f_lo, k.lo, 1.0f - k.frac);
        add_footprint_taps<B>(taps, k.f_hi, k.hi, k.frac);
      } else {
        add_footprint_taps<B>(taps, k.f_lo, k.lo, 1.0f);
      }
    }
  }
  const unsigned lane = threadIdx.x & 31u;
  const bool vector = grad_stride == 4 && channels <= 4;
  if (B != DR_BOUNDARY_CUBE && MODE != DR_FILTER_NEAREST) {
    // Off a cube, a level's four taps form a quad that (off[0], off[3]) identifies (off[0] alone
    // when wrapping): lanes sharing a quad sum all four taps' contributions at once, with one
    // match per level instead of one per tap.
    constexpr int kSides = MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR ? 2 : 1;
    for (int c0 = 0; c0 < channels; c0 += 4) {
      const int group = min(4, channels - c0);
      float g[4];
      bool any_g = false;
      for (int cc = 0; cc < 4; ++cc) {
        g[cc] = live && cc < group ? __ldcs(grad_out + p * channels + c0 + cc) : 0.0f;
        any_g |= g[cc] != 0.0f;
      }
#pragma unroll
      for (int side = 0; side < kSides; ++side) {
        const Footprint& f = side ? k.f_hi : k.f_lo;
        const int level = side ? k.hi : k.lo;
        const float scale =
            MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR ? (side ? k.frac : 1.0f - k.frac) : 1.0f;
        const bool act = any_g && scale != 0.0f;
        const unsigned any = __ballot_sync(0xffffffffu, act);
        if (any == 0u) continue;
        unsigned peers = 1u << lane;
        if (act) {
          peers = __match_any_sync(
              any, (static_cast<unsigned long long>(level) << 48) | static_cast<unsigned long long>(f.off[0]));
          if (B != DR_BOUNDARY_WRAP) peers &= __match_any_sync(any, static_cast<unsigned long long>(f.off[3]));
        }
        const float gx = 1.0f - f.fx, gy = 1.0f - f.fy;
        const float wq[4] = {scale * (gx * gy), scale * (f.fx * gy), scale * (gx * f.fy),
                             scale * (f.fx * f.fy)};
        constexpr int NC = RGB ? 3 : 4;  // values per tap
        float v[4 * NC];
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int cc = 0; cc < NC; ++cc) v[NC * t + cc] = act && f.ok[t] ? g[cc] * wq[t] : 0.0f;
        segmented_sum<4 * NC>(peers, v);
        if (!act || (peers & ((1u << lane) - 1u)) != 0u) continue;
        if (peers == 0xffffffffu) {  // the whole warp on one quad (lane 0)
          const bool same = hot.level == level && hot.c0 == c0 && hot.off[0] == f.off[0] &&
                            hot.off[3] == f.off[3];
          if (same) {
#pragma unroll
            for (int i = 0; i < 4 * NC; ++i) hot.v[i] += v[i];
            continue;
          }
          if (!pending) {
            incoming.level = level;
            incoming.c0 = c0;
#pragma unroll
            for (int t = 0; t < 4; ++t) incoming.off[t] = f.off[t];
#pragma unroll
            for (int i = 0; i < 4 * NC; ++i) incoming.v[i] = v[i];
            pending = true;
            continue;
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          // The group's sum decides, not the leader's own weight or validity: other lanes of the
          // quad have other bilinear weights, and with zero padding other valid taps (a quad's
          // four offsets are the same for the whole group; invalid taps contributed zero).
          bool zero = true;
#pragma unroll
          for (int cc = 0; cc < NC; ++cc) zero = zero && v[NC * t + cc] == 0.0f;
          if (zero) continue;
          float* dst = L.grad[level] + f.off[t] * grad_stride + c0;
          if constexpr (RGB) {
            red_add_v4(dst, v[3 * t], v[3 * t + 1], v[3 * t + 2], 0.0f);
          } else if (vector) {
            red_add_v4(dst, v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]);
          } else {
            for (int cc = 0; cc < group; ++cc)
              if (v[4 * t + cc] != 0.0f) red_add(dst + cc, v[4 * t + cc]);
          }
        }
      }
    }
  } else {
  for (int c0 = 0; c0 < channels; c0 += 4) {
    const int group = min(4, channels - c0);
    float g[4];
    bool any_g = false;
    for (int cc = 0; cc < 4; ++cc) {
      g[cc] = live && cc < group ? __ldcs(grad_out + p * channels + c0 + cc) : 0.0f;
      any_g |= g[cc] != 0.0f;
    }
    for (int t = 0; t < 8; ++t) {
      const bool act = any_g && t < taps.n && taps.w[t] != 0.0f;
      const unsigned any = __ballot_sync(0xffffffffu, act);
      if (any == 0u) continue;
      const unsigned long long key =
          act ? (static_cast<unsigned long long>(taps.level[t]) << 48) | static_cast<unsigned long long>(taps.off[t])
              : 0ull;
      unsigned peers = 1u << lane;
      if (act) peers = __match_any_sync(any, key);
      float v[4];
      for (int cc = 0; cc < 4; ++cc) v[cc] = act ? g[cc] * taps.w[t] : 0.0f;
      segmented_sum<4>(peers, v);
      if (!act || (peers & ((1u << lane) - 1u)) != 0u) continue;
      float* dst = L.grad[taps.level[t]] + taps.off[t] * grad_stride + c0;
      if (vector) {
        red_add_v4(dst, v[0], v[1], v[2], v[3]);
      } else {
        for (int cc = 0; cc < group; ++cc)
          if (v[cc] != 0.0f) red_add(dst + cc, v[cc]);
      }
    }
  }
  }
  // With the interpolation (and rasterizer) chained in, pixels past the image go on to the
  // epilogue too (inside = false; they read and write nothing).
  constexpr bool chained = CHAIN != 0;
  if (!inside && !chained) return;
  const bool coord_grads = grad_uv != nullptr || grad_uv_da != nullptr || grad_bias != nullptr ||
                           chained;
  if (!coord_grads) return;
  float g_fx_lo = 0.f, g_fy_lo = 0.f, g_fx_hi = 0.f, g_fy_hi = 0.f, g_frac = 0.f;
  if (live && MODE != DR_FILTER_NEAREST) {
    const float w_hi = k.frac, w_lo = 1.0f - k.frac;
    // With RGB the channel count is known at compile time and the loop unrolls, so that all
    // channels' texel gathers are in flight together.
    const int nch = RGB ? 3 : channels;
#pragma unroll
    for (int c = 0; c < (RGB ? 3 : channels); ++c) {
      const float g = grad_out[p * nch + c];
      const float g_lo = MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR ? g * w_lo : g;
      float t[4];
      const float lower = bilinear_value<B>(L.ptr[k.lo], k.f_lo, nch, c, t);
      {
        const Footprint& f = k.f_lo;
        float dfx = (1.0f - f.fy) * (t[1] - t[0]) + f.fy * (t[3] - t[2]);
        float dfy = (1.0f - f.fx) * (t[2] - t[0]) + f.fx * (t[3] - t[1]);
        if (B == DR_BOUNDARY_CUBE) {
          const float third = (t[0] + t[1] + t[2] + t[3]) / 3.0f;
          dfx += f.dmiss_dx * third;
          dfy += f.dmiss_dy * third;
        }
        g_fx_lo += g_lo * dfx;
        g_fy_lo += g_lo * dfy;
      }
      if (MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR) {
        const float upper = bilinear_value<B>(L.ptr[k.hi], k.f_hi, nch, c, t);
        const Footprint& f = k.f_hi;
        float dfx = (1.0f - f.fy) * (t[1] - t[0]) + f.fy * (t[3] - t[2]);
        float dfy = (1.0f - f.fx) * (t[2] - t[0]) + f.fx * (t[3] - t[1]);
        if (B == DR_BOUNDARY_CUBE) {
          const float third = (t[0] + t[1] + t[2] + t[3]) / 3.0f;
          dfx += f.dmiss_dx * third;
          dfy += f.dmiss_dy * third;
        }
        g_fx_hi += g * w_hi * dfx;
        g_fy_hi += g * w_hi * dfy;
        g_frac += g * (upper - lower);
      }
    }
  }
  // Gradient of the coordinates (u, v) or, for a cube, of the face coordinates (s, t).
  float g_u = 0.f, g_v = 0.f;
  if (live && MODE != DR_FILTER_NEAREST) {
    g_u = g_fx_lo * k.f_lo.slope_x * static_cast<float>(L.w[k.lo]);
    g_v = g_fy_lo * k.f_lo.slope_y * static_cast<float>(L.h[k.lo]);
    if (MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR) {
      g_u += g_fx_hi * k.f_hi.slope_x * static_cast<float>(L.w[k.hi]);
      g_v += g_fy_hi * k.f_hi.slope_y * static_cast<float>(L.h[k.hi]);
    }
  }
  // Gradient of the level of detail: only trilinear filtering depends on it smoothly; it is
  // clamped to the available levels.
  float g_lod = 0.f;
  if (live && MODE == DR_FILTER_LINEAR_MIPMAP_LINEAR) {
    const float top = static_cast<float>(L.num_levels - 1);
    if (k.lod_raw >= 0.0f && k.lod_raw <= top) g_lod = g_frac;
  }
  if (grad_bias != nullptr && inside) grad_bias[p] = g_lod;
  float g_da[4] = {0.f, 0.f, 0.f, 0.f};
  if (live && k.has_da && g_lod != 0.0f) level_of_detail_bwd(k.da, L.h[0], L.w[0], g_lod, g_da);
  if (B == DR_BOUNDARY_CUBE) {
    float g_dir[3] = {0.f, 0.f, 0.f}, g_dir_da[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) cube_project_bwd(k.cube, g_u, g_v, k.has_da ? g_da : nullptr, g_dir, g_dir_da);
    if (grad_uv != nullptr && inside) write_record<3>(grad_uv, p, gst.uv, gst.uv_first, g_dir);
    if (grad_uv_da != nullptr && inside)
      write_record<6>(grad_uv_da, p, gst.uv_da, gst.da_first, g_dir_da);
  } else {
    const float g_uv[2] = {g_u, g_v};
    if constexpr (chained) {
      chain_interpolation<CHAIN == 2>(chain, p, view, col, row, width, height, inside, g_uv, g_da);
      return;
    }
    if (grad_uv != nullptr) write_record<2>(grad_uv, p, gst.uv, gst.uv_first, g_uv);
    if (grad_uv_da != nullptr) write_record<4>(grad_uv_da, p, gst.uv_da, gst.da_first, g_da);
  }
}

// Persistent blocks walk the 16 x 16 pixel tiles of all views; each warp keeps its hot quad across
// the tiles it visits and flushes it at the end.
template <int MODE, int B, bool RGB, int CHAIN>
__global__ void __launch_bounds__(256, B == DR_BOUNDARY_CUBE ? 2 : 3) texture_bwd_kernel(
    const Levels L, int channels, int grad_stride, const float* __restrict__ uv,
    const float* __restrict__ uv_da, const float* __restrict__ bias, const Strides st, int height,
    int width, const float* __restrict__ grad_out, float* __restrict__ grad_uv,
    float* __restrict__ grad_uv_da, float* __restrict__ grad_bias, const GradLayout gst,
    const InterpChain chain, long long tiles_x, long long tiles_per_view, long long tiles) {
  constexpr int NC = RGB ? 3 : 4;
  __shared__ HotQuad hot[8][2];
  const int warp = threadIdx.x >> 5;
  const bool leader = (threadIdx.x & 31u) == 0u;
  if (leader) hot[warp][0].level = hot[warp][1].level = -1;
  __syncwarp();
  int held = 0;
  bool pending = false;
  for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const long long view = tile / tiles_per_view;
    const long long in_view = tile - view * tiles_per_view;
    const long long ty = in_view / tiles_x;
    const int col = static_cast<int>((in_view - ty * tiles_x) * 16) + (threadIdx.x & 15);
    const int row = static_cast<int>(ty * 16) + (threadIdx.x >> 4);
    texture_bwd_tile<MODE, B, RGB, CHAIN>(L, channels, grad_stride, uv, uv_da, bias, st, height, width,
                                   grad_out, grad_uv, grad_uv_da, grad_bias, gst, chain, col,
                                   row, view, hot[warp][held], hot[warp][held ^ 1], pending);
    if (pending) {  // lane 0 only: the new quad replaces the held one
      flush_quad<NC>(L, hot[warp][held], channels, grad_stride);
      held ^= 1;
      pending = false;
    }
  }
  __syncwarp();
  if (leader) flush_quad<NC>(L, hot[warp][held], channels, grad_stride);
}

// ---------------------------------------------------------------------------------------------
// Mip chain (reference.py:449-488): bin j of the coarse level spans [j n, (j + 1) n] and texel i
// of the fine level [i m, (i + 1) m] in units of 1 / (n m), m = ceil(n / 2); the weight is the
// overlap divided by n (0.5 and 0.5 for even n, three taps for odd n).
// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ float halving_weight(int j, int i, int n, int m) {
  const long long lo = max(static_cast<long long>(j) * n, static_cast<long long>(i) * m);
  const long long hi = min(static_cast<long long>(j + 1) * n, static_cast<long long>(i + 1) * m);
  return hi > lo ? static_cast<float>(hi - lo) / static_cast<float>(n) : 0.0f;
}

// One block per output row (image, row); its threads walk the row's (texel, channel) elements.
// Even sizes take the pair-mean path: the area weights are all 1/2, which makes the sum exact in
// either order.
__global__ void __launch_bounds__(256) mip_down_kernel(const float* __restrict__ src, int h, int w,
                                                       int channels, float* __restrict__ dst) {
  const int oh = (h + 1) / 2, ow = (w + 1) / 2;
  const long long out_row = blockIdx.x;
  const long long img = out_row / oh;
  const int j = static_cast<int>(out_row - img * oh);
  const float* image = src + img * h * static_cast<long long>(w) * channels;
  float* out = dst + out_row * ow * channels;
  const int n = ow * channels;
  const bool even = (h % 2 == 0) && (w % 2 == 0);
  const int r0 = static_cast<int>(static_cast<long long>(j) * h / oh);
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int k = e / channels, c = e - k * channels;
    if (even) {
      const float* a = image + (static_cast<long long>(2 * j) * w + 2 * k) * channels + c;
      const float* b = a + static_cast<long long>(w) * channels;
      out[e] = 0.25f * ((__ldg(a) + __ldg(a + channels)) + (__ldg(b) + __ldg(b + channels)));
      continue;
    }
    const int c0 = static_cast<int>(static_cast<long long>(k) * w / ow);
    float acc = 0.0f;
    for (int r = r0; r < min(r0 + 3, h); ++r) {
      const float wr = h > 1 ? halving_weight(j, r, h, oh) : 1.0f;
      if (wr == 0.0f) continue;
      float row = 0.0f;
      for (int q = c0; q < min(c0 + 3, w); ++q) {
        const float wc = w > 1 ? halving_weight(k, q, w, ow) : 1.0f;
        if (wc != 0.0f) row += wc * __ldg(image + (static_cast<long long>(r) * w + q) * channels + c);
      }
      acc += wr * row;
    }
    out[e] = acc;
  }
}

// Even sizes with at most 4 channels: one thread per coarse texel (grid: coarse columns in x,
// coarse rows in y, images in z), the pair sums in the order of mip_down_kernel, so the values
// are the same.
template <int C>
__global__ void __launch_bounds__(256) mip_down_even_kernel(const float* __restrict__ src, int h,
                                                            int w, float* __restrict__ dst) {
  const int ow = w / 2, oh = h / 2;
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  const int j = blockIdx.y;
  if (k >= ow) return;
  const long long img = blockIdx.z;
  const float* a = src + ((img * h + 2 * j) * w + 2 * k) * C;
  const float* b = a + static_cast<long long>(w) * C;
  float* out = dst + ((img * oh + j) * ow + k) * C;
#pragma unroll
  for (int c = 0; c < C; ++c)
    out[c] = 0.25f * ((__ldg(a + c) + __ldg(a + C + c)) + (__ldg(b + c) + __ldg(b + C + c)));
}

// Adjoint of mip_down_kernel in gather form: one block per fine row; each fine element adds the
// weighted gradients of the coarse texels whose bins overlap it.
__global__ void __launch_bounds__(256) mip_down_bwd_kernel(const float* __restrict__ grad_dst,
                                                           int h, int w, int channels,
                                                           float* __restrict__ grad_src,
                                                           bool aligned16, float* __restrict__ out,
                                                           int out_channels) {
  const int oh = (h + 1) / 2, ow = (w + 1) / 2;
  const long long in_row = blockIdx.x;
  const long long img = in_row / h;
  const int r = static_cast<int>(in_row - img * h);
  const float* coarse = grad_dst + img * oh * static_cast<long long>(ow) * channels;
  float* fine = grad_src + in_row * w * channels;
  // With `out`, the sum goes to its first out_channels channels instead of back into grad_src.
  float* out_row = out == nullptr ? nullptr : out + in_row * w * out_channels;
  const int n = w * channels;
  const bool even = (h % 2 == 0) && (w % 2 == 0);
  if (even && channels == 4 && aligned16) {
    // Four-channel texels (the padded gradients of three-channel textures): one 16-byte load of
    // the coarse texel and one 16-byte read-modify-write per fine texel.
    const float4* c4 = reinterpret_cast<const float4*>(coarse) + static_cast<long long>(r / 2) * ow;
    float4* f4 = reinterpret_cast<float4*>(fine);
    for (int q = threadIdx.x; q < w; q += blockDim.x) {
      const float4 g = __ldg(c4 + q / 2);
      float4 v = f4[q];
      v.x += 0.25f * g.x;
      v.y += 0.25f * g.y;
      v.z += 0.25f * g.z;
      v.w += 0.25f * g.w;
      if (out_row == nullptr) {
        f4[q] = v;
      } else {
        const float vv[4] = {v.x, v.y, v.z, v.w};
        for (int c = 0; c < out_channels; ++c) out_row[q * out_channels + c] = vv[c];
      }
    }
    return;
  }
  // Coarse bins overlapping fine texel i: j in [floor(i m / n), ceil((i + 1) m / n) - 1].
  const int j0 = static_cast<int>(static_cast<long long>(r) * oh / h);
  const int j1 = static_cast<int>((static_cast<long long>(r + 1) * oh + h - 1) / h) - 1;
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int q = e / channels, c = e - q * channels;
    if (even) {
      const float v = fine[e] + 0.25f * __ldg(coarse + (static_cast<long long>(r / 2) * ow + q / 2) * channels + c);
      if (out_row == nullptr) fine[e] = v;
      else if (c < out_channels) out_row[q * out_channels + c] = v;
      continue;
    }
    const int k0 = static_cast<int>(static_cast<long long>(q) * ow / w);
    const int k1 = static_cast<int>((static_cast<long long>(q + 1) * ow + w - 1) / w) - 1;
    float acc = 0.0f;
    for (int j = j0; j <= j1; ++j) {
      const float wr = h > 1 ? halving_weight(j, r, h, oh) : 1.0f;
      float row = 0.0f;
      for (int k = k0; k <= k1; ++k) {
        const float wc = w > 1 ? halving_weight(k, q, w, ow) : 1.0f;
        row += wc * __ldg(coarse + (static_cast<long long>(j) * ow + k) * channels + c);
      }
      acc += wr * row;
    }
    if (out_row == nullptr) fine[e] += acc;
    else if (c < out_channels) out_row[q * out_channels + c] = fine[e] + acc;
  }
}

// Several levels of an even mip chain in one launch: a block reduces a 2^n x 2^n tile of the
// source level (n <= kChainLevels) to one texel of level source + n through shared memory and
// writes every intermediate level's texels of the tile. The averages are mip_down_even_kernel's,
// in its order, so the levels are bit for bit those of one launch per level. Grid: source tiles
// across in x, down in y, images in z.
constexpr int kChainLevels = 6;

struct ChainLevels {
  float* level[kChainLevels];
};

template <int C>
__global__ void __launch_bounds__(256) mip_chain_even_kernel(const float* __restrict__ src, int h,
                                                             int w, int n, ChainLevels dst) {
  __shared__ float buf[32 * 32 * C];
  const long long img = blockIdx.z;
  int side = (1 << n) / 2;  // texels per side of the tile in the level being made
  int lh = h / 2, lw = w / 2;
  int y0 = blockIdx.y * side, x0 = blockIdx.x * side;  // the tile's first texel in that level
  for (int i = threadIdx.x; i < side * side; i += blockDim.x) {
    const int j = i / side, k = i - j * side;
    const float* a = src + ((img * h + 2 * (y0 + j)) * static_cast<long long>(w) + 2 * (x0 + k)) * C;
    const float* b = a + static_cast<long long>(w) * C;
    float* out = dst.level[0] + ((img * lh + y0 + j) * static_cast<long long>(lw) + x0 + k) * C;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const float v = 0.25f * ((__ldg(a + c) + __ldg(a + C + c)) + (__ldg(b + c) + __ldg(b + C + c)));
      out[c] = v;
      buf[i * C + c] = v;
    }
  }
  for (int l = 1; l < n; ++l) {
    const int ns = side / 2;  // at most 16, so at most one texel per thread
    const int t = threadIdx.x;
    float v[C];
    __syncthreads();
    if (t < ns * ns) {
      const int j = t / ns, k = t - j * ns;
      const float* a = buf + (2 * j * side + 2 * k) * C;
      const float* b = a + side * C;
#pragma unroll
      for (int c = 0; c < C; ++c) v[c] = 0.25f * ((a[c] + a[C + c]) + (b[c] + b[C + c]));
    }
    __syncthreads();
    lh /= 2;
    lw /= 2;
    y0 /= 2;
    x0 /= 2;
    if (t < ns * ns) {
      const int j = t / ns, k = t - j * ns;
      float* out = dst.level[l] + ((img * lh + y0 + j) * static_cast<long long>(lw) + x0 + k) * C;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        out[c] = v[c];
        buf[t * C + c] = v[c];
      }
    }
    side = ns;
  }
}

// The adjoint of a run of n even halvings (2 <= n <= kChainLevels) in one launch: the gradient
// totals are pushed from the run's coarsest level f + n, whose totals are final (coarser runs go
// first), down to level f. A block owns one texel of level f + n and the 2^d x 2^d tile under it in
// each level f + n - d; level by level, total_l = grad_l + 1/4 total_{l+1}(parent), the sum
// mip_down_bwd_kernel forms for one level, so the results are bit for bit those of one launch per
// level. The block first loads the gradients of its tiles of levels f + n .. f + 1 (1365 texels
// for n = 6) into shared memory in one round of independent loads, turns them into totals there,
// coarsest first, and then streams level f, whose totals go back in place or, with out, to its
// first out_channels channels; grad levels f + 1 .. f + n - 1 are left unspecified. Shared slots:
// level f + n - d at (4^d - 1) / 3, row-major with side 2^d. Grid: level f + n texels across in
// x, down in y, images in z.
struct ChainGrads {
  float* level[kChainLevels + 1];  // [0] level f (fine) .. [n] level f + n (coarse)
};

// Shared texels of the levels above the fine one: (4^6 - 1) / 3.
constexpr int kChainSlots = 1365;

template <int C>
__global__ void __launch_bounds__(256) mip_chain_even_bwd_kernel(ChainGrads g, int hf, int wf,
                                                                 int n, float* __restrict__ out,
                                                                 int out_channels) {
  __shared__ __align__(16) float buf[kChainSlots * C];
  const long long img = blockIdx.z;
  const int slots = ((1 << (2 * n)) - 1) / 3;
  // Slot s holds level f + n - d, d = floor(log4(3 s + 1)), texel s - (4^d - 1) / 3 of its tile.
  auto element = [&](int s, int& d, int& idx) -> long long {
    d = (31 - __clz(3 * s + 1)) >> 1;
    idx = s - ((1 << (2 * d)) - 1) / 3;
    const int k = n - d, side = 1 << d;
    const int j = idx >> d, q = idx & (side - 1);
    const long long lh = hf >> k, lw = wf >> k;
    return ((img * lh + static_cast<long long>(blockIdx.y) * side + j) * lw +
            static_cast<long long>(blockIdx.x) * side + q) * C;
  };
  {
    constexpr int kRounds = (kChainSlots + 255) / 256;
    float v[kRounds][C];
#pragma unroll
    for (int m = 0; m < kRounds; ++m) {
      const int s = threadIdx.x + 256 * m;
      if (s < slots) {
        int d, idx;
        const long long e = element(s, d, idx);
        const float* src = g.level[0];
#pragma unroll
        for (int k = 1; k <= kChainLevels; ++k)
          if (k == n - d) src = g.level[k];
        src += e;
#pragma unroll
        for (int c = 0; c < C; ++c) v[m][c] = src[c];
      }
    }
#pragma unroll
    for (int m = 0; m < kRounds; ++m) {
      const int s = threadIdx.x + 256 * m;
      if (s < slots) {
#pragma unroll
        for (int c = 0; c < C; ++c) buf[s * C + c] = v[m][c];
      }
    }
  }
  // Totals of levels f + n - 1 .. f + 1 (the top texel's is final).
  for (int d = 1; d < n; ++d) {
    __syncthreads();
    const int base = ((1 << (2 * d)) - 1) / 3, pbase = ((1 << (2 * d - 2)) - 1) / 3;
    const int side = 1 << d, half = side >> 1;
    for (int i = threadIdx.x; i < side * side; i += blockDim.x) {
      const int j = i >> d, q = i & (side - 1);
      const float* pv = buf + (pbase + (j >> 1) * half + (q >> 1)) * C;
      float* cv = buf + (base + i) * C;
#pragma unroll
      for (int c = 0; c < C; ++c) cv[c] = cv[c] + 0.25f * pv[c];
    }
  }
  __syncthreads();
  // Level f, four texels per thread at a time with their loads issued first.
  const int side = 1 << n, half = side >> 1;
  const int pbase = ((1 << (2 * n - 2)) - 1) / 3;
  const long long lw = wf;
  const long long row0 = static_cast<long long>(blockIdx.y) * side;
  const long long col0 = static_cast<long long>(blockIdx.x) * side;
  float* level = g.level[0];
  for (int i0 = threadIdx.x; i0 < side * side; i0 += 4 * blockDim.x) {
    float v[4][C];
    long long e[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * blockDim.x;
      e[u] = -1;
      if (i < side * side) {
        const int j = i >> n, q = i & (side - 1);
        e[u] = ((img * hf + row0 + j) * lw + col0 + q) * C;
        if constexpr (C == 4) {
          const float4 gl = *reinterpret_cast<const float4*>(level + e[u]);
          v[u][0] = gl.x;
          v[u][1] = gl.y;
          v[u][2] = gl.z;
          v[u][3] = gl.w;
        } else {
#pragma unroll
          for (int c = 0; c < C; ++c) v[u][c] = level[e[u] + c];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * blockDim.x;
      if (e[u] < 0) continue;
      const int j = i >> n, q = i & (side - 1);
      const float* pv = buf + (pbase + (j >> 1) * half + (q >> 1)) * C;
#pragma unroll
      for (int c = 0; c < C; ++c) v[u][c] = v[u][c] + 0.25f * pv[c];
      if (out != nullptr) {
        float* o = out + (e[u] / C) * out_channels;
#pragma unroll
        for (int c = 0; c < C; ++c)
          if (c < out_channels) o[c] = v[u][c];
      } else if constexpr (C == 4) {
        *reinterpret_cast<float4*>(level + e[u]) = make_float4(v[u][0], v[u][1], v[u][2], v[u][3]);
      } else {
#pragma unroll
        for (int c = 0; c < C; ++c) level[e[u] + c] = v[u][c];
      }
    }
  }
}

template <int MODE, int B>
void launch_fwd(const Levels& L, int channels, const float* uv, const float* uv_da,
                const float* bias, Strides st, long long total, long long ppi, float* out,
                cudaStream_t s) {
  // Up to four channels a thread's own (12- or 16-byte) stores coalesce well enough, and the
  // block barrier of staging costs more (3 channels on config 5: 1.78 ms staged, 1.64 ms direct).
  const size_t stage_bytes = sizeof(float) * 256 * static_cast<size_t>(channels);
  const bool staged = channels > 4 && stage_bytes <= 48 * 1024;
  if (channels == 3 && !staged)
    texture_fwd_kernel<MODE, B, 3><<<blocks_for(total, 256), 256, 0, s>>>(
        L, channels, uv, uv_da, bias, st, total, ppi, out, false);
  else
    texture_fwd_kernel<MODE, B, 0><<<blocks_for(total, 256), 256, staged ? stage_bytes : 0, s>>>(
        L, channels, uv, uv_da, bias, st, total, ppi, out, staged);
}

template <int MODE, int B>
void launch_bwd(const Levels& L, int channels, int grad_stride, const float* uv,
                const float* uv_da, const float* bias, Strides st, int batch, int height,
                int width, const float* grad_out, float* grad_uv, float* grad_uv_da,
                float* grad_bias, GradLayout gst, const InterpChain& chain, cudaStream_t s) {
  const long long tiles_x = (width + 15) / 16;
  const long long tiles_per_view = tiles_x * ((height + 15) / 16);
  const long long tiles = tiles_per_view * batch;
  constexpr bool quads = B != DR_BOUNDARY_CUBE && MODE != DR_FILTER_NEAREST;
  auto launch = [&](auto kernel) {
    const long long grid = min(tiles, static_cast<long long>(resident_blocks(kernel, 256)));
    kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(L, channels, grad_stride, uv, uv_da, bias,
                                                      st, height, width, grad_out, grad_uv,
                                                      grad_uv_da, grad_bias, gst, chain, tiles_x,
                                                      tiles_per_view, tiles);
  };
  const bool rgb = quads && channels == 3 && grad_stride == 4;
  if constexpr (B != DR_BOUNDARY_CUBE && MODE != DR_FILTER_NEAREST) {
    if (chain.grad_pos != nullptr) {
      if (rgb) launch(texture_bwd_kernel<MODE, B, true, 2>);
      else launch(texture_bwd_kernel<MODE, B, false, 2>);
      return;
    }
    if (chain.grad_rast != nullptr) {
      if (rgb) launch(texture_bwd_kernel<MODE, B, true, 1>);
      else launch(texture_bwd_kernel<MODE, B, false, 1>);
      return;
    }
  }
  if (rgb)
    launch(texture_bwd_kernel<MODE, B, quads, 0>);
  else
    launch(texture_bwd_kernel<MODE, B, false, 0>);
}

template <int B, typename F>
void dispatch_mode(int mode, F&& f) {
  switch (mode) {
    case 0: f(std::integral_constant<int, 0>{}, std::integral_constant<int, B>{}); break;
    case 1: f(std::integral_constant<int, 1>{}, std::integral_constant<int, B>{}); break;
    case 2: f(std::integral_constant<int, 2>{}, std::integral_constant<int, B>{}); break;
    default: f(std::integral_constant<int, 3>{}, std::integral_constant<int, B>{}); break;
  }
}

template <typename F>
void dispatch(int mode, int boundary, F&& f) {
  switch (boundary) {
    case 0: dispatch_mode<0>(mode, f); break;
    case 1: dispatch_mode<1>(mode, f); break;
    case 2: dispatch_mode<2>(mode, f); break;
    default: dispatch_mode<3>(mode, f); break;
  }
}

int make_levels(const float* const* level_ptr, float* const* grad_ptr, const int32_t* level_h,
                const int32_t* level_w, const int64_t* level_batch_stride, int32_t num_levels,
                int32_t channels, int32_t filter_mode, int32_t boundary_mode, int64_t batch,
                Levels& L) {
  if (channels < 1) return DR_ERR_INVALID_ARGUMENT;
  if (num_levels < 1 || num_levels > DR_MAX_LEVELS || level_ptr == nullptr || level_h == nullptr ||
      level_w == nullptr || level_batch_stride == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  if (filter_mode < 0 || filter_mode > 3 || boundary_mode < 0 || boundary_mode > 3)
    return DR_ERR_INVALID_ARGUMENT;
  L.num_levels = num_levels;
  for (int l = 0; l < DR_MAX_LEVELS; ++l) {
    const bool used = l < num_levels;
    L.ptr[l] = used ? level_ptr[l] : nullptr;
    L.grad[l] = used && grad_ptr != nullptr ? grad_ptr[l] : nullptr;
    L.h[l] = used ? level_h[l] : 1;
    L.w[l] = used ? level_w[l] : 1;
    L.bstride[l] = used ? level_batch_stride[l] / channels : 0;
    // A level is shared by all views (stride 0) or holds one image per view.
    const long long image = static_cast<long long>(L.h[l]) * L.w[l] *
                            (boundary_mode == DR_BOUNDARY_CUBE ? 6 : 1);
    L.texels[l] = L.bstride[l] > 0 ? L.bstride[l] * (batch > 0 ? batch : 1) : image;
    if (used && (L.ptr[l] == nullptr || L.h[l] < 1 || L.w[l] < 1 || L.bstride[l] < 0))
      return DR_ERR_INVALID_ARGUMENT;
    if (used && grad_ptr != nullptr && L.grad[l] == nullptr) return DR_ERR_INVALID_ARGUMENT;
    if (used && boundary_mode == DR_BOUNDARY_CUBE && L.h[l] != L.w[l]) return DR_ERR_INVALID_ARGUMENT;
  }
  return DR_OK;
}

}  // namespace
}  // namespace dr

using namespace dr;

extern "C" int dr_texture_fwd(const float* const* level_ptr, const int32_t* level_h,
                              const int32_t* level_w, const int64_t* level_batch_stride,
                              int32_t num_levels, int32_t channels, const float* uv,
                              int64_t uv_stride, const float* uv_da, int64_t uv_da_stride,
                              const float* bias, int64_t batch,
                              int32_t height, int32_t width, int32_t filter_mode,
                              int32_t boundary_mode, float* out, void* stream) {
  Levels L;
  int status = make_levels(level_ptr, nullptr, level_h, level_w, level_batch_stride, num_levels,
                           channels, filter_mode, boundary_mode, batch, L);
  if (status != DR_OK) return status;
  if (channels < 1 || batch < 0 || height < 0 || width < 0) return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0) return DR_OK;
  if (uv == nullptr || out == nullptr) return DR_ERR_INVALID_ARGUMENT;
  const long long ppi = static_cast<long long>(height) * width;
  const int uv_width = boundary_mode == DR_BOUNDARY_CUBE ? 3 : 2;
  const int da_width = boundary_mode == DR_BOUNDARY_CUBE ? 6 : 4;
  const Strides st = {uv_stride > 0 ? uv_stride : uv_width, uv_da_stride > 0 ? uv_da_stride : da_width};
  if (st.uv < uv_width || (uv_da != nullptr && st.uv_da < da_width)) return DR_ERR_INVALID_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  dispatch(filter_mode, boundary_mode, [&](auto m, auto b) {
    launch_fwd<decltype(m)::value, decltype(b)::value>(L, channels, uv, uv_da, bias, st, total,
                                                       ppi, out, s);
  });
  return launch_status();
}

namespace {

int texture_bwd_impl(const float* const* level_ptr, float* const* grad_level_ptr,
                              const int32_t* level_h, const int32_t* level_w,
                              const int64_t* level_batch_stride, int32_t num_levels,
                              int32_t channels, int32_t grad_channel_stride, const float* uv,
                              int64_t uv_stride, const float* uv_da, int64_t uv_da_stride,
                              const float* bias, int64_t batch, int32_t height, int32_t width,
                              int32_t filter_mode, int32_t boundary_mode, const float* grad_out,
                              float* grad_uv, int64_t grad_uv_stride, int32_t grad_uv_first,
                              float* grad_uv_da, int64_t grad_uv_da_stride,
                              int32_t grad_uv_da_first, float* grad_bias, const InterpChain& chain,
                              void* stream) {
  if (grad_level_ptr == nullptr) return DR_ERR_INVALID_ARGUMENT;
  Levels L;
  int status = make_levels(level_ptr, grad_level_ptr, level_h, level_w, level_batch_stride,
                           num_levels, channels, filter_mode, boundary_mode, batch, L);
  if (status != DR_OK) return status;
  if (channels < 1 || batch < 0 || height < 0 || width < 0) return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0) return DR_OK;
  if (uv == nullptr || grad_out == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (grad_uv_da != nullptr && uv_da == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (grad_bias != nullptr && bias == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (batch > 65535 || height >= (1 << 20) || width >= (1 << 20)) return DR_ERR_TOO_LARGE;
  if (grad_channel_stride < channels) return DR_ERR_INVALID_ARGUMENT;
  const int uv_width = boundary_mode == DR_BOUNDARY_CUBE ? 3 : 2;
  const int da_width = boundary_mode == DR_BOUNDARY_CUBE ? 6 : 4;
  const Strides st = {uv_stride > 0 ? uv_stride : uv_width, uv_da_stride > 0 ? uv_da_stride : da_width};
  if (st.uv < uv_width || (uv_da != nullptr && st.uv_da < da_width)) return DR_ERR_INVALID_ARGUMENT;
  const GradLayout gst = {grad_uv_stride > 0 ? grad_uv_stride : uv_width,
                          grad_uv_da_stride > 0 ? grad_uv_da_stride : da_width,
                          grad_uv_first < 0 ? -1 : grad_uv_first,
                          grad_uv_da_first < 0 ? -1 : grad_uv_da_first};
  if (gst.uv < uv_width || gst.uv_da < da_width) return DR_ERR_INVALID_ARGUMENT;
  if (gst.uv_first + uv_width > gst.uv || gst.da_first + da_width > gst.uv_da)
    return DR_ERR_INVALID_ARGUMENT;
  if (grad_channel_stride == 4) {
    for (int l = 0; l < num_levels; ++l)
      if ((reinterpret_cast<uintptr_t>(grad_level_ptr[l]) & 15u) != 0) return DR_ERR_INVALID_ARGUMENT;
  }
  cudaStream_t s = as_stream(stream);
  dispatch(filter_mode, boundary_mode, [&](auto m, auto b) {
    launch_bwd<decltype(m)::value, decltype(b)::value>(L, channels, grad_channel_stride, uv, uv_da,
                                                       bias, st, static_cast<int>(batch), height,
                                                       width, grad_out, grad_uv, grad_uv_da,
                                                       grad_bias, gst, chain, s);
  });
  return launch_status();
}

}  // namespace

extern "C" int dr_texture_bwd(const float* const* level_ptr, float* const* grad_level_ptr,
                              const int32_t* level_h, const int32_t* level_w,
                              const int64_t* level_batch_stride, int32_t num_levels,
                              int32_t channels, int32_t grad_channel_stride, const float* uv,
                              int64_t uv_stride, const float* uv_da, int64_t uv_da_stride,
                              const float* bias, int64_t batch, int32_t height, int32_t width,
                              int32_t filter_mode, int32_t boundary_mode, const float* grad_out,
                              float* grad_uv, int64_t grad_uv_stride, int32_t grad_uv_first,
                              float* grad_uv_da, int64_t grad_uv_da_stride,
                              int32_t grad_uv_da_first, float* grad_bias, void* stream) {
  const InterpChain none = {};
  return texture_bwd_impl(level_ptr, grad_level_ptr, level_h, level_w, level_batch_stride,
                          num_levels, channels, grad_channel_stride, uv, uv_stride, uv_da,
                          uv_da_stride, bias, batch, height, width, filter_mode, boundary_mode,
                          grad_out, grad_uv, grad_uv_stride, grad_uv_first, grad_uv_da,
                          grad_uv_da_stride, grad_uv_da_first, grad_bias, none, stream);
}

namespace {

// The interpolation part of an InterpChain from the entry points' arguments, validated.
int interp_chain(int32_t filter_mode, int32_t boundary_mode, int64_t batch, int32_t height,
                 int32_t width, const float* uv_da, const float* rast, const int32_t* tri,
                 int64_t num_tri, const float* attr, int64_t attr_batch, int64_t num_vert,
                 int32_t attr_channels, int32_t cu, int32_t cv, int32_t du, int32_t dv,
                 bool want_db, InterpChain& chain) {
  if (boundary_mode == DR_BOUNDARY_CUBE || filter_mode < 1 || filter_mode > 3)
    return DR_ERR_INVALID_ARGUMENT;
  if (batch < 0 || height < 0 || width < 0 || num_tri < 0 || num_tri >= (1LL << 31) ||
      num_vert < 0 || attr_channels < 1)
    return DR_ERR_INVALID_ARGUMENT;
  if (attr_batch != 1 && attr_batch != batch) return DR_ERR_INVALID_ARGUMENT;
  if (cu < 0 || cu >= attr_channels || cv < 0 || cv >= attr_channels) return DR_ERR_INVALID_ARGUMENT;
  if (want_db && (uv_da == nullptr || filter_mode != 3 || du < 0 || du >= attr_channels ||
                  dv < 0 || dv >= attr_channels))
    return DR_ERR_INVALID_ARGUMENT;
  if (batch * static_cast<long long>(height) * width > 0) {
    if (rast == nullptr || (reinterpret_cast<uintptr_t>(rast) & 15u) != 0)
      return DR_ERR_INVALID_ARGUMENT;
    if (num_tri > 0 && tri == nullptr) return DR_ERR_INVALID_ARGUMENT;
    if (num_vert > 0 && attr == nullptr) return DR_ERR_INVALID_ARGUMENT;
  }
  chain = InterpChain{};
  chain.rast = reinterpret_cast<const float4*>(rast);
  chain.tri = tri;
  chain.attr = attr;
  chain.attr_view_stride = attr_batch == 1 ? 0 : num_vert * attr_channels;
  chain.num_vert = num_vert;
  chain.attr_channels = attr_channels;
  chain.num_tri = static_cast<int>(num_tri);
  chain.cu = cu;
  chain.cv = cv;
  chain.du = du;
  chain.dv = dv;
  return DR_OK;
}

}  // namespace

extern "C" int dr_texture_bwd_interp(
    const float* const* level_ptr, float* const* grad_level_ptr, const int32_t* level_h,
    const int32_t* level_w, const int64_t* level_batch_stride, int32_t num_levels,
    int32_t channels, int32_t grad_channel_stride, const float* uv, int64_t uv_stride,
    const float* uv_da, int64_t uv_da_stride, const float* bias, int64_t batch, int32_t height,
    int32_t width, int32_t filter_mode, int32_t boundary_mode, const float* grad_out,
    float* grad_bias, const float* rast, const int32_t* tri, int64_t num_tri, const float* attr,
    int64_t attr_batch, int64_t num_vert, int32_t attr_channels, int32_t cu, int32_t cv,
    int32_t du, int32_t dv, float* grad_rast, float* grad_db, void* stream) {
  InterpChain chain;
  const int status = interp_chain(filter_mode, boundary_mode, batch, height, width, uv_da, rast,
                                  tri, num_tri, attr, attr_batch, num_vert, attr_channels, cu, cv,
                                  du, dv, grad_db != nullptr, chain);
  if (status != DR_OK) return status;
  const uintptr_t align = reinterpret_cast<uintptr_t>(grad_rast) | reinterpret_cast<uintptr_t>(grad_db);
  if (batch * static_cast<long long>(height) * width > 0 && (grad_rast == nullptr || (align & 15u) != 0))
    return DR_ERR_INVALID_ARGUMENT;
  chain.grad_rast = reinterpret_cast<float4*>(grad_rast);
  chain.grad_db = reinterpret_cast<float4*>(grad_db);
  return texture_bwd_impl(level_ptr, grad_level_ptr, level_h, level_w, level_batch_stride,
                          num_levels, channels, grad_channel_stride, uv, uv_stride, uv_da,
                          uv_da_stride, bias, batch, height, width, filter_mode, boundary_mode,
                          grad_out, nullptr, 0, -1, nullptr, 0, -1, grad_bias, chain, stream);
}

extern "C" int dr_texture_bwd_resolve(
    const float* const* level_ptr, float* const* grad_level_ptr, const int32_t* level_h,
    const int32_t* level_w, const int64_t* level_batch_stride, int32_t num_levels,
    int32_t channels, int32_t grad_channel_stride, const float* uv, int64_t uv_stride,
    const float* uv_da, int64_t uv_da_stride, const float* bias, int64_t batch, int32_t height,
    int32_t width, int32_t filter_mode, int32_t boundary_mode, const float* grad_out,
    float* grad_bias, const float* rast, const int32_t* tri, int64_t num_tri, const float* attr,
    int64_t attr_batch, int64_t num_vert, int32_t attr_channels, int32_t cu, int32_t cv,
    int32_t du, int32_t dv, const int64_t* keys, const float* pos, int64_t pos_batch,
    int64_t pos_num_vert, int32_t rast_db_gradient, float* grad_pos, void* stream) {
  const bool want_db = rast_db_gradient != 0;
  InterpChain chain;
  const int status = interp_chain(filter_mode, boundary_mode, batch, height, width, uv_da, rast,
                                  tri, num_tri, attr, attr_batch, num_vert, attr_channels, cu, cv,
                                  du, dv, want_db, chain);
  if (status != DR_OK) return status;
  if (pos_batch != 1 && pos_batch != batch) return DR_ERR_INVALID_ARGUMENT;
  if (pos_num_vert < 0 || num_tri > (1LL << 24)) return DR_ERR_INVALID_ARGUMENT;
  if (batch * static_cast<long long>(height) * width > 0) {
    const uintptr_t align = reinterpret_cast<uintptr_t>(pos) | reinterpret_cast<uintptr_t>(grad_pos);
    if (keys == nullptr || pos == nullptr || grad_pos == nullptr || (align & 15u) != 0)
      return DR_ERR_INVALID_ARGUMENT;
  }
  chain.keys = reinterpret_cast<const long long*>(keys);
  chain.pos = pos;
  chain.pos_view_stride = pos_batch == 1 ? 0 : pos_num_vert;
  chain.pos_num_vert = pos_num_vert;
  chain.grad_pos = grad_pos;
  chain.resolve_db = want_db;
  return texture_bwd_impl(level_ptr, grad_level_ptr, level_h, level_w, level_batch_stride,
                          num_levels, channels, grad_channel_stride, uv, uv_stride, uv_da,
                          uv_da_stride, bias, batch, height, width, filter_mode, boundary_mode,
                          grad_out, nullptr, 0, -1, nullptr, 0, -1, grad_bias, chain, stream);
}

extern "C" int dr_texture_chain_bwd(const float* grad_uv, const float* grad_uv_da, int64_t batch,
                                    int32_t height, int32_t width, const int32_t* tri,
                                    int64_t num_tri, const float* attr, int64_t attr_batch,
                                    int64_t num_vert, int32_t attr_channels, int32_t cu,
                                    int32_t cv, int32_t du, int32_t dv, const int64_t* keys,
                                    const float* pos, int64_t pos_batch, int64_t pos_num_vert,
                                    int32_t rast_db_gradient, float* grad_pos, void* stream) {
  const bool want_db = rast_db_gradient != 0;
  if (batch < 0 || height < 0 || width < 0 || num_tri < 0 || num_tri > (1LL << 24) ||
      num_vert < 0 || pos_num_vert < 0 || attr_channels < 1)
    return DR_ERR_INVALID_ARGUMENT;
  if ((attr_batch != 1 && attr_batch != batch) || (pos_batch != 1 && pos_batch != batch))
    return DR_ERR_INVALID_ARGUMENT;
  if (cu < 0 || cu >= attr_channels || cv < 0 || cv >= attr_channels) return DR_ERR_INVALID_ARGUMENT;
  if (want_db && (grad_uv_da == nullptr || du < 0 || du >= attr_channels || dv < 0 ||
                  dv >= attr_channels))
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0) return DR_OK;
  const uintptr_t align = reinterpret_cast<uintptr_t>(pos) | reinterpret_cast<uintptr_t>(grad_pos) |
                          reinterpret_cast<uintptr_t>(grad_uv_da);
  if (grad_uv == nullptr || keys == nullptr || pos == nullptr || grad_pos == nullptr ||
      (align & 15u) != 0 || (reinterpret_cast<uintptr_t>(grad_uv) & 7u) != 0)
    return DR_ERR_INVALID_ARGUMENT;
  if (num_tri > 0 && tri == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (num_vert > 0 && attr == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (batch > 65535 || height > 65535) return DR_ERR_TOO_LARGE;
  InterpChain c = {};
  c.tri = tri;
  c.attr = attr;
  c.attr_view_stride = attr_batch == 1 ? 0 : num_vert * attr_channels;
  c.num_vert = num_vert;
  c.attr_channels = attr_channels;
  c.num_tri = static_cast<int>(num_tri);
  c.cu = cu;
  c.cv = cv;
  c.du = du;
  c.dv = dv;
  c.keys = reinterpret_cast<const long long*>(keys);
  c.pos = pos;
  c.pos_view_stride = pos_batch == 1 ? 0 : pos_num_vert;
  c.pos_num_vert = pos_num_vert;
  c.grad_pos = grad_pos;
  c.resolve_db = want_db;
  const dim3 grid((width + 255) / 256, static_cast<unsigned>(height), static_cast<unsigned>(batch));
  chain_parts_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      c, reinterpret_cast<const float2*>(grad_uv),
      want_db ? reinterpret_cast<const float4*>(grad_uv_da) : nullptr, height, width);
  return launch_status();
}

extern "C" int dr_mip_downsample(const float* src, int64_t images, int32_t h, int32_t w,
                                 int32_t channels, float* dst, void* stream) {
  if (images < 0 || h < 1 || w < 1 || channels < 1 || src == nullptr || dst == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  const long long rows = images * ((h + 1) / 2);
  if (rows == 0) return DR_OK;
  if (rows >= (1LL << 31)) return DR_ERR_TOO_LARGE;
  cudaStream_t s = as_stream(stream);
  if (h % 2 == 0 && w % 2 == 0 && channels <= 4 && h / 2 <= 65535 && images <= 65535) {
    const dim3 grid((w / 2 + 255) / 256, h / 2, static_cast<unsigned>(images));
    switch (channels) {
      case 1: mip_down_even_kernel<1><<<grid, 256, 0, s>>>(src, h, w, dst); break;
      case 2: mip_down_even_kernel<2><<<grid, 256, 0, s>>>(src, h, w, dst); break;
      case 3: mip_down_even_kernel<3><<<grid, 256, 0, s>>>(src, h, w, dst); break;
      default: mip_down_even_kernel<4><<<grid, 256, 0, s>>>(src, h, w, dst); break;
    }
    return launch_status();
  }
  mip_down_kernel<<<static_cast<unsigned>(rows), 256, 0, s>>>(src, h, w, channels, dst);
  return launch_status();
}

extern "C" int dr_mip_downsample_bwd(const float* grad_dst, int64_t images, int32_t h, int32_t w,
                                     int32_t channels, float* grad_src, float* out,
                                     int32_t out_channels, void* stream) {
  if (images < 0 || h < 1 || w < 1 || channels < 1 || grad_dst == nullptr || grad_src == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  if (out != nullptr && (out_channels < 1 || out_channels > channels)) return DR_ERR_INVALID_ARGUMENT;
  const long long rows = images * h;
  if (rows == 0) return DR_OK;
  if (rows >= (1LL << 31)) return DR_ERR_TOO_LARGE;
  const bool aligned16 = ((reinterpret_cast<uintptr_t>(grad_dst) | reinterpret_cast<uintptr_t>(grad_src)) & 15u) == 0;
  mip_down_bwd_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(
      grad_dst, h, w, channels, grad_src, aligned16, out, out_channels);
  return launch_status();
}
namespace {

// Sizes of level l of a chain whose base is h x w (the reference's rounding up).
void level_size(int h, int w, int l, int& lh, int& lw) {
  lh = h;
  lw = w;
  for (int i = 0; i < l; ++i) {
    lh = (lh + 1) / 2;
    lw = (lw + 1) / 2;
  }
}

// Largest n <= limit such that halving h x w n times stays even every time.
int even_run(int h, int w, int limit) {
  int n = 0;
  while (n < limit && h % 2 == 0 && w % 2 == 0) {
    h /= 2;
    w /= 2;
    ++n;
  }
  return n;
}

}  // namespace

extern "C" int dr_mip_build(const float* src, int64_t images, int32_t h, int32_t w,
                            int32_t channels, int32_t levels, float* const* dst, void* stream) {
  if (images < 0 || h < 1 || w < 1 || channels < 1 || levels < 0 || levels > DR_MAX_LEVELS - 1 ||
      src == nullptr || (levels > 0 && dst == nullptr))
    return DR_ERR_INVALID_ARGUMENT;
  for (int l = 0; l < levels; ++l)
    if (dst[l] == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (images == 0 || levels == 0) return DR_OK;
  cudaStream_t s = as_stream(stream);
  const float* cur = src;
  int ch = h, cw = w;
  for (int l = 0; l < levels;) {
    const int n = even_run(ch, cw, min(kChainLevels, levels - l));
    if (n >= 2 && channels <= 4 && images <= 65535 && (ch >> n) <= 65535) {
      ChainLevels cl = {};
      for (int i = 0; i < n; ++i) cl.level[i] = dst[l + i];
      const dim3 grid(static_cast<unsigned>(cw >> n), static_cast<unsigned>(ch >> n),
                      static_cast<unsigned>(images));
      switch (channels) {
        case 1: mip_chain_even_kernel<1><<<grid, 256, 0, s>>>(cur, ch, cw, n, cl); break;
        case 2: mip_chain_even_kernel<2><<<grid, 256, 0, s>>>(cur, ch, cw, n, cl); break;
        case 3: mip_chain_even_kernel<3><<<grid, 256, 0, s>>>(cur, ch, cw, n, cl); break;
        default: mip_chain_even_kernel<4><<<grid, 256, 0, s>>>(cur, ch, cw, n, cl); break;
      }
      const int status = launch_status();
      if (status != DR_OK) return status;
      cur = dst[l + n - 1];
      ch >>= n;
      cw >>= n;
      l += n;
      continue;
    }
    const int status = dr_mip_downsample(cur, images, ch, cw, channels, dst[l], stream);
    if (status != DR_OK) return status;
    cur = dst[l];
    ch = (ch + 1) / 2;
    cw = (cw + 1) / 2;
    ++l;
  }
  return DR_OK;
}

extern "C" int dr_mip_build_bwd(float* const* grad_levels, int64_t images, int32_t h, int32_t w,
                                int32_t channels, int32_t levels, float* out, int32_t out_channels,
                                void* stream) {
  if (images < 0 || h < 1 || w < 1 || channels < 1 || levels < 0 || levels > DR_MAX_LEVELS - 1 ||
      grad_levels == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  for (int l = 0; l <= levels; ++l)
    if (grad_levels[l] == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (out != nullptr && (out_channels < 1 || out_channels > channels || levels == 0))
    return DR_ERR_INVALID_ARGUMENT;
  if (images == 0 || levels == 0) return DR_OK;
  // The forward chain's steps (dr_mip_build: runs of even halvings, single halvings otherwise),
  // undone coarsest first. Runs take the tiled adjoint (mip_chain_even_bwd_kernel) when their
  // texels are 16-byte aligned or not 4-channel; every other step is one mip_down_bwd_kernel
  // launch. (A single pass over the base that reads every coarser level per texel was slower on
  // config 5: 0.31 against 0.20 ms for one launch per level.)
  int first[DR_MAX_LEVELS], count[DR_MAX_LEVELS], steps = 0;
  {
    int ch = h, cw = w;
    for (int l = 0; l < levels;) {
      const int n = even_run(ch, cw, min(kChainLevels, levels - l));
      const bool run = n >= 2 && channels <= 4 && images <= 65535 && (ch >> n) <= 65535;
      first[steps] = l;
      count[steps] = run ? n : 1;
      ++steps;
      if (run) {
        ch >>= n;
        cw >>= n;
        l += n;
      } else {
        ch = (ch + 1) / 2;
        cw = (cw + 1) / 2;
        ++l;
      }
    }
  }
  cudaStream_t s = as_stream(stream);
  for (int i = steps - 1; i >= 0; --i) {
    const int f = first[i], n = count[i];
    int lh, lw;
    level_size(h, w, f, lh, lw);
    float* dst = f == 0 ? out : nullptr;
    bool tiled = n >= 2;
    if (tiled && channels == 4) {
      uintptr_t bits = 0;
      for (int k = 0; k <= n; ++k) bits |= reinterpret_cast<uintptr_t>(grad_levels[f + k]);
      tiled = (bits & 15u) == 0;
    }
    if (tiled) {
      ChainGrads cg = {};
      for (int k = 0; k <= n; ++k) cg.level[k] = grad_levels[f + k];
      const dim3 grid(static_cast<unsigned>(lw >> n), static_cast<unsigned>(lh >> n),
                      static_cast<unsigned>(images));
      switch (channels) {
        case 1: mip_chain_even_bwd_kernel<1><<<grid, 256, 0, s>>>(cg, lh, lw, n, dst, out_channels); break;
        case 2: mip_chain_even_bwd_kernel<2><<<grid, 256, 0, s>>>(cg, lh, lw, n, dst, out_channels); break;
        case 3: mip_chain_even_bwd_kernel<3><<<grid, 256, 0, s>>>(cg, lh, lw, n, dst, out_channels); break;
        default: mip_chain_even_bwd_kernel<4><<<grid, 256, 0, s>>>(cg, lh, lw, n, dst, out_channels); break;
      }
      const int status = launch_status();
      if (status != DR_OK) return status;
      continue;
    }
    for (int l = f + n; l > f; --l) {
      level_size(h, w, l - 1, lh, lw);
      const int status = dr_mip_downsample_bwd(grad_levels[l], images, lh, lw, channels,
                                               grad_levels[l - 1], l == 1 ? out : nullptr,
                                               out_channels, stream);
      if (status != DR_OK) return status;
    }
  }
  return DR_OK;
}

DR_DEFINE_FAULT_QUERY(texture)
