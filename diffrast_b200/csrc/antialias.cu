// Silhouette antialiasing on B200 (diffrast reference.py:202-265, :675-814).
//
// For every horizontally or vertically adjacent pixel pair showing different triangles, the
// triangle seen at each pixel is followed towards the other pixel: the first of its edges crossed
// on the way (within a rounding slack) gives the crossing t, which counts when the edge is a
// silhouette and is handled by this axis; the nearer side wins when both find one. The pixel
// whose half holds the crossing blends |t - 1/2| of the other's colour.
//
// B200 design:
//   - Pixel tiles with a one-pixel halo: each pair is evaluated once per block into shared memory
//     and every pixel writes only its own output, so the forward pass and the colour gradient need
//     no atomics and are deterministic. The position gradient of a pair is scattered once, by the
//     block where its left or upper pixel is an output pixel.
//   - The silhouette test runs on the fly for the one edge a pair crosses, instead of classifying
//     every edge of every view beforehand. It needs the crossed triangle's own vertices (already
//     loaded for the crossing) and one more: the vertex opposite the edge in the adjacent
//     triangle, read from a per-edge table (dr_edge_opposite_vertices) built once per index
//     buffer from the adjacency, so the test costs one dependent load.
//   - Edge adjacency is built with a device hash table on 64-bit vertex-pair keys (count, first and
//     second edge per key): no sort, deterministic, identical to the reference's result.
// The edge tests use explicitly rounded operations in the reference's order so that the set of
// blended edges matches it bit for bit; the side test of the silhouette classification rounds like
// the CPU cross product of PyTorch, each component fma(a_i, b_j, -(a_j * b_i)).
#include <cstdint>

#include "common.cuh"
#include "edge_hash.cuh"
#include "warp_reduce.cuh"

namespace dr {
namespace {

struct AaCtx {
  const float* color;
  const float4* rast;
  const float* pos;
  const int* tri;
  const int* opposite;  // [num_tri, 3] vertex across each edge, -1 for a silhouette by topology
  long long pos_batch, num_vert;
  int num_tri;
  int height, width, channels;
};

// Triangle id of a rast pixel as the reference reads it for antialiasing: round(id + 1) - 1, with
// ids past the end of tri counted as background (-1). Values below -1 are kept distinct from -1
// only as far as the outcome needs: they cover nothing, so all map to -2.
__device__ __forceinline__ int aa_triangle(float id_plus_one, int num_tri) {
  const float r = rintf(id_plus_one);
  if (!(r >= 0.0f)) return -2;
  if (r > static_cast<float>(num_tri)) return -1;
  return static_cast<int>(r) - 1;
}

struct Tri2 {
  int idx[3];
  float x[3], y[3], w[3];
};

__device__ __forceinline__ Tri2 load_tri(const AaCtx& a, long long pb, int t) {
  Tri2 v;
  const long long base = pb * a.num_vert;
  for (int k = 0; k < 3; ++k) {
    v.idx[k] = static_cast<int>(
        checked_index(__ldg(a.tri + 3 * static_cast<long long>(t) + k), a.num_vert, kSiteVertex));
    const float4 p = __ldg(reinterpret_cast<const float4*>(a.pos) + base + v.idx[k]);
    v.x[k] = p.x;
    v.y[k] = p.y;
    v.w[k] = p.w;
  }
  return v;
}

// Sign test of the silhouette classification: sign((l . p) * p_w) with l = a x b in (x, y, w).
__device__ __forceinline__ float side_sign(const float l[3], const float4& p) {
  const float d = add(add(mul(l[0], p.x), mul(l[1], p.y)), mul(l[2], p.w));
  const float s = mul(d, p.w);
  return s > 0.0f ? 1.0f : (s < 0.0f ? -1.0f : (s == 0.0f ? 0.0f : s));
}

// Whether edge k of triangle t is a silhouette in view pb (reference.py:790-814): unshared, shared
// by several, or shared with a triangle whose opposite vertex lies on the same side of it. v holds
// t's vertex indices and clip-space x, y, w.
// The side test with the opposite vertex's position po already loaded.
__device__ __forceinline__ bool silhouette_side(const Tri2& v, int k, const float4& po) {
  const int i = (k + 1) % 3, j = (k + 2) % 3;
  const float A[3] = {v.x[i], v.y[i], v.w[i]}, B[3] = {v.x[j], v.y[j], v.w[j]};
  float l[3];
  for (int c = 0; c < 3; ++c) {
    const int ci = (c + 1) % 3, cj = (c + 2) % 3;
    l[c] = __fmaf_rn(A[ci], B[cj], -mul(A[cj], B[ci]));
  }
  const float s1 = side_sign(l, make_float4(v.x[k], v.y[k], 0.0f, v.w[k]));
  return mul(s1, side_sign(l, po)) > 0.0f;
}

__device__ __forceinline__ bool silhouette_of(const AaCtx& a, long long pb, const Tri2& v, int t,
                                              int k) {
  const int opp = __ldg(a.opposite + 3 * static_cast<long long>(t) + k);
  if (opp < 0) return true;
  const int i = (k + 1) % 3, j = (k + 2) % 3;
  const float A[3] = {v.x[i], v.y[i], v.w[i]}, B[3] = {v.x[j], v.y[j], v.w[j]};
  float l[3];
  for (int c = 0; c < 3; ++c) {
    const int ci = (c + 1) % 3, cj = (c + 2) % 3;
    l[c] = __fmaf_rn(A[ci], B[cj], -mul(A[cj], B[ci]));
  }
  const float s1 = side_sign(l, make_float4(v.x[k], v.y[k], 0.0f, v.w[k]));
  const float s2 = side_sign(l, __ldg(reinterpret_cast<const float4*>(a.pos) + pb * a.num_vert +
                                      checked_index(opp, a.num_vert, kSiteOpposite)));
  return mul(s1, s2) > 0.0f;
}

struct Crossing {
  bool found;
  float t;
  int edge;
};

// reference.py:675-727 for one pixel pair side: triangle t seen at src, followed towards dst.
// As in the reference, a = x - px w and c = y - py w are formed once per vertex and point and
// shared by the three edge functions and the slack (reference.py:274-278, :730-746). The terms of
// the source point are computed once (SrcTerms) and shared by the directions a pixel's triangle is
// followed in: for a horizontal step the destination's c equal the source's, for a vertical step
// its a, bit for bit, so only the other half is formed again.
struct SrcTerms {
  float as[3], cs[3], es[3];
  float sign;
  float rx[3], ry[3];
};

__device__ __forceinline__ SrcTerms src_terms(const Tri2& v, float sx, float sy) {
  SrcTerms S;
  for (int k = 0; k < 3; ++k) {
    S.as[k] = sub(v.x[k], mul(sx, v.w[k]));
    S.cs[k] = sub(v.y[k], mul(sy, v.w[k]));
  }
  for (int k = 0; k < 3; ++k) {
    const int i = (k + 1) % 3, j = (k + 2) % 3;
    S.es[k] = cross2(S.as[i], S.cs[j], S.as[j], S.cs[i]);
  }
  S.sign = add(add(S.es[0], S.es[1]), S.es[2]) < 0.0f ? -1.0f : 1.0f;
  for (int k = 0; k < 3; ++k) {
    S.rx[k] = add(fabsf(v.x[k]), fabsf(v.w[k]));
    S.ry[k] = add(fabsf(v.y[k]), fabsf(v.w[k]));
  }
  return S;
}

// Crossing of triangle t (vertices v, source terms S) towards (d, sy) when horizontal, else
// towards (sx, d), before the silhouette test: found means an edge is crossed and handled by this
// axis; the caller completes it with the silhouette test of that edge.
__device__ __forceinline__ Crossing crossing_candidate(const AaCtx& a, const Tri2& v,
                                                       const SrcTerms& S, float d, bool horizontal) {
  Crossing r = {false, 0.0f, 0};
  float ad[3], cd[3];
  for (int k = 0; k < 3; ++k) {
    ad[k] = horizontal ? sub(v.x[k], mul(d, v.w[k])) : S.as[k];
    cd[k] = horizontal ? S.cs[k] : sub(v.y[k], mul(d, v.w[k]));
  }
  float ed[3];
  for (int k = 0; k < 3; ++k) {
    const int i = (k + 1) % 3, j = (k + 2) % 3;
    ed[k] = cross2(ad[i], cd[j], ad[j], cd[i]);
  }
  bool any = false;
  float best = __int_as_float(0x7f800000);
  int edge = 0;
  for (int k = 0; k < 3; ++k) {
    const int i = (k + 1) % 3, j = (k + 2) % 3;
    const float span = sub(S.es[k], ed[k]);
    const float ai = fabsf(ad[i]), aj = fabsf(ad[j]), ci = fabsf(cd[i]), cj = fabsf(cd[j]);
    const float terms = add(add(add(mul(add(S.rx[i], ai), cj), mul(add(S.rx[j], aj), ci)),
                                mul(S.ry[j], ai)),
                            mul(S.ry[i], aj));
    const float slack = mul(terms, kEdgeTie);
    const bool crossed = (mul(ed[k], S.sign) <= slack) && (mul(span, S.sign) > mul(2.0f, slack));
    any |= crossed;
    const float tk = crossed ? dvd(S.es[k], span) : __int_as_float(0x7f800000);
    if (k == 0 || tk < best) {
      best = tk;
      edge = k;
    }
  }
  if (!any) return r;
  // Which axis handles the edge, from its two vertices alone (reference.py:749-765).
  const int i = (edge + 1) % 3, j = (edge + 2) % 3;
  const float steep = mul(mul(fabsf(cross2(v.w[j], v.y[i], v.w[i], v.y[j])),
                              static_cast<float>(a.height)),
                          kAxisTie);
  const float flat = mul(fabsf(cross2(v.x[j], v.w[i], v.x[i], v.w[j])), static_cast<float>(a.width));
  const bool along = horizontal ? (steep >= flat) : (flat > steep);
  if (!along) return r;
  r.found = true;
  r.t = best;
  r.edge = edge;
  return r;
}

__device__ __forceinline__ Crossing crossing_dir(const AaCtx& a, long long pb, int t, const Tri2& v,
                                                 const SrcTerms& S, float d, bool horizontal) {
  Crossing r = crossing_candidate(a, v, S, d, horizontal);
  if (r.found && !silhouette_of(a, pb, v, t, r.edge)) r.found = false;
  return r;
}

// v holds triangle t's clip-space x, y, w and vertex indices.
__device__ __forceinline__ Crossing crossing_of(const AaCtx& a, long long pb, int t, const Tri2& v,
                                                float sx, float sy, float dx, float dy,
                                                bool horizontal) {
  return crossing_dir(a, pb, t, v, src_terms(v, sx, sy), horizontal ? dx : dy, horizontal);
}

__device__ __forceinline__ Crossing crossing(const AaCtx& a, long long pb, int t, float sx,
                                             float sy, float dx, float dy, bool horizontal) {
  if (t < 0) return {false, 0.0f, 0};
  return crossing_of(a, pb, t, load_tri(a, pb, t), sx, sy, dx, dy, horizontal);
}

struct Pair {
  bool active, use_p;
  float t, bp, bq;
  int owner, edge;
  float sx, sy, dx, dy;  // crossing measured from (sx, sy) towards (dx, dy)
};

// Pair of pixel P = (row, col) and its right (horizontal) or lower neighbour Q in view b.
__device__ __forceinline__ Pair eval_pair(const AaCtx& a, long long b, int row, int col,
                                          bool horizontal) {
  Pair r;
  r.active = false;
  r.bp = r.bq = 0.0f;
  const long long hw = static_cast<long long>(a.height) * a.width;
  const long long p = b * hw + static_cast<long long>(row) * a.width + col;
  const long long q = p + (horizontal ? 1 : a.width);
  const int row_q = horizontal ? row : row + 1, col_q = horizontal ? col + 1 : col;
  const float4 rp = a.rast[p], rq = a.rast[q];
  const int id_p = aa_triangle(rp.w, a.num_tri), id_q = aa_triangle(rq.w, a.num_tri);
  if (id_p == id_q) return r;
  const long long pb = a.pos_batch == 1 ? 0 : b;
  const float xp = pixel_centre(col, a.width), yp = pixel_centre(row, a.height);
  const float xq = pixel_centre(col_q, a.width), yq = pixel_centre(row_q, a.height);
  const Crossing cp = crossing(a, pb, id_p, xp, yp, xq, yq, horizontal);
  const Crossing cq = crossing(a, pb, id_q, xq, yq, xp, yp, horizontal);
  r.use_p = cp.found && (!cq.found || rp.z <= rq.z);
  const bool use_q = cq.found && !r.use_p;
  r.active = r.use_p || use_q;
  if (!r.active) return r;
  r.t = r.use_p ? cp.t : sub(1.0f, cq.t);
  if (r.t < 0.5f) r.bp = sub(0.5f, r.t); else r.bq = sub(r.t, 0.5f);
  r.owner = r.use_p ? id_p : id_q;
  r.edge = r.use_p ? cp.edge : cq.edge;
  r.sx = r.use_p ? xp : xq;
  r.sy = r.use_p ? yp : yq;
  r.dx = r.use_p ? xq : xp;
  r.dy = r.use_p ? yq : yp;
  return r;
}

// The pairs of every pixel as the forward pass found them, so that the backward pass reads them
// instead of repeating the edge tests: for the right (low nibble) and lower (high nibble) pair
// of pixel p, bit 3 = active, bit 2 = the crossing was found from p's side, bits 0-1 = the edge
// of the owning triangle; t[p] holds the two crossings t (zero when inactive) and verts[p] the
// vertex indices of the two crossed edges (right pair in x, y; lower pair in z, w; written only
// for pixels with an active pair).
struct PairRecords {
  float2* t;
  uint8_t* code;
  int4* verts;
};

// Vertex (edge + k) % 3 of the pair's owning triangle: k = 1, 2 give the crossed edge's ends.
__device__ __forceinline__ int edge_vertex(const AaCtx& a, const Pair& r, int k) {
  return static_cast<int>(checked_index(
      __ldg(a.tri + 3 * static_cast<long long>(r.owner) + (r.edge + k) % 3), a.num_vert,
      kSiteVertex));
}

// Blend coefficients (bp, bq) of a recorded pair, as eval_pair forms them from t.
__device__ __forceinline__ float2 recorded_blend(unsigned code, float t) {
  if (!(code & 8u)) return make_float2(0.f, 0.f);
  return t < 0.5f ? make_float2(sub(0.5f, t), 0.f) : make_float2(0.f, sub(t, 0.5f));
}

// Pixel tiling of the backward pass that repeats the edge tests (aa_bwd_kernel): a block of
// 32 x 8 threads covers a 31 x 7 tile of output pixels plus a one-pixel halo to the left and above.
// Each thread evaluates the right pair of its pixel (unless it is in the halo row) and the lower
// pair (unless it is in the halo column) once, into shared memory; every output pixel then reads
// its four pairs from there.
constexpr int kAaThreadsX = 32, kAaThreadsY = 8;
constexpr int kAaTileX = kAaThreadsX - 1, kAaTileY = kAaThreadsY - 1;

// Forward pass. A block of 32 x 16 threads covers 30 x 14 output pixels plus a one-pixel halo all
// round. Each thread follows its own pixel's triangle, loaded once, towards each neighbour that
// shows another triangle (the source terms shared by the up to four directions) and leaves the
// crossings in shared memory; each output pixel then decides its four pairs from both sides'
// crossings, blends, writes only itself (no colour atomics, deterministic) and records its right
// and lower pairs for the backward pass.
constexpr int kFwdX = 32, kFwdY = 16;
constexpr int kFwdTileX = kFwdX - 2, kFwdTileY = kFwdY - 2;
enum AaDirection { kRight = 0, kLeft = 1, kDown = 2, kUp = 3 };

struct PairOutcome {
  bool active, use_p;
  float t, bp, bq;
  int edge;
};

// eval_pair's decision from the two sides' crossings: code bit 2 = found, bits 0-1 = edge.
__device__ __forceinline__ PairOutcome decide_pair(int id_p, int id_q, float zp, float zq,
                                                   unsigned cp, float tp, unsigned cq, float tq) {
  PairOutcome r;
  r.active = false;
  r.use_p = false;
  r.t = r.bp = r.bq = 0.0f;
  r.edge = 0;
  if (id_p == id_q) return r;
  const bool fp = (cp & 4u) != 0u, fq = (cq & 4u) != 0u;
  r.use_p = fp && (!fq || zp <= zq);
  const bool use_q = fq && !r.use_p;
  r.active = r.use_p || use_q;
  if (!r.active) return r;
  r.t = r.use_p ? tp : sub(1.0f, tq);
  if (r.t < 0.5f) r.bp = sub(0.5f, r.t); else r.bq = sub(r.t, 0.5f);
  r.edge = static_cast<int>((r.use_p ? cp : cq) & 3u);
  return r;
}

__device__ __forceinline__ int owner_vertex(const AaCtx& a, int owner, int edge, int k) {
  return static_cast<int>(checked_index(
      __ldg(a.tri + 3 * static_cast<long long>(owner) + (edge + k) % 3), a.num_vert, kSiteVertex));
}

// Squared-error loss fused into the antialias passes: the forward pass writes the residual
// out - target and adds up its squares per block into partial[block]; the backward pass takes the
// upstream gradient grad_out (when given) plus s residual, s = 2 scale dL.
struct FusedLoss {
  const float* target;
  float* residual;
  float* partial;
};

// One block per 30 x 14 output pixels of a view (a 32 x 16 thread tile with a one-pixel halo).
// NC > 0: exactly NC colour channels, known at compile time: constant address arithmetic in the
// blend loop, which stays rolled (unrolled, its loads spill under the 40-register cap).
template <bool kLoss, int NC>
__global__ void __launch_bounds__(kFwdX * kFwdY, 3) aa_fwd_kernel(const AaCtx a,
                                                                   float* __restrict__ out,
                                                                   PairRecords rec,
                                                                   FusedLoss loss) {
  __shared__ int s_id[kFwdY][kFwdX];
  __shared__ float s_z[kFwdY][kFwdX];
  __shared__ float s_t[4][kFwdY][kFwdX];
  __shared__ unsigned char s_c[4][kFwdY][kFwdX];
  __shared__ float s_cx[kFwdX], s_cy[kFwdY];
  const int tx = threadIdx.x % kFwdX, ty = threadIdx.x / kFwdX;
  const int col0 = blockIdx.x * kFwdTileX - 1, row0 = blockIdx.y * kFwdTileY - 1;
  const int col = col0 + tx, row = row0 + ty;
  const long long b = blockIdx.z;
  const long long pb = a.pos_batch == 1 ? 0 : b;
  const bool in_image = col >= 0 && col < a.width && row >= 0 && row < a.height;
  const long long p = (b * a.height + row) * a.width + col;
  int id = -3;
  float z = 0.0f;
  if (in_image) {
    const float4 r = a.rast[p];
    id = aa_triangle(r.w, a.num_tri);
    z = r.z;
  }
  s_id[ty][tx] = id;
  s_z[ty][tx] = z;
  if (threadIdx.x < kFwdX) s_cx[threadIdx.x] = pixel_centre(col0 + threadIdx.x, a.width);
  else if (threadIdx.x < kFwdX + kFwdY)
    s_cy[threadIdx.x - kFwdX] = pixel_centre(row0 + threadIdx.x - kFwdX, a.height);
  __syncthreads();
  // Directions needed by the output pixels' pairs, towards a neighbour showing another triangle.
  const bool out_row = ty >= 1 && ty <= kFwdY - 2, out_col = tx >= 1 && tx <= kFwdX - 2;
  bool need[4];
  need[kRight] = out_row && tx <= kFwdX - 2 && col + 1 < a.width && s_id[ty][tx + 1] != id;
  need[kLeft] = out_row && tx >= 1 && col >= 1 && s_id[ty][tx - 1] != id;
  need[kDown] = out_col && ty <= kFwdY - 2 && row + 1 < a.height && s_id[ty + 1][tx] != id;
  need[kUp] = out_col && ty >= 1 && row >= 1 && s_id[ty - 1][tx] != id;
  unsigned code[4] = {0u, 0u, 0u, 0u};
  float tc[4] = {0.f, 0.f, 0.f, 0.f};
  if (in_image && id >= 0 && (need[0] || need[1] || need[2] || need[3])) {
    const Tri2 v = load_tri(a, pb, id);
    const SrcTerms S = src_terms(v, s_cx[tx], s_cy[ty]);
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      if (!need[d]) continue;
      const float dst = d == kRight ? s_cx[tx + 1]
                        : d == kLeft ? s_cx[tx - 1]
                        : d == kDown ? s_cy[ty + 1]
                                     : s_cy[ty - 1];
      const Crossing c = crossing_candidate(a, v, S, dst, d < 2);
      if (c.found) {
        code[d] = 4u | static_cast<unsigned>(c.edge);
        tc[d] = c.t;
      }
    }
    // Silhouette tests of the candidate edges, their loads issued together.
    int opp[4];
#pragma unroll
    for (int d = 0; d < 4; ++d)
      opp[d] = code[d] ? __ldg(a.opposite + 3 * static_cast<long long>(id) + (code[d] & 3u)) : -1;
    float4 po[4];
#pragma unroll
    for (int d = 0; d < 4; ++d)
      po[d] = opp[d] >= 0 ? __ldg(reinterpret_cast<const float4*>(a.pos) + pb * a.num_vert +
                                  checked_index(opp[d], a.num_vert, kSiteOpposite))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int d = 0; d < 4; ++d)
      if (code[d] && opp[d] >= 0 && !silhouette_side(v, static_cast<int>(code[d] & 3u), po[d]))
        code[d] = 0u;
  }
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    s_c[d][ty][tx] = static_cast<unsigned char>(code[d]);
    s_t[d][ty][tx] = tc[d];
  }
  __syncthreads();
  const bool emit = in_image && out_row && out_col;
  if (!kLoss && !emit) return;
  float sq = 0.0f;
  if (emit) {
    const PairOutcome right =
        col + 1 < a.width
            ? decide_pair(id, s_id[ty][tx + 1], z, s_z[ty][tx + 1], code[kRight], tc[kRight],
                          s_c[kLeft][ty][tx + 1], s_t[kLeft][ty][tx + 1])
            : decide_pair(0, 0, 0.f, 0.f, 0u, 0.f, 0u, 0.f);
    const PairOutcome left =
        col >= 1 ? decide_pair(s_id[ty][tx - 1], id, s_z[ty][tx - 1], z, s_c[kRight][ty][tx - 1],
                               s_t[kRight][ty][tx - 1], code[kLeft], tc[kLeft])
                 : decide_pair(0, 0, 0.f, 0.f, 0u, 0.f, 0u, 0.f);
    const PairOutcome down =
        row + 1 < a.height
            ? decide_pair(id, s_id[ty + 1][tx], z, s_z[ty + 1][tx], code[kDown], tc[kDown],
                          s_c[kUp][ty + 1][tx], s_t[kUp][ty + 1][tx])
            : decide_pair(0, 0, 0.f, 0.f, 0u, 0.f, 0u, 0.f);
    const PairOutcome up =
        row >= 1 ? decide_pair(s_id[ty - 1][tx], id, s_z[ty - 1][tx], z, s_c[kDown][ty - 1][tx],
                               s_t[kDown][ty - 1][tx], code[kUp], tc[kUp])
                 : decide_pair(0, 0, 0.f, 0.f, 0u, 0.f, 0u, 0.f);
    if (rec.code != nullptr) {
      unsigned codes = 0u;
      int4 verts = make_int4(0, 0, 0, 0);
      if (right.active) {
        codes = 8u | (right.use_p ? 4u : 0u) | static_cast<unsigned>(right.edge);
        const int owner = right.use_p ? id : s_id[ty][tx + 1];
        verts.x = owner_vertex(a, owner, right.edge, 1);
        verts.y = owner_vertex(a, owner, right.edge, 2);
      }
      if (down.active) {
        codes |= (8u | (down.use_p ? 4u : 0u) | static_cast<unsigned>(down.edge)) << 4;
        const int owner = down.use_p ? id : s_id[ty + 1][tx];
        verts.z = owner_vertex(a, owner, down.edge, 1);
        verts.w = owner_vertex(a, owner, down.edge, 2);
      }
      rec.t[p] = make_float2(right.t, down.t);
      rec.code[p] = static_cast<uint8_t>(codes);
      // Edge vertices are read only for active pairs.
      if (codes & 0x88u) rec.verts[p] = verts;
    }
    // Blend in the reference's accumulation order: right pair (this pixel first), left pair
    // (second), lower pair (first), upper pair (second).
    const float k[4] = {right.bp, left.bq, down.bp, up.bq};
    const long long other[4] = {p + 1, p - 1, p + a.width, p - a.width};
    const int C = NC > 0 ? NC : a.channels;
    auto blend = [&](int c) {
      const float self = __ldg(a.color + p * C + c);
      float value = self;
      for (int i = 0; i < 4; ++i) {
        if (k[i] != 0.0f) value = add(value, mul(k[i], sub(__ldg(a.color + other[i] * C + c), self)));
      }
      out[p * C + c] = value;
      if (kLoss) {
        const float d = value - __ldg(loss.target + p * C + c);
        loss.residual[p * C + c] = d;
        sq = fmaf(d, d, sq);
      }
    };
    if constexpr (NC > 0) {
#pragma unroll 1
      for (int c = 0; c < NC; ++c) blend(c);
    } else {
      for (int c = 0; c < C; ++c) blend(c);
    }
  }
  if (kLoss) {
    __shared__ float warp_sq[kFwdX * kFwdY / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 31u) == 0u) warp_sq[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      float total = 0.0f;
      for (int i = 0; i < kFwdX * kFwdY / 32; ++i) total += warp_sq[i];
      loss.partial[(static_cast<long long>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x +
                   blockIdx.x] = total;
    }
  }
}

// Position gradient of the crossing t of a pair, chained into the two vertices of its edge:
// t = e_s / (e_s - e_d), e = a_i c_j - a_j c_i with a = x - px w, c = y - py w.
__device__ __forceinline__ void edge_gradient(const AaCtx& a, float* grad_pos, long long pb, int vi,
                                              int vj, const Pair& r, float grad_t) {
  const long long base = pb * a.num_vert;
  vi = static_cast<int>(checked_index(vi, a.num_vert, kSiteVertex));
  vj = static_cast<int>(checked_index(vj, a.num_vert, kSiteVertex));
  const float4 pi = __ldg(reinterpret_cast<const float4*>(a.pos) + base + vi);
  const float4 pj = __ldg(reinterpret_cast<const float4*>(a.pos) + base + vj);
  const float ai_s = pi.x - r.sx * pi.w, aj_s = pj.x - r.sx * pj.w;
  const float ci_s = pi.y - r.sy * pi.w, cj_s = pj.y - r.sy * pj.w;
  const float ai_d = pi.x - r.dx * pi.w, aj_d = pj.x - r.dx * pj.w;
  const float ci_d = pi.y - r.dy * pi.w, cj_d = pj.y - r.dy * pj.w;
  const float e_s = ai_s * cj_s - aj_s * ci_s;
  const float e_d = ai_d * cj_d - aj_d * ci_d;
  float denom = e_s - e_d;
  if (denom == 0.0f) denom = 1.0f;
  const float g_s = grad_t * -e_d / (denom * denom);
  const float g_d = grad_t * e_s / (denom * denom);
  const float gx_i = g_s * cj_s + g_d * cj_d;
  const float gx_j = -(g_s * ci_s + g_d * ci_d);
  const float gy_i = -(g_s * aj_s + g_d * aj_d);
  const float gy_j = g_s * ai_s + g_d * ai_d;
  const float gw_i = g_s * (r.sy * aj_s - r.sx * cj_s) + g_d * (r.dy * aj_d - r.dx * cj_d);
  const float gw_j = g_s * (r.sx * ci_s - r.sy * ai_s) + g_d * (r.dx * ci_d - r.dy * ai_d);
  red_add_v4(grad_pos + (base + vi) * 4, gx_i, gy_i, 0.0f, gw_i);
  red_add_v4(grad_pos + (base + vj) * 4, gx_j, gy_j, 0.0f, gw_j);
}

__device__ __forceinline__ void add_edge_gradient(const AaCtx& a, float* grad_pos, long long pb,
                                                  const Pair& r, float grad_t) {
  edge_gradient(a, grad_pos, pb, edge_vertex(a, r, 1), edge_vertex(a, r, 2), r, grad_t);
}

__global__ void __launch_bounds__(256, 5) aa_bwd_kernel(const AaCtx a,
                                                     const float* __restrict__ grad_out,
                                                     float boost, float* __restrict__ grad_color,
                                                     float* __restrict__ grad_pos) {
  __shared__ float2 hk[kAaThreadsY][kAaThreadsX], vk[kAaThreadsY][kAaThreadsX];
  const int tx = threadIdx.x % kAaThreadsX, ty = threadIdx.x / kAaThreadsX;
  const int col = blockIdx.x * kAaTileX + tx - 1, row = blockIdx.y * kAaTileY + ty - 1;
  const long long b = blockIdx.z;
  const bool in_image = col >= 0 && col < a.width && row >= 0 && row < a.height;
  const bool interior = in_image && tx >= 1 && ty >= 1;
  const long long pb = a.pos_batch == 1 ? 0 : b;
  const long long p = (b * a.height + row) * a.width + col;
  const int C = a.channels;
  Pair own[2];
  own[0].active = own[1].active = false;
  own[0].bp = own[0].bq = own[1].bp = own[1].bq = 0.0f;
  if (in_image && ty >= 1 && col + 1 < a.width) own[0] = eval_pair(a, b, row, col, true);
  if (in_image && tx >= 1 && row + 1 < a.height) own[1] = eval_pair(a, b, row, col, false);
  hk[ty][tx] = make_float2(own[0].bp, own[0].bq);
  vk[ty][tx] = make_float2(own[1].bp, own[1].bq);
  __syncthreads();
  if (!interior) return;
  // As the first pixel of a pair (P = p, Q): grad_color[p] += -bp g[p] + bq g[Q]; as the second
  // pixel of a pair (P, Q = p): grad_color[p] += bp g[P] - bq g[p].
  const float2 right = hk[ty][tx], left = hk[ty][tx - 1], down = vk[ty][tx], up = vk[ty - 1][tx];
  const float kp[4] = {-right.x, -left.y, -down.x, -up.y};
  const float kq[4] = {right.y, left.x, down.y, up.x};
  const long long other[4] = {p + 1, p - 1, p + a.width, p - a.width};
  float grad_t[2] = {0.f, 0.f};
  for (int c = 0; c < C; ++c) {
    const float g_self = grad_out[p * C + c];
    float value = g_self;
    for (int i = 0; i < 4; ++i) {
      if (kp[i] != 0.0f || kq[i] != 0.0f) value += kp[i] * g_self + kq[i] * grad_out[other[i] * C + c];
    }
    grad_color[p * C + c] = value;
    for (int d = 0; d < 2; ++d) {
      if (!own[d].active) continue;
      const long long q = other[d == 0 ? 0 : 2];
      const float c_p = __ldg(a.color + p * C + c), c_q = __ldg(a.color + q * C + c);
      // d/dt of (1/2 - t)(c_q - c_p) below the midpoint and (t - 1/2)(c_p - c_q) above it.
      grad_t[d] += own[d].t < 0.5f ? -g_self * (c_q - c_p) : grad_out[q * C + c] * (c_p - c_q);
    }
  }
  // The pairs whose first pixel is interior here are owned by this block: scatter their
  // position gradients once.
  for (int d = 0; d < 2; ++d) {
    if (!own[d].active) continue;
    const float g = grad_t[d] * boost;
    if (g == 0.0f) continue;
    // When the edge belongs to Q's triangle, t = 1 - t_q.
    add_edge_gradient(a, grad_pos, pb, own[d], own[d].use_p ? g : -g);
  }
}

// Position gradient of pixel (row, col)'s own right (horizontal) or lower pair, recorded with
// code c4 and crossing gradient g.
__device__ __forceinline__ void recorded_edge_gradient(const AaCtx& a, float* grad_pos,
                                                       long long pb, int row, int col, unsigned c4,
                                                       int vi, int vj, bool horizontal, float g) {
  const int row_q = horizontal ? row : row + 1, col_q = horizontal ? col + 1 : col;
  Pair r;
  r.use_p = (c4 & 4u) != 0u;
  const float xp = pixel_centre(col, a.width), yp = pixel_centre(row, a.height);
  const float xq = horizontal ? pixel_centre(col_q, a.width) : xp;
  const float yq = horizontal ? yp : pixel_centre(row_q, a.height);
  r.sx = r.use_p ? xp : xq;
  r.sy = r.use_p ? yp : yq;
  r.dx = r.use_p ? xq : xp;
  r.dy = r.use_p ? yq : yp;
  // When the edge belongs to Q's triangle, t = 1 - t_q.
  edge_gradient(a, grad_pos, pb, vi, vj, r, r.use_p ? g : -g);
}

// The upstream gradient of output element i: grad (when given) plus, with a fused squared-error
// loss, s residual[i] with s = 2 scale dL.
struct Upstream {
  const float* grad;
  const float* residual;
  const float* loss_grad;  // device scalar dL
  float scale2;
};

// Upstream modes of the recorded backward pass: the output's gradient only, the fused loss only
// (the pass is linear in the upstream gradient, so it runs on the residual and scales its results
// by s once), or both.
enum UpstreamMode { kGradOnly = 0, kLossOnly = 1, kGradAndLoss = 2 };

template <int kMode>
__device__ __forceinline__ float upstream(const Upstream& u, float s, long long i) {
  if (kMode == kGradOnly) return u.grad[i];
  if (kMode == kLossOnly) return __ldg(u.residual + i);
  return fmaf(s, __ldg(u.residual + i), u.grad[i]);
}

// Backward pass from the pairs recorded by the forward pass: one thread per pixel (grid: columns
// in x, rows in y, views in z), no edge tests. Same arithmetic as aa_bwd_kernel for the colour
// gradient and for the crossings of the pixel's own (right and lower) pairs, whose position
// gradients it scatters. With K > 0 channels known at compile time, every input the pixel can
// need is loaded up front, unconditionally, so that the loads overlap instead of each waiting for
// the record that decides it; K = 0 handles any channel count. kMode (UpstreamMode) says where the
// upstream gradient comes from.
template <int K, int kMode>
__global__ void __launch_bounds__(256, 5) aa_bwd_recorded_kernel(const AaCtx a,
                                                              const float2* __restrict__ rec_t,
                                                              const uint8_t* __restrict__ rec_code,
                                                              const int4* __restrict__ rec_verts,
                                                              const Upstream u, float boost,
                                                              float* __restrict__ grad_color,
                                                              float* __restrict__ grad_pos,
                                                              int row0) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= a.width) return;
  const int row = row0 + static_cast<int>(blockIdx.y);
  const long long b = blockIdx.z;
  const long long p = (b * a.height + row) * a.width + col;
  const long long w = a.width;
  const bool has_l = col > 0, has_r = col + 1 < a.width, has_u = row > 0, has_d = row + 1 < a.height;
  const unsigned code = __ldg(rec_code + p);
  const unsigned code_l = has_l ? __ldg(rec_code + p - 1) & 15u : 0u;
  const unsigned code_u = has_u ? __ldg(rec_code + p - w) >> 4 : 0u;
  const float2 t = __ldg(rec_t + p);
  const float t_l = has_l ? __ldg(rec_t + p - 1).x : 0.f;
  const float t_u = has_u ? __ldg(rec_t + p - w).y : 0.f;
  const int4 verts = __ldg(rec_verts + p);
  const float s = kMode == kGradAndLoss ? u.scale2 * __ldg(u.loss_grad) : 0.0f;
  const int C = K > 0 ? K : a.channels;
  constexpr int R = K > 0 ? K : 1;
  float gs[R], gl[R], gr[R], gu[R], gd[R], cs[R], cr[R], cd[R];
  if (K > 0) {
#pragma unroll
    for (int c = 0; c < R; ++c) {
      gs[c] = upstream<kMode>(u, s, p * C + c);
      gl[c] = has_l ? upstream<kMode>(u, s, (p - 1) * C + c) : 0.f;
      gr[c] = has_r ? upstream<kMode>(u, s, (p + 1) * C + c) : 0.f;
      gu[c] = has_u ? upstream<kMode>(u, s, (p - w) * C + c) : 0.f;
      gd[c] = has_d ? upstream<kMode>(u, s, (p + w) * C + c) : 0.f;
      cs[c] = __ldg(a.color + p * C + c);
      cr[c] = has_r ? __ldg(a.color + (p + 1) * C + c) : 0.f;
      cd[c] = has_d ? __ldg(a.color + (p + w) * C + c) : 0.f;
    }
  }
  const float2 right = recorded_blend(code & 15u, t.x), down = recorded_blend(code >> 4, t.y);
  const float2 left = recorded_blend(code_l, t_l), up = recorded_blend(code_u, t_u);
  const bool own_r = (code & 8u) != 0u, own_d = (code & 0x80u) != 0u;
  const float s_end = kMode == kLossOnly ? u.scale2 * __ldg(u.loss_grad) : 1.0f;
  float grad_tr = 0.f, grad_td = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int i = K > 0 ? c : 0;
    if (K == 0) {
      gs[0] = upstream<kMode>(u, s, p * C + c);
      gl[0] = has_l ? upstream<kMode>(u, s, (p - 1) * C + c) : 0.f;
      gr[0] = has_r ? upstream<kMode>(u, s, (p + 1) * C + c) : 0.f;
      gu[0] = has_u ? upstream<kMode>(u, s, (p - w) * C + c) : 0.f;
      gd[0] = has_d ? upstream<kMode>(u, s, (p + w) * C + c) : 0.f;
      cs[0] = __ldg(a.color + p * C + c);
      cr[0] = has_r ? __ldg(a.color + (p + 1) * C + c) : 0.f;
      cd[0] = has_d ? __ldg(a.color + (p + w) * C + c) : 0.f;
    }
    const float g_self = gs[i];
    float value = g_self;
    // Right pair (first pixel), left (second), lower (first), upper (second), as aa_bwd_kernel.
    if (right.x != 0.0f || right.y != 0.0f) value += -right.x * g_self + right.y * gr[i];
    if (left.x != 0.0f || left.y != 0.0f) value += -left.y * g_self + left.x * gl[i];
    if (down.x != 0.0f || down.y != 0.0f) value += -down.x * g_self + down.y * gd[i];
    if (up.x != 0.0f || up.y != 0.0f) value += -up.y * g_self + up.x * gu[i];
    grad_color[p * C + c] = kMode == kLossOnly ? value * s_end : value;
    // d/dt of (1/2 - t)(c_q - c_p) below the midpoint and (t - 1/2)(c_p - c_q) above it.
    if (own_r) grad_tr += t.x < 0.5f ? -g_self * (cr[i] - cs[i]) : gr[i] * (cs[i] - cr[i]);
    if (own_d) grad_td += t.y < 0.5f ? -g_self * (cd[i] - cs[i]) : gd[i] * (cs[i] - cd[i]);
  }
  const long long pb = a.pos_batch == 1 ? 0 : b;
  if (kMode == kLossOnly) {
    grad_tr *= s_end;
    grad_td *= s_end;
  }
  if (own_r && grad_tr * boost != 0.0f)
    recorded_edge_gradient(a, grad_pos, pb, row, col, code & 15u, verts.x, verts.y, true,
                           grad_tr * boost);
  if (own_d && grad_td * boost != 0.0f)
    recorded_edge_gradient(a, grad_pos, pb, row, col, code >> 4, verts.z, verts.w, false,
                           grad_td * boost);
}

__global__ void __launch_bounds__(256) silhouette_kernel(const AaCtx a, long long total,
                                                         uint8_t* __restrict__ out) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= total) return;
  const long long per_view = 3LL * a.num_tri;
  const long long pb = i / per_view;
  const long long e = i - pb * per_view;
  const int t = static_cast<int>(e / 3);
  out[i] = silhouette_of(a, pb, load_tri(a, pb, t), t, static_cast<int>(e % 3)) ? 1 : 0;
}


// Vertex opposite each edge in the triangle across it: tri[neighbours[e]], or -1 without a single
// adjacent triangle (and for an index outside the edge range, which dr_edge_neighbours never gives).
__global__ void __launch_bounds__(256) opposite_kernel(const int* __restrict__ tri,
                                                       const long long* __restrict__ neighbours,
                                                       long long edges, int* __restrict__ opposite) {
  const long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (e >= edges) return;
  const long long n = neighbours[e];
  opposite[e] = (n >= 0 && n < edges) ? tri[n] : -1;
}

bool bad_aa_args(const float* color, const float* rast, const float* pos, int64_t pos_batch,
                 int64_t num_vert, const int32_t* tri, int64_t num_tri, const int32_t* opposite,
                 int64_t batch, int32_t height, int32_t width, int32_t channels) {
  if (pos_batch < 1 || (pos_batch != 1 && pos_batch != batch)) return true;
  if (num_vert < 0 || num_tri < 0 || num_tri >= (1LL << 29) || batch < 0 || height < 0 ||
      width < 0 || channels < 0)
    return true;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total > 0 && (color == nullptr || rast == nullptr)) return true;
  if ((reinterpret_cast<uintptr_t>(rast) & 15u) != 0 || (reinterpret_cast<uintptr_t>(pos) & 15u) != 0)
    return true;
  if (num_tri > 0 && (tri == nullptr || opposite == nullptr || pos == nullptr)) return true;
  return false;
}

AaCtx make_ctx(const float* color, const float* rast, const float* pos, int64_t pos_batch,
               int64_t num_vert, const int32_t* tri, int64_t num_tri, const int32_t* opposite,
               int32_t height, int32_t width, int32_t channels) {
  AaCtx a;
  a.color = color;
  a.rast = reinterpret_cast<const float4*>(rast);
  a.pos = pos;
  a.tri = tri;
  a.opposite = opposite;
  a.pos_batch = pos_batch;
  a.num_vert = num_vert;
  a.num_tri = static_cast<int>(num_tri);
  a.height = height;
  a.width = width;
  a.channels = channels;
  return a;
}

size_t pair_record_bytes(long long pixels) {
  const size_t n = static_cast<size_t>(pixels);
  return align256(sizeof(float2) * n) + align256(n) + align256(sizeof(int4) * n);
}

PairRecords pair_records(void* pairs, long long pixels) {
  if (pairs == nullptr) return {nullptr, nullptr, nullptr};
  const size_t n = static_cast<size_t>(pixels);
  char* p = static_cast<char*>(pairs);
  return {reinterpret_cast<float2*>(p), reinterpret_cast<uint8_t*>(p + align256(sizeof(float2) * n)),
          reinterpret_cast<int4*>(p + align256(sizeof(float2) * n) + align256(n))};
}

template <int kMode>
void launch_recorded(const AaCtx& a, const PairRecords& rec, const Upstream& u, float boost,
                     float* grad_color, float* grad_pos, long long batch, cudaStream_t s) {
  // Rows in y, launched 65535 at a time for taller images.
  for (int r0 = 0; r0 < a.height; r0 += 65535) {
    const dim3 grid((a.width + 255) / 256, static_cast<unsigned>(min(a.height - r0, 65535)),
                    static_cast<unsigned>(batch));
    switch (a.channels) {
      case 1:
        aa_bwd_recorded_kernel<1, kMode><<<grid, 256, 0, s>>>(a, rec.t, rec.code, rec.verts, u,
                                                              boost, grad_color, grad_pos, r0);
        break;
      case 3:
        aa_bwd_recorded_kernel<3, kMode><<<grid, 256, 0, s>>>(a, rec.t, rec.code, rec.verts, u,
                                                              boost, grad_color, grad_pos, r0);
        break;
      case 4:
        aa_bwd_recorded_kernel<4, kMode><<<grid, 256, 0, s>>>(a, rec.t, rec.code, rec.verts, u,
                                                              boost, grad_color, grad_pos, r0);
        break;
      default:
        aa_bwd_recorded_kernel<0, kMode><<<grid, 256, 0, s>>>(a, rec.t, rec.code, rec.verts, u,
                                                              boost, grad_color, grad_pos, r0);
    }
  }
}

dim3 fwd_grid(int64_t batch, int32_t height, int32_t width) {
  return dim3((width + kFwdTileX - 1) / kFwdTileX, (height + kFwdTileY - 1) / kFwdTileY,
              static_cast<unsigned>(batch));
}

}  // namespace
}  // namespace dr

using namespace dr;

extern "C" size_t dr_antialias_loss_partials(int64_t batch, int32_t height, int32_t width) {
  if (batch <= 0 || height <= 0 || width <= 0) return 0;
  const dim3 g = fwd_grid(batch, height, width);
  return static_cast<size_t>(g.x) * g.y * g.z;
}

extern "C" size_t dr_antialias_pair_bytes(int64_t batch, int32_t height, int32_t width) {
  if (batch < 0 || height < 0 || width < 0) return 0;
  return pair_record_bytes(batch * static_cast<long long>(height) * width);
}

extern "C" size_t dr_edge_neighbours_workspace_bytes(int64_t num_tri) {
  const unsigned long long slots = table_slots(num_tri < 0 ? 0 : num_tri);
  return align256(8 * slots) + 3 * align256(4 * slots);
}

extern "C" int dr_edge_neighbours(const int32_t* tri, int64_t num_tri, int64_t* neighbours,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (num_tri < 0 || num_tri >= (1LL << 29)) return DR_ERR_INVALID_ARGUMENT;
  if (num_tri == 0) return DR_OK;
  if (tri == nullptr || neighbours == nullptr || workspace == nullptr) return DR_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < dr_edge_neighbours_workspace_bytes(num_tri)) return DR_ERR_WORKSPACE_TOO_SMALL;
  const unsigned long long slots = table_slots(num_tri);
  char* p = static_cast<char*>(workspace);
  auto* keys = reinterpret_cast<unsigned long long*>(p);
  p += align256(8 * slots);
  int* count = reinterpret_cast<int*>(p);
  p += align256(4 * slots);
  int* first = reinterpret_cast<int*>(p);
  p += align256(4 * slots);
  int* second = reinterpret_cast<int*>(p);
  cudaStream_t s = as_stream(stream);
  cudaError_t err = cudaMemsetAsync(keys, 0xFF, 8 * slots, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(count, 0, 4 * slots, s);
  if (err != cudaSuccess) return static_cast<int>(err);
  const long long edges = 3 * num_tri;
  edge_insert_kernel<<<blocks_for(edges, 256), 256, 0, s>>>(tri, edges, keys, count, first, second,
                                                            slots - 1);
  edge_lookup_kernel<<<blocks_for(edges, 256), 256, 0, s>>>(
      tri, edges, keys, count, first, second, slots - 1, reinterpret_cast<long long*>(neighbours));
  return launch_status();
}

extern "C" int dr_edge_opposite_vertices(const int32_t* tri, const int64_t* neighbours,
                                         int64_t num_tri, int32_t* opposite, void* stream) {
  if (num_tri < 0 || num_tri >= (1LL << 29)) return DR_ERR_INVALID_ARGUMENT;
  if (num_tri == 0) return DR_OK;
  if (tri == nullptr || neighbours == nullptr || opposite == nullptr) return DR_ERR_INVALID_ARGUMENT;
  const long long edges = 3 * num_tri;
  opposite_kernel<<<blocks_for(edges, 256), 256, 0, as_stream(stream)>>>(
      tri, reinterpret_cast<const long long*>(neighbours), edges, opposite);
  return launch_status();
}

extern "C" int dr_silhouette_edges(const float* pos, int64_t pos_batch, int64_t num_vert,
                                   const int32_t* tri, int64_t num_tri, const int32_t* opposite,
                                   uint8_t* silhouette, void* stream) {
  if (pos_batch < 1 || num_tri < 0 || num_tri >= (1LL << 29) || num_vert < 0)
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = pos_batch * 3 * num_tri;
  if (total == 0) return DR_OK;
  if (pos == nullptr || tri == nullptr || opposite == nullptr || silhouette == nullptr ||
      (reinterpret_cast<uintptr_t>(pos) & 15u) != 0)
    return DR_ERR_INVALID_ARGUMENT;
  const AaCtx a = make_ctx(nullptr, nullptr, pos, pos_batch, num_vert, tri, num_tri, opposite, 1, 1, 0);
  silhouette_kernel<<<blocks_for(total, 256), 256, 0, as_stream(stream)>>>(a, total, silhouette);
  return launch_status();
}

extern "C" int dr_antialias_fwd(const float* color, const float* rast, const float* pos,
                                int64_t pos_batch, int64_t num_vert, const int32_t* tri,
                                int64_t num_tri, const int32_t* opposite, int64_t batch,
                                int32_t height, int32_t width, int32_t channels, float* out,
                                void* pairs, size_t pair_bytes, void* stream) {
  if (bad_aa_args(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, batch, height,
                  width, channels) ||
      out == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (pairs != nullptr && pair_bytes < pair_record_bytes(total)) return DR_ERR_WORKSPACE_TOO_SMALL;
  if (total == 0 || channels == 0) return DR_OK;
  if (num_tri == 0) {
    cudaError_t err = cudaMemcpyAsync(out, color, sizeof(float) * total * channels,
                                      cudaMemcpyDeviceToDevice, as_stream(stream));
    return static_cast<int>(err);
  }
  const AaCtx a = make_ctx(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, height,
                           width, channels);
  if (batch > 65535) return DR_ERR_TOO_LARGE;
  if (channels == 3)
    aa_fwd_kernel<false, 3><<<fwd_grid(batch, height, width), kFwdX * kFwdY, 0, as_stream(stream)>>>(
        a, out, pair_records(pairs, total), FusedLoss{nullptr, nullptr, nullptr});
  else
    aa_fwd_kernel<false, 0><<<fwd_grid(batch, height, width), kFwdX * kFwdY, 0, as_stream(stream)>>>(
        a, out, pair_records(pairs, total), FusedLoss{nullptr, nullptr, nullptr});
  return launch_status();
}

extern "C" int dr_antialias_mse_fwd(const float* color, const float* rast, const float* pos,
                                    int64_t pos_batch, int64_t num_vert, const int32_t* tri,
                                    int64_t num_tri, const int32_t* opposite, int64_t batch,
                                    int32_t height, int32_t width, int32_t channels,
                                    const float* target, float* out, float* residual,
                                    void* pairs, size_t pair_bytes, float* partial_sums,
                                    size_t partial_count, void* stream) {
  if (bad_aa_args(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, batch, height,
                  width, channels))
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0 || channels == 0) return DR_OK;
  if (out == nullptr || target == nullptr || residual == nullptr || pairs == nullptr ||
      partial_sums == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  if (pair_bytes < pair_record_bytes(total) ||
      partial_count < dr_antialias_loss_partials(batch, height, width))
    return DR_ERR_WORKSPACE_TOO_SMALL;
  if (batch > 65535) return DR_ERR_TOO_LARGE;
  const AaCtx a = make_ctx(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, height,
                           width, channels);
  if (channels == 3)
    aa_fwd_kernel<true, 3><<<fwd_grid(batch, height, width), kFwdX * kFwdY, 0, as_stream(stream)>>>(
        a, out, pair_records(pairs, total), FusedLoss{target, residual, partial_sums});
  else
    aa_fwd_kernel<true, 0><<<fwd_grid(batch, height, width), kFwdX * kFwdY, 0, as_stream(stream)>>>(
        a, out, pair_records(pairs, total), FusedLoss{target, residual, partial_sums});
  return launch_status();
}

extern "C" int dr_antialias_mse_bwd(const float* color, const float* rast, const float* pos,
                                    int64_t pos_batch, int64_t num_vert, const int32_t* tri,
                                    int64_t num_tri, const int32_t* opposite, int64_t batch,
                                    int32_t height, int32_t width, int32_t channels,
                                    const float* residual, const float* loss_grad, float scale,
                                    const float* grad_out, float pos_gradient_boost,
                                    const void* pairs, size_t pair_bytes, float* grad_color,
                                    float* grad_pos, void* stream) {
  if (bad_aa_args(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, batch, height,
                  width, channels))
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0 || channels == 0) return DR_OK;
  if (residual == nullptr || loss_grad == nullptr || pairs == nullptr || grad_color == nullptr ||
      (num_tri > 0 && grad_pos == nullptr))
    return DR_ERR_INVALID_ARGUMENT;
  if (pair_bytes < pair_record_bytes(total)) return DR_ERR_WORKSPACE_TOO_SMALL;
  if (batch > 65535) return DR_ERR_TOO_LARGE;
  const AaCtx a = make_ctx(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, height,
                           width, channels);
  const PairRecords rec = pair_records(const_cast<void*>(pairs), total);
  const Upstream u{grad_out, residual, loss_grad, 2.0f * scale};
  if (grad_out == nullptr)
    launch_recorded<kLossOnly>(a, rec, u, pos_gradient_boost, grad_color, grad_pos, batch,
                               as_stream(stream));
  else
    launch_recorded<kGradAndLoss>(a, rec, u, pos_gradient_boost, grad_color, grad_pos, batch,
                                  as_stream(stream));
  return launch_status();
}

extern "C" int dr_antialias_bwd(const float* color, const float* rast, const float* pos,
                                int64_t pos_batch, int64_t num_vert, const int32_t* tri,
                                int64_t num_tri, const int32_t* opposite, int64_t batch,
                                int32_t height, int32_t width, int32_t channels,
                                const float* grad_out, float pos_gradient_boost,
                                const void* pairs, size_t pair_bytes, float* grad_color,
                                float* grad_pos, void* stream) {
  if (bad_aa_args(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, batch, height,
                  width, channels) ||
      grad_out == nullptr || grad_color == nullptr || (num_tri > 0 && grad_pos == nullptr))
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (pairs != nullptr && pair_bytes < pair_record_bytes(total)) return DR_ERR_WORKSPACE_TOO_SMALL;
  if (total == 0 || channels == 0) return DR_OK;
  if (num_tri == 0) {
    cudaError_t err = cudaMemcpyAsync(grad_color, grad_out, sizeof(float) * total * channels,
                                      cudaMemcpyDeviceToDevice, as_stream(stream));
    return static_cast<int>(err);
  }
  const AaCtx a = make_ctx(color, rast, pos, pos_batch, num_vert, tri, num_tri, opposite, height,
                           width, channels);
  if (batch > 65535) return DR_ERR_TOO_LARGE;
  if (pairs != nullptr) {
    launch_recorded<kGradOnly>(a, pair_records(const_cast<void*>(pairs), total),
                           Upstream{grad_out, nullptr, nullptr, 0.0f}, pos_gradient_boost,
                           grad_color, grad_pos, batch, as_stream(stream));
    return launch_status();
  }
  const dim3 grid((width + kAaTileX - 1) / kAaTileX, (height + kAaTileY - 1) / kAaTileY, batch);
  aa_bwd_kernel<<<grid, 256, 0, as_stream(stream)>>>(a, grad_out,
                                                                        pos_gradient_boost,
                                                                        grad_color, grad_pos);
  return launch_status();
}
DR_DEFINE_FAULT_QUERY(antialias)
