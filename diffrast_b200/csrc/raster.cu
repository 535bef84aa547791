// Rasterization on B200: visibility as packed 64-bit depth|triangle keys, then resolve.
//
// Visibility (result identical to diffrast's reference, backends/reference.py:368-397):
//   1. setup_kernel, one thread per (view, triangle): culls and bounds the triangle in pixels.
//      Triangles whose box holds at most kWarpPixels pixels are rasterized by the warp directly:
//      the triangles are staged in shared memory, their rows are handed out to the lanes 32 at a
//      time (warp prefix sums), each lane bounds its row by the projected triangle's half-planes
//      widened by a safety margin, and the pixels inside those spans are handed out to the lanes
//      again, one exact test each. Thin diagonal triangles thus do not pay for their bounding box
//      and lanes stay busy. Keys are merged with 64-bit atomicMin. Larger triangles are appended
//      (warp-aggregated) to a list.
//   2. Device-side binning without host round trips beyond one counter read: per-tile counts,
//      one exclusive scan (pair offsets and 256-triangle work items), and a scatter into per-tile
//      triangle lists.
//   3. tile_kernel, persistent (a few blocks per SM pull work items from an atomic counter): a
//      16x16 block stages up to 256 triangles of its tile in shared memory (12 floats each), every
//      thread keeps the minimum key of its pixel in a register and merges it with one atomicMin.
// Resolve: one thread per pixel turns the key into rast = (u, v, z/w, id + 1) and rast_db; the
// backward pass chains the gradients of rast and rast_db into the three vertices and scatters
// them with float4 reductions.
#include <cstdint>

#include "common.cuh"
#include "resolve_adjoint.cuh"
#include "warp_reduce.cuh"

namespace dr {
namespace {

// One triangle that needs tile binning: its view (item) and triangle, and its inclusive pixel
// box. The record layout does not depend on the list capacity.
struct Binned {
  int b, t;
  int c0, c1, r0, r1;
};

// The (view, triangle) pairs a visibility pass draws. Instanced mode: every triangle in every
// view, flat index g = view * num_tri + triangle, positions per view. Range mode (range_start
// non-null): item b draws triangles range_start[b] .. + count, flat indices range_first[b] ..
// range_first[b + 1] - 1 (exclusive prefix sums of the counts), all items sharing one position
// buffer (pos_stride 0).
struct Items {
  int num_tri;
  int items;
  const int* range_start;
  const long long* range_first;
  long long pos_stride;  // vertices between the positions of consecutive views
  long long num_vert;    // vertices of one view's positions (bounds checks only)
};

// Sizes that bound the indices read from tri and from the keys (checked build only).
struct Bounds {
  int num_tri;
  long long num_vert;
};

// Vertex index k of triangle t, both checked against their buffers in the checked build.
__device__ __forceinline__ int tri_vertex(const int* __restrict__ tri, long long t, int k,
                                          int num_tri, long long num_vert) {
  t = checked_index(t, num_tri, kSiteTriangle);
  return static_cast<int>(checked_index(__ldg(tri + 3 * t + k), num_vert, kSiteVertex));
}

__device__ __forceinline__ void locate(const Items& it, long long g, int& b, int& t) {
  if (it.range_start == nullptr) {
    // g < 2^31 (checked by the host): a 32-bit division.
    const unsigned gu = static_cast<unsigned>(g), n = static_cast<unsigned>(it.num_tri);
    const unsigned q = gu / n;
    b = static_cast<int>(q);
    t = static_cast<int>(gu - q * n);
    return;
  }
  // Last item whose first flat index is <= g (empty items share their successor's).
  int lo = 0, hi = it.items - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(it.range_first + mid) <= g) lo = mid; else hi = mid - 1;
  }
  b = lo;
  t = __ldg(it.range_start + lo) + static_cast<int>(g - __ldg(it.range_first + lo));
}

struct SetupLayout {
  unsigned long long* counters;  // [0] binned triangles, [1] (triangle, tile) pairs
  float* centres;                // NDC x of every column, then y of every row
  Binned* binned;
};

SetupLayout setup_layout(const void* ws, int height, int width) {
  char* p = static_cast<char*>(const_cast<void*>(ws));
  SetupLayout l;
  l.counters = reinterpret_cast<unsigned long long*>(p);
  l.centres = reinterpret_cast<float*>(p + 256);
  l.binned = reinterpret_cast<Binned*>(p + 256 + align256(sizeof(float) * (height + width)));
  return l;
}

size_t setup_bytes(int64_t capacity, int height, int width) {
  return 256 + align256(sizeof(float) * static_cast<size_t>(height + width)) +
         align256(sizeof(Binned) * static_cast<size_t>(capacity));
}

__global__ void centres_kernel(float* __restrict__ centres, int height, int width) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < width) centres[i] = pixel_centre(i, width);
  else if (i < width + height) centres[i] = pixel_centre(i - width, height);
}

struct BinLayout {
  unsigned* tile_count;   // [tiles]
  unsigned* tile_cursor;  // [tiles]
  unsigned* tile_offset;  // [tiles + 1]
  unsigned* item_offset;  // [tiles + 1]
  unsigned* work;         // [1]
  unsigned* scan_totals;  // [2 (scan chunks + 1)]
  int* pairs;             // [num_pairs]
};

long long scan_chunks(int64_t tiles) { return (tiles + 4095) / 4096; }

BinLayout bin_layout(void* ws, int64_t tiles, int64_t num_pairs) {
  char* p = static_cast<char*>(ws);
  BinLayout l;
  const size_t t = align256(sizeof(unsigned) * static_cast<size_t>(tiles + 1));
  l.tile_count = reinterpret_cast<unsigned*>(p);
  p += t;
  l.tile_cursor = reinterpret_cast<unsigned*>(p);
  p += t;
  l.tile_offset = reinterpret_cast<unsigned*>(p);
  p += t;
  l.item_offset = reinterpret_cast<unsigned*>(p);
  p += t;
  l.work = reinterpret_cast<unsigned*>(p);
  p += 256;
  l.scan_totals = reinterpret_cast<unsigned*>(p);
  p += align256(sizeof(unsigned) * 2 * static_cast<size_t>(scan_chunks(tiles) + 1));
  l.pairs = reinterpret_cast<int*>(p);
  (void)num_pairs;
  return l;
}

size_t bin_bytes(int64_t tiles, int64_t num_pairs) {
  return 4 * align256(sizeof(unsigned) * static_cast<size_t>(tiles + 1)) + 256 +
         align256(sizeof(unsigned) * 2 * static_cast<size_t>(scan_chunks(tiles) + 1)) +
         align256(sizeof(int) * static_cast<size_t>(num_pairs));
}

__global__ void fill_keys_kernel(long long* __restrict__ keys, long long n) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride)
    keys[i] = kEmptyKey;
}

// Pixel centres within [lo, hi] (NDC) as an inclusive index range. The margin keeps centres on
// the boundary despite the rounding of x / w, which grows with the image size; extra pixels are
// tested exactly. Same margin as the reference's Triton setup (_triton_rasterize.py:113-123).
__device__ __forceinline__ void pixel_range(float lo, float hi, int size, int& first, int& last) {
  const float s = static_cast<float>(size);
  const float margin = 1e-3f + s * 1e-6f;
  float f = ceilf(((lo + 1.0f) * s - 1.0f) * 0.5f - margin);
  float l = floorf(((hi + 1.0f) * s - 1.0f) * 0.5f + margin);
  f = fminf(fmaxf(f, 0.0f), s);
  l = fminf(fmaxf(l, -1.0f), s - 1.0f);
  first = static_cast<int>(f);
  last = static_cast<int>(l);
}

// Hardware approximations (at most a few ulp from the exact results over the whole float range,
// subnormals included) for the margins and bounds that only decide which pixels get an exact test.
__device__ __forceinline__ float approx_rcp(float x) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float approx_sqrt(float x) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Direct triangles of a warp, staged so that any lane can work on any of them (structure of
// arrays, indexed by the triangle's rank among the warp's direct triangles).
// Rows a warp can have queued for exact tests (a power of two, at least 63).
constexpr int kRing = 64;

struct WarpTris {
  float4 v[3][32];     // clip-space vertices, for the exact test
  float4 edge[3][32];  // NDC half-planes A x + B y + C >= -D, stored as (1 / A, B, C + D, A)
  float4 aux[32];      // coverage_reach of the triangle (x, y), its index and view (as bits)
  // (first row - number of the triangle's first row among the warp's rows, first column, last
  // column, whether rows are bounded by the half-planes)
  int4 info[32];
  // Ring of rows with pixels to test: (triangle rank | row << 5, column of the row's pixel number
  // 0, number of pixels queued up to the row's end, the row's NDC centre as bits).
  int4 row[kRing];
};

// Occlusion pass state. The first visibility pass sets aside small triangles that face away in
// screen space (negative orientation: the far side of a closed, outward-facing mesh) as records
// (flat index, tile box x0 | x1 << 16, y0 | y1 << 16, ordered lower bound of their depth); once
// everything else is in the keys, the largest key of every 16 x 16 tile is taken, and a set-aside
// triangle whose depth bound lies above the largest key of every tile it touches cannot be the
// nearest anywhere and is skipped; the others are drawn as usual.
struct Occlusion {
  unsigned long long* count;   // records set aside
  int4* list;                  // [capacity]
  const long long* tile_max;   // [views, tiles_per_view]
  int tiles_x, tiles_per_view;
};

// Largest key of each 16 x 16 tile (grid: tiles x, tiles y, views).
__global__ void __launch_bounds__(256) tile_max_kernel(const long long* __restrict__ keys,
                                                       int height, int width,
                                                       long long* __restrict__ tile_max) {
  __shared__ long long warp_max[8];
  const int row = blockIdx.y * kTile + static_cast<int>(threadIdx.x) / kTile;
  const int col = blockIdx.x * kTile + static_cast<int>(threadIdx.x) % kTile;
  const long long b = blockIdx.z;
  long long m = -0x7FFFFFFFFFFFFFFFLL - 1;
  if (row < height && col < width) m = __ldg(keys + (b * height + row) * width + col);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long other = __shfl_xor_sync(0xffffffffu, m, o);
    m = other > m ? other : m;
  }
  if ((threadIdx.x & 31u) == 0u) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < 8; ++i) m = warp_max[i] > m ? warp_max[i] : m;
    tile_max[(b * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x] = m;
  }
}

// Lower bound of the depth z / w that the exact test can give anywhere inside a triangle whose
// vertices all have w > 0: the interpolated depth is a convex combination of the vertex depths
// (the edge functions share one sign and so do the weights e_k w_k), up to a few float32
// roundings of terms no larger than the largest |z_k / w_k|; 1e-5 of it covers them many times.
// Returned as the ordered high word of the packed key.
__device__ __forceinline__ int depth_floor_word(const Vert& v0, const Vert& v1, const Vert& v2) {
  const float d0 = v0.z / v0.w, d1 = v1.z / v1.w, d2 = v2.z / v2.w;
  const float mag = fmaxf(fmaxf(fabsf(d0), fabsf(d1)), fabsf(d2));
  const float lb = fminf(fminf(d0, d1), d2) - (1e-5f * mag + 1e-30f);
  if (!(lb == lb)) return -0x7FFFFFFF - 1;  // never set aside with a NaN bound
  return static_cast<int>(pack_key(lb, 0) >> 32);
}

// Four blocks per SM: up to 64 registers, a little faster than five blocks at 48 (measured on
// config 5: 6.50 against 6.54 ms).
template <int kPass>
__global__ void __launch_bounds__(256, 4) setup_kernel(
    const float* __restrict__ pos, const int* __restrict__ tri, const Items items,
    long long total, int height, int width, const float* __restrict__ centres,
    const long long* __restrict__ prev, long long* __restrict__ keys,
    unsigned long long* __restrict__ counters, Binned* __restrict__ binned, long long capacity,
    const Occlusion oc) {
  __shared__ WarpTris staged[8];
  const unsigned lane = threadIdx.x & 31u;
  WarpTris& w = staged[threadIdx.x >> 5];
  // Passes 0 (everything) and 1 (setting aside) take one item per thread; pass 2 walks the
  // records set aside with a grid-stride loop.
  const long long items_n = kPass == 2 ? static_cast<long long>(*oc.count) : total;
  const long long step = kPass == 2 ? static_cast<long long>(gridDim.x) * blockDim.x : items_n;
  for (long long first = blockIdx.x * static_cast<long long>(blockDim.x); first < items_n;
       first += step) {
    const long long item = first + threadIdx.x;
    long long g = item < items_n ? item : total;
    if (kPass == 2 && item < items_n) {
      const int4 rec = oc.list[item];
      g = rec.x;
      int vb, vt;
      locate(items, g, vb, vt);
      const long long* tm = oc.tile_max + static_cast<long long>(vb) * oc.tiles_per_view;
      const int tx0 = rec.y & 0xFFFF, tx1 = static_cast<int>(static_cast<unsigned>(rec.y) >> 16);
      const int ty0 = rec.z & 0xFFFF, ty1 = static_cast<int>(static_cast<unsigned>(rec.z) >> 16);
      long long m = -0x7FFFFFFFFFFFFFFFLL - 1;
      for (int ty = ty0; ty <= ty1; ++ty)
        for (int tx = tx0; tx <= tx1; ++tx) {
          const long long k = __ldg(tm + ty * oc.tiles_x + tx);
          m = k > m ? k : m;
        }
      if ((static_cast<long long>(rec.w) << 32) > m) g = total;  // behind every pixel it touches
    }
    bool large = false, direct = false;
    unsigned pairs = 0;
    int b = 0, t = 0, c0 = 0, c1 = -1, r0 = 0, r1 = -1;
    Vert v0 = {0.f, 0.f, 0.f, 1.f}, v1 = v0, v2 = v0;
    float nx[3] = {0.f, 0.f, 0.f}, ny[3] = {0.f, 0.f, 0.f};
    if (g < total) {
      locate(items, g, b, t);
      const int i0 = tri_vertex(tri, t, 0, items.num_tri, items.num_vert);
      const int i1 = tri_vertex(tri, t, 1, items.num_tri, items.num_vert);
      const int i2 = tri_vertex(tri, t, 2, items.num_tri, items.num_vert);
      const long long base = static_cast<long long>(b) * items.pos_stride;
      v0 = load_vert(pos, base + i0);
      v1 = load_vert(pos, base + i1);
      v2 = load_vert(pos, base + i2);
      // A triangle is invisible when all vertices are behind the camera or outside the same side
      // plane; every covered point is a non-negative combination of the vertices. Non-finite
      // vertices are never drawn (reference.py:334).
      bool culled = !(finite4(v0) && finite4(v1) && finite4(v2));
      culled |= (v0.w <= 0.0f) && (v1.w <= 0.0f) && (v2.w <= 0.0f);
      culled |= (v0.x > v0.w) && (v1.x > v1.w) && (v2.x > v2.w);
      culled |= (v0.x < -v0.w) && (v1.x < -v1.w) && (v2.x < -v2.w);
      culled |= (v0.y > v0.w) && (v1.y > v1.w) && (v2.y > v2.w);
      culled |= (v0.y < -v0.w) && (v1.y < -v1.w) && (v2.y < -v2.w);
      if (!culled) {
        const bool in_front = (v0.w > 0.0f) && (v1.w > 0.0f) && (v2.w > 0.0f);
        c0 = 0;
        c1 = width - 1;
        r0 = 0;
        r1 = height - 1;
        if (in_front) {
          // Projected vertices bound the pixels to test, never decide coverage; bounds are widened
          // by margins far above the error of the fast reciprocal used for ordinary w.
          const Vert* vs[3] = {&v0, &v1, &v2};
          for (int k = 0; k < 3; ++k) {
            const float wk = vs[k]->w;
            if (wk >= 1e-30f && wk <= 1e30f) {
              const float iw = __fdividef(1.0f, wk);
              nx[k] = vs[k]->x * iw;
              ny[k] = vs[k]->y * iw;
            } else {
              nx[k] = vs[k]->x / wk;
              ny[k] = vs[k]->y / wk;
            }
          }
          pixel_range(fminf(fminf(nx[0], nx[1]), nx[2]), fmaxf(fmaxf(nx[0], nx[1]), nx[2]), width,
                      c0, c1);
          pixel_range(fminf(fminf(ny[0], ny[1]), ny[2]), fmaxf(fmaxf(ny[0], ny[1]), ny[2]), height,
                      r0, r1);
        }
        if (c0 <= c1 && r0 <= r1) {
          const long long area = static_cast<long long>(c1 - c0 + 1) * (r1 - r0 + 1);
          if (in_front && area <= kWarpPixels) {
            direct = true;
            if (kPass == 1) {
              const float ex = (nx[1] - nx[0]) * (ny[2] - ny[0]);
              const float ey = (ny[1] - ny[0]) * (nx[2] - nx[0]);
              const float area2 = ex - ey;
              if (area2 < -1e-3f * (fabsf(ex) + fabsf(ey))) {
                direct = false;
                const unsigned aside = __activemask();
                const int rank_aside = __popc(aside & ((1u << lane) - 1u));
                const int leader = __ffs(aside) - 1;
                unsigned long long slot0 = 0;
                if (static_cast<int>(lane) == leader)
                  slot0 = atomicAdd(oc.count, static_cast<unsigned long long>(__popc(aside)));
                slot0 = __shfl_sync(aside, slot0, leader);
                const int tx0 = c0 / kTile, tx1 = c1 / kTile, ty0 = r0 / kTile, ty1 = r1 / kTile;
                oc.list[slot0 + rank_aside] =
                    make_int4(static_cast<int>(g), tx0 | (tx1 << 16), ty0 | (ty1 << 16),
                              depth_floor_word(v0, v1, v2));
              }
            }
          } else {
            large = true;
            const unsigned tx0 = c0 / kTile, tx1 = c1 / kTile, ty0 = r0 / kTile, ty1 = r1 / kTile;
            pairs = (tx1 - tx0 + 1) * (ty1 - ty0 + 1);
          }
        }
      }
    }
    // Stage the direct triangles in rank order. Their rows are distributed over the lanes (phase A:
    // each lane bounds one row by the triangle's half-planes), then the pixels inside those row
    // spans are distributed over the lanes again (phase B: one exact test per lane), so lanes stay
    // busy whatever the shape of the triangles.
    const unsigned direct_mask = __ballot_sync(0xffffffffu, direct);
    const int rank = __popc(direct_mask & ((1u << lane) - 1u));
    const int rows = direct ? r1 - r0 + 1 : 0;
    int end = rows;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, end, o);
      if (static_cast<int>(lane) >= o) end += y;
    }
    const int all_rows = __shfl_sync(0xffffffffu, end, 31);
    if (direct) {
      w.v[0][rank] = make_float4(v0.x, v0.y, v0.z, v0.w);
      w.v[1][rank] = make_float4(v1.x, v1.y, v1.z, v1.w);
      w.v[2][rank] = make_float4(v2.x, v2.y, v2.z, v2.w);
      const float2 reach = coverage_reach(v0, v1, v2);
      w.aux[rank] = make_float4(reach.x, reach.y, __int_as_float(t), __int_as_float(b));
      // Half-planes of the projected triangle, oriented inwards and widened by a margin that
      // covers the rounding of x / w and of the exact homogeneous test many times over. A triangle
      // whose projected orientation is not clear-cut keeps whole bounding-box rows.
      const float ex = (nx[1] - nx[0]) * (ny[2] - ny[0]), ey = (ny[1] - ny[0]) * (nx[2] - nx[0]);
      const float area2 = ex - ey;
      const bool spans = fabsf(area2) > 1e-3f * (fabsf(ex) + fabsf(ey));
      w.info[rank] = make_int4(r0 - (end - rows), c0, c1, spans ? 1 : 0);
      const float o = area2 > 0.0f ? 1.0f : -1.0f;
      const float size = static_cast<float>(max(width, height));
      const float delta = (0.01f + size * 1e-6f) * 2.0f / static_cast<float>(min(width, height));
      for (int k = 0; k < 3; ++k) {
        const int i = (k + 1) % 3, j = (k + 2) % 3;
        const float A = -o * (ny[j] - ny[i]), B = o * (nx[j] - nx[i]);
        const float C = -(A * nx[i] + B * ny[i]);
        const float D = delta * approx_sqrt(A * A + B * B) +
                        4e-6f * (fabsf(A) + fabsf(B)) * (1.0f + fabsf(nx[i]) + fabsf(ny[i]));
        // Row bounds are x >= (-(B y + C) - D) / A (A > 0) or x <= it (A < 0): keep 1 / A.
        w.edge[k][rank] = make_float4(A != 0.0f ? approx_rcp(A) : 0.0f, B, C + D, A);
      }
    }
    __syncwarp();
    // Rows with pixels to test join a ring of kRing records; exact tests run 32 pixels at a time as
    // soon as 32 are queued (and once more at the end), so that the pixels of consecutive row
    // batches share test iterations. After a drain fewer than 32 pixels (so at most 31 rows) are
    // pending and a batch adds at most 32 rows, so the ring never overwrites a pending row.
    int done = 0;           // triangles whose rows all precede this batch
    int queued_rows = 0;    // rows appended to the ring so far
    int consumed_rows = 0;  // rows whose pixels have all been tested
    int queued_px = 0;      // pixels appended so far
    int tested_px = 0;      // pixels tested so far
    for (int base = 0; base < all_rows; base += 32) {
      // Phase A. Bit e - base - 1 marks a triangle whose rows end at e within (base, base + 32];
      // the owner of row item base + lane is the number of triangles ending at or before it.
      unsigned bit = 0u;
      if (direct && end > base && end <= base + 32) bit = 1u << (end - base - 1);
      const unsigned ends = __reduce_or_sync(0xffffffffu, bit);
      const int item = base + static_cast<int>(lane);
      const int k = done + __popc(ends & ((1u << lane) - 1u));
      done += __popc(ends);
      int count = 0, row = 0, cl = 0;
      float py = 0.0f;
      if (item < all_rows) {
        const int4 info = w.info[k];
        row = info.x + item;
        cl = info.y;
        int cr = info.z;
        py = __ldg(centres + width + row);
        if (info.w) {
          float lo = -__int_as_float(0x7f800000), hi = __int_as_float(0x7f800000);
          bool empty = false;
          for (int e = 0; e < 3; ++e) {
            const float4 h = w.edge[e][k];  // (1 / A, B, C + D, A)
            const float rhs = -(h.y * py + h.z);
            if (h.w > 0.0f) lo = fmaxf(lo, rhs * h.x);
            else if (h.w < 0.0f) hi = fminf(hi, rhs * h.x);
            else empty |= rhs > 0.0f;
          }
          if (empty || !(lo <= hi)) {
            cr = cl - 1;
          } else {
            int sl, sr;
            pixel_range(lo, hi, width, sl, sr);
            cl = max(cl, sl);
            cr = min(cr, sr);
          }
        }
        count = max(0, cr - cl + 1);
      }
      // Append the rows that have pixels, numbering their pixels after those already queued.
      const unsigned busy = __ballot_sync(0xffffffffu, count > 0);
      const int slot = __popc(busy & ((1u << lane) - 1u));
      int pix_end = count;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, pix_end, o);
        if (static_cast<int>(lane) >= o) pix_end += y;
      }
      if (count > 0) {
        const int q = (queued_rows + slot) & (kRing - 1);
        const int last = queued_px + pix_end;  // pixels queued up to the end of this row
        // (triangle rank, row, column of pixel number 0 of this row's numbering, end)
        w.row[q] = make_int4(k | (row << 5), cl - (last - count), last, __float_as_int(py));
      }
      queued_rows += __popc(busy);
      queued_px += __shfl_sync(0xffffffffu, pix_end, 31);
      __syncwarp();
      // Phase B: one exact coverage test per lane.
      const bool final_batch = base + 32 >= all_rows;
      while (queued_px - tested_px >= 32 || (final_batch && queued_px > tested_px)) {
        // Rows ending within (tested_px, tested_px + 32] mark their last pixel; the owner of pixel
        // tested_px + lane is the number of such rows ending before it.
        const int n = consumed_rows + static_cast<int>(lane);
        unsigned pbit = 0u;
        if (n < queued_rows) {
          const int e = w.row[n & (kRing - 1)].z;
          if (e <= tested_px + 32) pbit = 1u << (e - tested_px - 1);
        }
        const unsigned pends = __reduce_or_sync(0xffffffffu, pbit);
        const int pitem = tested_px + static_cast<int>(lane);
        const int r = (consumed_rows + __popc(pends & ((1u << lane) - 1u))) & (kRing - 1);
        consumed_rows += __popc(pends);
        tested_px += 32;
        if (pitem >= queued_px) continue;
        const int4 rec = w.row[r];
        const int kk = rec.x & 31, y = rec.x >> 5, col = rec.y + pitem;
        const float4 a = w.v[0][kk], bb = w.v[1][kk], cc = w.v[2][kk];
        const float4 aux = w.aux[kk];
        const long long key = coverage_key({a.x, a.y, a.z, a.w}, {bb.x, bb.y, bb.z, bb.w},
                                           {cc.x, cc.y, cc.z, cc.w}, __ldg(centres + col),
                                           __int_as_float(rec.w), __float_as_int(aux.z), aux.x,
                                           aux.y);
        if (key == kEmptyKey) continue;
        const long long off = checked_index(
            (static_cast<long long>(__float_as_int(aux.w)) * height + y) * width + col,
            static_cast<long long>(items.items) * height * width, kSitePixel);
        if (prev != nullptr && !(key > __ldg(prev + off))) continue;
        atomicMin(keys + off, key);
      }
      tested_px = min(tested_px, queued_px);
      __syncwarp();
    }
    // Warp-aggregated append of the large triangles and of their pair counts.
    const unsigned mask = __ballot_sync(0xffffffffu, large);
    unsigned long long warp_pairs = pairs;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) warp_pairs += __shfl_xor_sync(0xffffffffu, warp_pairs, o);
    if (mask != 0u) {
      unsigned long long slot0 = 0;
      if (lane == 0) {
        slot0 = atomicAdd(counters, static_cast<unsigned long long>(__popc(mask)));
        atomicAdd(counters + 1, warp_pairs);
      }
      slot0 = __shfl_sync(0xffffffffu, slot0, 0);
      if (large) {
        const unsigned long long slot = slot0 + __popc(mask & ((1u << lane) - 1u));
        if (slot < static_cast<unsigned long long>(capacity)) binned[slot] = {b, t, c0, c1, r0, r1};
      }
    }
  }
}

// One warp per binned triangle; its lanes walk the triangle's tiles.
// Device-driven variant (count_on_device non-null): the count is the setup counter, and a list
// or pair total above its capacity (an incomplete list) is flagged in *overflow and nothing is
// scattered.
struct DeviceCounts {
  const unsigned long long* count_on_device;  // setup counter [0], or null
  long long capacity;                         // records in the binned list
  long long pair_capacity;                    // entries of the pair list
  unsigned long long* overflow;
};

template <bool kScatter>
__global__ void __launch_bounds__(256) bin_kernel(const Binned* __restrict__ binned,
                                                  long long count, int tiles_x, int tiles_per_image,
                                                  unsigned* __restrict__ tile_count,
                                                  const unsigned* __restrict__ tile_offset,
                                                  int* __restrict__ pairs, const DeviceCounts dc,
                                                  int num_tiles) {
  if (dc.count_on_device != nullptr) {
    count = static_cast<long long>(*dc.count_on_device);
    const bool over = count > dc.capacity ||
                      (kScatter && static_cast<long long>(tile_offset[num_tiles]) > dc.pair_capacity);
    if (over) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(dc.overflow, 1ull);
      return;
    }
  }
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
  const unsigned lane = threadIdx.x & 31u;
  for (long long i = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) / 32; i < count;
       i += warps) {
    const Binned rec = binned[i];
    const int b = rec.b;
    const int tx0 = rec.c0 / kTile, tx1 = rec.c1 / kTile, ty0 = rec.r0 / kTile, ty1 = rec.r1 / kTile;
    const int nx = tx1 - tx0 + 1;
    const int n = nx * (ty1 - ty0 + 1);
    for (int k = lane; k < n; k += 32) {
      const int tile = b * tiles_per_image + (ty0 + k / nx) * tiles_x + tx0 + k % nx;
      if (kScatter) {
        const unsigned slot = atomicAdd(tile_count + tile, 1u);
        pairs[tile_offset[tile] + slot] = static_cast<int>(i);
      } else {
        atomicAdd(tile_count + tile, 1u);
      }
    }
  }
}

// Exclusive scans of the per-tile pair counts and of their 256-triangle work items, in three
// passes over chunks of kScanChunk tiles: chunk totals (scan_totals_kernel), an exclusive scan of
// the totals in one block (scan_chunks_kernel), and each chunk's scan from its carry
// (scan_kernel).
constexpr int kScanPer = 4;
constexpr int kScanChunk = 1024 * kScanPer;

__device__ __forceinline__ unsigned work_items(unsigned pairs) { return (pairs + kChunk - 1) / kChunk; }

// Block-wide inclusive scan of (xa, xb) over 1024 threads; returns the block totals too.
__device__ __forceinline__ void block_scan2(unsigned& xa, unsigned& xb, unsigned& total_a,
                                            unsigned& total_b) {
  __shared__ unsigned warp_a[32], warp_b[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned ya = __shfl_up_sync(0xffffffffu, xa, o);
    const unsigned yb = __shfl_up_sync(0xffffffffu, xb, o);
    if (lane >= o) {
      xa += ya;
      xb += yb;
    }
  }
  if (lane == 31) {
    warp_a[warp] = xa;
    warp_b[warp] = xb;
  }
  __syncthreads();
  if (warp == 0) {
    unsigned wa = warp_a[lane], wb = warp_b[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned ya = __shfl_up_sync(0xffffffffu, wa, o);
      const unsigned yb = __shfl_up_sync(0xffffffffu, wb, o);
      if (lane >= o) {
        wa += ya;
        wb += yb;
      }
    }
    warp_a[lane] = wa;
    warp_b[lane] = wb;
  }
  __syncthreads();
  if (warp > 0) {
    xa += warp_a[warp - 1];
    xb += warp_b[warp - 1];
  }
  total_a = warp_a[31];
  total_b = warp_b[31];
  __syncthreads();
}

__global__ void __launch_bounds__(1024) scan_totals_kernel(const unsigned* __restrict__ count, int n,
                                                           unsigned* __restrict__ totals) {
  unsigned sa = 0, sb = 0;
#pragma unroll
  for (int j = 0; j < kScanPer; ++j) {
    const long long i = static_cast<long long>(blockIdx.x) * kScanChunk + threadIdx.x * kScanPer + j;
    const unsigned c = i < n ? count[i] : 0u;
    sa += c;
    sb += work_items(c);
  }
  unsigned ta, tb;
  block_scan2(sa, sb, ta, tb);
  if (threadIdx.x == 0) {
    totals[2 * blockIdx.x] = ta;
    totals[2 * blockIdx.x + 1] = tb;
  }
}

// Exclusive scan of the chunk totals in place; the grand totals go to totals[2 chunks, + 1].
__global__ void __launch_bounds__(1024) scan_chunks_kernel(unsigned* __restrict__ totals,
                                                           int chunks) {
  unsigned carry_a = 0, carry_b = 0;
  for (int base = 0; base < chunks; base += 1024) {
    const int i = base + static_cast<int>(threadIdx.x);
    const unsigned ca = i < chunks ? totals[2 * i] : 0u, cb = i < chunks ? totals[2 * i + 1] : 0u;
    unsigned xa = ca, xb = cb, ta, tb;
    block_scan2(xa, xb, ta, tb);
    if (i < chunks) {
      totals[2 * i] = carry_a + xa - ca;
      totals[2 * i + 1] = carry_b + xb - cb;
    }
    carry_a += ta;
    carry_b += tb;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    totals[2 * chunks] = carry_a;
    totals[2 * chunks + 1] = carry_b;
  }
}

__global__ void __launch_bounds__(1024) scan_kernel(const unsigned* __restrict__ count, int n,
                                                    const unsigned* __restrict__ totals, int chunks,
                                                    unsigned* __restrict__ offset,
                                                    unsigned* __restrict__ item_offset) {
  const long long base = static_cast<long long>(blockIdx.x) * kScanChunk + threadIdx.x * kScanPer;
  unsigned a[kScanPer], b[kScanPer], sa = 0, sb = 0;
#pragma unroll
  for (int j = 0; j < kScanPer; ++j) {
    const long long i = base + j;
    const unsigned c = i < n ? count[i] : 0u;
    a[j] = sa;
    b[j] = sb;
    sa += c;
    sb += work_items(c);
  }
  unsigned xa = sa, xb = sb, ta, tb;
  block_scan2(xa, xb, ta, tb);
  const unsigned pre_a = totals[2 * blockIdx.x] + xa - sa;
  const unsigned pre_b = totals[2 * blockIdx.x + 1] + xb - sb;
#pragma unroll
  for (int j = 0; j < kScanPer; ++j) {
    const long long i = base + j;
    if (i < n) {
      offset[i] = pre_a + a[j];
      item_offset[i] = pre_b + b[j];
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    offset[n] = totals[2 * chunks];
    item_offset[n] = totals[2 * chunks + 1];
  }
}

__global__ void __launch_bounds__(256) tile_kernel(
    const float* __restrict__ pos, const int* __restrict__ tri, long long pos_stride,
    const Bounds bd, int height, int width, int tiles_x, int tiles_per_image, int num_tiles,
    const float* __restrict__ centres,
    const long long* __restrict__ prev, long long* __restrict__ keys, const int* __restrict__ pairs,
    const Binned* __restrict__ binned, const unsigned* __restrict__ tile_offset,
    const unsigned* __restrict__ item_offset, unsigned* __restrict__ work, const DeviceCounts dc) {
  __shared__ float4 sv[3][kChunk];
  __shared__ int st[kChunk];
  __shared__ int4 sbox[kChunk];
  __shared__ int s_tile;
  __shared__ unsigned s_first, s_count;
  const int lx = threadIdx.x % kTile, ly = threadIdx.x / kTile;
  const unsigned total_items = item_offset[num_tiles];
  if (dc.count_on_device != nullptr &&
      (static_cast<long long>(*dc.count_on_device) > dc.capacity ||
       static_cast<long long>(tile_offset[num_tiles]) > dc.pair_capacity))
    return;  // flagged by bin_kernel
  for (;;) {
    if (threadIdx.x == 0) {
      const unsigned item = atomicAdd(work, 1u);
      int tile = -1;
      if (item < total_items) {
        // Last tile whose first item is <= item.
        int lo = 0, hi = num_tiles - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (item_offset[mid] <= item) lo = mid; else hi = mid - 1;
        }
        tile = lo;
        const unsigned first = tile_offset[tile] + (item - item_offset[tile]) * kChunk;
        const unsigned end = min(first + kChunk, tile_offset[tile + 1]);
        s_first = first;
        s_count = end - first;
      }
      s_tile = tile;
    }
    __syncthreads();
    const int tile = s_tile;
    if (tile < 0) break;
    const int n = static_cast<int>(s_count);
    if (threadIdx.x < n) {
      const Binned rec = binned[pairs[s_first + threadIdx.x]];
      const int b = rec.b, t = rec.t;
      const long long base = static_cast<long long>(b) * pos_stride;
      const float4* p4 = reinterpret_cast<const float4*>(pos);
      sv[0][threadIdx.x] = __ldg(p4 + base + tri_vertex(tri, t, 0, bd.num_tri, bd.num_vert));
      sv[1][threadIdx.x] = __ldg(p4 + base + tri_vertex(tri, t, 1, bd.num_tri, bd.num_vert));
      sv[2][threadIdx.x] = __ldg(p4 + base + tri_vertex(tri, t, 2, bd.num_tri, bd.num_vert));
      st[threadIdx.x] = t;
      sbox[threadIdx.x] = make_int4(rec.c0, rec.c1, rec.r0, rec.r1);
    }
    __syncthreads();
    const int image = tile / tiles_per_image;
    const int in_image = tile - image * tiles_per_image;
    const int row = (in_image / tiles_x) * kTile + ly;
    const int col = (in_image % tiles_x) * kTile + lx;
    if (row < height && col < width) {
      const float px = __ldg(centres + col), py = __ldg(centres + width + row);
      const long long off = (static_cast<long long>(image) * height + row) * width + col;
      const long long floor_key = prev != nullptr ? __ldg(prev + off) : -0x7FFFFFFFFFFFFFFFLL - 1;
      long long best = kEmptyKey;
      for (int i = 0; i < n; ++i) {
        const int4 box = sbox[i];
        if (col < box.x || col > box.y || row < box.z || row > box.w) continue;
        const float4 a = sv[0][i], b = sv[1][i], c = sv[2][i];
        const long long key = coverage_key({a.x, a.y, a.z, a.w}, {b.x, b.y, b.z, b.w},
                                           {c.x, c.y, c.z, c.w}, px, py, st[i]);
        if (key > floor_key && key < best) best = key;
      }
      if (best != kEmptyKey) atomicMin(keys + off, best);
    }
    __syncthreads();
  }
}

struct PixelTri {
  bool covered;
  int b, t;
  int i0, i1, i2;
  Vert v0, v1, v2;
  float px, py;
};

// Pixel (view b, row, col) of the resolve kernels' grid: columns in x, rows in y (from row0 on),
// views in z (from view b0 on). Images with more rows or views than a grid dimension holds
// (65535) take several launches.
struct ResolvePixel {
  int b, row, col;
  long long p;
  bool inside;
};

__device__ __forceinline__ ResolvePixel resolve_pixel(int b0, int row0, int height, int width) {
  ResolvePixel r;
  r.col = blockIdx.x * blockDim.x + threadIdx.x;
  r.row = row0 + static_cast<int>(blockIdx.y);
  r.b = b0 + static_cast<int>(blockIdx.z);
  r.inside = r.col < width;
  r.p = (static_cast<long long>(r.b) * height + r.row) * width + r.col;
  return r;
}

__device__ __forceinline__ PixelTri pixel_triangle(const float* __restrict__ pos,
                                                   const int* __restrict__ tri,
                                                   const long long* __restrict__ keys,
                                                   const ResolvePixel& rp, long long pos_stride,
                                                   const Bounds& bd, int height, int width) {
  PixelTri r;
  const long long key = keys[rp.p];
  r.covered = key != kEmptyKey;
  r.b = rp.b;
  const int row = rp.row, col = rp.col;
  r.px = pixel_centre(col, width);
  r.py = pixel_centre(row, height);
  r.t = static_cast<int>(key & 0xFFFFFFFFLL);
  if (r.covered) {
    r.i0 = tri_vertex(tri, r.t, 0, bd.num_tri, bd.num_vert);
    r.i1 = tri_vertex(tri, r.t, 1, bd.num_tri, bd.num_vert);
    r.i2 = tri_vertex(tri, r.t, 2, bd.num_tri, bd.num_vert);
    const long long base = static_cast<long long>(r.b) * pos_stride;
    r.v0 = load_vert(pos, base + r.i0);
    r.v1 = load_vert(pos, base + r.i1);
    r.v2 = load_vert(pos, base + r.i2);
  } else {
    r.i0 = r.i1 = r.i2 = 0;
    r.v0 = r.v1 = r.v2 = {0.0f, 0.0f, 0.0f, 1.0f};
  }
  return r;
}

// Pixels per thread of the resolve forward pass: each thread walks kResolvePix pixels of a row,
// 128 columns apart, one load phase at a time (keys, then vertex indices, then vertices), so that
// the loads of all its pixels are in flight together.
constexpr int kResolvePix = 2;
constexpr int kResolveThreads = 128;

// Graph-captured passes only: when the device word `overflow` is set (a captured pass outgrew
// its binning capacity since the host last cleared the word), the depth field of every covered
// pixel's key becomes kPoisonDepth; the triangle field, which the resolve passes index with, is
// kept. One 8-byte read per block when the word is clear.
__global__ void __launch_bounds__(256) poison_keys_kernel(const unsigned long long* __restrict__ overflow,
                                                          long long* __restrict__ keys,
                                                          long long count) {
  __shared__ unsigned long long flag;
  if (threadIdx.x == 0) flag = *overflow;
  __syncthreads();
  if (flag == 0) return;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += stride) {
    const long long key = keys[i];
    if (key == kEmptyKey) continue;
    keys[i] = (static_cast<long long>(kPoisonDepth) << 32) | (key & 0xFFFFFFFFLL);
  }
}

__global__ void __launch_bounds__(kResolveThreads) resolve_fwd_kernel(
    const float* __restrict__ pos, const int* __restrict__ tri, const long long* __restrict__ keys,
    int b0, int row0, long long pos_stride, const Bounds bd, int height, int width,
    float4* __restrict__ rast, float4* __restrict__ rast_db) {
  const int row = row0 + static_cast<int>(blockIdx.y);
  const long long b = b0 + static_cast<long long>(blockIdx.z);
  const long long row_start = (b * height + row) * width;
  const long long base = b * pos_stride;
  long long key[kResolvePix];
#pragma unroll
  for (int i = 0; i < kResolvePix; ++i) {
    const int col = blockIdx.x * (kResolveThreads * kResolvePix) + i * kResolveThreads + threadIdx.x;
    key[i] = col < width ? __ldcs(keys + row_start + col) : kEmptyKey;
  }
  int idx[kResolvePix][3];
#pragma unroll
  for (int i = 0; i < kResolvePix; ++i) {
    const long long t = key[i] & 0xFFFFFFFFLL;
#pragma unroll
    for (int k = 0; k < 3; ++k)
      idx[i][k] = key[i] != kEmptyKey ? tri_vertex(tri, t, k, bd.num_tri, bd.num_vert) : 0;
  }
  Vert v[kResolvePix][3];
#pragma unroll
  for (int i = 0; i < kResolvePix; ++i)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      v[i][k] = key[i] != kEmptyKey ? load_vert(pos, base + idx[i][k]) : Vert{0.f, 0.f, 0.f, 1.f};
  const float py = pixel_centre(row, height);
#pragma unroll
  for (int i = 0; i < kResolvePix; ++i) {
    const int col = blockIdx.x * (kResolveThreads * kResolvePix) + i * kResolveThreads + threadIdx.x;
    if (col >= width) continue;
    const long long p = row_start + col;
    if (key[i] == kEmptyKey) {
      rast[p] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (rast_db != nullptr) rast_db[p] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      continue;
    }
    if (static_cast<int>(key[i] >> 32) == kPoisonDepth) {
      const float nan = __int_as_float(0x7FC00000);
      rast[p] = make_float4(nan, nan, nan, static_cast<float>((key[i] & 0xFFFFFFFFLL) + 1));
      if (rast_db != nullptr) rast_db[p] = make_float4(nan, nan, nan, nan);
      continue;
    }
    const float px = pixel_centre(col, width);
    const Vert &v0 = v[i][0], &v1 = v[i][1], &v2 = v[i][2];
    const float a0 = v0.x - px * v0.w, a1 = v1.x - px * v1.w, a2 = v2.x - px * v2.w;
    const float c0 = v0.y - py * v0.w, c1 = v1.y - py * v1.w, c2 = v2.y - py * v2.w;
    const float e0 = a1 * c2 - a2 * c1, e1 = a2 * c0 - a0 * c2, e2 = a0 * c1 - a1 * c0;
    const float s = e0 + e1 + e2;
    const float u = e0 / s, vv = e1 / s;
    const float ew = e0 * v0.w + e1 * v1.w + e2 * v2.w;
    const float depth = (e0 * v0.z + e1 * v1.z + e2 * v2.z) / ew;
    __stcs(rast + p, make_float4(u, vv, depth, static_cast<float>((key[i] & 0xFFFFFFFFLL) + 1)));
    if (rast_db != nullptr) {
      // de/dpx = c x w and de/dpy = w x a (reference.py:281-290).
      const float dx0 = c1 * v2.w - c2 * v1.w, dx1 = c2 * v0.w - c0 * v2.w;
      const float dx2 = c0 * v1.w - c1 * v0.w;
      const float dy0 = v1.w * a2 - v2.w * a1, dy1 = v2.w * a0 - v0.w * a2;
      const float dy2 = v0.w * a1 - v1.w * a0;
      const float sx = dx0 + dx1 + dx2, sy = dy0 + dy1 + dy2;
      const float inv_s = 1.0f / s;
      const float scale_x = 2.0f / static_cast<float>(width) * inv_s;
      const float scale_y = 2.0f / static_cast<float>(height) * inv_s;
      __stcs(rast_db + p, make_float4((dx0 - u * sx) * scale_x, (dy0 - u * sy) * scale_y,
                                      (dx1 - vv * sx) * scale_x, (dy1 - vv * sy) * scale_y));
    }
  }
}

__global__ void __launch_bounds__(256) resolve_bwd_kernel(
    const float* __restrict__ pos, const int* __restrict__ tri, const long long* __restrict__ keys,
    int b0, int row0, long long pos_stride, const Bounds bd, int height, int width,
    const float4* __restrict__ grad_rast, const float4* __restrict__ grad_db,
    float* __restrict__ grad_pos) {
  const ResolvePixel rp = resolve_pixel(b0, row0, height, width);
  const long long p = rp.p;
  PixelTri q;
  if (rp.inside) {
    q = pixel_triangle(pos, tri, keys, rp, pos_stride, bd, height, width);
  } else {
    q.covered = false;
    q.b = 0;
    q.i0 = q.i1 = q.i2 = 0;
  }
  float gv[3][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  if (q.covered) {
    const float4 gr = grad_rast[p];
    const float4 gd = grad_db != nullptr ? grad_db[p] : make_float4(0.f, 0.f, 0.f, 0.f);
    resolve_adjoint(q.v0, q.v1, q.v2, q.px, q.py, gr, grad_db != nullptr, gd, width, height, gv);
  }
  const long long base = static_cast<long long>(q.b) * pos_stride;
  // Lanes showing the same triangle (a warp covers 32 pixels of one row) sum their vertex
  // gradients first; one of them adds the sums with three vector reductions.
  const unsigned act = __ballot_sync(0xffffffffu, q.covered);
  if (act == 0u) return;
  const unsigned lane = threadIdx.x & 31u;
  unsigned peers = 1u << lane;
  if (q.covered) peers = __match_any_sync(act, q.t);
  float v[12];
#pragma unroll
  for (int k = 0; k < 3; ++k)
#pragma unroll
    for (int c = 0; c < 4; ++c) v[4 * k + c] = gv[k][c];
  segmented_sum<12>(peers, v);
  if (!q.covered || (peers & ((1u << lane) - 1u)) != 0u) return;
#pragma unroll
  for (int k = 0; k < 3; ++k)
#pragma unroll
    for (int c = 0; c < 4; ++c) gv[k][c] = v[4 * k + c];
  red_add_v4(grad_pos + (base + q.i0) * 4, gv[0][0], gv[0][1], gv[0][2], gv[0][3]);
  red_add_v4(grad_pos + (base + q.i1) * 4, gv[1][0], gv[1][1], gv[1][2], gv[1][3]);
  red_add_v4(grad_pos + (base + q.i2) * 4, gv[2][0], gv[2][1], gv[2][2], gv[2][3]);
}

bool bad_raster_args(const float* pos, const int32_t* tri, int64_t batch, int64_t num_vert,
                     int64_t num_tri, int32_t height, int32_t width, int64_t pos_batch) {
  if (batch < 0 || num_vert < 0 || num_tri < 0 || height <= 0 || width <= 0) return true;
  if (pos_batch != 1 && pos_batch != batch) return true;
  if (height >= (1 << 20) || width >= (1 << 20)) return true;
  if (num_tri >= (1LL << 31)) return true;
  if ((reinterpret_cast<uintptr_t>(pos) & 15u) != 0) return true;
  if (batch > 0 && num_tri > 0 && (pos == nullptr || tri == nullptr)) return true;
  return false;
}

// Vertices between the positions of consecutive views: 0 when all views share pos.
long long pos_stride(int64_t pos_batch, int64_t num_vert) { return pos_batch == 1 ? 0 : num_vert; }

}  // namespace
}  // namespace dr

using namespace dr;

extern "C" size_t dr_raster_setup_workspace_bytes(int64_t capacity, int32_t height,
                                                  int32_t width) {
  return setup_bytes(capacity < 0 ? 0 : capacity, height < 0 ? 0 : height, width < 0 ? 0 : width);
}

namespace dr {
namespace {

// Occlusion workspace: the record count, the tile maxima, the records (one per item at most).
struct OcclusionLayout {
  unsigned long long* count;
  long long* tile_max;
  int4* list;
};

OcclusionLayout occlusion_layout(void* ws, int64_t batch, int height, int width) {
  char* p = static_cast<char*>(ws);
  const long long tiles = batch * static_cast<long long>((height + kTile - 1) / kTile) *
                          ((width + kTile - 1) / kTile);
  OcclusionLayout l;
  l.count = reinterpret_cast<unsigned long long*>(p);
  l.tile_max = reinterpret_cast<long long*>(p + 256);
  l.list = reinterpret_cast<int4*>(p + 256 + align256(sizeof(long long) * static_cast<size_t>(tiles)));
  return l;
}

size_t occlusion_bytes(int64_t total, int64_t batch, int height, int width) {
  const long long tiles = batch * static_cast<long long>((height + kTile - 1) / kTile) *
                          ((width + kTile - 1) / kTile);
  return 256 + align256(sizeof(long long) * static_cast<size_t>(tiles)) +
         align256(sizeof(int4) * static_cast<size_t>(total));
}

Occlusion make_occlusion(const OcclusionLayout& l, int height, int width) {
  const int tiles_x = (width + kTile - 1) / kTile, tiles_y = (height + kTile - 1) / kTile;
  return Occlusion{l.count, l.list, l.tile_max, tiles_x, tiles_x * tiles_y};
}

}  // namespace
}  // namespace dr

extern "C" size_t dr_raster_occlusion_workspace_bytes(int64_t total, int64_t batch,
                                                      int32_t height, int32_t width) {
  if (total < 0 || batch < 0 || height <= 0 || width <= 0) return 0;
  return occlusion_bytes(total, batch, height, width);
}

extern "C" int dr_raster_setup(const float* pos, int64_t pos_batch, const int32_t* tri,
                               int64_t batch, int64_t num_vert, int64_t num_tri,
                               const int32_t* range_start, const int64_t* range_first,
                               int64_t range_total, int32_t height, int32_t width,
                               const int64_t* prev_keys, int64_t* keys, void* workspace,
                               size_t workspace_bytes, int64_t capacity,
                               void* occlusion_workspace, size_t occlusion_workspace_bytes,
                               void* stream) {
  const bool ranged = range_start != nullptr;
  if (bad_raster_args(pos, tri, batch, num_vert, num_tri, height, width, pos_batch) ||
      capacity < 0 || keys == nullptr || workspace == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  if (ranged && (range_first == nullptr || range_total < 0 || range_total >= (1LL << 31)))
    return DR_ERR_INVALID_ARGUMENT;
  if (!ranged && batch * num_tri >= (1LL << 31)) return DR_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < setup_bytes(capacity, height, width)) return DR_ERR_WORKSPACE_TOO_SMALL;
  const long long total = ranged ? range_total : batch * num_tri;
  if (occlusion_workspace != nullptr &&
      occlusion_workspace_bytes < occlusion_bytes(total, batch, height, width))
    return DR_ERR_WORKSPACE_TOO_SMALL;
  cudaStream_t s = as_stream(stream);
  SetupLayout l = setup_layout(workspace, height, width);
  const long long pixels = batch * static_cast<long long>(height) * width;
  cudaError_t err = cudaMemsetAsync(l.counters, 0, 2 * sizeof(unsigned long long), s);
  if (err != cudaSuccess) return static_cast<int>(err);
  if (pixels > 0) {
    fill_keys_kernel<<<min(blocks_for(pixels, 256), 148u * 32u), 256, 0, s>>>(
        reinterpret_cast<long long*>(keys), pixels);
  }
  centres_kernel<<<blocks_for(height + width, 256), 256, 0, s>>>(l.centres, height, width);
  const Items items = {static_cast<int>(num_tri), static_cast<int>(batch), range_start,
                       reinterpret_cast<const long long*>(range_first),
                       pos_stride(pos_batch, num_vert), num_vert};
  if (occlusion_workspace != nullptr) {
    const OcclusionLayout ol = occlusion_layout(occlusion_workspace, batch, height, width);
    err = cudaMemsetAsync(ol.count, 0, sizeof(unsigned long long), s);
    if (err != cudaSuccess) return static_cast<int>(err);
    if (total > 0 && batch > 0) {
      setup_kernel<1><<<blocks_for(total, 256), 256, 0, s>>>(
          pos, tri, items, total, height, width, l.centres,
          reinterpret_cast<const long long*>(prev_keys), reinterpret_cast<long long*>(keys),
          l.counters, l.binned, capacity, make_occlusion(ol, height, width));
    }
  } else if (total > 0 && batch > 0) {
    setup_kernel<0><<<blocks_for(total, 256), 256, 0, s>>>(
        pos, tri, items, total, height, width, l.centres,
        reinterpret_cast<const long long*>(prev_keys), reinterpret_cast<long long*>(keys),
        l.counters, l.binned, capacity, Occlusion{nullptr, nullptr, nullptr, 0, 0});
  }
  return launch_status();
}

extern "C" int dr_raster_occluded(const float* pos, int64_t pos_batch, const int32_t* tri,
                                  int64_t batch, int64_t num_vert, int64_t num_tri,
                                  const int32_t* range_start, const int64_t* range_first,
                                  int64_t range_total, int32_t height, int32_t width,
                                  const int64_t* prev_keys, int64_t* keys,
                                  const void* setup_workspace, void* occlusion_workspace,
                                  size_t occlusion_workspace_bytes, void* stream) {
  const bool ranged = range_start != nullptr;
  if (bad_raster_args(pos, tri, batch, num_vert, num_tri, height, width, pos_batch) ||
      keys == nullptr || setup_workspace == nullptr || occlusion_workspace == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  if (ranged && (range_first == nullptr || range_total < 0 || range_total >= (1LL << 31)))
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = ranged ? range_total : batch * num_tri;
  if (!ranged && total >= (1LL << 31)) return DR_ERR_INVALID_ARGUMENT;
  if (occlusion_workspace_bytes < occlusion_bytes(total, batch, height, width))
    return DR_ERR_WORKSPACE_TOO_SMALL;
  if (total == 0 || batch == 0) return DR_OK;
  if (batch > 65535 || height >= (1 << 20)) return DR_ERR_TOO_LARGE;
  cudaStream_t s = as_stream(stream);
  SetupLayout l = setup_layout(setup_workspace, height, width);
  const OcclusionLayout ol = occlusion_layout(occlusion_workspace, batch, height, width);
  const Occlusion oc = make_occlusion(ol, height, width);
  tile_max_kernel<<<dim3(oc.tiles_x, oc.tiles_per_view / oc.tiles_x, static_cast<unsigned>(batch)),
                    256, 0, s>>>(reinterpret_cast<const long long*>(keys), height, width,
                                 ol.tile_max);
  const Items items = {static_cast<int>(num_tri), static_cast<int>(batch), range_start,
                       reinterpret_cast<const long long*>(range_first),
                       pos_stride(pos_batch, num_vert), num_vert};
  // Nothing is binned here (every record is a small triangle), so the list is not touched.
  const unsigned grid = static_cast<unsigned>(
      min(static_cast<long long>(blocks_for(total, 256)),
          static_cast<long long>(resident_blocks(setup_kernel<2>, 256))));
  setup_kernel<2><<<grid, 256, 0, s>>>(pos, tri, items, total, height, width, l.centres,
                                       reinterpret_cast<const long long*>(prev_keys),
                                       reinterpret_cast<long long*>(keys), l.counters, l.binned, 0,
                                       oc);
  return launch_status();
}

extern "C" int dr_raster_counts(const void* setup_workspace, int64_t* num_binned,
                                int64_t* num_pairs, void* stream) {
  if (setup_workspace == nullptr || num_binned == nullptr || num_pairs == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  unsigned long long host[2] = {0, 0};
  cudaStream_t s = as_stream(stream);
  cudaError_t err = cudaMemcpyAsync(host, setup_workspace, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return static_cast<int>(err);
  *num_binned = static_cast<int64_t>(host[0]);
  *num_pairs = static_cast<int64_t>(host[1]);
  return DR_OK;
}

extern "C" size_t dr_raster_bin_workspace_bytes(int64_t batch, int32_t height, int32_t width,
                                                int64_t num_pairs) {
  const int64_t tiles_x = (width + kTile - 1) / kTile, tiles_y = (height + kTile - 1) / kTile;
  return bin_bytes(batch * tiles_x * tiles_y, num_pairs < 0 ? 0 : num_pairs);
}

namespace dr {
namespace {

// Stage 2 with either host counts (dc.count_on_device null: num_binned and num_pairs exact) or the
// setup counters read on the device (num_binned and num_pairs are then capacities).
int launch_tiles(const float* pos, int64_t pos_batch, const int32_t* tri, int64_t batch,
                 int64_t num_vert, int64_t num_tri, int32_t height, int32_t width,
                 const int64_t* prev_keys,
                 int64_t* keys, const void* setup_workspace, int64_t num_binned,
                 int64_t num_pairs, void* bin_workspace, size_t bin_workspace_bytes,
                 const DeviceCounts& dc, cudaStream_t s) {
  const int tiles_x = (width + kTile - 1) / kTile, tiles_y = (height + kTile - 1) / kTile;
  const int64_t tiles = batch * tiles_x * tiles_y;
  if (tiles >= (1LL << 31)) return DR_ERR_TOO_LARGE;
  if (bin_workspace == nullptr || bin_workspace_bytes < bin_bytes(tiles, num_pairs))
    return DR_ERR_WORKSPACE_TOO_SMALL;
  // Only the first num_binned records are read; the caller reran setup with enough capacity.
  SetupLayout sl = setup_layout(setup_workspace, height, width);
  BinLayout bl = bin_layout(bin_workspace, tiles, num_pairs);
  const size_t tile_bytes = align256(sizeof(unsigned) * static_cast<size_t>(tiles + 1));
  cudaError_t err = cudaMemsetAsync(bl.tile_count, 0, 2 * tile_bytes, s);  // counts and cursors
  if (err == cudaSuccess) err = cudaMemsetAsync(bl.work, 0, sizeof(unsigned), s);
  if (err != cudaSuccess) return static_cast<int>(err);
  const int tiles_per_image = tiles_x * tiles_y;
  const int nt = static_cast<int>(tiles);
  const unsigned bin_blocks = min(blocks_for(num_binned * 32, 256), 148u * 16u);
  bin_kernel<false><<<bin_blocks, 256, 0, s>>>(sl.binned, num_binned, tiles_x, tiles_per_image,
                                               bl.tile_count, nullptr, nullptr, dc, nt);
  const int chunks = static_cast<int>(scan_chunks(tiles));
  scan_totals_kernel<<<chunks, 1024, 0, s>>>(bl.tile_count, nt, bl.scan_totals);
  scan_chunks_kernel<<<1, 1024, 0, s>>>(bl.scan_totals, chunks);
  scan_kernel<<<chunks, 1024, 0, s>>>(bl.tile_count, nt, bl.scan_totals, chunks, bl.tile_offset,
                                      bl.item_offset);
  bin_kernel<true><<<bin_blocks, 256, 0, s>>>(sl.binned, num_binned, tiles_x, tiles_per_image,
                                              bl.tile_cursor, bl.tile_offset, bl.pairs, dc, nt);
  tile_kernel<<<148 * 8, 256, 0, s>>>(pos, tri, pos_stride(pos_batch, num_vert),
                                      Bounds{static_cast<int>(num_tri), num_vert}, height, width,
                                      tiles_x, tiles_per_image, nt, sl.centres,
                                      reinterpret_cast<const long long*>(prev_keys),
                                      reinterpret_cast<long long*>(keys), bl.pairs, sl.binned,
                                      bl.tile_offset, bl.item_offset, bl.work, dc);
  return launch_status();
}

}  // namespace
}  // namespace dr

extern "C" int dr_raster_tiles(const float* pos, int64_t pos_batch, const int32_t* tri,
                               int64_t batch, int64_t num_vert, int64_t num_tri, int32_t height,
                               int32_t width, const int64_t* prev_keys, int64_t* keys,
                               const void* setup_workspace, int64_t num_binned, int64_t num_pairs,
                               void* bin_workspace, size_t bin_workspace_bytes, void* stream) {
  if (bad_raster_args(pos, tri, batch, num_vert, num_tri, height, width, pos_batch) ||
      keys == nullptr || setup_workspace == nullptr || num_binned < 0 || num_pairs < 0)
    return DR_ERR_INVALID_ARGUMENT;
  if (num_pairs >= (1LL << 31)) return DR_ERR_TOO_LARGE;
  if (num_binned == 0 || num_pairs == 0) return DR_OK;
  return launch_tiles(pos, pos_batch, tri, batch, num_vert, num_tri, height, width, prev_keys, keys,
                      setup_workspace, num_binned, num_pairs, bin_workspace, bin_workspace_bytes,
                      DeviceCounts{nullptr, 0, 0, nullptr}, as_stream(stream));
}

extern "C" int dr_raster_tiles_device(const float* pos, int64_t pos_batch, const int32_t* tri,
                                      int64_t batch, int64_t num_vert, int64_t num_tri,
                                      int32_t height, int32_t width, const int64_t* prev_keys,
                                      int64_t* keys, const void* setup_workspace,
                                      int64_t binned_capacity, int64_t pair_capacity,
                                      void* bin_workspace, size_t bin_workspace_bytes,
                                      uint64_t* overflow, void* stream) {
  if (bad_raster_args(pos, tri, batch, num_vert, num_tri, height, width, pos_batch) ||
      keys == nullptr || setup_workspace == nullptr || overflow == nullptr ||
      binned_capacity < 0 || pair_capacity < 0)
    return DR_ERR_INVALID_ARGUMENT;
  if (pair_capacity >= (1LL << 31)) return DR_ERR_TOO_LARGE;
  if (batch == 0 || num_tri == 0) return DR_OK;
  SetupLayout sl = setup_layout(setup_workspace, height, width);
  const DeviceCounts dc{sl.counters, binned_capacity, pair_capacity,
                        reinterpret_cast<unsigned long long*>(overflow)};
  return launch_tiles(pos, pos_batch, tri, batch, num_vert, num_tri, height, width, prev_keys, keys,
                      setup_workspace, binned_capacity > 0 ? binned_capacity : 1, pair_capacity,
                      bin_workspace, bin_workspace_bytes, dc, as_stream(stream));
}

extern "C" int dr_raster_poison_keys(const uint64_t* overflow, int64_t* keys, int64_t count,
                                     void* stream) {
  if (overflow == nullptr || count < 0 || (count > 0 && keys == nullptr))
    return DR_ERR_INVALID_ARGUMENT;
  if (count == 0) return DR_OK;
  poison_keys_kernel<<<min(blocks_for(count, 256), 148u * 4u), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const unsigned long long*>(overflow), reinterpret_cast<long long*>(keys),
      count);
  return launch_status();
}

extern "C" int dr_raster_resolve_fwd(const float* pos, int64_t pos_batch, const int32_t* tri,
                                     const int64_t* keys, int64_t batch, int64_t num_vert,
                                     int64_t num_tri,
                                     int32_t height, int32_t width, float* rast, float* rast_db,
                                     void* stream) {
  if (bad_raster_args(pos, tri, batch, num_vert, num_tri, height, width, pos_batch) ||
      keys == nullptr || rast == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0) return DR_OK;
  for (long long b0 = 0; b0 < batch; b0 += 65535)
    for (int r0 = 0; r0 < height; r0 += 65535) {
      const dim3 grid((width + kResolveThreads * kResolvePix - 1) / (kResolveThreads * kResolvePix),
                      static_cast<unsigned>(min(height - r0, 65535)),
                      static_cast<unsigned>(min(batch - b0, 65535LL)));
      resolve_fwd_kernel<<<grid, kResolveThreads, 0, as_stream(stream)>>>(
          pos, tri, reinterpret_cast<const long long*>(keys), static_cast<int>(b0), r0,
          pos_stride(pos_batch, num_vert), Bounds{static_cast<int>(num_tri), num_vert}, height,
          width, reinterpret_cast<float4*>(rast), reinterpret_cast<float4*>(rast_db));
    }
  return launch_status();
}

extern "C" int dr_raster_resolve_bwd(const float* pos, int64_t pos_batch, const int32_t* tri,
                                     const int64_t* keys, int64_t batch, int64_t num_vert,
                                     int64_t num_tri,
                                     int32_t height, int32_t width, const float* grad_rast,
                                     const float* grad_db, float* grad_pos, void* stream) {
  if (bad_raster_args(pos, tri, batch, num_vert, num_tri, height, width, pos_batch) ||
      keys == nullptr || grad_rast == nullptr || grad_pos == nullptr)
    return DR_ERR_INVALID_ARGUMENT;
  const long long total = batch * static_cast<long long>(height) * width;
  if (total == 0) return DR_OK;
  for (long long b0 = 0; b0 < batch; b0 += 65535)
    for (int r0 = 0; r0 < height; r0 += 65535) {
      const dim3 grid((width + 255) / 256, static_cast<unsigned>(min(height - r0, 65535)),
                      static_cast<unsigned>(min(batch - b0, 65535LL)));
      resolve_bwd_kernel<<<grid, 256, 0, as_stream(stream)>>>(
          pos, tri, reinterpret_cast<const long long*>(keys), static_cast<int>(b0), r0,
          pos_stride(pos_batch, num_vert), Bounds{static_cast<int>(num_tri), num_vert}, height,
          width, reinterpret_cast<const float4*>(grad_rast),
          reinterpret_cast<const float4*>(grad_db), grad_pos);
    }
  return launch_status();
}
DR_DEFINE_FAULT_QUERY(raster)
