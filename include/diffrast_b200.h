/*
 * diffrast_b200: C ABI of the B200 (sm_100a) kernels behind the diffrast render path
 * (rasterize -> interpolate -> texture -> antialias, forward and backward).
 *
 * Conventions
 *   - Every function returns an int status: 0 on success, a cudaError_t value (1..999) when a
 *     CUDA call or launch failed, or one of the DR_ERR_* codes below. dr_status_string() names it.
 *   - Tensor pointers are DEVICE pointers to contiguous row-major float32 / int32 / int64 data,
 *     16-byte aligned where a row has 4 floats (pos, rast, rast_db). Sizes are element counts.
 *   - Optional inputs are NULL when absent. Work is enqueued on `stream` (a cudaStream_t; NULL is
 *     the legacy default stream) and is asynchronous unless a function says otherwise.
 *   - The library allocates nothing: scratch memory is passed in as `workspace`, sized by the
 *     matching *_workspace_bytes() query.
 *   - Outputs are fully written (no need to clear them) unless a function says it accumulates.
 *
 * Citations name the reference project's files (paths under src/diffrast/ of sennecools/diffrast)
 * whose behaviour each entry point reproduces.
 */
#ifndef DIFFRAST_B200_H
#define DIFFRAST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DR_OK 0
#define DR_ERR_INVALID_ARGUMENT 10001
#define DR_ERR_WORKSPACE_TOO_SMALL 10002
#define DR_ERR_TOO_LARGE 10003
#define DR_ERR_EXCEEDS_STATIC_SCRATCH 10004

/* Filter modes (ops.py:22 FilterMode, without "auto", which the host resolves). */
#define DR_FILTER_NEAREST 0
#define DR_FILTER_LINEAR 1
#define DR_FILTER_LINEAR_MIPMAP_NEAREST 2
#define DR_FILTER_LINEAR_MIPMAP_LINEAR 3
/* Boundary modes (ops.py:23 BoundaryMode). */
#define DR_BOUNDARY_WRAP 0
#define DR_BOUNDARY_CLAMP 1
#define DR_BOUNDARY_ZERO 2
#define DR_BOUNDARY_CUBE 3
/* Most mip levels a lookup may use (a 2**31-texel-wide texture has 32). */
#define DR_MAX_LEVELS 32

int dr_version(void);
const char* dr_status_string(int status);

/* Bounds-checked build (libdiffrast_b200_checked.so, compiled with -DDR_CHECKED=1; no
 * counterpart in the reference, which has no debug build). Every index its kernels read from the
 * data (vertex indices in tri, triangle ids in rast and the visibility keys, opposite vertices,
 * attribute rows, texel offsets, key offsets) is checked against the buffer it addresses. A failed
 * check records (site << 48) | (index & 0xFFFFFFFFFFFF) in a device word (the first one wins)
 * and the access goes to element 0 instead, so no kernel faults. dr_checked_build() is 1 for that
 * library, 0 for the ordinary one; dr_check_faults() synchronizes the device, returns the first
 * record since the last call in *fault (0: none, always 0 in the ordinary build) and clears it;
 * dr_check_site_name() names a record's site (*fault >> 48). */
/* Zeroes `bytes` bytes of device memory at ptr on the stream (cudaMemsetAsync): the gradient
 * buffers that the backward scatters accumulate into. No counterpart in the reference. */
int dr_zero(void* ptr, size_t bytes, void* stream);

int dr_checked_build(void);
int dr_check_faults(uint64_t* fault);
const char* dr_check_site_name(int site);

/* ---------------------------------------------------------------------------------------------
 * Rasterize: visibility (three stages) and resolve.
 * Replaces the visibility pass of backends/triton.py:21-40 (rasterize_layer) and
 * backends/_triton_rasterize.py:295-307 (visible_keys); the result is the reference's
 * backends/reference.py:368-397 (_visible_triangles) exactly, as packed 64-bit keys
 * ((order-preserving depth bits << 32) | triangle, INT64_MAX where empty).
 *
 * pos [pos_batch, num_vert, 4] with pos_batch = batch, or 1 when all views share one position
 * buffer; tri [num_tri, 3], keys [batch, height, width], prev_keys: keys of the previous depth
 * layer (DepthPeeler, peeling.py:68-92) or NULL. height and width below 2**20.
 * Instanced mode (range_start NULL): every view draws every triangle; batch * num_tri below 2**31.
 * Range mode (ops.py:482-508, one pass for all items instead of one per item): view (item) b
 * draws tri[range_start[b] .. range_start[b] + count_b - 1], with range_first [batch + 1] the
 * exclusive prefix sums of the counts (range_first[batch] = range_total < 2**31); both are DEVICE
 * arrays, range_start int32 and range_first int64, checked by the caller (ranges inside tri).
 * Keys and rast ids hold indices into the whole tri, as range mode's ids are counted.
 * ------------------------------------------------------------------------------------------- */

/* Scratch of stage 1 for up to `capacity` triangles that need tile binning, at this resolution. */
size_t dr_raster_setup_workspace_bytes(int64_t capacity, int32_t height, int32_t width);

/* Stage 1: fills `keys` with EMPTY, culls, writes the keys of triangles whose pixel box holds at
 * most 512 pixels directly (keys not ordered after prev_keys are skipped), and lists the others
 * for binning. If more than
 * `capacity` triangles need binning the list is incomplete: dr_raster_counts() reports how many,
 * and the caller reruns this stage with a larger workspace (the direct writes are idempotent). */
int dr_raster_setup(const float* pos, int64_t pos_batch, const int32_t* tri, int64_t batch,
                    int64_t num_vert, int64_t num_tri, const int32_t* range_start,
                    const int64_t* range_first, int64_t range_total, int32_t height,
                    int32_t width, const int64_t* prev_keys, int64_t* keys, void* workspace,
                    size_t workspace_bytes, int64_t capacity, void* occlusion_workspace,
                    size_t occlusion_workspace_bytes, void* stream);

/* Scratch of the occlusion pass for `total` (view, triangle) items (batch * num_tri, or the
 * range total) at this resolution: about 16 bytes per item. */
size_t dr_raster_occlusion_workspace_bytes(int64_t total, int64_t batch, int32_t height,
                                           int32_t width);

/* Occlusion pass (no counterpart in the reference, which tests every triangle at every pixel of
 * its box). Given an occlusion workspace, dr_raster_setup sets aside the small triangles
 * whose projection has negative orientation (the far side of a closed mesh whose front faces are
 * counter-clockwise) instead of drawing them. After stage 2, dr_raster_occluded takes the largest
 * key of every 16 x 16 tile and draws the set-aside triangles, skipping each one whose depth,
 * bounded below from its vertices, lies above the largest key of every tile its pixel box
 * touches: such a triangle is behind what every one of its pixels already shows, so the keys are
 * exactly those of a single pass. Same arguments as dr_raster_setup otherwise. */
int dr_raster_occluded(const float* pos, int64_t pos_batch, const int32_t* tri, int64_t batch,
                       int64_t num_vert, int64_t num_tri, const int32_t* range_start,
                       const int64_t* range_first, int64_t range_total, int32_t height,
                       int32_t width, const int64_t* prev_keys, int64_t* keys,
                       const void* setup_workspace, void* occlusion_workspace,
                       size_t occlusion_workspace_bytes, void* stream);

/* Reads the two counters of stage 1: triangles to bin and (triangle, tile) pairs. Synchronises
 * `stream`. */
int dr_raster_counts(const void* setup_workspace, int64_t* num_binned, int64_t* num_pairs,
                     void* stream);

size_t dr_raster_bin_workspace_bytes(int64_t batch, int32_t height, int32_t width,
                                     int64_t num_pairs);

/* Stage 2: bins the listed triangles into 16x16 screen tiles and rasterizes each tile's list with
 * the list staged in shared memory, merging into `keys` with 64-bit atomic minima. */
int dr_raster_tiles(const float* pos, int64_t pos_batch, const int32_t* tri, int64_t batch,
                    int64_t num_vert, int64_t num_tri, int32_t height, int32_t width,
                    const int64_t* prev_keys,
                    int64_t* keys, const void* setup_workspace, int64_t num_binned,
                    int64_t num_pairs, void* bin_workspace, size_t bin_workspace_bytes,
                    void* stream);

/* Stage 2 without the host round trip of dr_raster_counts, so that a CUDA graph can capture the
 * rasterizer (no counterpart in the reference): the counts are read on the device from the setup
 * workspace. binned_capacity is the
 * capacity dr_raster_setup was given and pair_capacity the pair count bin_workspace is sized for
 * (dr_raster_bin_workspace_bytes). When a count exceeds its capacity nothing is binned, 1 is
 * OR-ed into the device word *overflow and the keys lack the binned triangles: the caller then
 * reruns with larger capacities. Launches the same kernels whether or not anything is binned. */
int dr_raster_tiles_device(const float* pos, int64_t pos_batch, const int32_t* tri, int64_t batch,
                           int64_t num_vert, int64_t num_tri, int32_t height, int32_t width,
                           const int64_t* prev_keys, int64_t* keys, const void* setup_workspace,
                           int64_t binned_capacity, int64_t pair_capacity, void* bin_workspace,
                           size_t bin_workspace_bytes, uint64_t* overflow, void* stream);

/* For CUDA-graph-captured rasterization (no counterpart in the reference): if the device word
 * *overflow is non-zero, marks every covered key of `keys` [count] as poisoned (its triangle index
 * kept, its depth replaced by a value no covered pixel has), so that dr_raster_resolve_fwd writes
 * NaN barycentrics, depth and derivatives there and everything computed from them is NaN. Called
 * after dr_raster_tiles_device (and dr_raster_occluded) with the same word; *overflow stays set
 * until the host clears it, so every captured pass replayed until then is poisoned. A no-op
 * (one read per block) while the word is zero. */
int dr_raster_poison_keys(const uint64_t* overflow, int64_t* keys, int64_t count, void* stream);

/* rast [batch, h, w, 4] = (u, v, z/w, id + 1) and rast_db [.., 4] = (du/dx, du/dy, dv/dx, dv/dy),
 * zeros where empty (reference.py:69-114; _triton_resolve.py:84-116). rast_db may be NULL.
 * A poisoned key (dr_raster_poison_keys) gives (NaN, NaN, NaN, id + 1) and a NaN rast_db. */
int dr_raster_resolve_fwd(const float* pos, int64_t pos_batch, const int32_t* tri,
                          const int64_t* keys, int64_t batch, int64_t num_vert, int64_t num_tri,
                          int32_t height, int32_t width, float* rast, float* rast_db,
                          void* stream);

/* Gradient of rast (and rast_db unless grad_db is NULL) with respect to pos, ACCUMULATED into
 * grad_pos [pos_batch, num_vert, 4] (clear it first) (_triton_resolve.py:156-284). */
int dr_raster_resolve_bwd(const float* pos, int64_t pos_batch, const int32_t* tri,
                          const int64_t* keys, int64_t batch, int64_t num_vert, int64_t num_tri,
                          int32_t height, int32_t width, const float* grad_rast,
                          const float* grad_db, float* grad_pos, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Interpolate (reference.py:117-146; _triton_interpolate.py:38-254).
 * attr [attr_batch, num_vert, channels] with attr_batch 1 (shared) or batch, its vertex rows
 * attr_stride floats apart (0 = channels; a multiple of 4 with a 16-byte aligned attr lets the
 * kernels read rows of up to 8 channels with 16-byte loads, so callers may pad rows); rast,
 * rast_db [batch, h, w, 4]; diff: DEVICE int32 [num_diff] channel indices in [0, channels) (NULL
 * when num_diff is 0); out [batch, h, w, channels]; out_da [batch, h, w, 2 * num_diff].
 * dr_interpolate_bwd reads attr and writes grad_attr with rows of `channels` floats. Ids past
 * num_tri are empty.
 * ------------------------------------------------------------------------------------------- */
int dr_interpolate_fwd(const float* attr, int64_t attr_batch, int64_t num_vert, int32_t channels,
                       int32_t attr_stride, const float* rast, const float* rast_db,
                       const int32_t* tri,
                       int64_t num_tri, const int32_t* diff, int32_t num_diff, int64_t batch,
                       int32_t height, int32_t width, float* out, float* out_da, void* stream);

/* grad_attr (NULL to skip) is ACCUMULATED (clear it first); grad_rast is written; grad_db is
 * written when grad_out_da is given and ignored otherwise (may be NULL). */
int dr_interpolate_bwd(const float* attr, int64_t attr_batch, int64_t num_vert, int32_t channels,
                       const float* rast, const float* rast_db, const int32_t* tri,
                       int64_t num_tri, const int32_t* diff, int32_t num_diff, int64_t batch,
                       int32_t height, int32_t width, const float* grad_out,
                       const float* grad_out_da, float* grad_attr, float* grad_rast,
                       float* grad_db, void* stream);

/* dr_interpolate_bwd with the output gradients given in pieces (no counterpart in the
 * reference, whose consumers hand back whole gradient images): grad_out [batch, h, w, channels]
 * and grad_out_da [batch, h, w, 2 num_diff] may each be NULL, and compact channel ranges may be
 * added: part [batch, h, w, part_count] holds the gradient of out channels part_first ..
 * part_first + part_count - 1, part_da [batch, h, w, da_count] that of out_da channels da_first ..
 * (either NULL to omit). Whatever is not given counts as zero. A lookup that read uv and uv_da
 * as channel slices of out and out_da hands its compact coordinate gradients over this way, so
 * no zero-padded gradient records are written or read. grad_db is written when grad_out_da or
 * part_da is given. */
int dr_interpolate_bwd_parts(const float* attr, int64_t attr_batch, int64_t num_vert,
                             int32_t channels, const float* rast, const float* rast_db,
                             const int32_t* tri, int64_t num_tri, const int32_t* diff,
                             int32_t num_diff, int64_t batch, int32_t height, int32_t width,
                             const float* grad_out, const float* grad_out_da, const float* part,
                             int32_t part_first, int32_t part_count, const float* part_da,
                             int32_t da_first, int32_t da_count, float* grad_attr,
                             float* grad_rast, float* grad_db, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Texture (reference.py:149-194, :491-672; _cube.py:44-143; _triton_texture.py:37-549).
 * Level l has `level_ptr[l]` -> [tex_batch(, 6), level_h[l], level_w[l], channels]; its batch
 * stride in elements is `level_batch_stride[l]` (0 when that level is shared by all views).
 * These four arrays are HOST arrays of `num_levels` entries (level 0 is the base texture).
 * For DR_BOUNDARY_CUBE, uv holds directions [batch, h, w, 3] and uv_da [batch, h, w, 6].
 * uv_stride / uv_da_stride: floats between consecutive pixels of uv / uv_da (0 for packed), so
 * channel slices of a wider tensor are read in place. uv_da and bias may be NULL.
 * out [batch, h, w, channels]; grad_uv and grad_uv_da are packed.
 * ------------------------------------------------------------------------------------------- */
int dr_texture_fwd(const float* const* level_ptr, const int32_t* level_h, const int32_t* level_w,
                   const int64_t* level_batch_stride, int32_t num_levels, int32_t channels,
                   const float* uv, int64_t uv_stride, const float* uv_da, int64_t uv_da_stride,
                   const float* bias, int64_t batch,
                   int32_t height, int32_t width, int32_t filter_mode, int32_t boundary_mode,
                   float* out, void* stream);

/* Texel gradients are ACCUMULATED into grad_level_ptr[l] (clear them first), laid out like the
 * levels but with grad_channel_stride (>= channels) floats per texel; with 4 (and channels <= 4,
 * 16-byte aligned buffers) each texel's gradient is added with one vector reduction. grad_uv,
 * grad_uv_da and grad_bias (each NULL to skip) are written. grad_uv and grad_uv_da have their own
 * pixel strides (0 = contiguous). With grad_uv_first = -1 the pointer addresses the gradient
 * itself and nothing else is written; with grad_uv_first = c >= 0 it addresses pixel records of
 * grad_uv_stride floats (such as the gradient of dr_interpolate_fwd's output, whose channels
 * c, c + 1 are uv): the gradient goes to channels c.. and every other float of each record is
 * set to zero, so that the caller need not clear them. Likewise grad_uv_da_first. */
int dr_texture_bwd(const float* const* level_ptr, float* const* grad_level_ptr,
                   const int32_t* level_h, const int32_t* level_w,
                   const int64_t* level_batch_stride, int32_t num_levels, int32_t channels,
                   int32_t grad_channel_stride, const float* uv, int64_t uv_stride,
                   const float* uv_da, int64_t uv_da_stride, const float* bias, int64_t batch,
                   int32_t height, int32_t width, int32_t filter_mode, int32_t boundary_mode,
                   const float* grad_out, float* grad_uv, int64_t grad_uv_stride,
                   int32_t grad_uv_first, float* grad_uv_da, int64_t grad_uv_da_stride,
                   int32_t grad_uv_da_first, float* grad_bias, void* stream);

/* dr_texture_bwd with the interpolation's backward pass for the lookup's coordinates fused in
 * (no counterpart in the reference, whose texture and interpolate backward passes run apart,
 * backends/_triton_texture.py and _triton_interpolate.py). uv and uv_da must be what
 * dr_interpolate_fwd made of rast, rast_db, tri and attr [attr_batch, num_vert, attr_channels]:
 * uv = attribute channels (cu, cv), uv_da = the derivative pairs of channels (du, dv). In place of
 * grad_uv and grad_uv_da, their gradients are chained through that interpolation and written as
 * grad_rast [batch, height, width, 4] (b0, b1, then zeros for z and the id) and grad_db
 * [batch, height, width, 4] (NULL when uv_da gets no gradient; then uv_da may still be given for
 * the level of detail) -- what dr_interpolate_bwd would write for the same coordinate gradients
 * and no attribute gradient. 2D textures only (not boundary mode 3), filter modes 1-3; rast,
 * grad_rast and grad_db 16-byte aligned. */
int dr_texture_bwd_interp(const float* const* level_ptr, float* const* grad_level_ptr,
                          const int32_t* level_h, const int32_t* level_w,
                          const int64_t* level_batch_stride, int32_t num_levels, int32_t channels,
                          int32_t grad_channel_stride, const float* uv, int64_t uv_stride,
                          const float* uv_da, int64_t uv_da_stride, const float* bias,
                          int64_t batch, int32_t height, int32_t width, int32_t filter_mode,
                          int32_t boundary_mode, const float* grad_out, float* grad_bias,
                          const float* rast, const int32_t* tri, int64_t num_tri,
                          const float* attr, int64_t attr_batch, int64_t num_vert,
                          int32_t attr_channels, int32_t cu, int32_t cv, int32_t du, int32_t dv,
                          float* grad_rast, float* grad_db, void* stream);

/* One mip step (reference.py:449-488): dst [images, (h + 1) / 2, (w + 1) / 2, channels] from
 * src [images, h, w, channels] by area weights; `images` = tex_batch, or 6 * tex_batch for a cube. */
int dr_mip_downsample(const float* src, int64_t images, int32_t h, int32_t w, int32_t channels,
                      float* dst, void* stream);

/* Adjoint of dr_mip_downsample: ACCUMULATES the gradient of dst into grad_src; or, with out
 * non-NULL, writes grad_src + that adjoint to out [images, h, w, out_channels] (the first
 * out_channels <= channels channels, dropping the padding of 4-channel gradients) and leaves
 * grad_src unchanged. */
int dr_mip_downsample_bwd(const float* grad_dst, int64_t images, int32_t h, int32_t w,
                          int32_t channels, float* grad_src, float* out, int32_t out_channels,
                          void* stream);

/* dr_texture_bwd_interp with the rasterizer's backward pass fused in as well (no counterpart in
 * the reference). rast, tri and pos must be what dr_raster_setup / dr_raster_resolve_fwd made
 * keys and rast from (pos [pos_batch, pos_num_vert, 4], pos_batch 1 or batch; at most 2^24
 * triangles), and attr's rows are those of the same vertex indices. In place of grad_rast and
 * grad_db, the gradients of the pixel's triangle's clip-space vertices are ACCUMULATED into
 * grad_pos (like pos) with vector reductions -- what dr_raster_resolve_bwd would
 * add for the rast / rast_db gradients dr_texture_bwd_interp would write (rast_db's only when
 * rast_db_gradient is nonzero, which needs filter mode 3 and uv_da). The pixel's triangle is read
 * from keys. pos and grad_pos 16-byte aligned. */
int dr_texture_bwd_resolve(const float* const* level_ptr, float* const* grad_level_ptr,
                           const int32_t* level_h, const int32_t* level_w,
                           const int64_t* level_batch_stride, int32_t num_levels,
                           int32_t channels, int32_t grad_channel_stride, const float* uv,
                           int64_t uv_stride, const float* uv_da, int64_t uv_da_stride,
                           const float* bias, int64_t batch, int32_t height, int32_t width,
                           int32_t filter_mode, int32_t boundary_mode, const float* grad_out,
                           float* grad_bias, const float* rast, const int32_t* tri,
                           int64_t num_tri, const float* attr, int64_t attr_batch,
                           int64_t num_vert, int32_t attr_channels, int32_t cu, int32_t cv,
                           int32_t du, int32_t dv, const int64_t* keys, const float* pos,
                           int64_t pos_batch, int64_t pos_num_vert, int32_t rast_db_gradient,
                           float* grad_pos, void* stream);

/* The chained position part of dr_texture_bwd_resolve on its own (no counterpart in the
 * reference): from a lookup's compact coordinate gradients grad_uv [batch, height, width, 2] and
 * grad_uv_da [batch, height, width, 4] (as dr_texture_bwd writes them with grad_uv_first = -1),
 * the interpolation's and the rasterizer's backward passes, ACCUMULATED into grad_pos like
 * dr_texture_bwd_resolve does (arguments as there). Lets a caller complete the texture gradient
 * first (dr_texture_bwd without the chain) and run this while that gradient is being reduced
 * across GPUs. One thread per pixel in short blocks; batch and height at most 65535. */
int dr_texture_chain_bwd(const float* grad_uv, const float* grad_uv_da, int64_t batch,
                         int32_t height, int32_t width, const int32_t* tri, int64_t num_tri,
                         const float* attr, int64_t attr_batch, int64_t num_vert,
                         int32_t attr_channels, int32_t cu, int32_t cv, int32_t du, int32_t dv,
                         const int64_t* keys, const float* pos, int64_t pos_batch,
                         int64_t pos_num_vert, int32_t rast_db_gradient, float* grad_pos,
                         void* stream);

/* The whole mip chain at once (reference.py:433-488; texture_construct_mip, ops.py:239-265):
 * levels 1 .. levels of src [images, h, w, channels] into dst[0 .. levels - 1], each
 * [images, h_l, w_l, channels] with h_l = (h_{l-1} + 1) / 2 (and w_l likewise), values equal to
 * repeated dr_mip_downsample. Runs of even halvings with at most 4 channels take one launch per
 * up to 6 levels. levels <= DR_MAX_LEVELS - 1. No counterpart in the reference's interface, which
 * builds the chain step by step. */
int dr_mip_build(const float* src, int64_t images, int32_t h, int32_t w, int32_t channels,
                 int32_t levels, float* const* dst, void* stream);

/* The adjoint of dr_mip_build: pushes the gradients of levels 1 .. levels (grad_levels[1 ..],
 * `channels` floats per texel, e.g. 4-channel padded) down into the base gradient grad_levels[0],
 * as repeated dr_mip_downsample_bwd from the coarsest level would (same values); with out non-NULL
 * the base result goes to out [images, h, w, out_channels] instead (levels >= 1 then) and
 * grad_levels[0] is left unchanged. The contents of grad_levels[1 ..] afterwards are unspecified
 * (they hold the partial sums). */
int dr_mip_build_bwd(float* const* grad_levels, int64_t images, int32_t h, int32_t w,
                     int32_t channels, int32_t levels, float* out, int32_t out_channels,
                     void* stream);

/* ---------------------------------------------------------------------------------------------
 * Antialias (reference.py:202-265, :675-814; topology.py; _triton_antialias.py).
 * neighbours [num_tri, 3] int64 from dr_edge_neighbours (reference.py:768-787); opposite
 * [num_tri, 3] int32 from dr_edge_opposite_vertices.
 * pos [pos_batch, num_vert, 4] with pos_batch 1 (shared across views) or batch.
 * ------------------------------------------------------------------------------------------- */
size_t dr_edge_neighbours_workspace_bytes(int64_t num_tri);

/* For edge 3 t + k (opposite vertex k) the other edge over the same vertex pair, or -1 when
 * none or several share it. Deterministic; needs no sort. */
int dr_edge_neighbours(const int32_t* tri, int64_t num_tri, int64_t* neighbours, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Same result as dr_edge_neighbours for callers that cannot allocate device memory (a plain FFI
 * binding without a device allocator, or a fixed device-memory budget): the hash table lives in a
 * 10 MiB file-scope device array instead of a caller workspace. No counterpart in the reference.
 * At most dr_edge_neighbours_noalloc_max_triangles() (65536) triangles; more is refused with
 * DR_ERR_EXCEEDS_STATIC_SCRATCH. The array is taken on a GPU when the library's module for it
 * loads there (with CUDA's default lazy loading, at this entry point's first call on that GPU;
 * with CUDA_MODULE_LOADING=EAGER, on every GPU the library loads on) and kept until process
 * exit. All calls share the array (each clears the part it uses), so calls that overlap on the
 * GPU race. Each call looks up the array's device address on the current device, so nothing
 * goes stale after a cudaDeviceReset; the first call on a device also loads the module there,
 * so make it before any stream capture. Allocates nothing. */
int64_t dr_edge_neighbours_noalloc_max_triangles(void);
int dr_edge_neighbours_noalloc(const int32_t* tri, int64_t num_tri, int64_t* neighbours,
                               void* stream);

/* opposite [num_tri, 3] int32: for edge 3 t + k the vertex opposite it in the adjacent triangle,
 * tri[neighbours[3 t + k]], or -1 where neighbours is -1 (no single adjacent triangle: a
 * silhouette by topology). Built once per index buffer; the antialias entry points take it in
 * place of neighbours, so that their silhouette test needs one dependent load
 * (reference.py:790-814 reads tri[neighbours] there). No counterpart in the reference. */
int dr_edge_opposite_vertices(const int32_t* tri, const int64_t* neighbours, int64_t num_tri,
                              int32_t* opposite, void* stream);

/* Silhouette flags [pos_batch, num_tri, 3] as bytes (reference.py:790-814). The antialias
 * kernels evaluate the same test on the fly for the edges they cross. */
int dr_silhouette_edges(const float* pos, int64_t pos_batch, int64_t num_vert,
                        const int32_t* tri, int64_t num_tri, const int32_t* opposite,
                        uint8_t* silhouette, void* stream);

/* Bytes of the pair records that dr_antialias_fwd can leave for dr_antialias_bwd (about 25 bytes
 * per pixel): per pixel, the crossing t, the outcome and the crossed edge of its right and lower
 * pixel pairs. */
size_t dr_antialias_pair_bytes(int64_t batch, int32_t height, int32_t width);

/* Forward pass (_triton_antialias.py:272-304). pairs may be NULL; otherwise the records of
 * dr_antialias_pair_bytes() bytes (pair_bytes at least that) are written. */
int dr_antialias_fwd(const float* color, const float* rast, const float* pos, int64_t pos_batch,
                     int64_t num_vert, const int32_t* tri, int64_t num_tri,
                     const int32_t* opposite, int64_t batch, int32_t height, int32_t width,
                     int32_t channels, float* out, void* pairs, size_t pair_bytes, void* stream);

/* Backward pass (_triton_antialias.py:306-320). grad_color is written; grad_pos
 * [pos_batch, num_vert, 4] is ACCUMULATED (clear it first). With pairs from a dr_antialias_fwd
 * call on the same color, rast, pos, tri and opposite, the edge tests are not repeated; with
 * pairs NULL they are. Both give the same result. */
int dr_antialias_bwd(const float* color, const float* rast, const float* pos, int64_t pos_batch,
                     int64_t num_vert, const int32_t* tri, int64_t num_tri,
                     const int32_t* opposite, int64_t batch, int32_t height, int32_t width,
                     int32_t channels, const float* grad_out, float pos_gradient_boost,
                     const void* pairs, size_t pair_bytes, float* grad_color, float* grad_pos,
                     void* stream);

/* ---- Antialias with a fused squared-error loss (no counterpart in the reference) -------------
 * The loss a fit puts right after antialias (the examples of diffrast take an MSE of the
 * antialiased image), computed inside the antialias passes: no separate loss kernels; the forward
 * pass leaves the residual out - target, from which the backward pass forms the output's
 * gradient on the fly. */

/* Number of floats of per-block partial sums of (out - target)^2 that dr_antialias_mse_fwd
 * writes; the loss is their sum times the caller's scale. */
size_t dr_antialias_loss_partials(int64_t batch, int32_t height, int32_t width);

/* dr_antialias_fwd (pairs required) that also writes residual = out - target and the partial
 * sums of residual^2; target and residual are [batch, height, width, channels]. */
int dr_antialias_mse_fwd(const float* color, const float* rast, const float* pos,
                         int64_t pos_batch, int64_t num_vert, const int32_t* tri, int64_t num_tri,
                         const int32_t* opposite, int64_t batch, int32_t height, int32_t width,
                         int32_t channels, const float* target, float* out, float* residual,
                         void* pairs, size_t pair_bytes, float* partial_sums, size_t partial_count,
                         void* stream);

/* Backward pass of loss = scale * sum (out - target)^2 (plus grad_out, the gradient of out, when
 * not NULL): the output's gradient is grad_out + 2 scale dL residual, dL the device scalar
 * *loss_grad, with residual and pairs from the dr_antialias_mse_fwd call. grad_color is written;
 * grad_pos is ACCUMULATED (clear it first). */
int dr_antialias_mse_bwd(const float* color, const float* rast, const float* pos,
                         int64_t pos_batch, int64_t num_vert, const int32_t* tri, int64_t num_tri,
                         const int32_t* opposite, int64_t batch, int32_t height, int32_t width,
                         int32_t channels, const float* residual, const float* loss_grad,
                         float scale, const float* grad_out, float pos_gradient_boost,
                         const void* pairs, size_t pair_bytes, float* grad_color, float* grad_pos,
                         void* stream);

/* ---- World-to-clip transform (the step ahead of the rasterizer in a multi-view fit) -------- */

/* clip [batch, num_vert, 4] = matrices [batch, 4, 4] (row-major) applied to the homogeneous
 * positions (p, 1), p [num_vert, 3]: diffrast examples/common.py:320-323 (to_clip), which the
 * reference computes with a torch matmul. clip must be 16-byte aligned. */
int dr_to_clip_fwd(const float* positions, int64_t num_vert, const float* matrices, int64_t batch,
                   float* clip, void* stream);

/* Gradients of dr_to_clip_fwd from grad_clip [batch, num_vert, 4] (16-byte aligned):
 * grad_positions [num_vert, 3] (written; sums over the views) and grad_matrices [batch, 4, 4]
 * (written). Either may be NULL. */
int dr_to_clip_bwd(const float* grad_clip, const float* positions, int64_t num_vert,
                   const float* matrices, int64_t batch, float* grad_positions,
                   float* grad_matrices, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Lambert shading from interpolated normals (the optional shading of a fused fit step; no
 * counterpart in the reference, whose examples shade with torch elementwise ops).
 * color [batch, h, w, channels]; normal: 3 floats per pixel, normal_stride floats apart (>= 3, so
 * a channel slice of interpolate's output is read in place); light [light_batch, 3] with
 * light_batch 1 or batch (normalised here). out = color * (ambient + max(0, n . l)) with n, l the
 * unit normal and light; a zero normal shades with the ambient term alone. The backward pass
 * writes grad_color [batch, h, w, channels] and grad_normal [batch, h, w, 3] (either may be NULL);
 * the light gets no gradient. batch at most 65535.
 * ------------------------------------------------------------------------------------------- */
int dr_lambert_fwd(const float* color, const float* normal, int64_t normal_stride,
                   const float* light, int64_t light_batch, float ambient, int64_t batch,
                   int32_t height, int32_t width, int32_t channels, float* out, void* stream);
int dr_lambert_bwd(const float* color, const float* normal, int64_t normal_stride,
                   const float* light, int64_t light_batch, float ambient, int64_t batch,
                   int32_t height, int32_t width, int32_t channels, const float* grad_out,
                   float* grad_color, float* grad_normal, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DIFFRAST_B200_H */
