// Library identification and status strings of the C ABI.
#include <cuda_runtime.h>

#include "common.cuh"

extern "C" int dr_version(void) { return 1; }

extern "C" const char* dr_status_string(int status) {
  switch (status) {
    case DR_OK:
      return "success";
    case DR_ERR_INVALID_ARGUMENT:
      return "invalid argument (shape, size, alignment or a missing pointer)";
    case DR_ERR_WORKSPACE_TOO_SMALL:
      return "workspace too small; query the *_workspace_bytes() function";
    case DR_ERR_TOO_LARGE:
      return "problem too large for 32-bit work lists; split the batch";
    case DR_ERR_EXCEEDS_STATIC_SCRATCH:
      return "input exceeds the fixed device array of the allocation-free entry point "
             "(dr_edge_neighbours_noalloc takes at most 65536 triangles)";
    default:
      return cudaGetErrorString(static_cast<cudaError_t>(status));
  }
}

// Fault words of the checked build, one per translation unit (defined there with
// DR_DEFINE_FAULT_QUERY).
extern "C" int dr_fault_raster(uint64_t* fault);
extern "C" int dr_fault_interpolate(uint64_t* fault);
extern "C" int dr_fault_texture(uint64_t* fault);
extern "C" int dr_fault_antialias(uint64_t* fault);
extern "C" int dr_fault_transform(uint64_t* fault);
extern "C" int dr_fault_shading(uint64_t* fault);

extern "C" int dr_checked_build(void) { return DR_CHECKED; }

extern "C" int dr_check_faults(uint64_t* fault) {
  if (fault == nullptr) return DR_ERR_INVALID_ARGUMENT;
  *fault = 0;
  if (!DR_CHECKED) return DR_OK;
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return static_cast<int>(err);
  int (*const units[])(uint64_t*) = {dr_fault_raster, dr_fault_interpolate, dr_fault_texture,
                                     dr_fault_antialias, dr_fault_transform,
                                     dr_fault_shading};
  for (auto query : units) {
    uint64_t value = 0;
    const int status = query(&value);
    if (status != DR_OK) return status;
    if (*fault == 0) *fault = value;
  }
  return DR_OK;
}

extern "C" const char* dr_check_site_name(int site) {
  switch (site) {
    case dr::kSiteTriangle:
      return "triangle index into tri";
    case dr::kSiteVertex:
      return "vertex index read from tri";
    case dr::kSiteOpposite:
      return "vertex index read from the opposite-vertex table";
    case dr::kSiteTexel:
      return "texel offset into a texture level";
    case dr::kSitePixel:
      return "pixel offset into the visibility keys";
    case dr::kSiteAttrRow:
      return "attribute row";
    default:
      return "unknown site";
  }
}

extern "C" int dr_zero(void* ptr, size_t bytes, void* stream) {
  if (bytes == 0) return DR_OK;
  if (ptr == nullptr) return DR_ERR_INVALID_ARGUMENT;
  return static_cast<int>(cudaMemsetAsync(ptr, 0, bytes, reinterpret_cast<cudaStream_t>(stream)));
}
