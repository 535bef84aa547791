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
