/* Plain C caller of the library, for tests/test_c_abi.py: the header must compile as C, and the
 * entry points must be callable through it without Python. Only calls that fail validation (and
 * so touch no GPU) are made. */
#include <stdio.h>
#include <string.h>

#include "diffrast_b200.h"

int main(void) {
  if (dr_version() < 1) return 1;
  if (strcmp(dr_status_string(DR_OK), "success") != 0) return 2;
  /* Negative sizes and missing pointers are refused before any CUDA call. */
  if (dr_raster_setup(NULL, 1, NULL, -1, 0, 0, NULL, NULL, 0, 4, 4, NULL, NULL, NULL, 0, 0, NULL,
                      0, NULL) != DR_ERR_INVALID_ARGUMENT)
    return 3;
  if (dr_to_clip_fwd(NULL, -1, NULL, 1, NULL, NULL) != DR_ERR_INVALID_ARGUMENT) return 4;
  if (dr_edge_neighbours_noalloc(NULL, dr_edge_neighbours_noalloc_max_triangles() + 1, NULL,
                                 NULL) != DR_ERR_EXCEEDS_STATIC_SCRATCH)
    return 5;
  if (dr_raster_setup_workspace_bytes(1000, 64, 64) < 20000) return 6;
  printf("c abi ok: %s\n", dr_status_string(DR_ERR_WORKSPACE_TOO_SMALL));
  return 0;
}
