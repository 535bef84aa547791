// Edge adjacency without any device allocation: dr_edge_neighbours_noalloc.
//
// Some callers cannot allocate device memory themselves: a program that binds this library
// through a plain C foreign-function interface with no device allocator of its own, or one that
// runs under a fixed device-memory budget where nothing may be allocated once it is running.
// They cannot provide the workspace that dr_edge_neighbours asks for. This variant builds the
// same hash table in a file-scope device array instead, so the caller passes only the index
// buffer and the output.
//
// Limits and sharing:
//   - At most kMaxTriangles (65536) triangles; larger inputs are refused with
//     DR_ERR_EXCEEDS_STATIC_SCRATCH before any GPU work.
//   - The array takes kScratchBytes (10 MiB) of device memory on a GPU from the moment this
//     file's device code is loaded there until the process exits. Under CUDA's lazy module loading
//     (the default) that is the first call of this entry point on that GPU; with
//     CUDA_MODULE_LOADING=EAGER it is every GPU the library is loaded on.
//   - Every call uses the same array and finds the previous call's contents in it; the part the
//     call uses is cleared first. Two calls whose work overlaps on the GPU (on different streams,
//     or from different threads) race on the array and give wrong results.
//   - In host code the array's name stands for a host-side shadow, not device memory, so each
//     call looks up the array's device address on the current device (cudaGetSymbolAddress) and
//     passes that to the kernels. Nothing is cached, so the address stays right after a
//     cudaDeviceReset or on another context. The first call on a GPU also loads the module there;
//     make that first call before any stream capture.
#include <cstdint>

#include "common.cuh"
#include "edge_hash.cuh"

namespace dr {
namespace {

constexpr long long kMaxTriangles = 65536;
// Hash slots for kMaxTriangles: the smallest power of two with room for twice the edges.
constexpr unsigned long long kMaxSlots = 524288;
static_assert(kMaxSlots >= 2ull * 3ull * kMaxTriangles, "table too small for the triangle limit");
// Keys (8 bytes), count, first and second edge (4 bytes each) per slot.
constexpr size_t kScratchBytes = 20 * kMaxSlots;

static __device__ __align__(256) unsigned char g_edge_scratch[kScratchBytes];

// Device address of g_edge_scratch on the current device, looked up on every call.
int scratch_address(void** out) {
  cudaError_t err = cudaGetSymbolAddress(out, g_edge_scratch);
  return err == cudaSuccess ? DR_OK : static_cast<int>(err);
}

}  // namespace
}  // namespace dr

using namespace dr;

extern "C" int64_t dr_edge_neighbours_noalloc_max_triangles(void) { return kMaxTriangles; }

extern "C" int dr_edge_neighbours_noalloc(const int32_t* tri, int64_t num_tri,
                                          int64_t* neighbours, void* stream) {
  if (num_tri < 0) return DR_ERR_INVALID_ARGUMENT;
  if (num_tri > kMaxTriangles) return DR_ERR_EXCEEDS_STATIC_SCRATCH;
  if (num_tri == 0) return DR_OK;
  if (tri == nullptr || neighbours == nullptr) return DR_ERR_INVALID_ARGUMENT;
  void* base = nullptr;
  int status = scratch_address(&base);
  if (status != DR_OK) return status;
  const unsigned long long slots = table_slots(num_tri);
  char* p = static_cast<char*>(base);
  auto* keys = reinterpret_cast<unsigned long long*>(p);
  int* count = reinterpret_cast<int*>(p + 8 * kMaxSlots);
  int* first = reinterpret_cast<int*>(p + 12 * kMaxSlots);
  int* second = reinterpret_cast<int*>(p + 16 * kMaxSlots);
  cudaStream_t s = as_stream(stream);
  // The array keeps the previous call's table: mark the slots in use as empty and their counts 0.
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
