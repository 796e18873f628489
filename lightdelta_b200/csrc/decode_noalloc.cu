// Packed-mode decode that allocates nothing: the scratch slots of the packed state path live in
// one static device array of this library instead of memory the caller allocates.
//
// Packed mode (the reference backend's python/lightdelta/backend.py:30-91, GDNBackend here) copies
// each request's source state out of the pool into a scratch buffer, runs the decode on the
// scratch, and commits every live step state back to its pool slot.  GDNBackend gets that scratch
// from the framework allocator.  Some callers cannot allocate device memory while they decode:
//   - a host that binds the C ABI from a runtime with no device allocator of its own (a Go, Java
//     or C serving loop that only ever receives pool and activation pointers);
//   - a serving engine that reserves the whole GPU for its state pools at start-up and forbids
//     later allocations;
//   - a latency-bound loop where cudaMalloc's implicit device-wide synchronisation would stall the
//     other streams of the process.
// ld_decode_packed_noalloc gives them the packed path with a fixed-size scratch region that every
// GPU which loads this library holds until the process exits.
//
// Scratch layout (g_packed_scratch, LD_NOALLOC_SCRATCH_BYTES):
//   [0, kMetaBytes)       per-call request plan, rewritten by plan_kernel on every call:
//                         source slot, valid flag, compact scratch indices, the all-ones accepted
//                         vector of the scratch decode and the commit destinations;
//   [kMetaBytes, end)     fp32 state slots [1 + n_requests * width, HV, 128, 128]; slot 0 is the
//                         scratch's null slot and is never read or written.
// Every call overwrites what it reads before reading it (the plan, then the gathered source
// states, then the decoded step states), so nothing has to start at zero, and two calls whose
// work overlaps on the GPU (other streams, other host threads) race on the same array.
//
// The four launches are the plan kernel below and the library's own gather, decode and scatter
// kernels, in stream order on the caller's stream.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "internal.h"
#include "launch.cuh"
#include "lightdelta_b200.h"

namespace ldb {
namespace {

constexpr int64_t kScratchBytes = LD_NOALLOC_SCRATCH_BYTES;
constexpr int64_t kMetaBytes = 32 * 1024;       // request plan in front of the state slots
constexpr int64_t kMaxPlanRows = 1024;          // entries per plan vector (>= n_requests * width)
constexpr int kPlanThreads = 128;
constexpr int kMaxDevices = 64;

// Plan vectors inside the metadata region (byte offsets), each kMaxPlanRows entries long.
constexpr int64_t kSourceOffset = 0;                                  // int32 source slot per request
constexpr int64_t kOnesOffset = kSourceOffset + 4 * kMaxPlanRows;     // int32 accepted = 1 per request
constexpr int64_t kCompactOffset = kOnesOffset + 4 * kMaxPlanRows;    // int32 scratch slot per (request, step)
constexpr int64_t kDestOffset = kCompactOffset + 4 * kMaxPlanRows;    // int32 commit slot per (request, step)
constexpr int64_t kValidOffset = kDestOffset + 4 * kMaxPlanRows;      // uint8 valid flag per request
static_assert(kValidOffset + kMaxPlanRows <= kMetaBytes, "the request plan must fit its region");
static_assert(kMetaBytes % 256 == 0, "state slots must start 256-byte aligned");

static __device__ __align__(256) unsigned char g_packed_scratch[kScratchBytes];

// The request plan of backend.py:38-49 and :87-89, one thread per request:
//   source = slots[r, clamp(accepted, 1, W) - 1];  valid = 1 <= accepted <= W and source > 0;
//   compact[r, t] = 1 + r * W + t when valid, else 0 (the scratch decode then writes nothing);
//   dest[r, t] = slots[r, t] for live steps (t < tokens of r) of valid requests with slot > 0.
__global__ void __launch_bounds__(kPlanThreads) packed_plan_kernel(const int32_t* slots, const int32_t* cu,
                                                                   const int32_t* accepted, int requests, int width,
                                                                   unsigned char* meta) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  const int r = blockIdx.x * kPlanThreads + threadIdx.x;
  if (r >= requests) return;
  int32_t* source = reinterpret_cast<int32_t*>(meta + kSourceOffset);
  int32_t* ones = reinterpret_cast<int32_t*>(meta + kOnesOffset);
  int32_t* compact = reinterpret_cast<int32_t*>(meta + kCompactOffset);
  int32_t* dest = reinterpret_cast<int32_t*>(meta + kDestOffset);
  uint8_t* valid = meta + kValidOffset;
  const int acc = accepted[r];
  const int pick = (acc < 1 ? 1 : (acc > width ? width : acc)) - 1;
  const int32_t src = slots[r * width + pick];
  const bool ok = acc >= 1 && acc <= width && src > 0;
  const int tokens = cu[r + 1] - cu[r];
  source[r] = src;
  valid[r] = ok ? 1 : 0;
  ones[r] = 1;
  for (int t = 0; t < width; ++t) {
    const int32_t slot = slots[r * width + t];
    compact[r * width + t] = ok ? 1 + r * width + t : 0;
    dest[r * width + t] = (ok && t < tokens && slot > 0) ? slot : 0;
  }
}

// Device address of g_packed_scratch on the current device.  The first call on each device looks
// it up (cudaGetSymbolAddress, with that device current) and keeps it for later calls.
int scratch_address(unsigned char** out) {
  static std::mutex mutex;
  static unsigned char* addresses[kMaxDevices] = {};
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (device < 0 || device >= kMaxDevices) return set_error(LD_ERR_INVALID, "device index %d unsupported", device);
  std::lock_guard<std::mutex> lock(mutex);
  if (addresses[device] == nullptr) {
    void* address = nullptr;
    err = cudaGetSymbolAddress(&address, g_packed_scratch);
    if (err != cudaSuccess || address == nullptr) {
      return set_error(LD_ERR_CUDA, "looking up the static packed-mode scratch: %s", cudaGetErrorString(err));
    }
    addresses[device] = static_cast<unsigned char*>(address);
  }
  *out = addresses[device];
  return LD_OK;
}

}  // namespace
}  // namespace ldb

extern "C" int ld_decode_packed_noalloc(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride,
                                        const void* b, int64_t b_row_stride, const float* a_log, const void* dt_bias,
                                        int dt_bias_dtype, const int32_t* indices, int64_t n_requests, int64_t width,
                                        const int32_t* cu, const int32_t* accepted, float* state, int64_t n_slots,
                                        int64_t slot_stride, const void* gate, int64_t gate_row_stride,
                                        const void* weight, int weight_dtype, void* out, int64_t n_tokens,
                                        int64_t num_k_heads, int64_t num_v_heads, float eps, void* stream) {
  using namespace ldb;
  int rc = check_decode_args(qkv, qkv_row_stride, a, a_row_stride, b, b_row_stride, a_log, dt_bias, dt_bias_dtype,
                             indices, n_requests, width, cu, accepted, state, n_slots, slot_stride, gate,
                             gate_row_stride, weight, weight_dtype, out, n_tokens, num_k_heads, num_v_heads, eps);
  if (rc != LD_OK || n_requests == 0) return rc;
  const int64_t slot_elems = num_v_heads * LD_HEAD_DIM * LD_HEAD_DIM;
  const int64_t scratch_slots = 1 + n_requests * width;
  const int64_t needed = scratch_slots * slot_elems * static_cast<int64_t>(sizeof(float));
  if (n_requests * width > kMaxPlanRows || needed > kScratchBytes - kMetaBytes) {
    return set_error(LD_ERR_INVALID,
                     "ld_decode_packed_noalloc: %lld requests x width %lld need %lld scratch slots of %lld bytes "
                     "(%lld bytes); the static scratch holds %lld bytes of state slots",
                     static_cast<long long>(n_requests), static_cast<long long>(width),
                     static_cast<long long>(scratch_slots), static_cast<long long>(slot_elems * 4),
                     static_cast<long long>(needed), static_cast<long long>(kScratchBytes - kMetaBytes));
  }
  unsigned char* base = nullptr;
  rc = scratch_address(&base);
  if (rc != LD_OK) return rc;
  unsigned char* meta = base;
  float* slots_base = reinterpret_cast<float*>(base + kMetaBytes);
  const int32_t* source = reinterpret_cast<const int32_t*>(meta + kSourceOffset);
  const int32_t* ones = reinterpret_cast<const int32_t*>(meta + kOnesOffset);
  const int32_t* compact = reinterpret_cast<const int32_t*>(meta + kCompactOffset);
  const int32_t* dest = reinterpret_cast<const int32_t*>(meta + kDestOffset);
  const uint8_t* valid = meta + kValidOffset;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const int requests = static_cast<int>(n_requests);
  const dim3 grid(static_cast<unsigned int>((requests + kPlanThreads - 1) / kPlanThreads));
  cudaError_t err = ldb::launch(packed_plan_kernel, grid, dim3(kPlanThreads), 0, s, 1, indices, cu, accepted,
                                requests, static_cast<int>(width), meta);
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "packed plan launch failed: %s", cudaGetErrorString(err));
  // Source states -> scratch rows 1 + r * width (zeros for invalid requests), backend.py:40-44.
  rc = ld_gather_state(state, n_slots, slot_stride, source, 1, valid, n_requests, slots_base + slot_elems,
                       width * slot_elems, slot_elems, stream);
  if (rc != LD_OK) return rc;
  // Decode on the scratch with accepted = 1, backend.py:80-85.
  rc = ld_decode(qkv, qkv_row_stride, a, a_row_stride, b, b_row_stride, a_log, dt_bias, dt_bias_dtype, compact,
                 n_requests, width, cu, ones, slots_base, scratch_slots, slot_elems, gate, gate_row_stride, weight,
                 weight_dtype, out, n_tokens, num_k_heads, num_v_heads, eps, stream);
  if (rc != LD_OK) return rc;
  // Commit the live step states to their pool slots, backend.py:87-91.
  return ld_scatter_state(slots_base + slot_elems, slot_elems, dest, 1, n_requests * width, state, n_slots,
                          slot_stride, slot_elems, stream);
}
