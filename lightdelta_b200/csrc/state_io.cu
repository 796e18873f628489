// Slot-indexed state-pool copies for sm_100a: gather, scatter and pool-to-pool commit.
//
// Contract: lightdelta::gather_state / scatter_state of the reference
// (csrc/state_io.cu:11-27 kernel, :44-69 launchers); copy_slots is the one-pass form of
// the packed-mode commit (python/lightdelta/backend.py:87-91) for states already in the pool.
//
// Design (B200): a pure HBM copy.  Each CTA moves one 32 KiB chunk of one slot row; every
// thread issues all eight of its 128-bit loads before its stores so that a resident set of
// CTAs keeps well over the ~40 KB per SM needed to cover HBM latency in flight.  A row whose
// slot is null (gather: or not valid) writes zeros without reading.  When a pointer, stride
// or the slot size is not a multiple of four floats, a scalar variant with the same chunking
// runs instead.
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "launch.cuh"
#include "lightdelta_b200.h"

namespace ldb {
namespace {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 8;
constexpr int64_t kChunkItems = static_cast<int64_t>(kCopyThreads) * kCopyUnroll;  // per CTA

enum CopyKind { kGather = 0, kScatter = 1, kPoolCopy = 2 };

__device__ unsigned int g_state_io_faults;

struct CopyArgs {
  const float* src;       // gather: pool; scatter: packed; pool copy: pool
  int64_t src_stride;     // floats between consecutive slots / rows of src
  float* dst;             // gather: packed; scatter: pool; pool copy: pool
  int64_t dst_stride;
  const int32_t* slots;   // gather / scatter slot vector; pool copy: source slots
  int64_t slots_stride;
  const int32_t* slots2;  // pool copy: destination slots
  int64_t slots2_stride;
  const uint8_t* valid;   // gather only
  int64_t n_pool_slots;
  int64_t slot_elems;     // floats per slot
  int64_t chunks_per_row;
};

template <int kKind, bool kVec>
__global__ void __launch_bounds__(kCopyThreads) slot_copy_kernel(const CopyArgs p) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  const int64_t row = blockIdx.x / p.chunks_per_row;
  const int64_t chunk = blockIdx.x - row * p.chunks_per_row;
  const bool report = chunk == 0 && threadIdx.x == 0;

  const float* src = nullptr;
  float* dst = nullptr;
  bool live = true;
  if constexpr (kKind == kGather) {
    const int slot = p.slots[row * p.slots_stride];
    if (slot >= p.n_pool_slots) {
      if (report) atomicOr(&g_state_io_faults, LD_FAULT_GATHER_SLOT_RANGE);
      live = false;
    } else {
      live = slot > 0 && p.valid[row] != 0;
    }
    src = p.src + (live ? static_cast<int64_t>(slot) * p.src_stride : 0);
    dst = p.dst + row * p.dst_stride;
  } else if constexpr (kKind == kScatter) {
    const int slot = p.slots[row * p.slots_stride];
    if (slot <= 0) return;  // null slot: skipped, slot 0 never written (state_io.cu:19)
    if (slot >= p.n_pool_slots) {
      if (report) atomicOr(&g_state_io_faults, LD_FAULT_SCATTER_SLOT_RANGE);
      return;
    }
    src = p.src + row * p.src_stride;
    dst = p.dst + static_cast<int64_t>(slot) * p.dst_stride;
  } else {
    const int from = p.slots[row * p.slots_stride];
    const int to = p.slots2[row * p.slots2_stride];
    if (from <= 0 || to <= 0 || from == to) return;
    if (from >= p.n_pool_slots || to >= p.n_pool_slots) {
      if (report) atomicOr(&g_state_io_faults, LD_FAULT_COPY_SLOT_RANGE);
      return;
    }
    src = p.src + static_cast<int64_t>(from) * p.src_stride;
    dst = p.dst + static_cast<int64_t>(to) * p.dst_stride;
  }

  if constexpr (kVec) {
    const int64_t count = p.slot_elems / 4;
    const int64_t base = chunk * kChunkItems + threadIdx.x;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    float4 v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t idx = base + u * kCopyThreads;
      v[u] = (live && idx < count) ? s4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t idx = base + u * kCopyThreads;
      if (idx < count) d4[idx] = v[u];
    }
  } else {
    const int64_t count = p.slot_elems;
    const int64_t base = chunk * kChunkItems + threadIdx.x;
    float v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t idx = base + u * kCopyThreads;
      v[u] = (live && idx < count) ? src[idx] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t idx = base + u * kCopyThreads;
      if (idx < count) dst[idx] = v[u];
    }
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

template <int kKind>
int launch_copy(CopyArgs& args, int64_t n, bool vec, void* stream, const char* name) {
  const int64_t items = vec ? args.slot_elems / 4 : args.slot_elems;
  args.chunks_per_row = (items + kChunkItems - 1) / kChunkItems;
  if (n * args.chunks_per_row > 0x7fffffffLL) {
    return set_error(LD_ERR_INVALID, "%s: %lld rows of %lld floats exceed the grid limit", name,
                     static_cast<long long>(n), static_cast<long long>(args.slot_elems));
  }
  const dim3 grid(static_cast<unsigned int>(n * args.chunks_per_row));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t err = vec ? ldb::launch(slot_copy_kernel<kKind, true>, grid, dim3(kCopyThreads), 0, s, 1, args)
                              : ldb::launch(slot_copy_kernel<kKind, false>, grid, dim3(kCopyThreads), 0, s, 1, args);
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "%s launch failed: %s", name, cudaGetErrorString(err));
  return ok();
}

int check_common(const char* name, int64_t n_pool_slots, int64_t pool_slot_stride, int64_t slot_elems,
                 int64_t n) {
  if (n < 0) return set_error(LD_ERR_INVALID, "%s: negative row count", name);
  if (slot_elems <= 0) return set_error(LD_ERR_INVALID, "%s: slot_elems must be positive", name);
  if (n_pool_slots < 1) return set_error(LD_ERR_INVALID, "%s: the pool must hold at least one slot", name);
  if (n_pool_slots > 1 && pool_slot_stride < slot_elems) {
    return set_error(LD_ERR_INVALID, "%s: pool slot stride is smaller than a slot", name);
  }
  return LD_OK;
}

}  // namespace

int state_io_faults(uint32_t* flags, int clear) {
  unsigned int value = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&value, g_state_io_faults, sizeof(value));
  if (err != cudaSuccess) {
    return set_error(LD_ERR_CUDA, "reading state_io fault word: %s", cudaGetErrorString(err));
  }
  if (clear) {
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(g_state_io_faults, &zero, sizeof(zero));
    if (err != cudaSuccess) {
      return set_error(LD_ERR_CUDA, "clearing state_io fault word: %s", cudaGetErrorString(err));
    }
  }
  *flags = value;
  return LD_OK;
}

}  // namespace ldb

extern "C" int ld_gather_state(const float* pool, int64_t n_pool_slots, int64_t pool_slot_stride,
                               const int32_t* slots, int64_t slots_stride, const uint8_t* valid, int64_t n,
                               float* out, int64_t out_row_stride, int64_t slot_elems, void* stream) {
  using namespace ldb;
  int rc = check_common("gather_state", n_pool_slots, pool_slot_stride, slot_elems, n);
  if (rc != LD_OK) return rc;
  if (n == 0) return ok();
  if (pool == nullptr || slots == nullptr || valid == nullptr || out == nullptr) {
    return set_error(LD_ERR_INVALID, "gather_state: a required pointer is NULL");
  }
  if (n > 1 && out_row_stride < slot_elems) {
    return set_error(LD_ERR_INVALID, "gather_state: packed row stride is smaller than a slot");
  }
  CopyArgs args{};
  args.src = pool;
  args.src_stride = pool_slot_stride;
  args.dst = out;
  args.dst_stride = out_row_stride;
  args.slots = slots;
  args.slots_stride = slots_stride;
  args.valid = valid;
  args.n_pool_slots = n_pool_slots;
  args.slot_elems = slot_elems;
  const bool vec = aligned16(pool) && aligned16(out) && pool_slot_stride % 4 == 0 &&
                   out_row_stride % 4 == 0 && slot_elems % 4 == 0;
  return launch_copy<kGather>(args, n, vec, stream, "gather_state");
}

extern "C" int ld_scatter_state(const float* packed, int64_t packed_row_stride, const int32_t* slots,
                                int64_t slots_stride, int64_t n, float* pool, int64_t n_pool_slots,
                                int64_t pool_slot_stride, int64_t slot_elems, void* stream) {
  using namespace ldb;
  int rc = check_common("scatter_state", n_pool_slots, pool_slot_stride, slot_elems, n);
  if (rc != LD_OK) return rc;
  if (n == 0) return ok();
  if (packed == nullptr || slots == nullptr || pool == nullptr) {
    return set_error(LD_ERR_INVALID, "scatter_state: a required pointer is NULL");
  }
  if (n > 1 && packed_row_stride < slot_elems) {
    return set_error(LD_ERR_INVALID, "scatter_state: packed row stride is smaller than a slot");
  }
  CopyArgs args{};
  args.src = packed;
  args.src_stride = packed_row_stride;
  args.dst = pool;
  args.dst_stride = pool_slot_stride;
  args.slots = slots;
  args.slots_stride = slots_stride;
  args.n_pool_slots = n_pool_slots;
  args.slot_elems = slot_elems;
  const bool vec = aligned16(pool) && aligned16(packed) && pool_slot_stride % 4 == 0 &&
                   packed_row_stride % 4 == 0 && slot_elems % 4 == 0;
  return launch_copy<kScatter>(args, n, vec, stream, "scatter_state");
}

extern "C" int ld_copy_slots(float* pool, int64_t n_pool_slots, int64_t pool_slot_stride, const int32_t* src,
                             int64_t src_stride, const int32_t* dst, int64_t dst_stride, int64_t n,
                             int64_t slot_elems, void* stream) {
  using namespace ldb;
  int rc = check_common("copy_slots", n_pool_slots, pool_slot_stride, slot_elems, n);
  if (rc != LD_OK) return rc;
  if (n == 0) return ok();
  if (pool == nullptr || src == nullptr || dst == nullptr) {
    return set_error(LD_ERR_INVALID, "copy_slots: a required pointer is NULL");
  }
  CopyArgs args{};
  args.src = pool;
  args.src_stride = pool_slot_stride;
  args.dst = pool;
  args.dst_stride = pool_slot_stride;
  args.slots = src;
  args.slots_stride = src_stride;
  args.slots2 = dst;
  args.slots2_stride = dst_stride;
  args.n_pool_slots = n_pool_slots;
  args.slot_elems = slot_elems;
  const bool vec = aligned16(pool) && pool_slot_stride % 4 == 0 && slot_elems % 4 == 0;
  return launch_copy<kPoolCopy>(args, n, vec, stream, "copy_slots");
}
