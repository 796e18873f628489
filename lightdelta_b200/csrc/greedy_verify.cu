// Greedy MTP verification on the device: per-row argmax of the target logits fused with the
// prefix check against the draft tokens.
//
// Semantics follow LightDeltaRejectionSampler.__call__
// (python/lightdelta/runtime/speculation.py:274-326): target = logits.argmax(-1) (first index
// of the maximum, NaN counted as the maximum, as torch does); per request the drafts
// input_ids[query_start_loc[r+1]-d, query_start_loc[r+1]) are accepted while they equal the
// target at logits rows cu_num_logits[r] + i; the first mismatch (or the end of the request's
// logits) stops, and the target at min(begin + accepted, end - 1) is the bonus token.  The
// reference runs this as a host loop with a device round trip per comparison; here one launch
// does it all.
//
// Work decomposition: one thread-block cluster of Q CTAs (Q = 1, 2, 4, 8; 16 on request) per
// request.  Every CTA scans a 1/Q slice of the vocabulary of the request's logits rows, two
// rows at a time, with 128-bit streaming loads (eight in flight per thread).  A NaN-propagating
// maximum of each vector decides whether its elements need an in-order scan, so the common
// case costs about one instruction per element.  (value, index) pairs reduce through warp
// shuffles and shared memory, and every CTA writes its per-row result into rank 0's shared
// memory (distributed shared memory).  Rank 0 combines the slices and its thread 0 runs the
// prefix check, whose request metadata was loaded when the kernel started, and writes the
// request's outputs.  Only the rows a request can consult are read: rows
// [begin, min(begin + d, end - 1)].  No scratch memory, no atomics on the data path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>

#include "internal.h"
#include "launch.cuh"
#include "lightdelta_b200.h"

namespace {

__device__ uint32_t g_verify_faults;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 8;
constexpr int kMaxRows = LD_MAX_VERIFY_STEPS + 1;
constexpr int kMaxCluster = 16;
__device__ __forceinline__ float negative_infinity() { return __int_as_float(0xff800000); }

struct VerifyArgs {
  const void* logits;
  int64_t n_logits;
  int64_t vocab;
  int64_t row_stride;  // elements between consecutive logits rows
  const int32_t* cu_num_logits;
  const int32_t* query_start_loc;
  const void* input_ids;
  int64_t n_input_ids;
  int tokens_i64;
  const int32_t* num_draft_tokens;
  const int32_t* seq_lens;
  const int32_t* prefill_len;
  int64_t n_requests;
  int steps;
  void* sampled;
  int32_t* num_sampled;
  int32_t* num_rejected;
  int64_t chunk;  // vocabulary elements per cluster rank (multiple of 8)
  int vector_ok;  // rows start 16-byte aligned
};

// (value, index) order of torch.argmax: NaN beats every number, larger beats smaller, and on
// equal values (or two NaNs) the smaller index wins.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  const bool vn = v != v;
  const bool bn = bv != bv;
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void consider(float v, int i, float& bv, int& bi) {
  if (better(v, i, bv, bi)) {
    bv = v;
    bi = i;
  }
}

__device__ __forceinline__ void warp_best(float& bv, int& bi) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, offset);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, offset);
    consider(ov, oi, bv, bi);
  }
}

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_float<__half>(__half v) {
  return __half2float(v);
}

// Running best of one thread, which visits its elements in increasing index order: a strictly
// larger value or the first NaN replaces the best, a NaN is never replaced, and bi < 0 means
// nothing seen yet.  Equal values therefore keep the first index, as torch.argmax does.
__device__ __forceinline__ void scan(float x, int idx, float& bv, int& bi) {
  if (bi < 0 || (!(x <= bv) && bv == bv)) {
    bv = x;
    bi = idx;
  }
}

// Maxima that return NaN when either input is NaN (PTX max.NaN, sm_80 and later).
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ uint32_t max_nan_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t max_nan_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Largest element of a 16-byte vector, NaN if any element is NaN.
template <typename T>
__device__ __forceinline__ float vector_max(const uint4& raw);
template <>
__device__ __forceinline__ float vector_max<float>(const uint4& raw) {
  return max_nan(max_nan(__uint_as_float(raw.x), __uint_as_float(raw.y)),
                 max_nan(__uint_as_float(raw.z), __uint_as_float(raw.w)));
}
template <>
__device__ __forceinline__ float vector_max<__nv_bfloat16>(const uint4& raw) {
  const uint32_t m = max_nan_bf16x2(max_nan_bf16x2(raw.x, raw.y), max_nan_bf16x2(raw.z, raw.w));
  return max_nan(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u));
}
template <>
__device__ __forceinline__ float vector_max<__half>(const uint4& raw) {
  const uint32_t m = max_nan_f16x2(max_nan_f16x2(raw.x, raw.y), max_nan_f16x2(raw.z, raw.w));
  return max_nan(__half2float(__ushort_as_half(static_cast<unsigned short>(m & 0xffffu))),
                 __half2float(__ushort_as_half(static_cast<unsigned short>(m >> 16))));
}

// Folds one 16-byte vector into the running best.  The vector's maximum decides in a few
// instructions whether any element can replace the best; only then are its elements scanned
// in index order.
template <typename T>
__device__ __forceinline__ void scan_vector(const uint4& raw, int first, float& bv, int& bi) {
  const float m = vector_max<T>(raw);
  if (bi >= 0 && (m <= bv || bv != bv)) return;
  constexpr int kElems = 16 / sizeof(T);
  T values[kElems];
  static_assert(sizeof(values) == sizeof(uint4), "vector size");
  memcpy(values, &raw, sizeof(raw));
#pragma unroll
  for (int e = 0; e < kElems; ++e) scan(to_float(values[e]), first + e, bv, bi);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned int cluster_rank() {
  unsigned int r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ unsigned int cluster_size() {
  unsigned int n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Stores a (value, index) pair at the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ void peer_store(float* local_value, int* local_index, unsigned int rank, float v, int i) {
  uint32_t rv, ri;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rv) : "r"(smem_u32(local_value)), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ri) : "r"(smem_u32(local_index)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(rv), "f"(v) : "memory");
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(ri), "r"(i) : "memory");
}

// Rows of the logits a request consults, mirroring the index arithmetic of
// speculation.py:292-314.  `ok` is false when the reference would raise (more drafts than
// steps) or index outside the logits; such requests produce -1 / 0 / 0.
struct RowPlan {
  int64_t begin, end, lo;
  int n;
  int drafts;
  bool ok;
  uint32_t fault;
};

__device__ __forceinline__ RowPlan plan_rows(const VerifyArgs& p, int64_t r) {
  RowPlan plan{};
  plan.begin = p.cu_num_logits[r];
  plan.end = p.cu_num_logits[r + 1];
  plan.drafts = p.num_draft_tokens[r];
  plan.ok = true;
  if (plan.drafts > p.steps) {  // speculation.py:305-306 raises
    plan.ok = false;
    plan.fault = LD_FAULT_VERIFY_DRAFTS;
    return plan;
  }
  int64_t lo, hi;
  if (plan.drafts == 0) {  // speculation.py:295-296: target[begin]
    lo = hi = plan.begin;
  } else if (plan.end > plan.begin) {
    lo = plan.begin;
    hi = min(plan.begin + static_cast<int64_t>(max(plan.drafts, 0)), plan.end - 1);
  } else {  // no logits: nothing is accepted and the bonus is target[end - 1]
    lo = hi = plan.end - 1;
  }
  if (lo < 0 || hi >= p.n_logits) {
    plan.ok = false;
    plan.fault = LD_FAULT_VERIFY_RANGE;
    return plan;
  }
  plan.lo = lo;
  plan.n = static_cast<int>(hi - lo + 1);
  return plan;
}

__device__ __forceinline__ int64_t load_token(const VerifyArgs& p, int64_t i) {
  return p.tokens_i64 ? static_cast<const int64_t*>(p.input_ids)[i]
                      : static_cast<int64_t>(static_cast<const int32_t*>(p.input_ids)[i]);
}

__device__ __forceinline__ void store_sampled(const VerifyArgs& p, int64_t r, int col, int64_t token) {
  const int64_t at = r * (p.steps + 1) + col;
  if (p.tokens_i64) {
    static_cast<int64_t*>(p.sampled)[at] = token;
  } else {
    static_cast<int32_t*>(p.sampled)[at] = static_cast<int32_t>(token);
  }
}

// Request metadata that rank 0 loads when the kernel starts, so that the prefix check at the
// end reads shared memory only.
struct Prefetch {
  long long draft[kMaxRows];  // draft tokens; valid where draft_ok[i] != 0
  int draft_ok[kMaxRows];     // draft i lies inside input_ids
  int prefill;                // seq_lens[r] < prefill_len[r]
};

__device__ __forceinline__ void prefetch_request(const VerifyArgs& p, int64_t r, const RowPlan& plan, Prefetch& pre) {
  if (threadIdx.x == 0) pre.prefill = p.seq_lens[r] < p.prefill_len[r];
  const int i = static_cast<int>(threadIdx.x) - 32;  // warp 1 loads the drafts
  if (i >= 0 && i < plan.drafts) {
    const int64_t at = static_cast<int64_t>(p.query_start_loc[r + 1]) - plan.drafts + i;
    const bool inside = at >= 0 && at < p.n_input_ids;
    pre.draft_ok[i] = inside;
    pre.draft[i] = inside ? load_token(p, at) : 0;
  }
}

// The host loop of speculation.py:292-325 for one request, given the targets of its rows.
__device__ void verify_request(const VerifyArgs& p, int64_t r, const RowPlan& plan, const int* target,
                               const Prefetch& pre) {
  for (int c = 0; c <= p.steps; ++c) store_sampled(p, r, c, -1);
  uint32_t fault = plan.fault;
  int sampled_count = 0, rejected = 0;
  if (plan.ok) {
    const bool prefill = pre.prefill != 0;
    if (plan.drafts == 0) {
      store_sampled(p, r, 0, target[0]);
      sampled_count = prefill ? 0 : 1;
    } else {
      int accepted = 0;
      bool ok = true;
      while (accepted < plan.drafts) {
        if (plan.begin + accepted >= plan.end) break;
        if (!pre.draft_ok[accepted]) {
          ok = false;
          break;
        }
        const int64_t draft = pre.draft[accepted];
        if (static_cast<int64_t>(target[plan.begin + accepted - plan.lo]) != draft) break;
        store_sampled(p, r, accepted, draft);
        ++accepted;
      }
      if (!ok) {
        fault |= LD_FAULT_VERIFY_RANGE;
        for (int c = 0; c <= p.steps; ++c) store_sampled(p, r, c, -1);
      } else {
        const int64_t bonus = min(plan.begin + accepted, plan.end - 1);
        store_sampled(p, r, accepted, target[bonus - plan.lo]);
        if (!prefill) {
          sampled_count = accepted + 1;
          rejected = static_cast<int>(plan.end - plan.begin) - (accepted + 1);
        }
      }
    }
  }
  p.num_sampled[r] = sampled_count;
  p.num_rejected[r] = rejected;
  if (fault) atomicOr(&g_verify_faults, fault);
}

// One thread's share of a pair of rows (the second may be absent): the slice's whole vectors,
// kUnroll / 2 loads per row per batch so that both rows' loads are in flight together, then the
// ragged end by scalar loads.  Per row the thread visits its elements in index order.
template <typename T>
__device__ __forceinline__ void scan_row_pair(const T* row0, const T* row1, bool two, int slice_begin,
                                              int slice_end, int vector_end, bool vector_ok, float (&bv)[2],
                                              int (&bi)[2]) {
  constexpr int kElems = 16 / sizeof(T);
  constexpr int kPerRow = kUnroll / 2;
  int scalar_from = slice_begin;
  if (vector_ok) {
    // Slices start on multiples of 8 elements, so every vector lies inside one slice.
    const int v_end = min(slice_end, vector_end) / kElems;
    const uint4* vec0 = reinterpret_cast<const uint4*>(row0);
    const uint4* vec1 = reinterpret_cast<const uint4*>(row1);
    for (int base = slice_begin / kElems + static_cast<int>(threadIdx.x); base < v_end;
         base += kThreads * kPerRow) {
      uint4 buf0[kPerRow], buf1[kPerRow];
#pragma unroll
      for (int u = 0; u < kPerRow; ++u) {
        const int v = base + u * kThreads;
        if (v < v_end) {
          buf0[u] = __ldcs(vec0 + v);
          if (two) buf1[u] = __ldcs(vec1 + v);
        }
      }
#pragma unroll
      for (int u = 0; u < kPerRow; ++u) {
        const int v = base + u * kThreads;
        if (v < v_end) {
          scan_vector<T>(buf0[u], v * kElems, bv[0], bi[0]);
          if (two) scan_vector<T>(buf1[u], v * kElems, bv[1], bi[1]);
        }
      }
    }
    scalar_from = max(slice_begin, vector_end);
  }
  for (int base = scalar_from + static_cast<int>(threadIdx.x); base < slice_end; base += kThreads * kPerRow) {
    T buf0[kPerRow], buf1[kPerRow];
#pragma unroll
    for (int u = 0; u < kPerRow; ++u) {
      const int i = base + u * kThreads;
      if (i < slice_end) {
        buf0[u] = row0[i];
        if (two) buf1[u] = row1[i];
      }
    }
#pragma unroll
    for (int u = 0; u < kPerRow; ++u) {
      const int i = base + u * kThreads;
      if (i < slice_end) {
        scan(to_float(buf0[u]), i, bv[0], bi[0]);
        if (two) scan(to_float(buf1[u]), i, bv[1], bi[1]);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) greedy_verify_kernel(const VerifyArgs p) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  __shared__ float warp_value[kMaxRows][kWarps];
  __shared__ int warp_index[kMaxRows][kWarps];
  __shared__ float slice_value[kMaxCluster][kMaxRows];  // rank 0: one entry per cluster rank
  __shared__ int slice_index[kMaxCluster][kMaxRows];
  __shared__ int target[kMaxRows];
  __shared__ Prefetch pre;

  const unsigned int ranks = cluster_size();
  const unsigned int rank = ranks > 1 ? cluster_rank() : 0u;
  if (ranks > 1) cluster_arrive_relaxed();  // first phase: every CTA of the cluster has started

  const int64_t r = blockIdx.x / ranks;
  const RowPlan plan = plan_rows(p, r);
  const int rows = plan.ok ? plan.n : 0;
  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  if (rank == 0 && plan.ok) prefetch_request(p, r, plan, pre);

  // Element offsets within a row fit in 32 bits (vocab <= 2^31 - 1).
  const int slice_begin = static_cast<int>(min(static_cast<int64_t>(rank) * p.chunk, p.vocab));
  const int slice_end = static_cast<int>(min(p.vocab, static_cast<int64_t>(slice_begin) + p.chunk));
  constexpr int kElems = 16 / sizeof(T);
  const int vector_end = p.vector_ok ? static_cast<int>(p.vocab / kElems) * kElems : 0;
  const T* first_row = static_cast<const T*>(p.logits) + plan.lo * p.row_stride;

  for (int j = 0; j < rows; j += 2) {
    const bool two = j + 1 < rows;
    const T* row0 = first_row + j * p.row_stride;
    float bv[2] = {negative_infinity(), negative_infinity()};
    int bi[2] = {-1, -1};
    scan_row_pair<T>(row0, two ? row0 + p.row_stride : row0, two, slice_begin, slice_end, vector_end,
                     p.vector_ok != 0, bv, bi);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !two) break;
      if (bi[k] < 0) {  // nothing in this thread's share: lose every comparison
        bv[k] = negative_infinity();
        bi[k] = INT32_MAX;
      }
      warp_best(bv[k], bi[k]);
      if (lane == 0) {
        warp_value[j + k][warp] = bv[k];
        warp_index[j + k][warp] = bi[k];
      }
    }
  }
  __syncthreads();
  // One thread per row folds the warps' results into this CTA's slice result.
  float own_value = negative_infinity();
  int own_index = INT32_MAX;
  if (tid < rows) {
    for (int w = 0; w < kWarps; ++w) consider(warp_value[tid][w], warp_index[tid][w], own_value, own_index);
  }

  if (ranks > 1) {
    cluster_wait();  // rank 0's shared memory is live from here on
    if (tid < rows) peer_store(&slice_value[rank][tid], &slice_index[rank][tid], 0, own_value, own_index);
    cluster_sync();  // second phase: every slice result has landed in rank 0
    if (rank != 0) return;
    if (tid < rows) {
      float bv = negative_infinity();
      int bi = INT32_MAX;
      for (unsigned int q = 0; q < ranks; ++q) consider(slice_value[q][tid], slice_index[q][tid], bv, bi);
      target[tid] = bi;
    }
  } else if (tid < rows) {
    target[tid] = own_index;
  }
  __syncthreads();
  if (tid == 0) verify_request(p, r, plan, target, pre);
}

std::atomic<int> g_cluster_override{0};

int device_sms() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  return sms;
}

// Cluster size: the largest Q (at most 8, the portable cluster limit) whose R x Q CTAs all fit
// on the GPU at once, so the launch runs as one wave, with slices of at least 4096 elements.
int pick_cluster(int64_t n_requests, int64_t vocab, int64_t resident_ctas) {
  const int forced = g_cluster_override.load(std::memory_order_relaxed);
  if (forced > 0) return forced;
  int q = 8;
  while (q > 1 && (n_requests * q > resident_ctas || vocab / (2 * q) < 4096)) q /= 2;
  return q;
}

template <typename T>
int resident_ctas_per_sm() {
  static const int blocks = [] {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, greedy_verify_kernel<T>, kThreads, 0) != cudaSuccess) b = 1;
    return b > 0 ? b : 1;
  }();
  return blocks;
}

template <typename T>
cudaError_t launch_verify(VerifyArgs args, int sms, cudaStream_t stream) {
  const int q = pick_cluster(args.n_requests, args.vocab, static_cast<int64_t>(resident_ctas_per_sm<T>()) * sms);
  args.chunk = ((args.vocab + q - 1) / q + 7) / 8 * 8;
  if (q > 8) {  // 16-CTA clusters are a non-portable size that each kernel opts into
    const cudaError_t err =
        cudaFuncSetAttribute(greedy_verify_kernel<T>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err != cudaSuccess) return err;
  }
  return ldb::launch(greedy_verify_kernel<T>, dim3(static_cast<unsigned int>(args.n_requests * q)), dim3(kThreads),
                     0, stream, static_cast<unsigned int>(q), args);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace ldb {

int verify_faults(uint32_t* flags, int clear) {
  uint32_t value = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&value, g_verify_faults, sizeof(value));
  if (err == cudaSuccess && clear) {
    const uint32_t zero = 0;
    err = cudaMemcpyToSymbol(g_verify_faults, &zero, sizeof(zero));
  }
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "ld_fault_flags: %s", cudaGetErrorString(err));
  *flags = value;
  return LD_OK;
}

}  // namespace ldb

extern "C" int ld_greedy_verify_cluster_override(int cluster) {
  if (cluster != 0 && cluster != 1 && cluster != 2 && cluster != 4 && cluster != 8 && cluster != 16) {
    return -LD_ERR_INVALID;
  }
  return g_cluster_override.exchange(cluster);
}

extern "C" int ld_greedy_verify(const void* logits, int logits_dtype, int64_t n_logits, int64_t vocab,
                                int64_t logits_row_stride, const int32_t* cu_num_logits,
                                const int32_t* query_start_loc, const void* input_ids, int token_dtype,
                                int64_t n_input_ids, const int32_t* num_draft_tokens, const int32_t* seq_lens,
                                const int32_t* prefill_len, int64_t n_requests, int64_t num_speculative_steps,
                                void* sampled, int32_t* num_sampled, int32_t* num_rejected, void* stream) {
  using ldb::set_error;
  if (logits_dtype != LD_DTYPE_F32 && logits_dtype != LD_DTYPE_BF16 && logits_dtype != LD_DTYPE_F16) {
    return set_error(LD_ERR_INVALID, "ld_greedy_verify: logits must be F32, BF16 or F16");
  }
  if (token_dtype != LD_DTYPE_I32 && token_dtype != LD_DTYPE_I64) {
    return set_error(LD_ERR_INVALID, "ld_greedy_verify: tokens must be I32 or I64");
  }
  if (n_requests < 0 || n_logits < 0 || n_input_ids < 0) {
    return set_error(LD_ERR_INVALID, "ld_greedy_verify: negative sizes");
  }
  if (num_speculative_steps < 0 || num_speculative_steps > LD_MAX_VERIFY_STEPS) {
    return set_error(LD_ERR_INVALID, "ld_greedy_verify: num_speculative_steps must be in [0, %d]",
                     LD_MAX_VERIFY_STEPS);
  }
  if (vocab < 1 || vocab > INT32_MAX || logits_row_stride < vocab) {
    return set_error(LD_ERR_INVALID, "ld_greedy_verify: need 1 <= vocab <= 2^31-1 and row stride >= vocab");
  }
  if (n_requests == 0) return ldb::ok();
  if (n_requests > INT32_MAX / kMaxCluster) return set_error(LD_ERR_INVALID, "ld_greedy_verify: too many requests");
  if ((n_logits > 0 && logits == nullptr) || cu_num_logits == nullptr || query_start_loc == nullptr ||
      (n_input_ids > 0 && input_ids == nullptr) || num_draft_tokens == nullptr || seq_lens == nullptr ||
      prefill_len == nullptr || sampled == nullptr || num_sampled == nullptr || num_rejected == nullptr) {
    return set_error(LD_ERR_INVALID, "ld_greedy_verify: NULL pointer argument");
  }
  const int sms = device_sms();
  if (sms <= 0) return set_error(LD_ERR_CUDA, "ld_greedy_verify: no CUDA device");

  VerifyArgs args{};
  args.logits = logits;
  args.n_logits = n_logits;
  args.vocab = vocab;
  args.row_stride = logits_row_stride;
  args.cu_num_logits = cu_num_logits;
  args.query_start_loc = query_start_loc;
  args.input_ids = input_ids;
  args.n_input_ids = n_input_ids;
  args.tokens_i64 = token_dtype == LD_DTYPE_I64;
  args.num_draft_tokens = num_draft_tokens;
  args.seq_lens = seq_lens;
  args.prefill_len = prefill_len;
  args.n_requests = n_requests;
  args.steps = static_cast<int>(num_speculative_steps);
  args.sampled = sampled;
  args.num_sampled = num_sampled;
  args.num_rejected = num_rejected;
  const int64_t elem = logits_dtype == LD_DTYPE_F32 ? 4 : 2;
  args.vector_ok = aligned16(logits) && (logits_row_stride * elem) % 16 == 0;

  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (logits_dtype == LD_DTYPE_F32) {
    err = launch_verify<float>(args, sms, s);
  } else if (logits_dtype == LD_DTYPE_BF16) {
    err = launch_verify<__nv_bfloat16>(args, sms, s);
  } else {
    err = launch_verify<__half>(args, sms, s);
  }
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "ld_greedy_verify: launch failed: %s", cudaGetErrorString(err));
  return ldb::ok();
}
