// Fused Gated DeltaNet decode / MTP verify for sm_100a.
//
// Contract: lightdelta::decode of the reference (csrc/gdn_decode.cu:130-354 kernel,
// :360-420 launcher), generalised to any num_k_heads / num_v_heads with K = V = 128.
// Mathematics: python/lightdelta/reference/gdn.py:70-128 (post_conv_gdn).
//
// Design (B200): the op is a read-modify-write stream over fp32 state slots, so it is
// HBM bound (about 1 flop per byte at one token).  One CTA owns one (request, value head)
// pair and keeps the whole 128x128 fp32 state in registers: 256 threads, each holding
// 4 rows x 16 columns (64 floats).  Eight lanes share a row; lane j of a row group owns
// columns {32c + 4j .. 32c + 4j + 3 : c = 0..3}, so every warp-wide 128-bit load or store
// touches four fully used 128-byte lines.  All 16 loads of a thread are issued before the
// activations are prepared, giving 64 KiB in flight per CTA (128 KiB per SM at two CTAs).
// Row dot products (S k and S q) are reduced with three xor-shuffles inside the 8-lane
// group.  Each step's state goes straight from registers to its destination slot.
// Tensor cores are not used: per token the work is a rank-1 update plus two GEMVs.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "internal.h"
#include "lightdelta_b200.h"

namespace ldb {
namespace {

constexpr int kDim = LD_HEAD_DIM;                      // K = V = 128
constexpr int kHeadElems = kDim * kDim;                // floats per (slot, value head)
constexpr int kThreads = 256;
constexpr int kLanesPerRow = 8;                        // lanes sharing one state row
constexpr int kRowGroups = kThreads / kLanesPerRow;    // 32 rows in flight per pass
constexpr int kRowsPerThread = kDim / kRowGroups;      // 4
constexpr int kVecPerRow = kDim / (4 * kLanesPerRow);  // float4 per lane per row: 4
constexpr int kMaxTokens = LD_MAX_WIDTH;

__device__ unsigned int g_decode_faults;

struct DecodeArgs {
  const __nv_bfloat16* qkv;
  int64_t qkv_row;
  const __nv_bfloat16* a;
  int64_t a_row;
  const __nv_bfloat16* b;
  int64_t b_row;
  const float* a_log;
  const void* dt_bias;
  const int32_t* indices;
  const int32_t* cu;
  const int32_t* accepted;
  float* state;
  int64_t n_slots;
  int64_t slot_stride;
  const __nv_bfloat16* gate;
  int64_t gate_row;
  const void* weight;
  __nv_bfloat16* out;
  int64_t n_tokens;
  int width;
  int num_k_heads;
  int num_v_heads;
  int heads_ratio;
  int dt_bias_bf16;
  int weight_bf16;
  float q_scale;
  float eps;
};

__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

// Loads 4 consecutive bf16 values as fp32.  kVec: one 8-byte load (caller guarantees alignment).
template <bool kVec>
__device__ __forceinline__ void load4_bf16(const __nv_bfloat16* p, float (&v)[4]) {
  if constexpr (kVec) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    v[0] = bf16_lo(raw.x);
    v[1] = bf16_hi(raw.x);
    v[2] = bf16_lo(raw.y);
    v[3] = bf16_hi(raw.y);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = __bfloat162float(p[e]);
  }
}

template <bool kVec>
__device__ __forceinline__ void store4_bf16(__nv_bfloat16* p, const float (&v)[4]) {
  if constexpr (kVec) {
    uint2 raw;
    raw.x = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[0]))) |
            (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[1]))) << 16);
    raw.y = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2]))) |
            (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[3]))) << 16);
    *reinterpret_cast<uint2*>(p) = raw;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = __float2bfloat16_rn(v[e]);
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) x += __shfl_xor_sync(0xffffffffu, x, offset);
  return x;
}

// Sum over the 8 lanes that share a state row (lanes differ in their low three bits).
__device__ __forceinline__ float row_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  return x;
}

__device__ __forceinline__ float load_param(const void* p, int index, int is_bf16) {
  return is_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[index])
                 : static_cast<const float*>(p)[index];
}

// softplus with torch's default threshold 20 (reference gdn.py:102, gdn_decode.cu:96-98).
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

template <bool kVecAct>
__global__ void __launch_bounds__(kThreads, 2) gdn_decode_kernel(const DecodeArgs p) {
  __shared__ float4 sh_q[kMaxTokens][kDim / 4];
  __shared__ float4 sh_k[kMaxTokens][kDim / 4];
  __shared__ float sh_v[kMaxTokens][kDim];
  __shared__ float sh_z[kMaxTokens][kDim];
  __shared__ float sh_o[kMaxTokens][kDim];
  __shared__ float sh_decay[kMaxTokens];
  __shared__ float sh_beta[kMaxTokens];
  __shared__ int sh_dst[kMaxTokens];

  const int HV = p.num_v_heads;
  const int request = blockIdx.x / HV;
  const int head = blockIdx.x - request * HV;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int W = p.width;

  const int bos = p.cu[request];
  const int eos = p.cu[request + 1];
  const int n = eos - bos;
  if (n <= 0) return;  // no tokens: nothing is written (reference gdn_decode.cu:150-152)
  if (bos < 0 || static_cast<int64_t>(eos) > p.n_tokens) {
    if (tid == 0) atomicOr(&g_decode_faults, LD_FAULT_DECODE_TOKENS);
    return;
  }
  const int acc = p.accepted[request];
  const int src = (acc >= 1 && acc <= W) ? p.indices[request * W + acc - 1] : 0;
  if (src <= 0 || n > W || src >= p.n_slots) {
    // Invalid request: zero outputs, no state writes (reference gdn_decode.cu:154-168).
    if (tid == 0) {
      if (n > W) atomicOr(&g_decode_faults, LD_FAULT_DECODE_TOKENS);
      if (src >= p.n_slots) atomicOr(&g_decode_faults, LD_FAULT_DECODE_SLOT_RANGE);
    }
    for (int idx = tid; idx < n * kDim; idx += kThreads) {
      const int64_t token = bos + idx / kDim;
      p.out[(token * HV + head) * kDim + (idx % kDim)] = __float2bfloat16_rn(0.0f);
    }
    return;
  }

  // ---- issue the 64 KiB state read first: 16 x 128-bit loads per thread ----
  const int j = tid & (kLanesPerRow - 1);
  const int g = tid / kLanesPerRow;
  const int64_t head_offset = static_cast<int64_t>(head) * kHeadElems + g * kDim + 4 * j;
  const float4* src_ptr =
      reinterpret_cast<const float4*>(p.state + static_cast<int64_t>(src) * p.slot_stride + head_offset);
  float4 s[kRowsPerThread][kVecPerRow];
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) {
      s[i][c] = src_ptr[(i * kRowGroups * kDim + c * 4 * kLanesPerRow) / 4];
    }
  }

  // ---- per-token activations: warp t prepares token t ----
  if (warp < n) {
    const int t = warp;
    const int64_t token = bos + t;
    const int H = p.num_k_heads;
    const int key_head = head / p.heads_ratio;
    const __nv_bfloat16* row = p.qkv + token * p.qkv_row;
    float q[4], k[4], v[4], z[4];
    load4_bf16<kVecAct>(row + key_head * kDim + 4 * lane, q);
    load4_bf16<kVecAct>(row + (H + key_head) * kDim + 4 * lane, k);
    load4_bf16<kVecAct>(row + (2 * H + head) * kDim + 4 * lane, v);
    load4_bf16<kVecAct>(p.gate + token * p.gate_row + head * kDim + 4 * lane, z);
    float q_sq = 0.0f, k_sq = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      q_sq += q[e] * q[e];
      k_sq += k[e] * k[e];
    }
    q_sq = warp_sum(q_sq);
    k_sq = warp_sum(k_sq);
    // L2 norm in fp32 as gdn.py:98-99; q then scaled by K^-1/2 as gdn.py:101.
    const float q_inv = 1.0f / sqrtf(q_sq + 1e-6f);
    const float k_inv = 1.0f / sqrtf(k_sq + 1e-6f);
    sh_q[t][lane] = make_float4(q[0] * q_inv * p.q_scale, q[1] * q_inv * p.q_scale,
                                q[2] * q_inv * p.q_scale, q[3] * q_inv * p.q_scale);
    sh_k[t][lane] = make_float4(k[0] * k_inv, k[1] * k_inv, k[2] * k_inv, k[3] * k_inv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sh_v[t][4 * lane + e] = v[e];
      sh_z[t][4 * lane + e] = z[e];
    }
    if (lane == 0) {
      // decay = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b): gdn.py:102-103.
      const float a_val = __bfloat162float(p.a[token * p.a_row + head]);
      const float b_val = __bfloat162float(p.b[token * p.b_row + head]);
      const float dt = load_param(p.dt_bias, head, p.dt_bias_bf16);
      sh_decay[t] = expf(-expf(p.a_log[head]) * softplus(a_val + dt));
      sh_beta[t] = 1.0f / (1.0f + expf(-b_val));
      int dst = p.indices[request * W + t];
      if (dst >= p.n_slots) {
        atomicOr(&g_decode_faults, LD_FAULT_DECODE_SLOT_RANGE);
        dst = 0;
      }
      sh_dst[t] = dst;
    }
  }
  __syncthreads();

  // ---- recurrence: state stays in registers across the T steps ----
  const int row0 = g;  // rows owned: g + 32 i
  for (int t = 0; t < n; ++t) {
    const float decay = sh_decay[t];
    const float beta = sh_beta[t];
    float4 kv[kVecPerRow];
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) kv[c] = sh_k[t][c * kLanesPerRow + j];

    float pred[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      float acc_hk = 0.0f;
#pragma unroll
      for (int c = 0; c < kVecPerRow; ++c) {
        s[i][c].x *= decay;
        s[i][c].y *= decay;
        s[i][c].z *= decay;
        s[i][c].w *= decay;
        acc_hk = fmaf(s[i][c].x, kv[c].x, acc_hk);
        acc_hk = fmaf(s[i][c].y, kv[c].y, acc_hk);
        acc_hk = fmaf(s[i][c].z, kv[c].z, acc_hk);
        acc_hk = fmaf(s[i][c].w, kv[c].w, acc_hk);
      }
      pred[i] = acc_hk;
    }
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) pred[i] = row_sum(pred[i]);

#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      const float delta = (sh_v[t][row0 + i * kRowGroups] - pred[i]) * beta;
#pragma unroll
      for (int c = 0; c < kVecPerRow; ++c) {
        s[i][c].x = fmaf(delta, kv[c].x, s[i][c].x);
        s[i][c].y = fmaf(delta, kv[c].y, s[i][c].y);
        s[i][c].z = fmaf(delta, kv[c].z, s[i][c].z);
        s[i][c].w = fmaf(delta, kv[c].w, s[i][c].w);
      }
    }

    float4 qv[kVecPerRow];
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) qv[c] = sh_q[t][c * kLanesPerRow + j];
    float o[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      float acc_hq = 0.0f;
#pragma unroll
      for (int c = 0; c < kVecPerRow; ++c) {
        acc_hq = fmaf(s[i][c].x, qv[c].x, acc_hq);
        acc_hq = fmaf(s[i][c].y, qv[c].y, acc_hq);
        acc_hq = fmaf(s[i][c].z, qv[c].z, acc_hq);
        acc_hq = fmaf(s[i][c].w, qv[c].w, acc_hq);
      }
      o[i] = acc_hq;
    }
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) o[i] = row_sum(o[i]);
    if (j == 0) {
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) {
        // The recurrence output is rounded to bf16 before the norm (gdn.py:116).
        sh_o[t][row0 + i * kRowGroups] = __bfloat162float(__float2bfloat16_rn(o[i]));
      }
    }

    const int dst = sh_dst[t];
    if (dst > 0) {
      float4* dst_ptr =
          reinterpret_cast<float4*>(p.state + static_cast<int64_t>(dst) * p.slot_stride + head_offset);
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) {
#pragma unroll
        for (int c = 0; c < kVecPerRow; ++c) {
          dst_ptr[(i * kRowGroups * kDim + c * 4 * kLanesPerRow) / 4] = s[i][c];
        }
      }
    }
  }
  __syncthreads();

  // ---- gated RMSNorm epilogue: warp t finishes token t (gdn.py:117-119) ----
  if (warp < n) {
    const int t = warp;
    const int64_t token = bos + t;
    float o[4];
    float sq = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      o[e] = sh_o[t][4 * lane + e];
      sq += o[e] * o[e];
    }
    sq = warp_sum(sq);
    const float rstd = 1.0f / sqrtf(sq / static_cast<float>(kDim) + p.eps);
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int dim = 4 * lane + e;
      const float z = sh_z[t][dim];
      const float silu = z / (1.0f + expf(-z));
      const float w = load_param(p.weight, dim, p.weight_bf16);
      y[e] = o[e] * rstd * w * silu;
    }
    store4_bf16<kVecAct>(p.out + (token * HV + head) * kDim + 4 * lane, y);
  }
}

bool aligned(const void* ptr, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(ptr) % bytes) == 0;
}

}  // namespace

int decode_faults(uint32_t* flags, int clear) {
  unsigned int value = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&value, g_decode_faults, sizeof(value));
  if (err != cudaSuccess) {
    return set_error(LD_ERR_CUDA, "reading decode fault word: %s", cudaGetErrorString(err));
  }
  if (clear) {
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(g_decode_faults, &zero, sizeof(zero));
    if (err != cudaSuccess) {
      return set_error(LD_ERR_CUDA, "clearing decode fault word: %s", cudaGetErrorString(err));
    }
  }
  *flags = value;
  return LD_OK;
}

}  // namespace ldb

extern "C" int ld_decode(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride,
                         const void* b, int64_t b_row_stride, const float* a_log, const void* dt_bias,
                         int dt_bias_dtype, const int32_t* indices, int64_t n_requests, int64_t width,
                         const int32_t* cu, const int32_t* accepted, float* state, int64_t n_slots,
                         int64_t slot_stride, const void* gate, int64_t gate_row_stride,
                         const void* weight, int weight_dtype, void* out, int64_t n_tokens,
                         int64_t num_k_heads, int64_t num_v_heads, float eps, void* stream) {
  using namespace ldb;
  if (width < 1 || width > LD_MAX_WIDTH) {
    return set_error(LD_ERR_INVALID, "decode/MTP supports 1 through %d tokens per request (got width %lld)",
                     LD_MAX_WIDTH, static_cast<long long>(width));
  }
  if (n_requests < 0 || n_tokens < 0) {
    return set_error(LD_ERR_INVALID, "n_requests and n_tokens must be non-negative");
  }
  if (num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads != 0) {
    return set_error(LD_ERR_INVALID, "num_v_heads (%lld) must be a positive multiple of num_k_heads (%lld)",
                     static_cast<long long>(num_v_heads), static_cast<long long>(num_k_heads));
  }
  if (!(eps > 0.0f) || !std::isfinite(eps)) {
    return set_error(LD_ERR_INVALID, "norm epsilon must be positive");
  }
  if ((dt_bias_dtype != LD_DTYPE_F32 && dt_bias_dtype != LD_DTYPE_BF16) ||
      (weight_dtype != LD_DTYPE_F32 && weight_dtype != LD_DTYPE_BF16)) {
    return set_error(LD_ERR_INVALID, "dt_bias and weight must be FP32 or BF16");
  }
  if (n_requests == 0) return ok();
  if (n_requests * num_v_heads > 0x7fffffffLL) {
    return set_error(LD_ERR_INVALID, "n_requests * num_v_heads exceeds the grid limit");
  }
  if (qkv == nullptr || a == nullptr || b == nullptr || a_log == nullptr || dt_bias == nullptr ||
      indices == nullptr || cu == nullptr || accepted == nullptr || state == nullptr ||
      gate == nullptr || weight == nullptr || (out == nullptr && n_tokens > 0)) {
    return set_error(LD_ERR_INVALID, "decode: a required pointer is NULL");
  }
  const int64_t qkv_width = (2 * num_k_heads + num_v_heads) * LD_HEAD_DIM;
  if (qkv_row_stride < qkv_width || a_row_stride < num_v_heads || b_row_stride < num_v_heads ||
      gate_row_stride < num_v_heads * LD_HEAD_DIM) {
    return set_error(LD_ERR_INVALID, "activation row strides are smaller than a row");
  }
  const int64_t slot_elems = num_v_heads * LD_HEAD_DIM * LD_HEAD_DIM;
  if (n_slots < 1 || (n_slots > 1 && slot_stride < slot_elems)) {
    return set_error(LD_ERR_INVALID, "state must hold at least one slot of [HV,128,128] with slot stride >= %lld",
                     static_cast<long long>(slot_elems));
  }
  if (!aligned(state, 16) || slot_stride % 4 != 0) {
    return set_error(LD_ERR_INVALID, "state must be 16-byte aligned with a slot stride divisible by 4");
  }
  DecodeArgs args;
  args.qkv = static_cast<const __nv_bfloat16*>(qkv);
  args.qkv_row = qkv_row_stride;
  args.a = static_cast<const __nv_bfloat16*>(a);
  args.a_row = a_row_stride;
  args.b = static_cast<const __nv_bfloat16*>(b);
  args.b_row = b_row_stride;
  args.a_log = a_log;
  args.dt_bias = dt_bias;
  args.indices = indices;
  args.cu = cu;
  args.accepted = accepted;
  args.state = state;
  args.n_slots = n_slots;
  args.slot_stride = slot_stride;
  args.gate = static_cast<const __nv_bfloat16*>(gate);
  args.gate_row = gate_row_stride;
  args.weight = weight;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.n_tokens = n_tokens;
  args.width = static_cast<int>(width);
  args.num_k_heads = static_cast<int>(num_k_heads);
  args.num_v_heads = static_cast<int>(num_v_heads);
  args.heads_ratio = static_cast<int>(num_v_heads / num_k_heads);
  args.dt_bias_bf16 = dt_bias_dtype == LD_DTYPE_BF16;
  args.weight_bf16 = weight_dtype == LD_DTYPE_BF16;
  // K^-1/2 evaluated in double and rounded once, as torch scales an fp32 tensor by a Python float.
  args.q_scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(LD_HEAD_DIM)));
  args.eps = eps;

  const bool vec_act = aligned(qkv, 8) && qkv_row_stride % 4 == 0 && aligned(gate, 8) &&
                       gate_row_stride % 4 == 0 && aligned(out, 8);
  const dim3 grid(static_cast<unsigned int>(n_requests * num_v_heads));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec_act) {
    gdn_decode_kernel<true><<<grid, kThreads, 0, s>>>(args);
  } else {
    gdn_decode_kernel<false><<<grid, kThreads, 0, s>>>(args);
  }
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return set_error(LD_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(err));
  }
  return ok();
}
