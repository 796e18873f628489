// Fused Gated DeltaNet decode / MTP verify for sm_100a.
//
// Contract: lightdelta::decode of the reference (csrc/gdn_decode.cu:130-354 kernel,
// :360-420 launcher), generalised to any num_k_heads / num_v_heads with K = V = 128.
// Mathematics: python/lightdelta/reference/gdn.py:70-128 (post_conv_gdn).
//
// The op is a read-modify-write stream over fp32 state slots: about one flop per byte at one
// token, so HBM bandwidth bounds it and tensor cores have nothing to do (per token the work is
// a rank-1 update plus two GEMVs per (sequence, value head)).
//
// Work unit ("item"): one (request, value head) pair, i.e. one 128x128 fp32 state (64 KiB)
// read once and written once per token step.
//
// Register tile shared by both kernels: 256 compute threads hold the whole state, 4 rows x 16
// columns each.  Eight lanes share a row; lane j of a row group owns columns
// {32c + 4j .. 32c + 4j + 3 : c = 0..3}, so each warp-wide 128-bit access touches four fully
// used 128-byte lines, and the row dot products S k and S q reduce with three xor-shuffles.
//
// gdn_decode_stream_kernel (large one-token launches): persistent, one CTA per SM.  A producer warp streams the
// states of the CTA's items into a 3-deep shared-memory ring with TMA bulk copies
// (cp.async.bulk, completion on an mbarrier) together with the items' q/k/v/gate rows, while
// 8 consumer warps run the recurrence on the register tile and store each step's state
// straight from registers.  Up to three 64 KiB states per SM are in flight at all times, so
// HBM never waits for a CTA's compute or store phase.  Every mbarrier wait is bounded
// (LD_FAULT_WAIT_TIMEOUT).  No thread-block cluster: each CTA reads only its own items
// from this GPU's memory.
//
// gdn_decode_rowreg_kernel: one CTA per item, loading the state straight into registers with
// 128-bit loads.  Used for multi-token verify, for one-token launches below kStreamItemsPerSm
// items per SM, and when the activation rows are not 16-byte aligned (TMA bulk copies need
// 16-byte aligned sources).
//
// A bf16 state pool (ld_decode_bf16_state) runs the one-CTA-per-item kernel on an fp32 tile widened
// on load and rounded to bf16 on store, each lane owning eight consecutive columns per half row
// ({64h + 8j .. 64h + 8j + 7 : h = 0, 1}, see tile_col) so that its state accesses stay 16 bytes
// wide; its one-token launches use gdn_decode_b16_kernel (namespace b16 below), which keeps two
// items in flight per CTA.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <algorithm>
#include <atomic>
#include <mutex>

#include "internal.h"
#include "launch.cuh"
#include "lightdelta_b200.h"

namespace ldb {
namespace {

constexpr int kDim = LD_HEAD_DIM;                      // K = V = 128
constexpr int kHeadElems = kDim * kDim;                // floats per (slot, value head)
constexpr int kRowBytes = kDim * 2;                    // one bf16 head row: 256 B
constexpr int kLanesPerRow = 8;                        // lanes sharing one state row
constexpr int kVecPerRow = kDim / (4 * kLanesPerRow);  // float4 per lane per row: 4

// Register tile with kRows rows per thread: kDim / kRows row groups of 8 lanes.
template <int kRows>
struct Tile {
  static constexpr int kRowGroups = kDim / kRows;             // rows covered per pass
  static constexpr int kThreads = kRowGroups * kLanesPerRow;  // 256 (4 rows) or 512 (2 rows)
};
constexpr int kMaxTokens = LD_MAX_WIDTH;
// One-token launches with at least this many (request, head) items per SM use the streaming
// kernel (fp32 and bf16 pools); smaller ones and multi-token verify use one CTA per item.
constexpr int kStreamItemsPerSm = 9;
constexpr int kStreamItemsPerSmBf16 = 7;

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
  float* state;                  // fp32 state pool (null when the pool is bf16)
  __nv_bfloat16* state_bf16;     // bf16 state pool (ld_decode_bf16_state), else null
  int64_t n_slots;
  int64_t slot_stride;
  const __nv_bfloat16* gate;
  int64_t gate_row;
  const void* weight;
  __nv_bfloat16* out;
  int64_t n_tokens;
  int64_t total_items;
  int width;
  int num_k_heads;
  int num_v_heads;
  int heads_ratio;
  int dt_bias_bf16;
  int weight_bf16;
  float q_scale;
  float eps;
  uint64_t wait_ns;   // bound of every in-kernel wait of the persistent kernel (ld_decode_wait_test)
  uint32_t extra_tx;  // test only: bytes each state load announces beyond what it copies (normally 0)
  int64_t prefetch_stride;  // one-CTA-per-item kernel: blocks resident at once (0: no L2 prefetch)
};

// The state pool of a launch as the kernel's element type.
template <typename StateT>
__device__ __forceinline__ StateT* state_base(const DecodeArgs& p);
template <>
__device__ __forceinline__ float* state_base<float>(const DecodeArgs& p) {
  return p.state;
}
template <>
__device__ __forceinline__ __nv_bfloat16* state_base<__nv_bfloat16>(const DecodeArgs& p) {
  return p.state_bf16;
}

// ------------------------------------------------------------------------------------------
// scalar helpers
// ------------------------------------------------------------------------------------------
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

// decay = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b): gdn.py:102-103.
__device__ __forceinline__ void token_gates(const DecodeArgs& p, int64_t token, int head, float& decay,
                                            float& beta) {
  const float a_val = __bfloat162float(p.a[token * p.a_row + head]);
  const float b_val = __bfloat162float(p.b[token * p.b_row + head]);
  const float dt = load_param(p.dt_bias, head, p.dt_bias_bf16);
  decay = expf(-expf(p.a_log[head]) * softplus(a_val + dt));
  beta = 1.0f / (1.0f + expf(-b_val));
}

// Paired fp32 arithmetic (sm_100's f32x2 forms): two independent IEEE fp32 operations per
// instruction, each lane rounded exactly as the scalar instruction would round it.
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 lo2(const float4& v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(const float4& v) { return make_float2(v.z, v.w); }

// One delta-rule step on the register tile (gdn.py:111-114), then o = S q for the tile's rows
// (gdn.py:115), reduced over the row group.  kv / qv are this lane's normalised k and q columns.
// The decay and the rank-1 update are element-wise (paired instructions, same rounding as the
// scalar form); each lane's partial dot products keep four partial sums (the .x/.y lanes of the
// low and high column pairs), added at the end.
template <int kRows>
__device__ __forceinline__ void tile_step(float4 (&s)[kRows][kVecPerRow], const float4 (&kv)[kVecPerRow],
                                          const float4 (&qv)[kVecPerRow], const float (&vrow)[kRows],
                                          float decay, float beta, float (&o)[kRows]) {
  const float2 decay2 = make_float2(decay, decay);
  float pred[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    float2 acc_lo = make_float2(0.0f, 0.0f), acc_hi = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) {
      const float2 lo = mul2(lo2(s[i][c]), decay2);
      const float2 hi = mul2(hi2(s[i][c]), decay2);
      s[i][c] = make_float4(lo.x, lo.y, hi.x, hi.y);
      acc_lo = fma2(lo, lo2(kv[c]), acc_lo);
      acc_hi = fma2(hi, hi2(kv[c]), acc_hi);
    }
    pred[i] = (acc_lo.x + acc_lo.y) + (acc_hi.x + acc_hi.y);
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) pred[i] = row_sum(pred[i]);
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    const float delta = (vrow[i] - pred[i]) * beta;
    const float2 delta2 = make_float2(delta, delta);
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) {
      const float2 lo = fma2(lo2(kv[c]), delta2, lo2(s[i][c]));
      const float2 hi = fma2(hi2(kv[c]), delta2, hi2(s[i][c]));
      s[i][c] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    float2 acc_lo = make_float2(0.0f, 0.0f), acc_hi = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) {
      acc_lo = fma2(lo2(s[i][c]), lo2(qv[c]), acc_lo);
      acc_hi = fma2(hi2(s[i][c]), hi2(qv[c]), acc_hi);
    }
    o[i] = (acc_lo.x + acc_lo.y) + (acc_hi.x + acc_hi.y);
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) o[i] = row_sum(o[i]);
}

// Writes the tile's row sets in the order kFirst, kFirst+1, ... (all indices compile-time, so the
// tile stays in registers).
// kStream: streaming stores (st.global.cs; the stored states are not read again by this launch).
template <int kRows, int kFirst, bool kStream>
__device__ __forceinline__ void store_rows_from(float4* ptr, const float4 (&s)[kRows][kVecPerRow]) {
#pragma unroll
  for (int step = 0; step < kRows; ++step) {
    const int i = (step + kFirst) % kRows;
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) {
      float4* at = &ptr[(i * Tile<kRows>::kRowGroups * kDim + c * 4 * kLanesPerRow) / 4];
      if constexpr (kStream) {
        __stcs(at, s[i][c]);
      } else {
        *at = s[i][c];
      }
    }
  }
}

// Stores a register tile to one head's state.  CTAs start at different row sets (blockIdx.x mod
// kRows): when every SM writes the same quarter of its head at the same moment the state writes
// concentrate on part of the memory system; staggering them measured 5-7% faster on B200.
// Measured on B200 (config 3, back to back): streaming stores take the one-CTA-per-item verify
// kernel from 112.6 to 111.1 us on an fp32 pool and from 66.2 to 65.3 us on a bf16 pool; the
// persistent fp32 decode kernel keeps plain stores (176.7 -> 177.7 us with them).
template <int kRows, bool kStream = false>
__device__ __forceinline__ void store_tile(float* dst_head, int g, int j, const float4 (&s)[kRows][kVecPerRow]) {
  float4* ptr = reinterpret_cast<float4*>(dst_head + g * kDim + 4 * j);
  static_assert(kRows <= 4, "rotation covers at most four row sets");
  switch (blockIdx.x % kRows) {
    case 0: store_rows_from<kRows, 0, kStream>(ptr, s); break;
    case 1: store_rows_from<kRows, 1 % kRows, kStream>(ptr, s); break;
    case 2: store_rows_from<kRows, 2 % kRows, kStream>(ptr, s); break;
    default: store_rows_from<kRows, 3 % kRows, kStream>(ptr, s); break;
  }
}

// Shared-memory or global state of one head -> register tile.
template <int kRows>
__device__ __forceinline__ void load_tile(const float* head, int g, int j, float4 (&s)[kRows][kVecPerRow]) {
  const float4* ptr = reinterpret_cast<const float4*>(head + g * kDim + 4 * j);
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) s[i][c] = ptr[(i * Tile<kRows>::kRowGroups * kDim + c * 4 * kLanesPerRow) / 4];
  }
}

// Column of the first of the four consecutive columns that float4 c of lane j holds.  fp32 tiles
// use {32c + 4j}: a warp-wide 128-bit access covers whole 128-byte lines of fp32 rows.  bf16
// pools use the wide map {64(c/2) + 8j + 4(c%2)}: each lane owns eight consecutive columns per
// half row, so one 128-bit access moves eight bf16 values and a warp-wide access again covers
// whole 128-byte lines.  Activations follow the map of the state they meet.
template <bool kWide>
__device__ __forceinline__ constexpr int tile_col(int c, int j) {
  return kWide ? 64 * (c >> 1) + 8 * j + 4 * (c & 1) : 32 * c + 4 * j;
}

__device__ __forceinline__ float4 widen_bf16x4(uint32_t lo, uint32_t hi) {
  return make_float4(__uint_as_float(lo << 16), __uint_as_float(lo & 0xffff0000u), __uint_as_float(hi << 16),
                     __uint_as_float(hi & 0xffff0000u));
}

// bf16 state pools: the same fp32 tile on the wide map, eight bf16 values (16 bytes) per access,
// widened exactly on load and rounded to nearest-even on store.
template <int kRows>
__device__ __forceinline__ void load_tile(const __nv_bfloat16* head, int g, int j, float4 (&s)[kRows][kVecPerRow]) {
  const __nv_bfloat16* base = head + g * kDim + 8 * j;
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
#pragma unroll
    for (int h = 0; h < kVecPerRow / 2; ++h) {
      const uint4 raw = *reinterpret_cast<const uint4*>(base + i * Tile<kRows>::kRowGroups * kDim + 64 * h);
      s[i][2 * h] = widen_bf16x4(raw.x, raw.y);
      s[i][2 * h + 1] = widen_bf16x4(raw.z, raw.w);
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int kRows, int kFirst, bool kStream>
__device__ __forceinline__ void store_rows_from(__nv_bfloat16* base, const float4 (&s)[kRows][kVecPerRow]) {
#pragma unroll
  for (int step = 0; step < kRows; ++step) {
    const int i = (step + kFirst) % kRows;
#pragma unroll
    for (int h = 0; h < kVecPerRow / 2; ++h) {
      const float4& a = s[i][2 * h];
      const float4& b = s[i][2 * h + 1];
      uint4* at = reinterpret_cast<uint4*>(base + i * Tile<kRows>::kRowGroups * kDim + 64 * h);
      const uint4 words =
          make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
      if constexpr (kStream) {
        __stcs(at, words);
      } else {
        *at = words;
      }
    }
  }
}

template <int kRows, bool kStream = false>
__device__ __forceinline__ void store_tile(__nv_bfloat16* dst_head, int g, int j, const float4 (&s)[kRows][kVecPerRow]) {
  __nv_bfloat16* base = dst_head + g * kDim + 8 * j;
  switch (blockIdx.x % kRows) {
    case 0: store_rows_from<kRows, 0, kStream>(base, s); break;
    case 1: store_rows_from<kRows, 1 % kRows, kStream>(base, s); break;
    case 2: store_rows_from<kRows, 2 % kRows, kStream>(base, s); break;
    default: store_rows_from<kRows, 3 % kRows, kStream>(base, s); break;
  }
}

// Gated RMSNorm of one token's 128 recurrence outputs (already bf16-rounded), gdn.py:117-119:
// out = bf16(o * rsqrt(mean(o^2) + eps) * w * silu(z)).  One warp, 4 values per lane.
template <bool kVec>
__device__ __forceinline__ void gated_rmsnorm_store(const float* o_row, const float (&z)[4], const float (&w)[4],
                                                    float eps, int lane, __nv_bfloat16* out_row) {
  float o[4];
  float sq = 0.0f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    o[e] = o_row[4 * lane + e];
    sq += o[e] * o[e];
  }
  sq = warp_sum(sq);
  const float rstd = 1.0f / sqrtf(sq / static_cast<float>(kDim) + eps);
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float silu = z[e] / (1.0f + expf(-z[e]));
    y[e] = o[e] * rstd * w[e] * silu;
  }
  store4_bf16<kVec>(out_row + 4 * lane, y);
}

__device__ __forceinline__ void l2_prefetch(const void* ptr, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

// Warms L2 with what item `item` reads first: its source head and its tokens' q, k, v and gate rows.
// Addresses come from the same validity rules as the item's own launch; anything invalid prefetches
// nothing.
template <typename StateT>
__device__ void prefetch_item(const DecodeArgs& p, int64_t item) {
  if (item >= p.total_items) return;
  const int HV = p.num_v_heads;
  const int W = p.width;
  const int request = static_cast<int>(item / HV);
  const int head = static_cast<int>(item - static_cast<int64_t>(request) * HV);
  const int acc = p.accepted[request];
  const int src = (acc >= 1 && acc <= W) ? p.indices[request * W + acc - 1] : 0;
  if (src <= 0 || src >= p.n_slots) return;
  // Heads are 16-byte aligned (pool base and slot stride are checked on the host).
  const StateT* head_ptr =
      state_base<StateT>(p) + static_cast<int64_t>(src) * p.slot_stride + static_cast<int64_t>(head) * kHeadElems;
  for (int q = 0; q < 4; ++q) l2_prefetch(head_ptr + q * (kHeadElems / 4), kHeadElems * sizeof(StateT) / 4);
  const int bos = p.cu[request];
  const int n = p.cu[request + 1] - bos;
  if (bos < 0 || n > W || static_cast<int64_t>(bos) + n > p.n_tokens) return;
  const int H = p.num_k_heads;
  const int key_head = head / p.heads_ratio;
  for (int t = 0; t < n; ++t) {
    const __nv_bfloat16* row = p.qkv + (bos + t) * p.qkv_row;
    const __nv_bfloat16* rows[4] = {row + key_head * kDim, row + (H + key_head) * kDim, row + (2 * H + head) * kDim,
                                    p.gate + (bos + t) * p.gate_row + head * kDim};
    for (int r = 0; r < 4; ++r) {
      if ((reinterpret_cast<uintptr_t>(rows[r]) & 15) == 0) l2_prefetch(rows[r], kRowBytes);
    }
  }
}

// ==========================================================================================
// Fallback kernel: one CTA per item, state loaded straight into registers.
// ==========================================================================================
template <bool kVecAct, typename StateT>
__global__ void __launch_bounds__(Tile<4>::kThreads, 2) gdn_decode_rowreg_kernel(const DecodeArgs p) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  __shared__ float4 sh_q[kMaxTokens][kDim / 4];
  __shared__ float4 sh_k[kMaxTokens][kDim / 4];
  __shared__ float sh_v[kMaxTokens][kDim];
  __shared__ float sh_z[kMaxTokens][kDim];
  __shared__ float sh_o[kMaxTokens][kDim];
  __shared__ float sh_decay[kMaxTokens];
  __shared__ float sh_beta[kMaxTokens];
  __shared__ int sh_dst[kMaxTokens];

  constexpr int kRows = 4;
  constexpr int kThreads = Tile<kRows>::kThreads;
  constexpr int kRowGroups = Tile<kRows>::kRowGroups;
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

  // Issue the 64 KiB state read first: 16 x 128-bit loads per thread.
  const int j = tid & (kLanesPerRow - 1);
  const int g = tid / kLanesPerRow;
  const int64_t head_offset = static_cast<int64_t>(head) * kHeadElems;
  float4 s[kRows][kVecPerRow];
  load_tile<kRows>(state_base<StateT>(p) + static_cast<int64_t>(src) * p.slot_stride + head_offset, g, j, s);

  // The block one wave later most likely runs on this SM next: warm L2 with its first reads now, so
  // that they start from L2 instead of HBM.  The last warp prepares no token.
  if (warp == kThreads / 32 - 1 && lane == 0 && p.prefetch_stride > 0) {
    prefetch_item<StateT>(p, blockIdx.x + p.prefetch_stride);
  }

  // Per-token activations: warp t prepares token t.
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
    sh_q[t][lane] = make_float4(q[0] * q_inv * p.q_scale, q[1] * q_inv * p.q_scale, q[2] * q_inv * p.q_scale,
                                q[3] * q_inv * p.q_scale);
    sh_k[t][lane] = make_float4(k[0] * k_inv, k[1] * k_inv, k[2] * k_inv, k[3] * k_inv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sh_v[t][4 * lane + e] = v[e];
      sh_z[t][4 * lane + e] = z[e];
    }
    if (lane == 0) {
      token_gates(p, token, head, sh_decay[t], sh_beta[t]);
      int dst = p.indices[request * W + t];
      if (dst >= p.n_slots) {
        atomicOr(&g_decode_faults, LD_FAULT_DECODE_SLOT_RANGE);
        dst = 0;
      }
      sh_dst[t] = dst;
    }
  }
  __syncthreads();

  for (int t = 0; t < n; ++t) {
    float4 kv[kVecPerRow], qv[kVecPerRow];
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) {
      kv[c] = sh_k[t][tile_col<sizeof(StateT) == 2>(c, j) / 4];
      qv[c] = sh_q[t][tile_col<sizeof(StateT) == 2>(c, j) / 4];
    }
    float vrow[kRows], o[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) vrow[i] = sh_v[t][g + i * kRowGroups];
    tile_step<kRows>(s, kv, qv, vrow, sh_decay[t], sh_beta[t], o);
    if (j == 0) {
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        // The recurrence output is rounded to bf16 before the norm (gdn.py:116).
        sh_o[t][g + i * kRowGroups] = __bfloat162float(__float2bfloat16_rn(o[i]));
      }
    }
    const int dst = sh_dst[t];
    if (dst > 0) {
      store_tile<kRows, true>(state_base<StateT>(p) + static_cast<int64_t>(dst) * p.slot_stride + head_offset, g, j,
                              s);
    }
  }
  __syncthreads();

  if (warp < n) {
    const int t = warp;
    float z[4], w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      z[e] = sh_z[t][4 * lane + e];
      w[e] = load_param(p.weight, 4 * lane + e, p.weight_bf16);
    }
    gated_rmsnorm_store<kVecAct>(sh_o[t], z, w, p.eps, lane, p.out + ((bos + t) * static_cast<int64_t>(HV) + head) * kDim);
  }
}

// ==========================================================================================
// Streaming kernel: persistent CTAs, TMA bulk prefetch of states into a shared-memory ring.
// ==========================================================================================
namespace stream {

constexpr int kStates = 3;                            // fp32 state ring depth (64 KiB each)

enum ItemKind : int { kSkip = 0, kZero = 1, kRun = 2 };

struct ItemInfo {
  int kind;
  int n;
  int bos;
  int pad;
  int dst[kMaxTokens];
  float decay[kMaxTokens];
  float beta[kMaxTokens];
  float k_inv[kMaxTokens];  // 1 / sqrt(sum k^2 + 1e-6), written by the producer once the rows land
  float q_inv[kMaxTokens];  // the same for q, times K^-1/2
};

struct ActStage {
  __nv_bfloat16 q[kMaxTokens][kDim];
  __nv_bfloat16 k[kMaxTokens][kDim];
  __nv_bfloat16 v[kMaxTokens][kDim];
  __nv_bfloat16 z[kMaxTokens][kDim];
  ItemInfo info;
};

// State ring of the fp32 streaming kernel: three 64 KiB stages, each with an activation stage
// behind it.  The consumer warps reduce the q / k norms themselves: done by the producer, its waits
// for each item's data cost 175.2 -> 192.1 us on config 2 (B200).
struct Smem {
  using State = float;
  static constexpr int kStateStages = kStates;
  static constexpr int kActStages = kStateStages + 1;
  static constexpr bool kStatesReadOnce = false;  // plain state loads (evict-first: 176.7 -> 178.3 us)
  float state[kStateStages][kHeadElems];
  ActStage act[kActStages];
  float out[2][kMaxTokens][kDim];
  unsigned long long full[kStateStages];
  unsigned long long empty_state[kStateStages];
  unsigned long long empty_act[kActStages];
  unsigned long long out_full[2];   // all consumer warps wrote their rows of out[b]
  unsigned long long out_empty[2];  // all consumer warps are past the epilogue that read out[b]
  int abort;
};
static_assert(sizeof(Smem) <= 227 * 1024, "the streaming kernel's ring must fit one CTA's shared memory");

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase of `bar` with the given parity; false once `limit_ns` have passed.
__device__ __noinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > limit_ns) return false;
  }
  return true;
}

// The same with an L2 evict-first policy, for data read once.
__device__ __forceinline__ void bulk_load_once(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// TMA bulk copy global -> this CTA's own shared memory (one destination), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Bounded wait whose outcome is the same for every lane of the warp.
__device__ __forceinline__ bool warp_wait(unsigned long long* bar, uint32_t parity, uint64_t limit_ns) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, limit_ns));
}

template <class S>
__device__ __forceinline__ void set_abort(S& sm) {
  atomicOr(&g_decode_faults, LD_FAULT_WAIT_TIMEOUT);
  *reinterpret_cast<volatile int*>(&sm.abort) = 1;
}

template <class S>
__device__ __forceinline__ bool aborted(const S& sm) { return *reinterpret_cast<const volatile int*>(&sm.abort) != 0; }

// Everything the producer needs to issue one item, resolved ahead of time by one lane.
struct ItemPlan {
  int kind;
  int src;
  int bos;
  int n;
  int dst[kMaxTokens];
  float decay[kMaxTokens];
  float beta[kMaxTokens];
};

// Resolves an item's source slot, token range, destination slots and gates (the validity rules of
// the reference kernel, gdn_decode.cu:150-168 and :303-316).  Items past the end plan as kSkip.
__device__ ItemPlan plan_item(const DecodeArgs& p, int64_t item) {
  ItemPlan plan;
  plan.kind = kSkip;
  plan.src = 0;
  plan.bos = 0;
  plan.n = 0;
#pragma unroll
  for (int t = 0; t < kMaxTokens; ++t) {
    plan.dst[t] = 0;
    plan.decay[t] = 0.0f;
    plan.beta[t] = 0.0f;
  }
  if (item >= p.total_items) return plan;
  const int HV = p.num_v_heads;
  const int W = p.width;
  const int request = static_cast<int>(item / HV);
  const int head = static_cast<int>(item - static_cast<int64_t>(request) * HV);
  const int bos = p.cu[request];
  const int eos = p.cu[request + 1];
  const int acc = p.accepted[request];
  const int n = eos - bos;
  plan.bos = bos;
  plan.n = n;
  if (n <= 0) return plan;
  if (bos < 0 || static_cast<int64_t>(eos) > p.n_tokens) {
    atomicOr(&g_decode_faults, LD_FAULT_DECODE_TOKENS);
    return plan;
  }
  const int src = (acc >= 1 && acc <= W) ? p.indices[request * W + acc - 1] : 0;
  if (src <= 0 || n > W || src >= p.n_slots) {
    if (n > W) atomicOr(&g_decode_faults, LD_FAULT_DECODE_TOKENS);
    if (src >= p.n_slots) atomicOr(&g_decode_faults, LD_FAULT_DECODE_SLOT_RANGE);
    plan.kind = kZero;
    return plan;
  }
  plan.kind = kRun;
  plan.src = src;
#pragma unroll
  for (int t = 0; t < kMaxTokens; ++t) {
    if (t < n) {
      int dst = p.indices[request * W + t];
      if (dst >= p.n_slots) {
        atomicOr(&g_decode_faults, LD_FAULT_DECODE_SLOT_RANGE);
        dst = 0;
      }
      plan.dst[t] = dst;
      token_gates(p, bos + t, head, plan.decay[t], plan.beta[t]);
    }
  }
  return plan;
}

// The producer's k-th item, once its rows have landed: the q and k norms of its tokens (the
// reduction every consumer warp would otherwise repeat), then the stage's `ready` arrival.
// Returns false when the wait for the rows gave up.
template <class S>
__device__ bool publish_norms(const DecodeArgs& p, S& sm, int k, int lane) {
  constexpr int kStates = S::kStateStages;
  constexpr int kActs = S::kActStages;
  const int s = k % kStates;
  const int a = k % kActs;
  if (!warp_wait(&sm.full[s], (k / kStates) & 1, p.wait_ns)) {
    if (lane == 0) set_abort(sm);
    return false;
  }
  ItemInfo& info = sm.act[a].info;
  if (info.kind == kRun) {
    for (int t = 0; t < info.n; ++t) {
      const uint2 kr = *reinterpret_cast<const uint2*>(&sm.act[a].k[t][4 * lane]);
      const uint2 qr = *reinterpret_cast<const uint2*>(&sm.act[a].q[t][4 * lane]);
      const float k0 = bf16_lo(kr.x), k1 = bf16_hi(kr.x), k2 = bf16_lo(kr.y), k3 = bf16_hi(kr.y);
      const float q0 = bf16_lo(qr.x), q1 = bf16_hi(qr.x), q2 = bf16_lo(qr.y), q3 = bf16_hi(qr.y);
      const float k_sq = warp_sum(k0 * k0 + k1 * k1 + k2 * k2 + k3 * k3);
      const float q_sq = warp_sum(q0 * q0 + q1 * q1 + q2 * q2 + q3 * q3);
      if (lane == 0) {
        info.k_inv[t] = 1.0f / sqrtf(k_sq + 1e-6f);
        info.q_inv[t] = 1.0f / sqrtf(q_sq + 1e-6f) * p.q_scale;
      }
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&sm.ready[a]);
  return true;
}

// Producer warp.  Every 32 items, lane i plans the CTA's item k + i, so the dependent metadata
// loads of 32 items share one round of memory latency; items are then issued in order from the
// planning lane's registers: wait for a free stage, publish the plan, start the TMA bulk copies.
template <class S>
__device__ void produce(const DecodeArgs& p, S& sm, int lane) {
  constexpr int kStates = S::kStateStages;
  constexpr int kActs = S::kActStages;
  const int HV = p.num_v_heads;
  const int H = p.num_k_heads;
  ItemPlan mine;
  int k = 0;
  for (int64_t item = blockIdx.x; item < p.total_items; item += gridDim.x, ++k) {
    if (aborted(sm)) break;
    const int owner = k & 31;
    if (owner == 0) mine = plan_item(p, item + static_cast<int64_t>(lane) * gridDim.x);
    const int kind = __shfl_sync(0xffffffffu, mine.kind, owner);
    const int src = __shfl_sync(0xffffffffu, mine.src, owner);
    const int bos = __shfl_sync(0xffffffffu, mine.bos, owner);
    const int n = __shfl_sync(0xffffffffu, mine.n, owner);
    int dst[kMaxTokens];
    float decay[kMaxTokens], beta[kMaxTokens];
#pragma unroll
    for (int t = 0; t < kMaxTokens; ++t) {
      dst[t] = __shfl_sync(0xffffffffu, mine.dst[t], owner);
      decay[t] = __shfl_sync(0xffffffffu, mine.decay[t], owner);
      beta[t] = __shfl_sync(0xffffffffu, mine.beta[t], owner);
    }
    const int head = static_cast<int>(item % HV);

    const int s = k % kStates;
    const int a = k % kActs;
    bool ok = true;
    if (k >= kStates) ok = warp_wait(&sm.empty_state[s], ((k / kStates) - 1) & 1, p.wait_ns);
    if (ok && k >= kActs) ok = warp_wait(&sm.empty_act[a], ((k / kActs) - 1) & 1, p.wait_ns);
    if (!ok) {
      if (lane == 0) set_abort(sm);
      break;
    }
    if (lane == 0) {
      ItemInfo& info = sm.act[a].info;
#pragma unroll
      for (int t = 0; t < kMaxTokens; ++t) {
        info.dst[t] = dst[t];
        info.decay[t] = decay[t];
        info.beta[t] = beta[t];
      }
      info.kind = kind;
      info.n = n;
      info.bos = bos;
      if (kind == kRun) {
        using State = typename S::State;
        constexpr uint32_t kStateBytes = kHeadElems * sizeof(State);
        mbar_arrive_expect_tx(&sm.full[s], kStateBytes + n * 4 * kRowBytes + p.extra_tx);
        const State* src_head =
            state_base<State>(p) + static_cast<int64_t>(src) * p.slot_stride + static_cast<int64_t>(head) * kHeadElems;
        // Four pieces, starting at a per-SM quarter (see store_tile).
        for (int q = 0; q < 4; ++q) {
          const int piece = (q + static_cast<int>(blockIdx.x)) & 3;
          if constexpr (S::kStatesReadOnce) {
            bulk_load_once(sm.state[s] + piece * (kHeadElems / 4), src_head + piece * (kHeadElems / 4),
                           kStateBytes / 4, &sm.full[s]);
          } else {
            bulk_load(sm.state[s] + piece * (kHeadElems / 4), src_head + piece * (kHeadElems / 4), kStateBytes / 4,
                      &sm.full[s]);
          }
        }
        const int key_head = head / p.heads_ratio;
        for (int t = 0; t < n; ++t) {
          const int64_t token = bos + t;
          const __nv_bfloat16* row = p.qkv + token * p.qkv_row;
          bulk_load(sm.act[a].q[t], row + key_head * kDim, kRowBytes, &sm.full[s]);
          bulk_load(sm.act[a].k[t], row + (H + key_head) * kDim, kRowBytes, &sm.full[s]);
          bulk_load(sm.act[a].v[t], row + (2 * H + head) * kDim, kRowBytes, &sm.full[s]);
          bulk_load(sm.act[a].z[t], p.gate + token * p.gate_row + head * kDim, kRowBytes, &sm.full[s]);
        }
      } else {
        mbar_arrive(&sm.full[s]);
      }
    }
    __syncwarp();
  }
  // Drain: every bulk copy this warp issued has landed before the CTA may exit.
  if (lane == 0) {
    for (int kk = k > kStates ? k - kStates : 0; kk < k; ++kk) {
      if (!mbar_wait(&sm.full[kk % kStates], (kk / kStates) & 1, p.wait_ns)) {
        set_abort(sm);
        break;
      }
    }
  }
}

// Reads this lane's 16 columns (tile_col<kWide>) of a bf16 head row from shared memory.
template <bool kWide>
__device__ __forceinline__ void load_row_cols(const __nv_bfloat16* row, int j, float4 (&v)[kVecPerRow], float& sq) {
  if constexpr (kWide) {
#pragma unroll
    for (int h = 0; h < kVecPerRow / 2; ++h) {
      const uint4 raw = *reinterpret_cast<const uint4*>(row + 64 * h + 8 * j);
      v[2 * h] = widen_bf16x4(raw.x, raw.y);
      v[2 * h + 1] = widen_bf16x4(raw.z, raw.w);
    }
  } else {
#pragma unroll
    for (int c = 0; c < kVecPerRow; ++c) {
      const uint2 raw = *reinterpret_cast<const uint2*>(row + tile_col<false>(c, j));
      v[c] = make_float4(bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y));
    }
  }
  sq = 0.0f;
#pragma unroll
  for (int c = 0; c < kVecPerRow; ++c) sq += v[c].x * v[c].x + v[c].y * v[c].y + v[c].z * v[c].z + v[c].w * v[c].w;
}

template <int kRows, class S>
__device__ void consume(const DecodeArgs& p, S& sm, int tid) {
  constexpr int kStates = S::kStateStages;
  constexpr int kActs = S::kActStages;
  using State = typename S::State;
  constexpr int kConsumers = Tile<kRows>::kThreads;
  constexpr int kRowGroups = Tile<kRows>::kRowGroups;
  const int HV = p.num_v_heads;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int j = tid & (kLanesPerRow - 1);
  const int g = tid / kLanesPerRow;
  float w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) w[e] = load_param(p.weight, 4 * lane + e, p.weight_bf16);
  int k = 0;
  int runs = 0;
  for (int64_t item = blockIdx.x; item < p.total_items; item += gridDim.x, ++k) {
    const int s = k % kStates;
    const int a = k % kActs;
    if (!warp_wait(&sm.full[s], (k / kStates) & 1, p.wait_ns)) {
      if (lane == 0) set_abort(sm);
      break;
    }
    const ItemInfo& info = sm.act[a].info;
    const int kind = info.kind;
    const int n = info.n;
    const int64_t bos = info.bos;
    const int head = static_cast<int>(item % HV);
    if (kind != kRun) {
      if (kind == kZero) {
        for (int idx = tid; idx < n * kDim; idx += kConsumers) {
          const int64_t token = bos + idx / kDim;
          p.out[(token * HV + head) * kDim + (idx % kDim)] = __float2bfloat16_rn(0.0f);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.empty_state[s]);
        mbar_arrive(&sm.empty_act[a]);
      }
      continue;
    }

    // State ring -> registers; the stage is released as soon as every warp has its tile.
    float4 tile[kRows][kVecPerRow];
    load_tile<kRows>(sm.state[s], g, j, tile);
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty_state[s]);

    const ActStage& act = sm.act[a];
    const int buf = runs & 1;
    const int use = runs >> 1;
    // out[buf] was last read by the epilogue two run items ago.
    if (use > 0 && !warp_wait(&sm.out_empty[buf], (use - 1) & 1, p.wait_ns)) {
      if (lane == 0) set_abort(sm);
      break;
    }
    float* o_buf = &sm.out[buf][0][0];
    const int64_t head_offset = static_cast<int64_t>(head) * kHeadElems;
    for (int t = 0; t < n; ++t) {
      float4 kv[kVecPerRow], qv[kVecPerRow];
      float k_sq, q_sq;
      load_row_cols<false>(act.k[t], j, kv, k_sq);
      load_row_cols<false>(act.q[t], j, qv, q_sq);
      // L2 norms in fp32 as gdn.py:98-99; q then scaled by K^-1/2 as gdn.py:101.
      k_sq = row_sum(k_sq);
      q_sq = row_sum(q_sq);
      const float k_inv = 1.0f / sqrtf(k_sq + 1e-6f);
      const float q_inv = 1.0f / sqrtf(q_sq + 1e-6f);
#pragma unroll
      for (int c = 0; c < kVecPerRow; ++c) {
        kv[c] = make_float4(kv[c].x * k_inv, kv[c].y * k_inv, kv[c].z * k_inv, kv[c].w * k_inv);
        qv[c] = make_float4(qv[c].x * q_inv * p.q_scale, qv[c].y * q_inv * p.q_scale,
                            qv[c].z * q_inv * p.q_scale, qv[c].w * q_inv * p.q_scale);
      }
      float vrow[kRows], o[kRows];
#pragma unroll
      for (int i = 0; i < kRows; ++i) vrow[i] = __bfloat162float(act.v[t][g + i * kRowGroups]);
      tile_step<kRows>(tile, kv, qv, vrow, info.decay[t], info.beta[t], o);
      if (j == 0) {
#pragma unroll
        for (int i = 0; i < kRows; ++i) {
          o_buf[t * kDim + g + i * kRowGroups] = __bfloat162float(__float2bfloat16_rn(o[i]));
        }
      }
      const int dst = info.dst[t];
      if (dst > 0) {
        store_tile<kRows>(state_base<State>(p) + static_cast<int64_t>(dst) * p.slot_stride + head_offset, g, j, tile);
      }
    }
    // Token et's gated RMSNorm runs on warp et (rotating it over the warps from item to item cost
    // 175 -> 192 us on config 2: with the HBM-bound fp32 pool the first warps have slack).
    const int et = warp;
    float z[4] = {0.f, 0.f, 0.f, 0.f};
    if (et < n) {
      const uint2 raw = *reinterpret_cast<const uint2*>(&act.z[et][4 * lane]);
      z[0] = bf16_lo(raw.x);
      z[1] = bf16_hi(raw.x);
      z[2] = bf16_lo(raw.y);
      z[3] = bf16_hi(raw.y);
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&sm.empty_act[a]);
      mbar_arrive(&sm.out_full[buf]);
    }
    if (et < n) {
      if (!warp_wait(&sm.out_full[buf], use & 1, p.wait_ns)) {  // every row's output of this item is in o_buf
        if (lane == 0) set_abort(sm);
        break;
      }
      gated_rmsnorm_store<true>(o_buf + et * kDim, z, w, p.eps, lane, p.out + ((bos + et) * HV + head) * kDim);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.out_empty[buf]);
    ++runs;
  }
}

// Block: Tile<kRows>::kThreads consumer threads followed by one producer warp, one CTA per SM.
// The register cap keeps the block launchable: its 9 warps are spread over the SM's four 16 K-register
// sub-partitions (at most 3 warps each), which allows 168 registers per thread.
template <int kRows>
__global__ void __maxnreg__(168) gdn_decode_stream_kernel(const DecodeArgs p) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  constexpr int kConsumers = Tile<kRows>::kThreads;
  constexpr int kConsumerWarps = kConsumers / 32;
  using S = Smem;
  constexpr int kStates = S::kStateStages;
  constexpr int kActs = S::kActStages;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kStates; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty_state[s], kConsumerWarps);
    }
    for (int a = 0; a < kActs; ++a) mbar_init(&sm.empty_act[a], kConsumerWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.out_full[b], kConsumerWarps);
      mbar_init(&sm.out_empty[b], kConsumerWarps);
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  if (tid >= kConsumers) {
    produce(p, sm, tid & 31);
  } else {
    consume<kRows, S>(p, sm, tid);
  }
}

// ------------------------------------------------------------------------------------------
// One-token decode on a bf16 pool: two items in flight per CTA.
//
// With half the state bytes per item, the per-item work of the consumer warps (a dependent chain
// of smem loads, two row reductions and the stores) is the bound rather than HBM, and a register
// tile of 64 fp32 values per thread leaves room for only 8 consumer warps.  Here each thread keeps
// its 4 x 16 state values packed as bf16 pairs (32 registers instead of 64) and widens them twice,
// once for S k and once for the update, S q and the stores; the bf16 k and q rows stay packed too,
// with their L2 norms folded into the reductions and the update (o = q_scale / |q| sum S' q,
// pred = sum (decay S) k / |k|, S' = decay S + (beta (v - pred) / |k|) k).  That frees enough
// registers for two groups of 8 consumer warps, each taking every other item of the CTA's ring, so
// one group's reductions and stores overlap the other's.  The producer warp and the ring are those
// of the streaming kernel (TMA bulk copies, producer-side q / k norms).
// ------------------------------------------------------------------------------------------
namespace b16 {

constexpr int kGroups = 2;
constexpr int kGroupWarps = 8;
constexpr int kGroupThreads = kGroupWarps * 32;          // 256: one Tile<4> per group
constexpr int kThreads = kGroups * kGroupThreads + 64;   // + producer warp + norm warp
constexpr int kRows = 4;
constexpr int kRowGroups = Tile<kRows>::kRowGroups;      // 32

struct ActStage1 {
  __nv_bfloat16 q[1][kDim];
  __nv_bfloat16 k[1][kDim];
  __nv_bfloat16 v[1][kDim];
  __nv_bfloat16 z[1][kDim];
  ItemInfo info;
};

// The producer's view (produce() / publish_norms()) plus per-group output buffers.  The producer
// only issues copies (it never waits for data); a norm warp of its own publishes each item's q / k
// norms on `ready` as soon as the item lands (norm_loop).
struct Smem {
  using State = __nv_bfloat16;
  static constexpr int kStateStages = 6;
  static constexpr int kActStages = 8;
  // State loads with an L2 evict-first policy and streaming state stores (RowWords::store): 95.6 ->
  // 93.8 us on config 2 (B200); either alone measured 95.7 (stores) and 96.2 us (loads).
  static constexpr bool kStatesReadOnce = true;
  __nv_bfloat16 state[kStateStages][kHeadElems];
  ActStage1 act[kActStages];
  float out[kGroups][2][kDim];
  unsigned long long full[kStateStages];
  unsigned long long empty_state[kStateStages];
  unsigned long long empty_act[kActStages];
  unsigned long long ready[kActStages];
  unsigned long long out_full[kGroups][2];
  unsigned long long out_empty[kGroups][2];
  int abort;
};
static_assert(sizeof(Smem) <= 227 * 1024, "the bf16 ring must fit one CTA's shared memory");

// Widens bf16 pair word w into (lo, hi) fp32.
__device__ __forceinline__ float2 widen2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// The same, widened again at each use: volatile, so that the compiler neither hoists the widened
// k and q words (reused by every row) out of the row loop nor keeps the decayed state of the first
// pass alive into the second -- either would hold 32 or 64 more fp32 values in registers.
__device__ __forceinline__ float2 widen2_each(uint32_t w) {
  uint32_t lo, hi;
  asm volatile("shl.b32 %0, %2, 16;\n\tand.b32 %1, %2, 0xffff0000;" : "=r"(lo), "=r"(hi) : "r"(w));
  return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}

// One thread's 16 columns of one state row, as bf16 pairs: loaded from the stage, widened for the
// two row products, and replaced by the updated row rounded to bf16.
struct RowWords {
  uint4 w[2];

  __device__ __forceinline__ void load(const __nv_bfloat16* row) {
    w[0] = *reinterpret_cast<const uint4*>(row);
    w[1] = *reinterpret_cast<const uint4*>(row + 64);
  }

  // Partial sum of (decay S) k over the thread's columns (k: the raw bf16 row).
  __device__ __forceinline__ float decayed_dot(float2 decay2, const uint4 (&kr)[2]) const {
    float2 acc_a = make_float2(0.0f, 0.0f), acc_b = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sw[4] = {w[h].x, w[h].y, w[h].z, w[h].w};
      const uint32_t kw[4] = {kr[h].x, kr[h].y, kr[h].z, kr[h].w};
      acc_a = fma2(mul2(widen2(sw[0]), decay2), widen2_each(kw[0]), acc_a);
      acc_b = fma2(mul2(widen2(sw[1]), decay2), widen2_each(kw[1]), acc_b);
      acc_a = fma2(mul2(widen2(sw[2]), decay2), widen2_each(kw[2]), acc_a);
      acc_b = fma2(mul2(widen2(sw[3]), decay2), widen2_each(kw[3]), acc_b);
    }
    return (acc_a.x + acc_a.y) + (acc_b.x + acc_b.y);
  }

  // S' = decay S + dk k (kept as bf16 pairs) and the partial sum of S' q.
  __device__ __forceinline__ float update(float2 decay2, float dk, const uint4 (&kr)[2], const uint4 (&qr)[2]) {
    const float2 dk2 = make_float2(dk, dk);
    float2 acc_a = make_float2(0.0f, 0.0f), acc_b = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sw[4] = {w[h].x, w[h].y, w[h].z, w[h].w};
      const uint32_t kw[4] = {kr[h].x, kr[h].y, kr[h].z, kr[h].w};
      const uint32_t qw[4] = {qr[h].x, qr[h].y, qr[h].z, qr[h].w};
      uint32_t nw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 upd = fma2(widen2_each(kw[e]), dk2, mul2(widen2_each(sw[e]), decay2));
        if (e & 1) {
          acc_b = fma2(upd, widen2_each(qw[e]), acc_b);
        } else {
          acc_a = fma2(upd, widen2_each(qw[e]), acc_a);
        }
        nw[e] = pack_bf16x2(upd.x, upd.y);
      }
      w[h] = make_uint4(nw[0], nw[1], nw[2], nw[3]);
    }
    return (acc_a.x + acc_a.y) + (acc_b.x + acc_b.y);
  }

  // Streaming stores (st.global.cs), with the evict-first state loads of this kernel's ring.
  __device__ __forceinline__ void store(__nv_bfloat16* row) const {
    __stcs(reinterpret_cast<uint4*>(row), w[0]);
    __stcs(reinterpret_cast<uint4*>(row + 64), w[1]);
  }
};

__device__ void consume(const DecodeArgs& p, Smem& sm, int group, int tid) {
  constexpr int kStates = Smem::kStateStages;
  constexpr int kActs = Smem::kActStages;
  const int HV = p.num_v_heads;
  const int lane = tid & 31;
  const int warp = tid >> 5;  // within the group
  const int j = tid & (kLanesPerRow - 1);
  const int g = tid / kLanesPerRow;
  int runs = 0;
  int k = group;
  for (int64_t item = blockIdx.x + static_cast<int64_t>(group) * gridDim.x; item < p.total_items;
       item += static_cast<int64_t>(kGroups) * gridDim.x, k += kGroups) {
    const int s = k % kStates;
    const int a = k % kActs;
    if (!warp_wait(&sm.full[s], (k / kStates) & 1, p.wait_ns) || !warp_wait(&sm.ready[a], (k / kActs) & 1, p.wait_ns)) {
      if (lane == 0) set_abort(sm);
      break;
    }
    const ItemInfo& info = sm.act[a].info;
    const int kind = info.kind;
    const int64_t bos = info.bos;
    const int head = static_cast<int>(item % HV);
    if (kind != kRun) {
      if (kind == kZero) {
        for (int idx = tid; idx < info.n * kDim; idx += kGroupThreads) {
          const int64_t token = bos + idx / kDim;
          p.out[(token * HV + head) * kDim + (idx % kDim)] = __float2bfloat16_rn(0.0f);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.empty_state[s]);
        mbar_arrive(&sm.empty_act[a]);
      }
      continue;
    }
    const ActStage1& act = sm.act[a];
    uint4 kr[2], qr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      kr[h] = *reinterpret_cast<const uint4*>(&act.k[0][64 * h + 8 * j]);
      qr[h] = *reinterpret_cast<const uint4*>(&act.q[0][64 * h + 8 * j]);
    }
    const float decay = info.decay[0], beta = info.beta[0];
    const float k_inv = info.k_inv[0], q_inv = info.q_inv[0];
    const float2 decay2 = make_float2(decay, decay);
    // This thread's rows g + 32 i, columns {64 h + 8 j .. + 7}, of the staged head and of the
    // destination head, one row at a time from its stage words to its stored words, starting at row
    // set blockIdx.x mod 4 (see store_tile).  Only 8 state words are live at a time: the 16 warps of
    // the two groups hide each other's latencies instead of a 64-value tile per thread.
    const __nv_bfloat16* srow = sm.state[s] + g * kDim + 8 * j;
    const int dst = info.dst[0];
    __nv_bfloat16* out_rows = dst > 0 ? state_base<__nv_bfloat16>(p) + static_cast<int64_t>(dst) * p.slot_stride +
                                            static_cast<int64_t>(head) * kHeadElems + g * kDim + 8 * j
                                      : nullptr;
    const int buf = runs & 1;
    const int use = runs >> 1;
    if (use > 0 && !warp_wait(&sm.out_empty[group][buf], (use - 1) & 1, p.wait_ns)) {
      if (lane == 0) set_abort(sm);
      break;
    }
    float* o_buf = sm.out[group][buf];
    const int first = blockIdx.x % kRows;
#pragma unroll 1
    for (int step = 0; step < kRows; ++step) {
      const int i = (first + step) % kRows;
      RowWords row;
      row.load(srow + i * kRowGroups * kDim);
      const float pred = row_sum(row.decayed_dot(decay2, kr)) * k_inv;
      const float v = __bfloat162float(act.v[0][g + i * kRowGroups]);
      // beta (v - pred) / |k|: the delta with k's norm folded in.
      const float o = row_sum(row.update(decay2, (v - pred) * beta * k_inv, kr, qr)) * q_inv;
      if (out_rows != nullptr) row.store(out_rows + i * kRowGroups * kDim);
      if (j == 0) o_buf[g + i * kRowGroups] = __bfloat162float(__float2bfloat16_rn(o));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty_state[s]);  // this warp's reads of the stage are done
    // The gated RMSNorm of the item's token runs on one warp of the group, rotating from item to item.
    const bool epilogue = warp == runs % kGroupWarps;
    float z[4] = {0.f, 0.f, 0.f, 0.f};
    float w[4] = {0.f, 0.f, 0.f, 0.f};
    if (epilogue) {
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = load_param(p.weight, 4 * lane + e, p.weight_bf16);
      const uint2 raw = *reinterpret_cast<const uint2*>(&act.z[0][4 * lane]);
      z[0] = bf16_lo(raw.x);
      z[1] = bf16_hi(raw.x);
      z[2] = bf16_lo(raw.y);
      z[3] = bf16_hi(raw.y);
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&sm.empty_act[a]);
      mbar_arrive(&sm.out_full[group][buf]);
    }
    if (epilogue) {
      if (!warp_wait(&sm.out_full[group][buf], use & 1, p.wait_ns)) {
        if (lane == 0) set_abort(sm);
        break;
      }
      gated_rmsnorm_store<true>(o_buf, z, w, p.eps, lane, p.out + (bos * HV + head) * kDim);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.out_empty[group][buf]);
    ++runs;
  }
}

// Norm warp: for each of the CTA's items in order, wait until it lands, reduce its q and k norms and
// arrive on the stage's `ready` barrier.  Measured on B200 (config 2, bf16 pool): done by the
// producer after issuing the next item, every issue waited for the previous item's copies, so at
// most two items were in flight (one item issued per 2.1 us against 1.8 us of work per item).
__device__ void norm_loop(const DecodeArgs& p, Smem& sm, int lane) {
  int k = 0;
  for (int64_t item = blockIdx.x; item < p.total_items; item += gridDim.x, ++k) {
    if (aborted(sm) || !publish_norms(p, sm, k, lane)) break;
  }
}

// Block: two groups of 8 consumer warps, the producer warp and the norm warp; one CTA per SM.
__global__ void __launch_bounds__(kThreads, 1) gdn_decode_b16_kernel(const DecodeArgs p) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < Smem::kStateStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty_state[s], kGroupWarps);
    }
    for (int a = 0; a < Smem::kActStages; ++a) {
      mbar_init(&sm.empty_act[a], kGroupWarps);
      mbar_init(&sm.ready[a], 1);
    }
    for (int grp = 0; grp < kGroups; ++grp) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&sm.out_full[grp][b], kGroupWarps);
        mbar_init(&sm.out_empty[grp][b], kGroupWarps);
      }
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  if (tid >= kGroups * kGroupThreads + 32) {
    norm_loop(p, sm, tid & 31);
  } else if (tid >= kGroups * kGroupThreads) {
    produce(p, sm, tid & 31);
  } else {
    consume(p, sm, tid / kGroupThreads, tid % kGroupThreads);
  }
}

}  // namespace b16

}  // namespace stream

bool aligned(const void* ptr, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(ptr) % bytes) == 0; }

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int sms = 0;
  bool stream_ready = false;
};

// Per-device launch facts: SM count, and the shared-memory opt-in of the streaming kernel.
int device_info(DeviceInfo& out) {
  static std::mutex mutex;
  static DeviceInfo infos[kMaxDevices];
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (device < 0 || device >= kMaxDevices) return set_error(LD_ERR_INVALID, "device index %d unsupported", device);
  std::lock_guard<std::mutex> lock(mutex);
  DeviceInfo& info = infos[device];
  if (!info.stream_ready) {
    err = cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "SM count: %s", cudaGetErrorString(err));
    err = cudaFuncSetAttribute(stream::gdn_decode_stream_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(sizeof(stream::Smem)));
    if (err == cudaSuccess) {
      err = cudaFuncSetAttribute(stream::b16::gdn_decode_b16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(stream::b16::Smem)));
    }
    if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "shared-memory opt-in: %s", cudaGetErrorString(err));
    info.stream_ready = true;
  }
  out = info;
  return LD_OK;
}

std::atomic<int> g_kernel_override{LD_DECODE_KERNEL_AUTO};
constexpr uint64_t kDefaultWaitNs = 1000000000ull;  // 1 s bound on every in-kernel wait
std::atomic<uint64_t> g_wait_ns{kDefaultWaitNs};
std::atomic<uint32_t> g_extra_tx{0};

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

namespace ldb {

// Host-side checks of ld_decode's arguments and the kernel argument block (shared with the
// fused conv entry point).  args.total_items stays 0 when there is nothing to launch.
int prepare_decode(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride,
                   const void* b, int64_t b_row_stride, const float* a_log, const void* dt_bias,
                   int dt_bias_dtype, const int32_t* indices, int64_t n_requests, int64_t width,
                   const int32_t* cu, const int32_t* accepted, void* state, int64_t n_slots,
                   int64_t slot_stride, const void* gate, int64_t gate_row_stride,
                   const void* weight, int weight_dtype, void* out, int64_t n_tokens,
                   int64_t num_k_heads, int64_t num_v_heads, float eps, bool state_bf16, DecodeArgs& args) {
  args.total_items = 0;
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
  if (4 * n_requests * num_v_heads > 0x7fffffffLL) {
    return set_error(LD_ERR_INVALID, "4 * n_requests * num_v_heads exceeds the grid limit");
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
  if (!aligned(state, 16) || slot_stride % (state_bf16 ? 8 : 4) != 0) {
    return set_error(LD_ERR_INVALID, "state must be 16-byte aligned with a slot stride divisible by %d",
                     state_bf16 ? 8 : 4);
  }
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
  args.state = state_bf16 ? nullptr : static_cast<float*>(state);
  args.state_bf16 = state_bf16 ? static_cast<__nv_bfloat16*>(state) : nullptr;
  args.n_slots = n_slots;
  args.slot_stride = slot_stride;
  args.gate = static_cast<const __nv_bfloat16*>(gate);
  args.gate_row = gate_row_stride;
  args.weight = weight;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.n_tokens = n_tokens;
  args.total_items = n_requests * num_v_heads;
  args.width = static_cast<int>(width);
  args.num_k_heads = static_cast<int>(num_k_heads);
  args.num_v_heads = static_cast<int>(num_v_heads);
  args.heads_ratio = static_cast<int>(num_v_heads / num_k_heads);
  args.dt_bias_bf16 = dt_bias_dtype == LD_DTYPE_BF16;
  args.weight_bf16 = weight_dtype == LD_DTYPE_BF16;
  // K^-1/2 evaluated in double and rounded once, as torch scales an fp32 tensor by a Python float.
  args.q_scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(LD_HEAD_DIM)));
  args.eps = eps;
  args.wait_ns = g_wait_ns.load(std::memory_order_relaxed);
  args.extra_tx = g_extra_tx.load(std::memory_order_relaxed);
  args.prefetch_stride = 0;
  return ok();
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
  DecodeArgs args;
  const int rc = prepare_decode(qkv, qkv_row_stride, a, a_row_stride, b, b_row_stride, a_log, dt_bias, dt_bias_dtype,
                                indices, n_requests, width, cu, accepted, state, n_slots, slot_stride, gate,
                                gate_row_stride, weight, weight_dtype, out, n_tokens, num_k_heads, num_v_heads, eps,
                                false, args);
  if (rc != LD_OK || args.total_items == 0) return rc;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // TMA bulk copies need 16-byte aligned sources: qkv and gate rows must start on 16 bytes.
  const bool bulk_ok = aligned(qkv, 16) && qkv_row_stride % 8 == 0 && aligned(gate, 16) &&
                       gate_row_stride % 8 == 0 && aligned(out, 8);
  int variant = bulk_ok ? g_kernel_override.load(std::memory_order_relaxed) : LD_DECODE_KERNEL_ROWREG;
  DeviceInfo info;
  if (variant != LD_DECODE_KERNEL_ROWREG) {
    const int rc = device_info(info);
    if (rc != LD_OK) return rc;
  }
  if (variant == LD_DECODE_KERNEL_AUTO) {
    // Measured on B200 (CUDA-graph replay, HV=32 and 48, T=1 launches of 288..8192 items, and
    // BASELINE configs 2 and 3): the one-CTA-per-item kernel is fastest for multi-token verify,
    // whose four state writes per item favour its two resident CTAs per SM, and for one-token
    // launches up to about 9 (request, head) items per SM (1,184 items: 26.5 vs 26.9 us); the
    // streaming kernel from there on (1,472 items: 33.7 vs 36.0 us; config 2: 175 vs 188 us).
    variant = (width == 1 && args.total_items >= kStreamItemsPerSm * info.sms) ? LD_DECODE_KERNEL_STREAM
                                                                              : LD_DECODE_KERNEL_ROWREG;
  }
  cudaError_t err;
  if (variant == LD_DECODE_KERNEL_STREAM) {
    const dim3 grid(static_cast<unsigned int>(std::min<int64_t>(args.total_items, info.sms)));
    err = ldb::launch(stream::gdn_decode_stream_kernel<4>, grid, dim3(Tile<4>::kThreads + 32),
                      sizeof(stream::Smem), s, 1, args);
  } else {
    const bool vec_act = aligned(qkv, 8) && qkv_row_stride % 4 == 0 && aligned(gate, 8) &&
                         gate_row_stride % 4 == 0 && aligned(out, 8);
    const dim3 grid(static_cast<unsigned int>(args.total_items));
    if (vec_act) {
      err = ldb::launch(gdn_decode_rowreg_kernel<true, float>, grid, dim3(Tile<4>::kThreads), 0, s, 1, args);
    } else {
      err = ldb::launch(gdn_decode_rowreg_kernel<false, float>, grid, dim3(Tile<4>::kThreads), 0, s, 1, args);
    }
  }
  if (err != cudaSuccess) {
    return set_error(LD_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(err));
  }
  return ok();
}

extern "C" int ld_decode_wait_test(int64_t limit_ns, int32_t extra_tx_bytes) {
  if (limit_ns < 0 || extra_tx_bytes < 0 || extra_tx_bytes > 1024) {
    return ldb::set_error(LD_ERR_INVALID, "ld_decode_wait_test: limit_ns >= 0 and 0 <= extra_tx_bytes <= 1024");
  }
  ldb::g_wait_ns.store(limit_ns == 0 ? ldb::kDefaultWaitNs : static_cast<uint64_t>(limit_ns));
  ldb::g_extra_tx.store(static_cast<uint32_t>(extra_tx_bytes));
  return ldb::ok();
}

extern "C" int ld_decode_kernel_override(int variant) {
  if (variant < LD_DECODE_KERNEL_AUTO || variant > LD_DECODE_KERNEL_STREAM) {
    return ldb::set_error(-LD_ERR_INVALID, "unknown decode kernel variant %d", variant);
  }
  return ldb::g_kernel_override.exchange(variant);
}

namespace ldb {

int check_decode_args(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride, const void* b,
                      int64_t b_row_stride, const float* a_log, const void* dt_bias, int dt_bias_dtype,
                      const int32_t* indices, int64_t n_requests, int64_t width, const int32_t* cu,
                      const int32_t* accepted, float* state, int64_t n_slots, int64_t slot_stride, const void* gate,
                      int64_t gate_row_stride, const void* weight, int weight_dtype, void* out, int64_t n_tokens,
                      int64_t num_k_heads, int64_t num_v_heads, float eps) {
  DecodeArgs args;
  return prepare_decode(qkv, qkv_row_stride, a, a_row_stride, b, b_row_stride, a_log, dt_bias, dt_bias_dtype, indices,
                        n_requests, width, cu, accepted, state, n_slots, slot_stride, gate, gate_row_stride, weight,
                        weight_dtype, out, n_tokens, num_k_heads, num_v_heads, eps, false, args);
}

}  // namespace ldb

extern "C" int ld_decode_bf16_state(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride,
                                    const void* b, int64_t b_row_stride, const float* a_log, const void* dt_bias,
                                    int dt_bias_dtype, const int32_t* indices, int64_t n_requests, int64_t width,
                                    const int32_t* cu, const int32_t* accepted, void* state, int64_t n_slots,
                                    int64_t slot_stride, const void* gate, int64_t gate_row_stride,
                                    const void* weight, int weight_dtype, void* out, int64_t n_tokens,
                                    int64_t num_k_heads, int64_t num_v_heads, float eps, void* stream) {
  using namespace ldb;
  DecodeArgs args;
  int rc = prepare_decode(qkv, qkv_row_stride, a, a_row_stride, b, b_row_stride, a_log, dt_bias, dt_bias_dtype,
                          indices, n_requests, width, cu, accepted, state, n_slots, slot_stride, gate, gate_row_stride,
                          weight, weight_dtype, out, n_tokens, num_k_heads, num_v_heads, eps, true, args);
  if (rc != LD_OK || args.total_items == 0) return rc;
  DeviceInfo info;
  rc = device_info(info);
  if (rc != LD_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // One-token launches of at least 7 items per SM run the two-group streaming kernel, smaller ones
  // and multi-token launches the one-CTA-per-item kernel.  Measured on B200 (HV=32, CUDA-graph
  // replay, T=1): 1,024 items 17.2 (one CTA per item) vs 17.0 us, 2,048 items 32.4 vs 28.7 us,
  // 4,096 items 72.6 vs 54.3 us; at T=4 (config 3) 71.2 us against 75.2 us for a multi-token form
  // of the streaming kernel, which was not kept.
  const bool bulk_ok = aligned(qkv, 16) && qkv_row_stride % 8 == 0 && aligned(gate, 16) &&
                       gate_row_stride % 8 == 0 && aligned(out, 8);
  const int forced = g_kernel_override.load(std::memory_order_relaxed);
  const bool streaming = bulk_ok && width == 1 && (forced == LD_DECODE_KERNEL_STREAM ||
                                     (forced != LD_DECODE_KERNEL_ROWREG && width == 1 &&
                                      args.total_items >= kStreamItemsPerSmBf16 * info.sms));
  cudaError_t err;
  if (streaming) {
    const dim3 grid(static_cast<unsigned int>(std::min<int64_t>(args.total_items, info.sms)));
    err = ldb::launch(stream::b16::gdn_decode_b16_kernel, grid, dim3(stream::b16::kThreads),
                      sizeof(stream::b16::Smem), s, 1, args);
  } else {
    const bool vec_act = aligned(qkv, 8) && qkv_row_stride % 4 == 0 && aligned(gate, 8) &&
                         gate_row_stride % 4 == 0 && aligned(out, 8);
    const dim3 grid(static_cast<unsigned int>(args.total_items));
    // Multi-token verify warms L2 with the next wave's first reads (two resident blocks per SM).
    // Measured on B200, config 3 on a bf16 pool: 71.7 us without, 69.0 us with the source heads,
    // 66.0 us with the heads and the q / k / v / gate rows (70.5 us two waves ahead).  On an fp32
    // pool, whose launch is HBM-bound, the heads cost 112.1 -> 117.6 us and the rows alone gain
    // nothing measurable (111.6 -> 111.4 us), so fp32 launches do not prefetch.
    args.prefetch_stride = width > 1 ? 2 * static_cast<int64_t>(info.sms) : 0;
    err = vec_act ? ldb::launch(gdn_decode_rowreg_kernel<true, __nv_bfloat16>, grid, dim3(Tile<4>::kThreads), 0, s, 1,
                                args)
                  : ldb::launch(gdn_decode_rowreg_kernel<false, __nv_bfloat16>, grid, dim3(Tile<4>::kThreads), 0, s,
                                1, args);
  }
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(err));
  return ok();
}
