// Causal depthwise conv1d state update of the GDN layer's q, k, v channels, and the conv + decode
// entry point.
//
// Semantics are vLLM's causal_conv1d_update as the reference's vLLM layer calls it
// (python/lightdelta/integration/vllm_layer.py:161-172 for speculative decode with
// num_accepted_tokens / query_start_loc, :199-207 for one-token decode), the step that produces
// the decode's q, k and v.  Per request r with conv slot c = slots[r] (skipped when c is the null
// block 0), tokens [cu[r], cu[r+1]) (n of them), window start o = accepted[r] - 1 and width w:
//   y_t = silu(bias + sum_j window_j * W[:, j] + x_t * W[:, w-1]), the window shifting by one
//         token after each step (fp32 accumulator from the bias; each bf16 x bf16 product rounded
//         to bf16; silu in fp32; y rounded to bf16), written over x in place;
//   the conv state positions [0, w - 2) take the window's positions [o + 1, o + w - 1), then
//   positions [w - 2, w - 2 + n) take the n inputs.
//
// One thread per (request, 8 channels) with 16-byte loads and stores where the layout allows
// (a scalar one-thread-per-channel form otherwise): a single HBM-bound pass (window, weights and
// inputs read, state and outputs written).  ld_conv_decode launches it and then the decode
// (ld_decode) on the post-conv activations; with programmatic dependent launch the decode's CTAs
// are scheduled while the conv finishes.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "launch.cuh"
#include "lightdelta_b200.h"

namespace {

__device__ uint32_t g_conv_faults;

constexpr int kThreads = 256;
constexpr int kMaxConvWidth = 4;

struct ConvUpdateArgs {
  __nv_bfloat16* x;  // [n_tokens, dim] rows x_row apart; post-conv values replace the inputs
  int64_t x_row;
  int64_t n_tokens;
  int64_t dim;
  __nv_bfloat16* state;  // element (slot, channel, position) at slot*s_slot + channel*s_dim + position*s_pos
  int64_t n_slots, s_slot, s_dim, s_pos;
  const __nv_bfloat16* weight;  // [dim, width], contiguous
  const __nv_bfloat16* bias;    // [dim] or null
  const int32_t* slots;
  int64_t slots_stride;
  const int32_t* accepted;  // null: every request's window starts at position 0
  const int32_t* cu;
  int max_tokens;  // tokens per request at most (the state holds width - 2 + max_tokens positions)
};

// silu(a) = a / (1 + exp(-a)) with the fast exponential and division intrinsics.  The result is
// rounded to bf16, so their few-ulp fp32 error changes under 1e-4 of outputs by one bf16 ulp
// (vLLM's Triton kernel also uses a fast exponential); the correctly rounded IEEE division made
// the whole config-2 update 1.75x slower (17.4 against 10.0 us per launch, back to back on B200).
__device__ __forceinline__ float silu(float a) { return __fdividef(a, 1.0f + __expf(-a)); }

template <int kWidth>
__global__ void __launch_bounds__(kThreads) conv_update_kernel(const ConvUpdateArgs p) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  const int64_t r = blockIdx.y;
  const int64_t channel = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (channel >= p.dim) return;
  const int slot = p.slots[r * p.slots_stride];
  if (slot == 0) return;  // null block
  if (slot < 0 || slot >= p.n_slots) {
    if (channel == 0) atomicOr(&g_conv_faults, LD_FAULT_CONV_SLOT_RANGE);
    return;
  }
  const int bos = p.cu[r];
  const int n = p.cu[r + 1] - bos;
  if (n <= 0) return;
  if (bos < 0 || bos + static_cast<int64_t>(n) > p.n_tokens || n > p.max_tokens) {
    if (channel == 0) atomicOr(&g_conv_faults, LD_FAULT_DECODE_TOKENS);
    return;
  }
  const int acc = p.accepted != nullptr ? p.accepted[r] : 1;
  if (acc < 1 || acc > p.max_tokens) return;  // no window position: the decode rejects the request too
  const int offset = acc - 1;

  __nv_bfloat16* cs = p.state + slot * p.s_slot + channel * p.s_dim;
  __nv_bfloat16 raw[kWidth - 1];
  float win[kWidth - 1], wt[kWidth];
#pragma unroll
  for (int q = 0; q < kWidth - 1; ++q) {
    raw[q] = cs[(offset + q) * p.s_pos];
    win[q] = __bfloat162float(raw[q]);
  }
#pragma unroll
  for (int j = 0; j < kWidth; ++j) wt[j] = __bfloat162float(p.weight[channel * kWidth + j]);
  const float bias = p.bias != nullptr ? __bfloat162float(p.bias[channel]) : 0.0f;
#pragma unroll
  for (int q = 0; q + 1 < kWidth - 1; ++q) cs[q * p.s_pos] = raw[q + 1];
  __nv_bfloat16* x = p.x + bos * p.x_row + channel;
  for (int t = 0; t < n; ++t) {
    const __nv_bfloat16 xin = x[t * p.x_row];
    const float xt = __bfloat162float(xin);
    float acc_f = bias;
#pragma unroll
    for (int j = 0; j < kWidth - 1; ++j) acc_f += __bfloat162float(__float2bfloat16_rn(win[j] * wt[j]));
    acc_f += __bfloat162float(__float2bfloat16_rn(xt * wt[kWidth - 1]));
#pragma unroll
    for (int j = 0; j + 1 < kWidth - 1; ++j) win[j] = win[j + 1];
    win[kWidth - 2] = xt;
    cs[(kWidth - 2 + t) * p.s_pos] = xin;
    x[t * p.x_row] = __float2bfloat16_rn(silu(acc_f));
  }
}

// Vector form: one thread per 8 consecutive channels, every access a 16-byte load or store --
// the window block ([8 channels][L] for a [slots, dim, L] state, [position][8 channels] rows for
// a [slots, L, dim] one), the weights [8][width], the inputs and outputs (8 channels of a token),
// and the new state.  Used when the layout allows it (16-byte aligned rows and blocks).
constexpr int kVec = 8;

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[kVec]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Each thread takes 8 consecutive channels of one request (kRequests): metadata first, then the
// window block and the inputs.  kL is the conv state length of a [slots, dim, L] state (0 for
// [slots, L, dim]) and kTokens the tokens per request at most; with them and a switch on the
// window start every index is a compile-time constant, so windows and blocks stay in registers.
constexpr int kRequests = 1;

struct VecRequest {
  int slot, bos, n, offset;
  bool live;
};

template <int kWidth, int kL, int kOffset>
__device__ __forceinline__ void window_at(const uint4 (&blk)[kL > 0 ? kL : 1], __nv_bfloat16 (&win)[kVec][kWidth - 1]) {
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(blk);
#pragma unroll
  for (int c = 0; c < kVec; ++c) {
#pragma unroll
    for (int q = 0; q < kWidth - 1; ++q) win[c][q] = e[c * kL + kOffset + q];
  }
}

template <int kWidth, int kL>
__device__ __forceinline__ void window_of(const uint4 (&blk)[kL > 0 ? kL : 1], int offset,
                                          __nv_bfloat16 (&win)[kVec][kWidth - 1]) {
  // offset <= kL - (kWidth - 1), checked on the host (L >= width - 2 + tokens, offset < tokens).
  if constexpr (kL >= kWidth - 1) {
    switch (offset) {
      case 0: window_at<kWidth, kL, 0>(blk, win); break;
      case 1: if constexpr (kL >= kWidth) window_at<kWidth, kL, 1>(blk, win); break;
      case 2: if constexpr (kL >= kWidth + 1) window_at<kWidth, kL, 2>(blk, win); break;
      default: if constexpr (kL >= kWidth + 2) window_at<kWidth, kL, 3>(blk, win); break;
    }
  }
}

template <int kWidth, int kL, int kTokens>
__global__ void __launch_bounds__(kThreads, kTokens == 1 ? 4 : 2) conv_update_vec_kernel(const ConvUpdateArgs p,
                                                                                  int64_t n_requests) {
  ldb::grid_dependency_wait();
  ldb::allow_dependent_launch();
  constexpr bool kDimFirst = kL > 0;
  constexpr int kBlk = kL > 0 ? kL : 1;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kRequests;
  const int64_t ch0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * kVec;
  if (ch0 >= p.dim) return;
  // Round 1: metadata of every request, weights and bias.
  VecRequest rq[kRequests];
  int acc[kRequests], eos[kRequests];
#pragma unroll
  for (int k = 0; k < kRequests; ++k) {
    const int64_t r = r0 + k;
    rq[k].live = r < n_requests;
    rq[k].slot = rq[k].bos = eos[k] = 0;
    acc[k] = 1;
    if (rq[k].live) {
      rq[k].slot = p.slots[r * p.slots_stride];
      rq[k].bos = p.cu[r];
      eos[k] = p.cu[r + 1];
      acc[k] = p.accepted != nullptr ? p.accepted[r] : 1;
    }
  }
  uint4 wraw4[kWidth];
#pragma unroll
  for (int piece = 0; piece < kWidth; ++piece) wraw4[piece] = reinterpret_cast<const uint4*>(p.weight + ch0 * kWidth)[piece];
  uint4 bias4 = make_uint4(0, 0, 0, 0);
  if (p.bias != nullptr) bias4 = *reinterpret_cast<const uint4*>(p.bias + ch0);
#pragma unroll
  for (int k = 0; k < kRequests; ++k) {
    if (!rq[k].live) continue;
    const int slot = rq[k].slot, bos = rq[k].bos, n = eos[k] - bos;
    rq[k].n = n;
    rq[k].offset = acc[k] - 1;
    if (slot == 0 || n <= 0) {
      rq[k].live = false;
    } else if (slot < 0 || slot >= p.n_slots) {
      if (ch0 == 0) atomicOr(&g_conv_faults, LD_FAULT_CONV_SLOT_RANGE);
      rq[k].live = false;
    } else if (bos < 0 || static_cast<int64_t>(eos[k]) > p.n_tokens || n > p.max_tokens) {
      if (ch0 == 0) atomicOr(&g_conv_faults, LD_FAULT_DECODE_TOKENS);
      rq[k].live = false;
    } else if (acc[k] < 1 || acc[k] > p.max_tokens) {
      rq[k].live = false;
    }
  }
  // Round 2: window (block) and inputs of every live request.
  uint4 blk[kRequests][kBlk];
  uint4 rows[kRequests][kWidth - 1 > 0 ? kWidth - 1 : 1];
  uint4 inputs[kRequests][kTokens];
#pragma unroll
  for (int k = 0; k < kRequests; ++k) {
    if (!rq[k].live) continue;
    const __nv_bfloat16* base = p.state + rq[k].slot * p.s_slot + ch0 * p.s_dim;
    const __nv_bfloat16* x = p.x + rq[k].bos * p.x_row + ch0;
#pragma unroll
    for (int t = 0; t < kTokens; ++t) {
      if (t < rq[k].n) inputs[k][t] = *reinterpret_cast<const uint4*>(x + t * p.x_row);
    }
    if constexpr (kDimFirst) {
#pragma unroll
      for (int piece = 0; piece < kBlk; ++piece) blk[k][piece] = reinterpret_cast<const uint4*>(base)[piece];
    } else {
#pragma unroll
      for (int q = 0; q < kWidth - 1; ++q) rows[k][q] = *reinterpret_cast<const uint4*>(base + (rq[k].offset + q) * p.s_pos);
    }
  }
  const __nv_bfloat16* wraw = reinterpret_cast<const __nv_bfloat16*>(wraw4);
  const __nv_bfloat16* braw = reinterpret_cast<const __nv_bfloat16*>(&bias4);
#pragma unroll
  for (int k = 0; k < kRequests; ++k) {
    if (!rq[k].live) continue;
    __nv_bfloat16 win[kVec][kWidth - 1];
    if constexpr (kDimFirst) {
      window_of<kWidth, kL>(blk[k], rq[k].offset, win);
    } else {
#pragma unroll
      for (int q = 0; q < kWidth - 1; ++q) {
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&rows[k][q]);
#pragma unroll
        for (int c = 0; c < kVec; ++c) win[c][q] = e[c];
      }
    }
    float w[kVec][kWidth - 1];
#pragma unroll
    for (int c = 0; c < kVec; ++c) {
#pragma unroll
      for (int q = 0; q < kWidth - 1; ++q) w[c][q] = __bfloat162float(win[c][q]);
    }
    __nv_bfloat16* x = p.x + rq[k].bos * p.x_row + ch0;
#pragma unroll
    for (int t = 0; t < kTokens; ++t) {
      if (t < rq[k].n) {
        float xt[kVec];
        unpack8(inputs[k][t], xt);
        __align__(16) __nv_bfloat16 y[kVec];
#pragma unroll
        for (int c = 0; c < kVec; ++c) {
          float acc_f = __bfloat162float(braw[c]);
#pragma unroll
          for (int j = 0; j < kWidth - 1; ++j) {
            acc_f += __bfloat162float(__float2bfloat16_rn(w[c][j] * __bfloat162float(wraw[c * kWidth + j])));
          }
          acc_f += __bfloat162float(__float2bfloat16_rn(xt[c] * __bfloat162float(wraw[c * kWidth + kWidth - 1])));
#pragma unroll
          for (int j = 0; j + 1 < kWidth - 1; ++j) w[c][j] = w[c][j + 1];
          w[c][kWidth - 2] = xt[c];
          y[c] = __float2bfloat16_rn(silu(acc_f));
        }
        *reinterpret_cast<uint4*>(x + t * p.x_row) = *reinterpret_cast<const uint4*>(y);
      }
    }
    // New state: positions [0, kWidth - 2) take window positions [offset + 1, ...), then the inputs.
    __nv_bfloat16* base = p.state + rq[k].slot * p.s_slot + ch0 * p.s_dim;
    if constexpr (kDimFirst) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(blk[k]);
#pragma unroll
      for (int c = 0; c < kVec; ++c) {
#pragma unroll
        for (int q = 0; q + 1 < kWidth - 1; ++q) e[c * kL + q] = win[c][q + 1];
#pragma unroll
        for (int t = 0; t < kTokens; ++t) {
          if (kWidth - 2 + t < kL && t < rq[k].n) {
            e[c * kL + kWidth - 2 + t] = reinterpret_cast<const __nv_bfloat16*>(&inputs[k][t])[c];
          }
        }
      }
#pragma unroll
      for (int piece = 0; piece < kBlk; ++piece) reinterpret_cast<uint4*>(base)[piece] = blk[k][piece];
    } else {
#pragma unroll
      for (int q = 0; q + 1 < kWidth - 1; ++q) {
        __align__(16) __nv_bfloat16 row[kVec];
#pragma unroll
        for (int c = 0; c < kVec; ++c) row[c] = win[c][q + 1];
        *reinterpret_cast<uint4*>(base + q * p.s_pos) = *reinterpret_cast<const uint4*>(row);
      }
#pragma unroll
      for (int t = 0; t < kTokens; ++t) {
        if (t < rq[k].n) *reinterpret_cast<uint4*>(base + (kWidth - 2 + t) * p.s_pos) = inputs[k][t];
      }
    }
  }
}

template <int kWidth, int kL>
cudaError_t launch_vec(const ConvUpdateArgs& args, int64_t n_requests, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned int>((args.dim / kVec + kThreads - 1) / kThreads),
                  static_cast<unsigned int>((n_requests + kRequests - 1) / kRequests));
  if (args.max_tokens == 1) {
    return ldb::launch(conv_update_vec_kernel<kWidth, kL, 1>, grid, dim3(kThreads), 0, stream, 1, args, n_requests);
  }
  return ldb::launch(conv_update_vec_kernel<kWidth, kL, LD_MAX_WIDTH>, grid, dim3(kThreads), 0, stream, 1, args,
                     n_requests);
}

bool aligned2(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 1u) == 0; }
bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

template <int kWidth>
cudaError_t launch_width(const ConvUpdateArgs& args, int64_t n_requests, int64_t state_len, cudaStream_t stream) {
  const bool dim_first = args.s_pos == 1 && args.s_dim == state_len;
  const bool token_first = args.s_dim == 1 && args.s_pos % kVec == 0;
  const bool vec = (dim_first || token_first) && args.dim % kVec == 0 && aligned16(args.x) && args.x_row % kVec == 0 &&
                   aligned16(args.state) && args.s_slot % kVec == 0 && aligned16(args.weight) &&
                   (args.bias == nullptr || aligned16(args.bias)) && state_len <= kMaxConvWidth - 2 + LD_MAX_WIDTH;
  if (vec && token_first) return launch_vec<kWidth, 0>(args, n_requests, stream);
  if (vec && dim_first) {
    switch (state_len) {
      case 2: if constexpr (kWidth <= 3) return launch_vec<kWidth, 2>(args, n_requests, stream); break;
      case 3: return launch_vec<kWidth, 3>(args, n_requests, stream);
      case 4: return launch_vec<kWidth, 4>(args, n_requests, stream);
      case 5: return launch_vec<kWidth, 5>(args, n_requests, stream);
      case 6: return launch_vec<kWidth, 6>(args, n_requests, stream);
      default: break;
    }
  }
  const dim3 grid(static_cast<unsigned int>((args.dim + kThreads - 1) / kThreads), static_cast<unsigned int>(n_requests));
  return ldb::launch(conv_update_kernel<kWidth>, grid, dim3(kThreads), 0, stream, 1, args);
}

int launch_conv_update(const ConvUpdateArgs& args, int64_t n_requests, int width, int64_t state_len,
                       cudaStream_t stream) {
  using ldb::set_error;
  cudaError_t err;
  switch (width) {
    case 2: err = launch_width<2>(args, n_requests, state_len, stream); break;
    case 3: err = launch_width<3>(args, n_requests, state_len, stream); break;
    default: err = launch_width<4>(args, n_requests, state_len, stream); break;
  }
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "conv update launch failed: %s", cudaGetErrorString(err));
  return ldb::ok();
}

// Host checks shared by both entry points; fills `args`.
int prepare_conv(void* x, int64_t x_row_stride, int64_t n_tokens, int64_t dim, void* conv_state, int64_t n_conv_slots,
                 int64_t conv_slot_stride, int64_t conv_dim_stride, int64_t conv_pos_stride, int64_t conv_state_len,
                 const void* conv_weight, const void* conv_bias, int64_t conv_width, const int32_t* slots,
                 int64_t slots_stride, const int32_t* accepted, const int32_t* cu, int64_t n_requests,
                 int64_t max_tokens, ConvUpdateArgs& args) {
  using ldb::set_error;
  if (conv_width < 2 || conv_width > kMaxConvWidth) {
    return set_error(LD_ERR_INVALID, "conv: kernel width must be 2 through %d", kMaxConvWidth);
  }
  if (max_tokens < 1 || max_tokens > LD_MAX_WIDTH) {
    return set_error(LD_ERR_INVALID, "conv: 1 through %d tokens per request", LD_MAX_WIDTH);
  }
  if (conv_state_len < conv_width - 2 + max_tokens) {
    return set_error(LD_ERR_INVALID, "conv: state length %lld < width - 2 + %lld tokens",
                     static_cast<long long>(conv_state_len), static_cast<long long>(max_tokens));
  }
  if (n_requests < 0 || n_tokens < 0 || dim < 1 || n_requests > 65535) {
    return set_error(LD_ERR_INVALID, "conv: need 0 <= requests <= 65535, tokens >= 0 and dim >= 1");
  }
  if (x_row_stride < dim || n_conv_slots < 1 || conv_slot_stride < 0 || conv_dim_stride < 1 || conv_pos_stride < 1 ||
      slots_stride < 1) {
    return set_error(LD_ERR_INVALID, "conv: invalid strides or slot count");
  }
  // Each request updates its window in place, so two (slot, channel, position) triples must never
  // share an element: channel and position strides must not overlap inside a slot, and slots must
  // not overlap each other.
  const bool dims_disjoint =
      conv_dim_stride >= conv_state_len * conv_pos_stride || conv_pos_stride >= dim * conv_dim_stride;
  const int64_t slot_extent = (dim - 1) * conv_dim_stride + (conv_state_len - 1) * conv_pos_stride + 1;
  if (!dims_disjoint || (n_conv_slots > 1 && conv_slot_stride < slot_extent)) {
    return set_error(LD_ERR_INVALID, "conv: the conv state's strides make slots, channels or positions overlap");
  }
  if (n_requests > 0 && (x == nullptr || conv_state == nullptr || conv_weight == nullptr || slots == nullptr ||
                         cu == nullptr)) {
    return set_error(LD_ERR_INVALID, "conv: a required pointer is NULL");
  }
  if (!aligned2(x) || !aligned2(conv_state) || !aligned2(conv_weight) || !aligned2(conv_bias)) {
    return set_error(LD_ERR_INVALID, "conv: bf16 tensors must be 2-byte aligned");
  }
  args.x = static_cast<__nv_bfloat16*>(x);
  args.x_row = x_row_stride;
  args.n_tokens = n_tokens;
  args.dim = dim;
  args.state = static_cast<__nv_bfloat16*>(conv_state);
  args.n_slots = n_conv_slots;
  args.s_slot = conv_slot_stride;
  args.s_dim = conv_dim_stride;
  args.s_pos = conv_pos_stride;
  args.weight = static_cast<const __nv_bfloat16*>(conv_weight);
  args.bias = static_cast<const __nv_bfloat16*>(conv_bias);
  args.slots = slots;
  args.slots_stride = slots_stride;
  args.accepted = accepted;
  args.cu = cu;
  args.max_tokens = static_cast<int>(max_tokens);
  return LD_OK;
}

}  // namespace

namespace ldb {

int conv_faults(uint32_t* flags, int clear) {
  uint32_t value = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&value, g_conv_faults, sizeof(value));
  if (err == cudaSuccess && clear) {
    const uint32_t zero = 0;
    err = cudaMemcpyToSymbol(g_conv_faults, &zero, sizeof(zero));
  }
  if (err != cudaSuccess) return set_error(LD_ERR_CUDA, "ld_fault_flags: %s", cudaGetErrorString(err));
  *flags = value;
  return LD_OK;
}

}  // namespace ldb

extern "C" int ld_conv_update(void* x, int64_t x_row_stride, int64_t n_tokens, int64_t dim, void* conv_state,
                              int64_t n_conv_slots, int64_t conv_slot_stride, int64_t conv_dim_stride,
                              int64_t conv_pos_stride, int64_t conv_state_len, const void* conv_weight,
                              const void* conv_bias, int64_t conv_width, const int32_t* slots, int64_t slots_stride,
                              const int32_t* accepted, const int32_t* cu, int64_t n_requests, int64_t max_tokens,
                              void* stream) {
  ConvUpdateArgs args{};
  const int rc = prepare_conv(x, x_row_stride, n_tokens, dim, conv_state, n_conv_slots, conv_slot_stride,
                              conv_dim_stride, conv_pos_stride, conv_state_len, conv_weight, conv_bias, conv_width,
                              slots, slots_stride, accepted, cu, n_requests, max_tokens, args);
  if (rc != LD_OK) return rc;
  if (n_requests == 0) return ldb::ok();
  return launch_conv_update(args, n_requests, static_cast<int>(conv_width), conv_state_len,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int ld_conv_decode(void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride, const void* b,
                              int64_t b_row_stride, const float* a_log, const void* dt_bias, int dt_bias_dtype,
                              const int32_t* indices, int64_t n_requests, int64_t width, const int32_t* cu,
                              const int32_t* accepted, float* state, int64_t n_slots, int64_t slot_stride,
                              const void* gate, int64_t gate_row_stride, const void* weight, int weight_dtype,
                              void* out, int64_t n_tokens, int64_t num_k_heads, int64_t num_v_heads, float eps,
                              void* conv_state, int64_t n_conv_slots, int64_t conv_slot_stride,
                              int64_t conv_dim_stride, int64_t conv_pos_stride, int64_t conv_state_len,
                              const void* conv_weight, const void* conv_bias, int64_t conv_width, void* stream) {
  // Every argument is checked before anything is launched, so a rejected call changes nothing.
  int rc = ldb::check_decode_args(qkv, qkv_row_stride, a, a_row_stride, b, b_row_stride, a_log, dt_bias,
                                  dt_bias_dtype, indices, n_requests, width, cu, accepted, state, n_slots,
                                  slot_stride, gate, gate_row_stride, weight, weight_dtype, out, n_tokens,
                                  num_k_heads, num_v_heads, eps);
  if (rc != LD_OK) return rc;
  if (n_requests == 0) return ldb::ok();
  ConvUpdateArgs conv{};
  const int64_t dim = (2 * num_k_heads + num_v_heads) * LD_HEAD_DIM;
  rc = prepare_conv(qkv, qkv_row_stride, n_tokens, dim, conv_state, n_conv_slots, conv_slot_stride, conv_dim_stride,
                    conv_pos_stride, conv_state_len, conv_weight, conv_bias, conv_width, indices, width, accepted, cu,
                    n_requests, width, conv);
  if (rc != LD_OK) return rc;
  rc = launch_conv_update(conv, n_requests, static_cast<int>(conv_width), conv_state_len,
                          static_cast<cudaStream_t>(stream));
  if (rc != LD_OK) return rc;
  return ld_decode(qkv, qkv_row_stride, a, a_row_stride, b, b_row_stride, a_log, dt_bias, dt_bias_dtype, indices,
                   n_requests, width, cu, accepted, state, n_slots, slot_stride, gate, gate_row_stride, weight,
                   weight_dtype, out, n_tokens, num_k_heads, num_v_heads, eps, stream);
}
