// torch.library registration of the lightdelta operator namespace on top of the C ABI.
//
// Schemas are identical to the reference's (csrc/register.cpp:4-11) so that callers written
// against torch.ops.lightdelta (python/lightdelta/backend.py:25-27, :82-84;
// python/lightdelta/integration/vllm_layer.py:114, :132) run unchanged.  Tensor checks keep
// the reference's preconditions and messages (csrc/gdn_decode.cu:367-403,
// csrc/state_io.cu:29-49) with one generalisation: the head counts come from the tensors
// instead of being fixed at 16/48, so HV=32 pools are accepted as well as HV=48.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "lightdelta_b200.h"

namespace lightdelta_b200 {
namespace {

void check_rc(int rc) { TORCH_CHECK(rc == LD_OK, ld_last_error()); }

int dtype_code(const at::Tensor& t) { return t.scalar_type() == at::kBFloat16 ? LD_DTYPE_BF16 : LD_DTYPE_F32; }

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

}  // namespace

namespace {

struct DecodeGeometry {
  int64_t h, hv, n;
};

// The reference launcher's tensor checks (csrc/gdn_decode.cu:367-403), head counts from the tensors.
DecodeGeometry check_decode(const at::Tensor& qkv, const at::Tensor& a, const at::Tensor& b, const at::Tensor& a_log,
                            const at::Tensor& dt_bias, const at::Tensor& indices, const at::Tensor& cu,
                            const at::Tensor& accepted, const at::Tensor& state, const at::Tensor& gate,
                            const at::Tensor& weight, const at::Tensor& out, double eps,
                            at::ScalarType state_type = at::kFloat) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16, "qkv must be CUDA BF16");
  for (const auto& t : {a, b, gate, out}) {
    TORCH_CHECK(t.device() == qkv.device() && t.scalar_type() == at::kBFloat16 && t.stride(-1) == 1,
                "activations must be BF16 with dense rows");
  }
  TORCH_CHECK(a_log.device() == qkv.device() && a_log.scalar_type() == at::kFloat && a_log.stride(-1) == 1,
              "state and A_log must be CUDA FP32 with dense rows");
  TORCH_CHECK(state.device() == qkv.device() && state.scalar_type() == state_type && state.stride(-1) == 1,
              state_type == at::kFloat ? "state and A_log must be CUDA FP32 with dense rows"
                                       : "state must be CUDA BF16 with dense rows");
  for (const auto& t : {indices, cu, accepted}) {
    TORCH_CHECK(t.device() == qkv.device() && t.scalar_type() == at::kInt && t.is_contiguous(),
                "metadata must be contiguous CUDA int32");
  }
  for (const auto& t : {dt_bias, weight}) {
    TORCH_CHECK(t.device() == qkv.device() && t.is_contiguous() &&
                    (t.scalar_type() == at::kFloat || t.scalar_type() == at::kBFloat16),
                "weights must be contiguous FP32/BF16");
  }
  TORCH_CHECK(state.dim() == 4 && state.size(2) == LD_HEAD_DIM && state.size(3) == LD_HEAD_DIM &&
                  state.stride(2) == LD_HEAD_DIM && state.stride(1) == LD_HEAD_DIM * LD_HEAD_DIM,
              "state must be [slots,HV,128,128]");
  const int64_t hv = state.size(1);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) % LD_HEAD_DIM == 0 &&
                  qkv.size(1) / LD_HEAD_DIM > hv && (qkv.size(1) / LD_HEAD_DIM - hv) % 2 == 0,
              "qkv must be [tokens,(2*H+HV)*128] with HV=state.size(1)");
  const int64_t h = (qkv.size(1) / LD_HEAD_DIM - hv) / 2;
  TORCH_CHECK(hv % h == 0, "value heads must be a multiple of key heads");
  TORCH_CHECK(indices.dim() == 2 && indices.size(1) >= 1 && indices.size(1) <= LD_MAX_WIDTH,
              "decode/MTP supports 1 through 4 tokens per request");
  const auto n = qkv.size(0);
  TORCH_CHECK(a.sizes() == at::IntArrayRef({n, hv}) && b.sizes() == a.sizes() &&
                  gate.sizes() == at::IntArrayRef({n, hv, LD_HEAD_DIM}) && out.sizes() == gate.sizes() &&
                  out.is_contiguous() && gate.stride(1) == LD_HEAD_DIM,
              "invalid activation shape or output layout");
  TORCH_CHECK(a_log.numel() == hv && dt_bias.numel() == hv && weight.numel() == LD_HEAD_DIM,
              "invalid weight shapes");
  TORCH_CHECK(cu.dim() == 1 && cu.numel() == indices.size(0) + 1 && accepted.dim() == 1 &&
                  accepted.numel() == indices.size(0),
              "invalid request metadata shapes");
  TORCH_CHECK(eps > 0, "norm epsilon must be positive");
  return DecodeGeometry{h, hv, n};
}

}  // namespace

void decode(const at::Tensor& qkv, const at::Tensor& a, const at::Tensor& b, const at::Tensor& a_log,
            const at::Tensor& dt_bias, const at::Tensor& indices, const at::Tensor& cu,
            const at::Tensor& accepted, at::Tensor state, const at::Tensor& gate, const at::Tensor& weight,
            at::Tensor out, double eps) {
  TORCH_CHECK(qkv.is_cuda(), "qkv must be CUDA BF16");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const DecodeGeometry geo = check_decode(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out,
                                          eps);
  if (indices.size(0) == 0) return;
  check_rc(ld_decode(qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                     a_log.data_ptr<float>(), dt_bias.data_ptr(), dtype_code(dt_bias),
                     indices.data_ptr<int32_t>(), indices.size(0), indices.size(1), cu.data_ptr<int32_t>(),
                     accepted.data_ptr<int32_t>(), state.data_ptr<float>(), state.size(0), state.stride(0),
                     gate.data_ptr(), gate.stride(0), weight.data_ptr(), dtype_code(weight), out.data_ptr(),
                     geo.n, geo.h, geo.hv, static_cast<float>(eps), stream_of(qkv)));
}

// Extension (no reference schema): decode on a bf16 state pool, the fp32 recurrence of decode
// with each stored step rounded to bf16.
void decode_bf16_state(const at::Tensor& qkv, const at::Tensor& a, const at::Tensor& b, const at::Tensor& a_log,
                       const at::Tensor& dt_bias, const at::Tensor& indices, const at::Tensor& cu,
                       const at::Tensor& accepted, at::Tensor state, const at::Tensor& gate,
                       const at::Tensor& weight, at::Tensor out, double eps) {
  TORCH_CHECK(qkv.is_cuda(), "qkv must be CUDA BF16");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const DecodeGeometry geo = check_decode(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out,
                                          eps, at::kBFloat16);
  if (indices.size(0) == 0) return;
  check_rc(ld_decode_bf16_state(qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                                a_log.data_ptr<float>(), dt_bias.data_ptr(), dtype_code(dt_bias),
                                indices.data_ptr<int32_t>(), indices.size(0), indices.size(1),
                                cu.data_ptr<int32_t>(), accepted.data_ptr<int32_t>(), state.data_ptr(),
                                state.size(0), state.stride(0), gate.data_ptr(), gate.stride(0), weight.data_ptr(),
                                dtype_code(weight), out.data_ptr(), geo.n, geo.h, geo.hv, static_cast<float>(eps),
                                stream_of(qkv)));
}

namespace {

struct ConvTensors {
  at::Tensor weight;
  const void* bias;
};

// Checks of the conv state, weight and bias against a [tokens, dim] activation matrix.
ConvTensors check_conv(const at::Tensor& x, const at::Tensor& conv_state, const at::Tensor& conv_weight,
                       const c10::optional<at::Tensor>& conv_bias) {
  const int64_t dim = x.size(1);
  TORCH_CHECK(conv_state.device() == x.device() && conv_state.scalar_type() == at::kBFloat16 &&
                  conv_state.dim() == 3 && conv_state.size(1) == dim,
              "conv_state must be a CUDA BF16 [slots, dim, L] view");
  const at::Tensor w = conv_weight.dim() == 3 ? conv_weight.view({conv_weight.size(0), conv_weight.size(2)})
                                                : conv_weight;
  TORCH_CHECK(w.device() == x.device() && w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.size(0) == dim &&
                  w.is_contiguous(),
              "conv_weight must be a contiguous CUDA BF16 [dim, width] (or [dim, 1, width]) tensor");
  const void* bias_ptr = nullptr;
  if (conv_bias.has_value() && conv_bias->defined()) {
    TORCH_CHECK(conv_bias->device() == x.device() && conv_bias->scalar_type() == at::kBFloat16 &&
                    conv_bias->numel() == dim && conv_bias->is_contiguous(),
                "conv_bias must be a contiguous CUDA BF16 [dim] tensor");
    bias_ptr = conv_bias->data_ptr();
  }
  return ConvTensors{w, bias_ptr};
}

}  // namespace

// Extension (no reference schema): the causal conv1d state update that produces q, k, v (vLLM's
// causal_conv1d_update as vllm_layer.py:161-172 and :199-207 call it), in place on x.
void conv_update(at::Tensor x, at::Tensor conv_state, const at::Tensor& conv_weight,
                 const c10::optional<at::Tensor>& conv_bias, const at::Tensor& slots,
                 const c10::optional<at::Tensor>& accepted, const at::Tensor& cu, int64_t max_tokens) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "x must be a CUDA BF16 [tokens, dim] matrix with dense rows");
  const c10::cuda::CUDAGuard guard(x.device());
  const ConvTensors conv = check_conv(x, conv_state, conv_weight, conv_bias);
  TORCH_CHECK(slots.device() == x.device() && slots.scalar_type() == at::kInt && slots.dim() == 1,
              "slots must be a CUDA int32 vector");
  const int64_t n = slots.numel();
  TORCH_CHECK(cu.device() == x.device() && cu.scalar_type() == at::kInt && cu.is_contiguous() && cu.numel() == n + 1,
              "cu must be a contiguous CUDA int32 [requests + 1] vector");
  const int32_t* accepted_ptr = nullptr;
  if (accepted.has_value() && accepted->defined()) {
    TORCH_CHECK(accepted->device() == x.device() && accepted->scalar_type() == at::kInt &&
                    accepted->is_contiguous() && accepted->numel() == n,
                "accepted must be a contiguous CUDA int32 [requests] vector");
    accepted_ptr = accepted->data_ptr<int32_t>();
  }
  if (n == 0) return;
  check_rc(ld_conv_update(x.data_ptr(), x.stride(0), x.size(0), x.size(1), conv_state.data_ptr(), conv_state.size(0),
                          conv_state.stride(0), conv_state.stride(1), conv_state.stride(2), conv_state.size(2),
                          conv.weight.data_ptr(), conv.bias, conv.weight.size(1), slots.data_ptr<int32_t>(),
                          slots.stride(0), accepted_ptr, cu.data_ptr<int32_t>(), n, max_tokens, stream_of(x)));
}

// Extension (no reference schema): conv update then decode, as vllm_layer.py:161-174 and
// :199-220 run them; qkv holds the pre-conv activations and receives the post-conv ones.
void conv_decode(at::Tensor qkv, at::Tensor conv_state, const at::Tensor& conv_weight,
                 const c10::optional<at::Tensor>& conv_bias, const at::Tensor& a, const at::Tensor& b,
                 const at::Tensor& a_log, const at::Tensor& dt_bias, const at::Tensor& indices, const at::Tensor& cu,
                 const at::Tensor& accepted, at::Tensor state, const at::Tensor& gate, const at::Tensor& weight,
                 at::Tensor out, double eps) {
  TORCH_CHECK(qkv.is_cuda(), "qkv must be CUDA BF16");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const DecodeGeometry geo = check_decode(qkv, a, b, a_log, dt_bias, indices, cu, accepted, state, gate, weight, out,
                                          eps);
  const ConvTensors conv = check_conv(qkv, conv_state, conv_weight, conv_bias);
  if (indices.size(0) == 0) return;
  check_rc(ld_conv_decode(qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                          a_log.data_ptr<float>(), dt_bias.data_ptr(), dtype_code(dt_bias),
                          indices.data_ptr<int32_t>(), indices.size(0), indices.size(1), cu.data_ptr<int32_t>(),
                          accepted.data_ptr<int32_t>(), state.data_ptr<float>(), state.size(0), state.stride(0),
                          gate.data_ptr(), gate.stride(0), weight.data_ptr(), dtype_code(weight), out.data_ptr(),
                          geo.n, geo.h, geo.hv, static_cast<float>(eps), conv_state.data_ptr(), conv_state.size(0),
                          conv_state.stride(0), conv_state.stride(1), conv_state.stride(2), conv_state.size(2),
                          conv.weight.data_ptr(), conv.bias, conv.weight.size(1), stream_of(qkv)));
}

namespace {
void check_pool(const at::Tensor& pool, const at::Tensor& slots, const at::Tensor& packed) {
  TORCH_CHECK(pool.is_cuda() && pool.scalar_type() == at::kFloat && pool.dim() == 4 && pool.stride(3) == 1 &&
                  pool.stride(2) == pool.size(3) && pool.stride(1) == pool.size(2) * pool.size(3),
              "pool must be CUDA FP32 with dense inner dimensions");
  TORCH_CHECK(slots.device() == pool.device() && slots.scalar_type() == at::kInt && slots.dim() == 1,
              "slots must be a CUDA int32 vector");
  TORCH_CHECK(packed.device() == pool.device() && packed.scalar_type() == at::kFloat && packed.dim() == 4 &&
                  packed.size(0) == slots.numel() && packed.sizes().slice(1) == pool.sizes().slice(1) &&
                  packed.stride(3) == 1 && packed.stride(2) == packed.size(3) &&
                  packed.stride(1) == packed.size(2) * packed.size(3),
              "invalid packed layout");
}
}  // namespace

void gather_state(const at::Tensor& pool, const at::Tensor& slots, const at::Tensor& valid, at::Tensor out) {
  check_pool(pool, slots, out);
  TORCH_CHECK(valid.device() == pool.device() && valid.scalar_type() == at::kBool &&
                  valid.sizes() == slots.sizes() && valid.is_contiguous(),
              "valid must be a CUDA bool vector");
  if (slots.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(pool.device());
  const int64_t elements = pool.size(1) * pool.size(2) * pool.size(3);
  check_rc(ld_gather_state(pool.data_ptr<float>(), pool.size(0), pool.stride(0), slots.data_ptr<int32_t>(),
                           slots.stride(0), reinterpret_cast<const uint8_t*>(valid.data_ptr<bool>()),
                           slots.numel(), out.data_ptr<float>(), out.stride(0), elements, stream_of(pool)));
}

void scatter_state(const at::Tensor& packed, const at::Tensor& slots, at::Tensor pool) {
  check_pool(pool, slots, packed);
  if (slots.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(pool.device());
  const int64_t elements = pool.size(1) * pool.size(2) * pool.size(3);
  check_rc(ld_scatter_state(packed.data_ptr<float>(), packed.stride(0), slots.data_ptr<int32_t>(),
                            slots.stride(0), slots.numel(), pool.data_ptr<float>(), pool.size(0), pool.stride(0),
                            elements, stream_of(pool)));
}

// Extension (no reference schema): pool[dst[i]] = pool[src[i]] for live, distinct slot pairs.
void copy_state(at::Tensor pool, const at::Tensor& src, const at::Tensor& dst) {
  TORCH_CHECK(pool.is_cuda() && pool.scalar_type() == at::kFloat && pool.dim() == 4 && pool.stride(3) == 1 &&
                  pool.stride(2) == pool.size(3) && pool.stride(1) == pool.size(2) * pool.size(3),
              "pool must be CUDA FP32 with dense inner dimensions");
  for (const auto& t : {src, dst}) {
    TORCH_CHECK(t.device() == pool.device() && t.scalar_type() == at::kInt && t.dim() == 1,
                "slots must be a CUDA int32 vector");
  }
  TORCH_CHECK(src.numel() == dst.numel(), "source and destination slot vectors differ in length");
  if (src.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(pool.device());
  const int64_t elements = pool.size(1) * pool.size(2) * pool.size(3);
  check_rc(ld_copy_slots(pool.data_ptr<float>(), pool.size(0), pool.stride(0), src.data_ptr<int32_t>(),
                         src.stride(0), dst.data_ptr<int32_t>(), dst.stride(0), src.numel(), elements,
                         stream_of(pool)));
}

// Extension (no reference schema): the device form of LightDeltaRejectionSampler.__call__
// (python/lightdelta/runtime/speculation.py:274-326), writing every entry of its three outputs.
void greedy_verify(const at::Tensor& logits, const at::Tensor& cu_num_logits, const at::Tensor& query_start_loc,
                   const at::Tensor& input_ids, const at::Tensor& num_draft_tokens, const at::Tensor& seq_lens,
                   const at::Tensor& prefill_len, at::Tensor sampled, at::Tensor num_sampled,
                   at::Tensor num_rejected) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1 &&
                  (logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16 ||
                   logits.scalar_type() == at::kHalf),
              "logits must be a CUDA FP32/BF16/FP16 matrix with dense rows");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t n = num_draft_tokens.numel();
  for (const auto& t : {cu_num_logits, query_start_loc, num_draft_tokens, seq_lens, prefill_len}) {
    TORCH_CHECK(t.device() == logits.device() && t.scalar_type() == at::kInt && t.is_contiguous() && t.dim() == 1,
                "request metadata must be contiguous CUDA int32 vectors");
  }
  TORCH_CHECK(cu_num_logits.numel() == n + 1 && query_start_loc.numel() == n + 1 && seq_lens.numel() == n &&
                  prefill_len.numel() == n,
              "invalid request metadata shapes");
  TORCH_CHECK(input_ids.device() == logits.device() && input_ids.dim() == 1 && input_ids.is_contiguous() &&
                  (input_ids.scalar_type() == at::kInt || input_ids.scalar_type() == at::kLong),
              "input_ids must be a contiguous CUDA int32/int64 vector");
  TORCH_CHECK(sampled.device() == logits.device() && sampled.scalar_type() == input_ids.scalar_type() &&
                  sampled.dim() == 2 && sampled.size(0) == n && sampled.size(1) >= 1 && sampled.is_contiguous(),
              "sampled must be a contiguous [requests, steps+1] tensor of the input_ids dtype");
  for (const auto& t : {num_sampled, num_rejected}) {
    TORCH_CHECK(t.device() == logits.device() && t.scalar_type() == at::kInt && t.is_contiguous() &&
                    t.dim() == 1 && t.numel() == n,
                "num_sampled and num_rejected must be contiguous CUDA int32 [requests]");
  }
  if (n == 0) return;
  const int logits_dtype = logits.scalar_type() == at::kFloat      ? LD_DTYPE_F32
                           : logits.scalar_type() == at::kBFloat16 ? LD_DTYPE_BF16
                                                                   : LD_DTYPE_F16;
  const int token_dtype = input_ids.scalar_type() == at::kLong ? LD_DTYPE_I64 : LD_DTYPE_I32;
  check_rc(ld_greedy_verify(logits.data_ptr(), logits_dtype, logits.size(0), logits.size(1), logits.stride(0),
                            cu_num_logits.data_ptr<int32_t>(), query_start_loc.data_ptr<int32_t>(),
                            input_ids.data_ptr(), token_dtype, input_ids.numel(),
                            num_draft_tokens.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                            prefill_len.data_ptr<int32_t>(), n, sampled.size(1) - 1, sampled.data_ptr(),
                            num_sampled.data_ptr<int32_t>(), num_rejected.data_ptr<int32_t>(), stream_of(logits)));
}

}  // namespace lightdelta_b200

TORCH_LIBRARY(lightdelta, m) {
  m.def(
      "decode(Tensor qkv, Tensor a, Tensor b, Tensor a_log, Tensor dt_bias, "
      "Tensor indices, Tensor cu, Tensor accepted, Tensor(s!) state, Tensor gate, "
      "Tensor weight, Tensor(o!) out, float eps) -> ()");
  m.def(
      "decode_bf16_state(Tensor qkv, Tensor a, Tensor b, Tensor a_log, Tensor dt_bias, "
      "Tensor indices, Tensor cu, Tensor accepted, Tensor(s!) state, Tensor gate, "
      "Tensor weight, Tensor(o!) out, float eps) -> ()");
  m.def("gather_state(Tensor pool, Tensor slots, Tensor valid, Tensor(o!) out) -> ()");
  m.def("scatter_state(Tensor packed, Tensor slots, Tensor(p!) pool) -> ()");
  m.def("copy_state(Tensor(p!) pool, Tensor src, Tensor dst) -> ()");
  m.def(
      "conv_update(Tensor(x!) x, Tensor(c!) conv_state, Tensor conv_weight, Tensor? conv_bias, Tensor slots, "
      "Tensor? accepted, Tensor cu, int max_tokens) -> ()");
  m.def(
      "conv_decode(Tensor(q!) qkv, Tensor(c!) conv_state, Tensor conv_weight, Tensor? conv_bias, Tensor a, Tensor b, "
      "Tensor a_log, Tensor dt_bias, Tensor indices, Tensor cu, Tensor accepted, Tensor(s!) state, Tensor gate, "
      "Tensor weight, Tensor(o!) out, float eps) -> ()");
  m.def(
      "greedy_verify(Tensor logits, Tensor cu_num_logits, Tensor query_start_loc, Tensor input_ids, "
      "Tensor num_draft_tokens, Tensor seq_lens, Tensor prefill_len, Tensor(a!) sampled, "
      "Tensor(b!) num_sampled, Tensor(c!) num_rejected) -> ()");
}

TORCH_LIBRARY_IMPL(lightdelta, CUDA, m) {
  m.impl("decode", lightdelta_b200::decode);
  m.impl("decode_bf16_state", lightdelta_b200::decode_bf16_state);
  m.impl("gather_state", lightdelta_b200::gather_state);
  m.impl("scatter_state", lightdelta_b200::scatter_state);
  m.impl("copy_state", lightdelta_b200::copy_state);
  m.impl("greedy_verify", lightdelta_b200::greedy_verify);
  m.impl("conv_decode", lightdelta_b200::conv_decode);
  m.impl("conv_update", lightdelta_b200::conv_update);
}
