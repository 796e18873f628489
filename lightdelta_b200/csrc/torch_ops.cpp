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

void decode(const at::Tensor& qkv, const at::Tensor& a, const at::Tensor& b, const at::Tensor& a_log,
            const at::Tensor& dt_bias, const at::Tensor& indices, const at::Tensor& cu,
            const at::Tensor& accepted, at::Tensor state, const at::Tensor& gate, const at::Tensor& weight,
            at::Tensor out, double eps) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16, "qkv must be CUDA BF16");
  const c10::cuda::CUDAGuard guard(qkv.device());
  for (const auto& t : {a, b, gate, out}) {
    TORCH_CHECK(t.device() == qkv.device() && t.scalar_type() == at::kBFloat16 && t.stride(-1) == 1,
                "activations must be BF16 with dense rows");
  }
  for (const auto& t : {a_log, state}) {
    TORCH_CHECK(t.device() == qkv.device() && t.scalar_type() == at::kFloat && t.stride(-1) == 1,
                "state and A_log must be CUDA FP32 with dense rows");
  }
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
  if (indices.size(0) == 0) return;
  check_rc(ld_decode(qkv.data_ptr(), qkv.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                     a_log.data_ptr<float>(), dt_bias.data_ptr(), dtype_code(dt_bias),
                     indices.data_ptr<int32_t>(), indices.size(0), indices.size(1), cu.data_ptr<int32_t>(),
                     accepted.data_ptr<int32_t>(), state.data_ptr<float>(), state.size(0), state.stride(0),
                     gate.data_ptr(), gate.stride(0), weight.data_ptr(), dtype_code(weight), out.data_ptr(),
                     n, h, hv, static_cast<float>(eps), stream_of(qkv)));
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

}  // namespace lightdelta_b200

TORCH_LIBRARY(lightdelta, m) {
  m.def(
      "decode(Tensor qkv, Tensor a, Tensor b, Tensor a_log, Tensor dt_bias, "
      "Tensor indices, Tensor cu, Tensor accepted, Tensor(s!) state, Tensor gate, "
      "Tensor weight, Tensor(o!) out, float eps) -> ()");
  m.def("gather_state(Tensor pool, Tensor slots, Tensor valid, Tensor(o!) out) -> ()");
  m.def("scatter_state(Tensor packed, Tensor slots, Tensor(p!) pool) -> ()");
  m.def("copy_state(Tensor(p!) pool, Tensor src, Tensor dst) -> ()");
}

TORCH_LIBRARY_IMPL(lightdelta, CUDA, m) {
  m.impl("decode", lightdelta_b200::decode);
  m.impl("gather_state", lightdelta_b200::gather_state);
  m.impl("scatter_state", lightdelta_b200::scatter_state);
  m.impl("copy_state", lightdelta_b200::copy_state);
}
