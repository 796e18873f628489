// TEST INFRASTRUCTURE ONLY: the reference's own decode kernel at any value-head ratio.
//
// The reference's launcher (csrc/gdn_decode.cu:360-420) hard-codes H=16, HV=48 and the kernel
// instantiation gdn_decode_post_conv_mtp_kernel<float, 3, false>; the kernel template itself
// (csrc/gdn_decode.cu:130-354) takes H and HV at run time and the value heads per key head as
// a template argument.  This translation unit compiles the reference file unmodified (it is
// included from the reference checkout by oracle/build_ref.py, never copied) and adds one C
// entry point that launches the template with ratio 2 (the BASELINE geometry H=16, HV=32) or 3,
// with the launch shape and arguments the stock launcher uses.  Built into oracle/_ref/ and used
// only by the tests and by bench.py's reference arm to run the reference kernel beside ours.
#include "csrc/gdn_decode.cu"

extern "C" int ref_decode_launch(const void* qkv, int64_t qkv_row, const void* a, int64_t a_row, const void* b,
                                 int64_t b_row, const float* a_log, const void* dt_bias, int dt_bias_bf16,
                                 const int* indices, int requests, int width, const int* cu, const int* accepted,
                                 float* state, int64_t slot_stride, const void* gate, int64_t gate_row,
                                 const void* weight, int weight_bf16, void* out, int num_k_heads, int num_v_heads,
                                 float eps, void* stream) {
  if (requests <= 0) return 0;
  if (num_k_heads <= 0 || width < 1 || width > 4) return -1;
  const GdnDecodeStrides strides{qkv_row, a_row, b_row, gate_row, slot_stride};
  const dim3 grid(static_cast<unsigned int>(requests), static_cast<unsigned int>(num_v_heads));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int dt_type = dt_bias_bf16 ? kDtBiasBFloat16 : kDtBiasFloat32;
  const float scale = 0.08838834764831845f;  // the stock launcher's K^-1/2 (csrc/gdn_decode.cu:416)
#define LD_REF_LAUNCH(RATIO)                                                                              \
  gdn_decode_post_conv_mtp_kernel<float, RATIO, false><<<grid, kThreads, 0, s>>>(                         \
      static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(a),                       \
      static_cast<const __nv_bfloat16*>(b), a_log, dt_bias, indices, cu, accepted, state,                 \
      static_cast<const __nv_bfloat16*>(gate), weight, static_cast<__nv_bfloat16*>(out), num_k_heads,     \
      num_v_heads, width, dt_type, weight_bf16 != 0, scale, eps, strides)
  if (num_v_heads == 2 * num_k_heads) {
    LD_REF_LAUNCH(2);
  } else if (num_v_heads == 3 * num_k_heads) {
    LD_REF_LAUNCH(3);
  } else {
    return -1;
  }
#undef LD_REF_LAUNCH
  return static_cast<int>(cudaGetLastError());
}
