// Internal helpers shared by the translation units of liblightdelta_b200.so.
#pragma once

#include <cstdint>

namespace ldb {

// Records a formatted message for ld_last_error() on the calling thread and returns `code`.
int set_error(int code, const char* fmt, ...);
// Clears the calling thread's message and returns LD_OK.
int ok();

// ld_decode's host-side argument checks without a launch (LD_OK, or the error ld_decode returns).
int check_decode_args(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride, const void* b,
                      int64_t b_row_stride, const float* a_log, const void* dt_bias, int dt_bias_dtype,
                      const int32_t* indices, int64_t n_requests, int64_t width, const int32_t* cu,
                      const int32_t* accepted, float* state, int64_t n_slots, int64_t slot_stride, const void* gate,
                      int64_t gate_row_stride, const void* weight, int weight_dtype, void* out, int64_t n_tokens,
                      int64_t num_k_heads, int64_t num_v_heads, float eps);

// Whether kernels launch with programmatic dependent launch (ld_programmatic_launch).
bool programmatic_launch_enabled();

// Per-translation-unit device fault words (see LD_FAULT_* in lightdelta_b200.h).
int decode_faults(uint32_t* flags, int clear);
int state_io_faults(uint32_t* flags, int clear);
int verify_faults(uint32_t* flags, int clear);
int conv_faults(uint32_t* flags, int clear);

}  // namespace ldb
