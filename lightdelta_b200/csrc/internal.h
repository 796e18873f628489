// Internal helpers shared by the translation units of liblightdelta_b200.so.
#pragma once

#include <cstdint>

namespace ldb {

// Records a formatted message for ld_last_error() on the calling thread and returns `code`.
int set_error(int code, const char* fmt, ...);
// Clears the calling thread's message and returns LD_OK.
int ok();

// Whether kernels launch with programmatic dependent launch (ld_programmatic_launch).
bool programmatic_launch_enabled();

// Per-translation-unit device fault words (see LD_FAULT_* in lightdelta_b200.h).
int decode_faults(uint32_t* flags, int clear);
int state_io_faults(uint32_t* flags, int clear);
int verify_faults(uint32_t* flags, int clear);

}  // namespace ldb
