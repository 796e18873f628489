// Library-wide C entry points: error reporting, version and the device fault word.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "lightdelta_b200.h"
#include "internal.h"

namespace ldb {
namespace {
thread_local std::string g_last_error;
std::atomic<int> g_programmatic_launch{1};
}  // namespace

bool programmatic_launch_enabled() { return g_programmatic_launch.load(std::memory_order_relaxed) != 0; }

int set_error(int code, const char* fmt, ...) {
  char buffer[512];
  va_list args;
  va_start(args, fmt);
  std::vsnprintf(buffer, sizeof(buffer), fmt, args);
  va_end(args);
  g_last_error = buffer;
  return code;
}

int ok() {
  g_last_error.clear();
  return LD_OK;
}

const char* last_error() { return g_last_error.c_str(); }

}  // namespace ldb

extern "C" const char* ld_last_error(void) { return ldb::last_error(); }

extern "C" const char* ld_version(void) { return "lightdelta_b200 0.1.0 (sm_100a)"; }

extern "C" int ld_programmatic_launch(int enable) {
  if (enable < 0) return ldb::g_programmatic_launch.load();
  return ldb::g_programmatic_launch.exchange(enable != 0 ? 1 : 0);
}

extern "C" int ld_fault_flags(uint32_t* flags, int clear) {
  if (flags == nullptr) return ldb::set_error(LD_ERR_INVALID, "ld_fault_flags: flags is NULL");
  uint32_t decode = 0, state_io = 0, verify = 0, conv = 0;
  int rc = ldb::decode_faults(&decode, clear);
  if (rc != LD_OK) return rc;
  rc = ldb::state_io_faults(&state_io, clear);
  if (rc != LD_OK) return rc;
  rc = ldb::verify_faults(&verify, clear);
  if (rc != LD_OK) return rc;
  rc = ldb::conv_faults(&conv, clear);
  if (rc != LD_OK) return rc;
  *flags = decode | state_io | verify | conv;
  return ldb::ok();
}
