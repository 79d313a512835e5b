// Shared host-side helpers: status codes, the thread-local error message and
// the exception type used between internal layers and the C ABI boundary.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "jal.h"

namespace jal {

struct JalError : std::runtime_error {
  int code;
  JalError(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw JalError(code, buf);
}

void set_last_error(const std::string &msg);

// Runs `f` and converts exceptions into a status code + last error.
template <class F>
int guard(F &&f) {
  try {
    f();
    return JAL_OK;
  } catch (const JalError &e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc &) {
    set_last_error("host allocation failed");
    return JAL_ERR_INVALID_ARGUMENT;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return JAL_ERR_INVALID_ARGUMENT;
  }
}

}  // namespace jal

#define JAL_CUDA(call)                                                        \
  do {                                                                        \
    cudaError_t err__ = (call);                                               \
    if (err__ != cudaSuccess)                                                 \
      ::jal::fail(JAL_ERR_CUDA, "%s failed: %s (%s:%d)", #call,              \
                  cudaGetErrorString(err__), __FILE__, __LINE__);             \
  } while (0)
