// Library-level C ABI: status messages, version and the device error words.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

int jt_fail(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return code;
}

int jt_cuda_check(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return JT_OK;
  return jt_fail(JT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

extern "C" int32_t jt_abi_version(void) { return JT_ABI_VERSION; }

extern "C" const char* jt_last_error(void) { return g_last_error; }

extern "C" int jt_read_device_errors(uint32_t* errors) {
  if (errors == nullptr) return jt_fail(JT_ERR_INVALID, "jt_read_device_errors: null output");
  uint32_t a = 0, b = 0, c = 0;
  int rc = jt_read_errors_kv(&a);
  if (rc != JT_OK) return rc;
  rc = jt_read_errors_attn(&b);
  if (rc != JT_OK) return rc;
  rc = jt_read_errors_rope(&c);
  if (rc != JT_OK) return rc;
  uint32_t d = 0, e = 0;
  rc = jt_read_errors_accept(&d);
  if (rc != JT_OK) return rc;
  rc = jt_read_errors_meta(&e);
  if (rc != JT_OK) return rc;
  uint32_t f = 0;
  rc = jt_read_errors_rowlin(&f);
  if (rc != JT_OK) return rc;
  uint32_t g = 0;
  rc = jt_read_errors_f32(&g);
  if (rc != JT_OK) return rc;
  *errors = a | b | c | d | e | f | g;
  return JT_OK;
}
