// Error reporting and version of the h3b C ABI.
#include "common.cuh"

#include <cstring>

namespace h3b {

namespace {
thread_local char g_last_error[512] = {0};
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = 0; }

}  // namespace h3b

namespace h3b {
int gemm_status_async(int* dst, int clear, cudaStream_t stream);
int attn_status_async(int* dst, int clear, cudaStream_t stream);
int rows_status_async(int* dst, int clear, cudaStream_t stream);
int peer_status_async(int* dst, int clear, cudaStream_t stream);
}  // namespace h3b

extern "C" const char* h3b_last_error(void) { return h3b::g_last_error; }

extern "C" int h3b_status_async(int* dst, int clear, cudaStream_t stream) {
  h3b::clear_error();
  H3B_REQUIRE(dst, "status_async: null destination");
  if (int rc = h3b::gemm_status_async(dst, clear, stream)) return rc;
  if (int rc = h3b::attn_status_async(dst + 1, clear, stream)) return rc;
  if (int rc = h3b::rows_status_async(dst + 2, clear, stream)) return rc;
  return h3b::peer_status_async(dst + 3, clear, stream);
}

extern "C" const char* h3b_version(void) { return "h3b 0.1 sm_100a"; }
