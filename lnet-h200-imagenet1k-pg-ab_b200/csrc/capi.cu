// Error plumbing, launch accounting and version of the lnet_b200 C ABI.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace lnet {

static thread_local std::string g_last_error;
static thread_local int g_launches = 0;

int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_check(cudaError_t err, const char *what) {
  if (err == cudaSuccess) return LNET_OK;
  return fail(LNET_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

void reset_launches() { g_launches = 0; }
void count_launch(int n) { g_launches += n; }
int launch_count() { return g_launches; }

int after_launch(const char *what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(LNET_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(err));
  ++g_launches;
  return LNET_OK;
}

}  // namespace lnet

extern "C" const char *lnet_b200_last_error(void) { return lnet::g_last_error.c_str(); }
extern "C" int lnet_b200_last_launch_count(void) { return lnet::g_launches; }
extern "C" const char *lnet_b200_version(void) { return "lnet_b200 0.1.0 (sm_100a)"; }
