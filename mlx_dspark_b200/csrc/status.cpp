// Error plumbing of the C ABI: a thread-local message behind dspark_last_error().
#include <cstdarg>
#include <cstdio>

#include <cuda_runtime.h>

#include "../../include/dspark_b200.h"

namespace dspark {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

// kernels launched by this thread through the library (dspark_launch_count)
static thread_local long long g_launches = 0;
void note_launch() { ++g_launches; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return set_error(DSPARK_ERR_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return DSPARK_OK;
}

}  // namespace dspark

extern "C" int dspark_version(void) { return 10000; /* 1.0.0 */ }

extern "C" const char* dspark_last_error(void) { return dspark::g_last_error; }

extern "C" long long dspark_launch_count(void) { return dspark::g_launches; }
