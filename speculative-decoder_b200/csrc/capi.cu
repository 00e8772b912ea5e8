// Library-wide C ABI helpers: version, the per-thread text of the last host-side error, and the
// bounded-wait check.
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

extern "C" int specb200_set_error(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : "");
  return code;
}

extern "C" int specb200_version(void) { return 10000; }

extern "C" const char* specb200_last_error(void) { return g_last_error; }

namespace {
// One thread waits, with the helper every pipeline uses for its mbarrier waits, on a phase of
// a barrier that expects one arrival and never gets it: the wait gives up after
// SPECB200_SPIN_LIMIT_CYCLES, records SPECB200_ERR_TIMEOUT and raises the CTA's abort flag.
// Nothing else is in flight, so the context stays usable.
__global__ void wait_probe_kernel(int32_t* status, int32_t* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    specb200::mbar_init(&bar, 1);
    abort_flag = 0;
    specb200::fence_mbar_init();
    const bool ok = specb200::mbar_wait_bounded(&bar, 0, status, &abort_flag);
    *gave_up = ok ? 0 : (abort_flag ? 1 : 2);
  }
}
}  // namespace

extern "C" int specb200_wait_probe(int32_t* status, int32_t* gave_up, void* stream) {
  if (!status || !gave_up) return specb200_set_error(SPECB200_ERR_ARG, "wait_probe: null pointer");
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, gave_up);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPECB200_OK : specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
}
