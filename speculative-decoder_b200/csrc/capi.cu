// Library-wide C ABI helpers: version and the per-thread text of the last host-side error.
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
