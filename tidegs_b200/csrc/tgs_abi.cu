// Library information entry points and host-side error plumbing.
#include <stdarg.h>
#include <string.h>

#include <mutex>

#include "tgs_common.cuh"

namespace tgs {

namespace {
thread_local char g_last_error[1024] = {0};
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace tgs

extern "C" int tgs_version(void) { return TGS_ABI_VERSION; }

extern "C" int tgs_last_error(char* buf, size_t len) {
  const size_t n = strlen(tgs::g_last_error);
  if (buf != nullptr && len > 0) {
    const size_t m = n < len - 1 ? n : len - 1;
    memcpy(buf, tgs::g_last_error, m);
    buf[m] = '\0';
  }
  return static_cast<int>(n);
}

extern "C" int tgs_h2d_blocks(void* const* dev_dst, const void* const* host_src,
                              const int64_t* bytes, int32_t n, void* stream) {
  TGS_CHECK_ARG(n >= 0, "tgs_h2d_blocks: n=%d < 0", n);
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(dev_dst && host_src && bytes, "tgs_h2d_blocks: null array");
  cudaStream_t s = tgs::as_stream(stream);
  for (int32_t k = 0; k < n; ++k) {
    TGS_CHECK_ARG(bytes[k] >= 0, "tgs_h2d_blocks: bytes[%d]=%lld < 0", k, (long long)bytes[k]);
    if (bytes[k] == 0) continue;
    TGS_CUDA(cudaMemcpyAsync(dev_dst[k], host_src[k], static_cast<size_t>(bytes[k]),
                             cudaMemcpyHostToDevice, s));
  }
  return TGS_OK;
}
