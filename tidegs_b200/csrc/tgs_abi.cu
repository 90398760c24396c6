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

namespace tgs {
namespace {

__global__ void copy_words_kernel(uint32_t* __restrict__ dst, const uint32_t* __restrict__ src,
                                  int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

__global__ void copy_vec4_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                 int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

}  // namespace
}  // namespace tgs

extern "C" int tgs_copy_small(void* dst, const void* src, int64_t bytes, void* stream) {
  TGS_CHECK_ARG(bytes >= 0, "tgs_copy_small: bytes < 0");
  if (bytes == 0) return TGS_OK;
  TGS_CHECK_ARG(dst && src, "tgs_copy_small: NULL pointer");
  TGS_CHECK_ARG((bytes & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 3) == 0 &&
                    (reinterpret_cast<uintptr_t>(src) & 3) == 0,
                "tgs_copy_small: addresses and size must be 4-byte aligned");
  cudaStream_t s = tgs::as_stream(stream);
  const int64_t cap = static_cast<int64_t>(tgs::sm_count()) * 4;
  if ((bytes & 15) == 0 && tgs::aligned16(dst) && tgs::aligned16(src)) {
    const int64_t n = bytes / 16;
    const int grid = static_cast<int>(std::min<int64_t>(tgs::ceil_div<int64_t>(n, 256), cap));
    tgs::copy_vec4_kernel<<<grid, 256, 0, s>>>(static_cast<uint4*>(dst),
                                               static_cast<const uint4*>(src), n);
  } else {
    const int64_t n = bytes / 4;
    const int grid = static_cast<int>(std::min<int64_t>(tgs::ceil_div<int64_t>(n, 256), cap));
    tgs::copy_words_kernel<<<grid, 256, 0, s>>>(static_cast<uint32_t*>(dst),
                                                static_cast<const uint32_t*>(src), n);
  }
  TGS_LAUNCH_CHECK();
  return TGS_OK;
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

extern "C" int tgs_d2h_blocks(void* const* host_dst, const void* const* dev_src,
                              const int64_t* bytes, int32_t n, void* stream) {
  TGS_CHECK_ARG(n >= 0, "tgs_d2h_blocks: n=%d < 0", n);
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(host_dst && dev_src && bytes, "tgs_d2h_blocks: null array");
  cudaStream_t s = tgs::as_stream(stream);
  for (int32_t k = 0; k < n; ++k) {
    TGS_CHECK_ARG(bytes[k] >= 0, "tgs_d2h_blocks: bytes[%d]=%lld < 0", k, (long long)bytes[k]);
    if (bytes[k] == 0) continue;
    TGS_CUDA(cudaMemcpyAsync(host_dst[k], dev_src[k], static_cast<size_t>(bytes[k]),
                             cudaMemcpyDeviceToHost, s));
  }
  return TGS_OK;
}
