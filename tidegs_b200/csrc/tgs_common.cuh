// Shared helpers for the tidegs_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include "tidegs_b200.h"

namespace tgs {

// ---------------------------------------------------------------------------
// Host-side error plumbing: every entry point returns a status and leaves a
// message in a thread-local buffer (tgs_last_error).
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

#define TGS_CHECK_ARG(cond, ...)              \
  do {                                        \
    if (!(cond)) {                            \
      ::tgs::set_error(__VA_ARGS__);          \
      return TGS_ERR_INVALID_ARG;             \
    }                                         \
  } while (0)

#define TGS_CUDA(call)                                                      \
  do {                                                                      \
    cudaError_t e_ = (call);                                                \
    if (e_ != cudaSuccess) {                                                \
      ::tgs::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                       __FILE__, __LINE__);                                 \
      return TGS_ERR_CUDA;                                                  \
    }                                                                       \
  } while (0)

#define TGS_LAUNCH_CHECK()                                                  \
  do {                                                                      \
    cudaError_t e_ = cudaGetLastError();                                    \
    if (e_ != cudaSuccess) {                                                \
      ::tgs::set_error("kernel launch failed: %s (%s:%d)",                 \
                       cudaGetErrorString(e_), __FILE__, __LINE__);         \
      return TGS_ERR_CUDA;                                                  \
    }                                                                       \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device id).
int sm_count();

// ---------------------------------------------------------------------------
// Row layout constants (component order = reference COMPONENT_SPECS order).
// ---------------------------------------------------------------------------
constexpr int kNumComp = TGS_NUM_COMPONENTS;
constexpr int kRowWidth = TGS_ROW_WIDTH;

__host__ __device__ constexpr int comp_width(int c) {
  return c == 0 ? 3 : c == 1 ? 1 : c == 2 ? 3 : c == 3 ? 4 : c == 4 ? 3 : 45;
}
// First column of component c in the UNIFIED order xyz|opacity|scaling|rotation|dc|rest.
__host__ __device__ constexpr int unified_offset(int c) {
  return c == 0 ? 0 : c == 1 ? 3 : c == 2 ? 4 : c == 3 ? 7 : c == 4 ? 11 : 14;
}
// First column of component c in the CACHE order xyz|scaling|rotation|opacity|dc|rest.
__host__ __device__ constexpr int cache_offset(int c) {
  return c == 0 ? 0 : c == 1 ? 10 : c == 2 ? 3 : c == 3 ? 6 : c == 4 ? 11 : 14;
}
__host__ __device__ constexpr int layout_offset(int layout, int c) {
  return layout == TGS_LAYOUT_UNIFIED ? unified_offset(c) : cache_offset(c);
}
// Component holding UNIFIED column j (0 <= j < 59).
__host__ __device__ constexpr int unified_comp_of(int j) {
  return j < 3 ? 0 : j < 4 ? 1 : j < 7 ? 2 : j < 11 ? 3 : j < 14 ? 4 : 5;
}
// Component holding column j of `layout`.
__host__ __device__ constexpr int layout_comp_of(int layout, int j) {
  return layout == TGS_LAYOUT_UNIFIED
             ? unified_comp_of(j)
             : (j < 3 ? 0 : j < 6 ? 2 : j < 10 ? 3 : j < 11 ? 1 : j < 14 ? 4 : 5);
}

// Selects entry c of a 6-entry kernel-parameter array with constant offsets
// (a dynamic index would copy the whole parameter block to local memory).
template <typename T>
__device__ __forceinline__ T pick6(const T (&arr)[kNumComp], int c) {
  switch (c) {
    case 0: return arr[0];
    case 1: return arr[1];
    case 2: return arr[2];
    case 3: return arr[3];
    case 4: return arr[4];
    default: return arr[5];
  }
}

// ---------------------------------------------------------------------------
// Device error word helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void report_error(int32_t* err, int code, int64_t index,
                                             int32_t aux = 0) {
  if (err == nullptr) return;
  if (atomicCAS(reinterpret_cast<int*>(err), 0, code) == 0) {
    err[1] = static_cast<int32_t>(static_cast<uint64_t>(index) & 0xffffffffu);
    err[2] = static_cast<int32_t>(static_cast<uint64_t>(index) >> 32);
    err[3] = aux;
  }
}

__device__ __forceinline__ int load_error(const int32_t* err) {
  if (err == nullptr) return 0;
  return *reinterpret_cast<const volatile int32_t*>(err);
}

// ---------------------------------------------------------------------------
// Exactly rounded fp32 arithmetic. The optimizer math uses these so that no
// multiply-add pair is contracted into an FMA: each operation rounds once,
// which is what the CPU oracle (numpy fp32) computes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, non-tensor) wrappers. No multicast form is used
// anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

// Raises the phase's expected byte count without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One bounded probe of phase completion.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(phase)
      : "memory");
  return done != 0;
}

// Waits for `phase` of `bar` with an iteration limit. Returns false when the
// limit was reached (the caller records TGS_DEV_WAIT_TIMEOUT and bails out).
constexpr uint32_t kWaitLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    if (mbar_try_wait(bar, phase)) return true;
  }
  return false;
}

// Bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bulk copy shared -> global in the current bulk async-group.
__device__ __forceinline__ void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_addr(smem_src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk groups still READ shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until all committed bulk groups have completed (writes visible).
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__host__ __device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

template <typename T>
__host__ __device__ __forceinline__ T ceil_div(T a, T b) {
  return (a + b - 1) / b;
}

}  // namespace tgs
