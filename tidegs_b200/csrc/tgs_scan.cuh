// Block-wide and device-wide prefix sums shared by the ordered compactions.
#pragma once

#include "tgs_common.cuh"

namespace tgs {
namespace {

// Exclusive scan of one int per thread over the CTA (blockDim.x a multiple
// of 32, at most 1024); *total receives the CTA sum. Every thread must call it.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) warp_sums[lane] = s;
  }
  __syncthreads();
  total = warp_sums[(blockDim.x >> 5) - 1];
  const int base = warp == 0 ? 0 : warp_sums[warp - 1];
  __syncthreads();
  return base + x - v;
}

// Exclusive scan of n_tiles int64 counts in place, by one CTA of 1024
// threads; *total_out receives the sum.
__global__ void __launch_bounds__(1024) scan_counts_kernel(int64_t* __restrict__ counts,
                                                           int64_t n_tiles,
                                                           int64_t* __restrict__ total_out) {
  __shared__ int64_t warp_sums[32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t b = 0; b < n_tiles; b += blockDim.x) {
    const int64_t i = b + threadIdx.x;
    const int64_t v = i < n_tiles ? counts[i] : 0;
    int64_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int64_t s = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const int64_t wbase = warp == 0 ? 0 : warp_sums[warp - 1];
    if (i < n_tiles) counts[i] = carry + wbase + x - v;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) *total_out = carry;
}

}  // namespace
}  // namespace tgs
