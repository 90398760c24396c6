// Dirty-block tracking on a bit-packed bitmap and its order-preserving
// compactions.
//
// Reference behaviour followed (bool bitmap + index_select/nonzero there):
//   strategies/tide_engine/double_buffer_gpu.py:494-543
#include "tgs_common.cuh"

namespace tgs {
namespace {

__global__ void dirty_mark_kernel(uint32_t* __restrict__ bitmap, int64_t num_blocks,
                                  const int64_t* __restrict__ ids, int64_t n, int value) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t id = ids[i];
    if (id < 0 || id >= num_blocks) continue;  // not a block of this bitmap
    const uint32_t bit = 1u << (id & 31);
    if (value) atomicOr(bitmap + (id >> 5), bit);
    else atomicAnd(bitmap + (id >> 5), ~bit);
  }
}

constexpr int kSelectThreads = 1024;

// Block-wide exclusive scan of 0/1 flags via warp ballots. Returns the rank
// of the calling thread's flag; `total` gets the CTA-wide count.
__device__ __forceinline__ int ballot_rank(bool flag, int* warp_counts, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned bal = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(bal & ((1u << lane) - 1u));
  if (lane == 0) warp_counts[warp] = __popc(bal);
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int c = lane < nw ? warp_counts[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, c, o);
      if (lane >= o) c += y;
    }
    if (lane < nw) warp_counts[lane] = c;  // inclusive
  }
  __syncthreads();
  total = warp_counts[(blockDim.x >> 5) - 1];
  const int base = warp == 0 ? 0 : warp_counts[warp - 1];
  __syncthreads();
  return base + in_warp;
}

// One CTA walks the id list in order; each pass ranks its 1024 flags with
// ballots and appends behind the running total, so output order = input order.
__global__ void __launch_bounds__(kSelectThreads) dirty_select_kernel(
    const uint32_t* __restrict__ bitmap, int64_t num_blocks, const int64_t* __restrict__ ids,
    int64_t n, int64_t* __restrict__ out, int64_t* __restrict__ count) {
  __shared__ int warp_counts[32];
  int64_t written = 0;
  for (int64_t base = 0; base < n; base += kSelectThreads) {
    const int64_t i = base + threadIdx.x;
    int64_t id = 0;
    bool flag = false;
    if (i < n) {
      id = ids[i];
      flag = id >= 0 && id < num_blocks && ((bitmap[id >> 5] >> (id & 31)) & 1u);
    }
    int total;
    const int rank = ballot_rank(flag, warp_counts, total);
    if (flag) out[written + rank] = id;
    written += total;
  }
  if (threadIdx.x == 0) *count = written;
}

// All set bits, ascending: thread t of a pass owns word base+t; word popcounts
// are ranked with a CTA scan and each thread writes its word's bit indices.
__global__ void __launch_bounds__(kSelectThreads) dirty_list_kernel(
    const uint32_t* __restrict__ bitmap, int64_t num_bits, int64_t* __restrict__ out,
    int64_t* __restrict__ count) {
  __shared__ int warp_sums[32];
  const int64_t n_words = (num_bits + 31) >> 5;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t written = 0;
  for (int64_t base = 0; base < n_words; base += kSelectThreads) {
    const int64_t w = base + threadIdx.x;
    uint32_t word = 0;
    if (w < n_words) {
      word = bitmap[w];
      const int64_t valid = num_bits - (w << 5);
      if (valid < 32) word &= (1u << valid) - 1u;
    }
    const int c = __popc(word);
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int s = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    int64_t pos = written + (warp == 0 ? 0 : warp_sums[warp - 1]) + (x - c);
    while (word != 0u) {
      const int b = __ffs(word) - 1;
      out[pos++] = (w << 5) + b;
      word &= word - 1u;
    }
    written += warp_sums[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = written;
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_dirty_mark(uint32_t* bitmap, int64_t num_blocks, const int64_t* ids,
                              int64_t n, int32_t value, void* stream) {
  TGS_CHECK_ARG(n >= 0 && num_blocks >= 0, "tgs_dirty_mark: bad sizes");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(bitmap && ids, "tgs_dirty_mark: NULL pointer");
  const int grid = static_cast<int>(std::min<int64_t>(ceil_div<int64_t>(n, 256), 4096));
  dirty_mark_kernel<<<grid, 256, 0, as_stream(stream)>>>(bitmap, num_blocks, ids, n, value);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_dirty_select(const uint32_t* bitmap, int64_t num_blocks, const int64_t* ids,
                                int64_t n, int64_t* out_ids, int64_t* dev_count, void* stream) {
  TGS_CHECK_ARG(n >= 0 && num_blocks >= 0, "tgs_dirty_select: bad sizes");
  TGS_CHECK_ARG(dev_count != nullptr, "tgs_dirty_select: dev_count is NULL");
  cudaStream_t s = as_stream(stream);
  if (n == 0) {
    TGS_CUDA(cudaMemsetAsync(dev_count, 0, sizeof(int64_t), s));
    return TGS_OK;
  }
  TGS_CHECK_ARG(bitmap && ids && out_ids, "tgs_dirty_select: NULL pointer");
  dirty_select_kernel<<<1, kSelectThreads, 0, s>>>(bitmap, num_blocks, ids, n, out_ids,
                                                    dev_count);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_dirty_list(const uint32_t* bitmap, int64_t num_blocks, int64_t* out_ids,
                              int64_t* dev_count, void* stream) {
  TGS_CHECK_ARG(num_blocks >= 0, "tgs_dirty_list: num_blocks < 0");
  TGS_CHECK_ARG(dev_count != nullptr, "tgs_dirty_list: dev_count is NULL");
  cudaStream_t s = as_stream(stream);
  if (num_blocks == 0) {
    TGS_CUDA(cudaMemsetAsync(dev_count, 0, sizeof(int64_t), s));
    return TGS_OK;
  }
  TGS_CHECK_ARG(bitmap && out_ids, "tgs_dirty_list: NULL pointer");
  dirty_list_kernel<<<1, kSelectThreads, 0, s>>>(bitmap, num_blocks, out_ids, dev_count);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}
