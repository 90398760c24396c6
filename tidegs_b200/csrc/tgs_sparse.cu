// Touched-only gradient accumulation of a camera batch.
//
// Reference behaviour followed (strategies/tide_engine/engine.py):
//   :1801-1807  touched rows = union of the cameras' local filters, ascending
//               (bool mask, scatter_ True, nonzero): tgs_dirty_mark marks the
//               bits, bitmap_count/write_kernel list them in order
//   :1815       local_to_global[touched] (gather_i64_kernel)
//   :2434-2471  per camera, searchsorted of its filter into the touched rows
//               and scatter_add_ of the six gradient components
//               (sparse_accum_kernel, one launch for all six)
#include "tgs_common.cuh"
#include "tgs_scan.cuh"

namespace tgs {
namespace {

// ---------------------------------------------------------------------------
// Bitmap -> ascending positions of its set bits, over tiles of
// kListTileWords words: (1) per-tile popcounts, (2) one-CTA scan of the
// counts, (3) per tile a CTA-wide rank of each word, then each thread writes
// its word's bits in ascending order.
// ---------------------------------------------------------------------------
constexpr int kListThreads = 256;
constexpr int kListWordsPerThread = 4;
constexpr int kListTileWords = kListThreads * kListWordsPerThread;

__device__ __forceinline__ uint32_t word_bits(const uint32_t* __restrict__ bitmap, int64_t w,
                                              int64_t num_bits) {
  if (w * 32 >= num_bits) return 0u;
  uint32_t v = bitmap[w];
  const int64_t tail = num_bits - w * 32;
  if (tail < 32) v &= (1u << tail) - 1u;
  return v;
}

__global__ void __launch_bounds__(kListThreads) bitmap_count_kernel(
    const uint32_t* __restrict__ bitmap, int64_t num_bits, int64_t* __restrict__ tile_counts) {
  __shared__ int warp_sums[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kListTileWords;
  int cnt = 0;
#pragma unroll
  for (int j = 0; j < kListWordsPerThread; ++j)
    cnt += __popc(word_bits(bitmap, base + j * kListThreads + threadIdx.x, num_bits));
  int total;
  block_exclusive_scan(cnt, warp_sums, total);
  if (threadIdx.x == 0) tile_counts[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kListThreads) bitmap_write_kernel(
    const uint32_t* __restrict__ bitmap, int64_t num_bits,
    const int64_t* __restrict__ tile_offsets, int64_t* __restrict__ out,
    int32_t* __restrict__ pos_map) {
  __shared__ int warp_sums[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kListTileWords;
  int64_t offset = tile_offsets[blockIdx.x];
  for (int j = 0; j < kListWordsPerThread; ++j) {
    const int64_t w = base + j * kListThreads + threadIdx.x;
    uint32_t bits = word_bits(bitmap, w, num_bits);
    int total;
    const int rank = block_exclusive_scan(__popc(bits), warp_sums, total);
    int64_t o = offset + rank;
    while (bits != 0u) {
      const int64_t b = w * 32 + (__ffs(bits) - 1);
      if (pos_map != nullptr) pos_map[b] = static_cast<int32_t>(o);
      out[o++] = b;
      bits &= bits - 1u;
    }
    offset += total;
  }
}

__global__ void bitmap_set_kernel(uint32_t* __restrict__ bitmap, int64_t num_bits,
                                  const int64_t* __restrict__ ids, int64_t n,
                                  int32_t* __restrict__ err) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = ids[i];
    if (b < 0 || b >= num_bits) {
      report_error(err, TGS_DEV_ID_OUT_OF_RANGE, i);
      continue;
    }
    atomicOr(bitmap + (b >> 5), 1u << (b & 31));
  }
}

__global__ void gather_i64_kernel(int64_t* __restrict__ out, const int64_t* __restrict__ src,
                                  int64_t n_src, const int64_t* __restrict__ idx, int64_t n,
                                  int32_t* __restrict__ err) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = idx[i];
    if (j < 0 || j >= n_src) {
      report_error(err, TGS_DEV_ID_OUT_OF_RANGE, i);
      out[i] = -1;
    } else {
      out[i] = src[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Accumulation: warp per filter row, lane l adds UNIFIED columns 2l and 2l+1
// (as in the optimizer kernel). A warp resolves the touched positions of 32
// filter rows at once (one binary search per lane) into a shared table, then
// streams the rows kAccumUnroll at a time, loads before stores.
// ---------------------------------------------------------------------------
constexpr int kAccumThreads = 256;
constexpr int kAccumWarps = kAccumThreads / 32;
constexpr int kAccumUnroll = 4;

struct AccumParams {
  const int64_t* touched;
  int64_t n_touched;
  const int32_t* pos_map;
  int64_t pos_map_len;
  const int64_t* filter;
  int64_t n_filter;
  const float* src[kNumComp];
  int64_t stride[kNumComp];
  float* acc[kNumComp];
  int32_t* err;
};

// First index p in [0, n) with a[p] >= x (n if none).
__device__ __forceinline__ int64_t lower_bound_i64(const int64_t* __restrict__ a, int64_t n,
                                                   int64_t x) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (__ldg(a + mid) < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

template <bool kUnique>
__global__ void __launch_bounds__(kAccumThreads) sparse_accum_kernel(const AccumParams a) {
  __shared__ int64_t s_pos[kAccumWarps][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const float* sbase[2];
  float* abase[2];
  int64_t sstride[2];
  int width[2];
  bool on[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = 2 * lane + e;
    const bool act = j < kRowWidth;
    const int c = act ? unified_comp_of(j) : 0;
    const int k = act ? j - unified_offset(c) : 0;
    const float* s = pick6(a.src, c);
    on[e] = act && s != nullptr;
    sbase[e] = s != nullptr ? s + k : nullptr;
    abase[e] = pick6(a.acc, c) + k;
    sstride[e] = pick6(a.stride, c);
    width[e] = comp_width(c);
  }
  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * kAccumWarps + warp;
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kAccumWarps;
  for (int64_t chunk = warp_id; chunk * 32 < a.n_filter; chunk += warp_stride) {
    const int64_t row0 = chunk * 32;
    const int nr = static_cast<int>(min64(32, a.n_filter - row0));
    if (lane < nr) {
      const int64_t f = a.filter[row0 + lane];
      int64_t p;
      if (a.pos_map != nullptr) {
        p = (f >= 0 && f < a.pos_map_len) ? static_cast<int64_t>(a.pos_map[f]) : -1;
      } else {
        p = lower_bound_i64(a.touched, a.n_touched, f);
        if (p >= a.n_touched || __ldg(a.touched + p) != f) p = -1;
      }
      if (p < 0) report_error(a.err, TGS_DEV_ID_NOT_TOUCHED, row0 + lane);
      s_pos[warp][lane] = p;
    }
    __syncwarp();
    for (int r = 0; r < nr; r += kAccumUnroll) {
      float x0[kAccumUnroll], x1[kAccumUnroll], y0[kAccumUnroll], y1[kAccumUnroll];
      int64_t pos[kAccumUnroll];
#pragma unroll
      for (int u = 0; u < kAccumUnroll; ++u) {
        const int rr = r + u;  // warp-uniform
        pos[u] = rr < nr ? s_pos[warp][rr] : -1;
        x0[u] = x1[u] = y0[u] = y1[u] = 0.f;
        if (pos[u] >= 0) {
          const int64_t row = row0 + rr;
          if (on[0]) x0[u] = sbase[0][row * sstride[0]];
          if (on[1]) x1[u] = sbase[1][row * sstride[1]];
          if (kUnique) {
            if (on[0]) y0[u] = abase[0][pos[u] * width[0]];
            if (on[1]) y1[u] = abase[1][pos[u] * width[1]];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kAccumUnroll; ++u) {
        if (pos[u] < 0) continue;
        if (kUnique) {
          if (on[0]) abase[0][pos[u] * width[0]] = fadd(y0[u], x0[u]);
          if (on[1]) abase[1][pos[u] * width[1]] = fadd(y1[u], x1[u]);
        } else {
          if (on[0]) atomicAdd(abase[0] + pos[u] * width[0], x0[u]);
          if (on[1]) atomicAdd(abase[1] + pos[u] * width[1], x1[u]);
        }
      }
    }
    __syncwarp();  // the table is rewritten by the next chunk
  }
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int64_t tgs_bitmap_list_scratch_words(int64_t num_bits) {
  const int64_t words = ceil_div<int64_t>(std::max<int64_t>(num_bits, 0), 32);
  return ceil_div<int64_t>(words, kListTileWords) + 1;
}

extern "C" int tgs_bitmap_list(const uint32_t* bitmap, int64_t num_bits, int64_t* out_ids,
                               int64_t* dev_count, int64_t* scratch, int32_t* pos_map,
                               void* stream) {
  TGS_CHECK_ARG(num_bits >= 0, "tgs_bitmap_list: num_bits < 0");
  TGS_CHECK_ARG(dev_count != nullptr && scratch != nullptr, "tgs_bitmap_list: NULL count/scratch");
  cudaStream_t s = as_stream(stream);
  if (num_bits == 0) {
    TGS_CUDA(cudaMemsetAsync(dev_count, 0, sizeof(int64_t), s));
    return TGS_OK;
  }
  TGS_CHECK_ARG(bitmap != nullptr && out_ids != nullptr, "tgs_bitmap_list: NULL pointer");
  const int64_t words = ceil_div<int64_t>(num_bits, 32);
  const int64_t tiles = ceil_div<int64_t>(words, kListTileWords);
  TGS_CHECK_ARG(tiles < (1ll << 31), "tgs_bitmap_list: num_bits too large");
  bitmap_count_kernel<<<static_cast<unsigned>(tiles), kListThreads, 0, s>>>(bitmap, num_bits,
                                                                            scratch);
  TGS_LAUNCH_CHECK();
  scan_counts_kernel<<<1, 1024, 0, s>>>(scratch, tiles, dev_count);
  TGS_LAUNCH_CHECK();
  bitmap_write_kernel<<<static_cast<unsigned>(tiles), kListThreads, 0, s>>>(
      bitmap, num_bits, scratch, out_ids, pos_map);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_bitmap_set(uint32_t* bitmap, int64_t num_bits, const int64_t* ids, int64_t n,
                              int32_t* err, void* stream) {
  TGS_CHECK_ARG(n >= 0 && num_bits >= 0, "tgs_bitmap_set: bad sizes");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(bitmap && ids, "tgs_bitmap_set: NULL pointer");
  const int grid = static_cast<int>(
      std::min<int64_t>(ceil_div<int64_t>(n, 256), static_cast<int64_t>(sm_count()) * 8));
  bitmap_set_kernel<<<grid, 256, 0, as_stream(stream)>>>(bitmap, num_bits, ids, n, err);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_gather_i64(int64_t* out, const int64_t* src, int64_t n_src,
                              const int64_t* idx, int64_t n, int32_t* err, void* stream) {
  TGS_CHECK_ARG(n >= 0 && n_src >= 0, "tgs_gather_i64: bad sizes");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(out && src && idx, "tgs_gather_i64: NULL pointer");
  const int grid = static_cast<int>(
      std::min<int64_t>(ceil_div<int64_t>(n, 256), static_cast<int64_t>(sm_count()) * 8));
  gather_i64_kernel<<<grid, 256, 0, as_stream(stream)>>>(out, src, n_src, idx, n, err);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_sparse_grad_accumulate(const TgsSparseAccumArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_sparse_grad_accumulate: args is NULL");
  TGS_CHECK_ARG(a->n_filter >= 0 && a->n_touched >= 0, "tgs_sparse_grad_accumulate: bad sizes");
  if (a->n_filter == 0) return TGS_OK;
  TGS_CHECK_ARG(a->filter != nullptr && (a->touched != nullptr || a->n_touched == 0),
                "tgs_sparse_grad_accumulate: NULL ids");
  AccumParams p;
  p.touched = a->touched;
  p.n_touched = a->n_touched;
  p.pos_map = a->pos_map;
  p.pos_map_len = a->pos_map != nullptr ? a->pos_map_len : 0;
  p.filter = a->filter;
  p.n_filter = a->n_filter;
  p.err = a->err;
  for (int c = 0; c < kNumComp; ++c) {
    p.src[c] = a->src[c];
    p.stride[c] = a->src_stride[c];
    p.acc[c] = a->acc[c];
    if (a->src[c] != nullptr) {
      TGS_CHECK_ARG(a->acc[c] != nullptr, "tgs_sparse_grad_accumulate: component %d has no output",
                    c);
      TGS_CHECK_ARG(a->src_stride[c] >= comp_width(c),
                    "tgs_sparse_grad_accumulate: stride %lld of component %d below its width",
                    (long long)a->src_stride[c], c);
    }
  }
  const int64_t warps = ceil_div<int64_t>(a->n_filter, 32);
  const int grid = static_cast<int>(std::min<int64_t>(ceil_div<int64_t>(warps, kAccumWarps),
                                                      static_cast<int64_t>(sm_count()) * 8));
  if (a->unique_filter) sparse_accum_kernel<true><<<grid, kAccumThreads, 0, as_stream(stream)>>>(p);
  else sparse_accum_kernel<false><<<grid, kAccumThreads, 0, as_stream(stream)>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}
