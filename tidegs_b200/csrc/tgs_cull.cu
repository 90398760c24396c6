// Block frustum culling (storage/gaussian_block.py:264-511 FrustumCuller,
// 6-plane path :429-465; plane extraction :145-228 stays on the host).
//
// Each block is a bounding sphere of its xyz bounds: center = (min+max)/2,
// radius = |max-min|/2 * 1.15 (gaussian_block.py:286-298). A block is visible
// to a camera when its signed distance to each of the camera's 6 normalized
// planes is >= -radius. The reference evaluates these in numpy float32 with
// every operation rounded once and the sums strictly left to right
// (((a0+a1)+a2) for the norm, (((p0c0+p1c1)+p2c2)+p3) for the distance); the
// kernels use the same exactly rounded operations in the same order, so the
// visible sets are identical.
//
// Each camera's candidates are split into slices of 4096; a counting pass
// and a writing pass run as (slice, camera) grids, so a camera batch fills
// the SMs. The writing pass starts each slice at the sum of the earlier
// slices' counts and appends the visible ids chunk by chunk (warp ballots and
// a CTA prefix sum), i.e. in candidate order (the reference's np.where /
// boolean-mask order).
#include "tgs_common.cuh"

namespace tgs {
namespace {

constexpr int kCullThreads = 1024;
constexpr int kCullWarps = kCullThreads / 32;
constexpr float kRadiusMargin = 1.15f;  // float32 value of the reference's 1.15

__global__ void sphere_kernel(const float* __restrict__ bounds, int64_t n,
                              float* __restrict__ centers, float* __restrict__ radii) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float* b = bounds + i * 6;
    float d[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float lo = b[k], hi = b[3 + k];
      centers[i * 3 + k] = fdiv(fadd(lo, hi), 2.0f);
      d[k] = fsub(hi, lo);
    }
    const float s = fadd(fadd(fmul(d[0], d[0]), fmul(d[1], d[1])), fmul(d[2], d[2]));
    radii[i] = fmul(fdiv(fsqrt(s), 2.0f), kRadiusMargin);
  }
}

struct CullParams {
  const float* centers;   // [n_blocks, 3]
  const float* radii;     // [n_blocks]
  int64_t n_blocks;
  const int64_t* subset;  // candidate block ids, or NULL for 0..n_blocks-1
  int64_t n_items;
  const float* planes;    // [n_cameras, 6, 4]
  int64_t* out_ids;       // [n_cameras, out_stride]
  int64_t out_stride;
  int64_t* out_counts;    // [n_cameras]
  int64_t* slice_counts;  // [n_cameras, n_slices]
  int n_slices;
  int32_t* err;
};

// Candidates per CTA in both passes: a camera's candidates are split into
// slices so that a batch of cameras spreads over the SMs.
constexpr int kCullSlice = 4 * kCullThreads;

// Whether candidate i is visible to the camera whose planes are in pl; *id
// receives the block id.
__device__ __forceinline__ bool candidate_visible(const CullParams& a, const float* pl, int64_t i,
                                                  int64_t* id, bool report) {
  if (i >= a.n_items) return false;
  const int64_t b = a.subset != nullptr ? a.subset[i] : i;
  *id = b;
  if (b < 0 || b >= a.n_blocks) {
    if (report) report_error(a.err, TGS_DEV_ID_OUT_OF_RANGE, i);
    return false;
  }
  const float cx = a.centers[b * 3], cy = a.centers[b * 3 + 1], cz = a.centers[b * 3 + 2];
  const float neg_r = -a.radii[b];
  bool vis = true;
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    const float d = fadd(fadd(fadd(fmul(pl[j * 4], cx), fmul(pl[j * 4 + 1], cy)),
                              fmul(pl[j * 4 + 2], cz)),
                         pl[j * 4 + 3]);
    vis = vis && (d >= neg_r);
  }
  return vis;
}

// Pass 1, grid (slice, camera): visible candidates per slice.
__global__ void __launch_bounds__(kCullThreads) cull_count_kernel(const CullParams a) {
  __shared__ float pl[24];
  __shared__ int warp_n[kCullWarps];
  const int tid = threadIdx.x;
  const int64_t cam = blockIdx.y;
  if (tid < 24) pl[tid] = a.planes[cam * 24 + tid];
  __syncthreads();
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * kCullSlice;
  int n = 0;
  for (int k = 0; k < kCullSlice; k += kCullThreads) {
    int64_t id = 0;
    n += candidate_visible(a, pl, begin + k + tid, &id, true) ? 1 : 0;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  if ((tid & 31) == 0) warp_n[tid >> 5] = n;
  __syncthreads();
  if (tid < 32) {
    int v = warp_n[tid];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (tid == 0) a.slice_counts[cam * a.n_slices + blockIdx.x] = v;
  }
}

// Pass 2, grid (slice, camera): the slice's visible ids in candidate order at
// the slice's offset (sum of the earlier slices' counts); the last slice
// writes the camera's total.
__global__ void __launch_bounds__(kCullThreads) cull_write_kernel(const CullParams a) {
  __shared__ float pl[24];
  __shared__ int warp_off[kCullWarps];
  __shared__ int chunk_total;
  __shared__ int64_t slice_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t cam = blockIdx.y;
  if (tid < 24) pl[tid] = a.planes[cam * 24 + tid];
  if (tid < 32) {
    int64_t sum = 0;
    for (int s = lane; s < static_cast<int>(blockIdx.x); s += 32)
      sum += a.slice_counts[cam * a.n_slices + s];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) slice_base = sum;
  }
  __syncthreads();
  int64_t* out = a.out_ids + cam * a.out_stride;
  int64_t base = slice_base;
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * kCullSlice;
  for (int k = 0; k < kCullSlice; k += kCullThreads) {
    int64_t id = 0;
    const bool vis = candidate_visible(a, pl, begin + k + tid, &id, false);
    const unsigned m = __ballot_sync(0xffffffffu, vis);
    if (lane == 0) warp_off[warp] = __popc(m);
    __syncthreads();
    if (warp == 0) {
      const int v = warp_off[lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      warp_off[lane] = incl - v;
      if (lane == 31) chunk_total = incl;
    }
    __syncthreads();
    if (vis) out[base + warp_off[warp] + __popc(m & ((1u << lane) - 1u))] = id;
    base += chunk_total;
    __syncthreads();
  }
  if (tid == 0 && static_cast<int>(blockIdx.x) == a.n_slices - 1) a.out_counts[cam] = base;
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_block_spheres(const float* bounds, int64_t n_blocks, float* centers,
                                 float* radii, void* stream) {
  TGS_CHECK_ARG(n_blocks >= 0, "tgs_block_spheres: n_blocks < 0");
  if (n_blocks == 0) return TGS_OK;
  TGS_CHECK_ARG(bounds && centers && radii, "tgs_block_spheres: NULL pointer");
  const int grid = static_cast<int>(
      std::min<int64_t>(ceil_div<int64_t>(n_blocks, 256), static_cast<int64_t>(sm_count()) * 8));
  sphere_kernel<<<grid, 256, 0, as_stream(stream)>>>(bounds, n_blocks, centers, radii);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int64_t tgs_frustum_cull_slices(int64_t n_items) {
  return n_items <= 0 ? 1 : ceil_div<int64_t>(n_items, kCullSlice);
}

extern "C" int tgs_frustum_cull(const TgsCullArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_frustum_cull: args is NULL");
  TGS_CHECK_ARG(a->n_blocks >= 0 && a->n_items >= 0 && a->n_cameras >= 0,
                "tgs_frustum_cull: negative size");
  if (a->n_cameras == 0) return TGS_OK;
  TGS_CHECK_ARG(a->n_cameras <= 65535, "tgs_frustum_cull: at most 65535 cameras per call");
  TGS_CHECK_ARG(a->planes && a->out_counts && a->slice_counts,
                "tgs_frustum_cull: NULL planes, counts or slice counts");
  TGS_CHECK_ARG(a->n_items == 0 || (a->centers && a->radii && a->out_ids),
                "tgs_frustum_cull: NULL blocks or output");
  TGS_CHECK_ARG(a->out_stride >= a->n_items, "tgs_frustum_cull: out_stride < n_items");
  if (a->subset == nullptr)
    TGS_CHECK_ARG(a->n_items == a->n_blocks, "tgs_frustum_cull: without a subset, n_items "
                  "must equal n_blocks");
  const int64_t slices = tgs_frustum_cull_slices(a->n_items);
  TGS_CHECK_ARG(slices < (1ll << 31), "tgs_frustum_cull: too many candidates");
  CullParams p;
  p.centers = a->centers;
  p.radii = a->radii;
  p.n_blocks = a->n_blocks;
  p.subset = a->subset;
  p.n_items = a->n_items;
  p.planes = a->planes;
  p.out_ids = a->out_ids;
  p.out_stride = a->out_stride;
  p.out_counts = a->out_counts;
  p.slice_counts = a->slice_counts;
  p.n_slices = static_cast<int>(slices);
  p.err = a->err;
  const dim3 grid(static_cast<unsigned>(slices), static_cast<unsigned>(a->n_cameras));
  cudaStream_t s = as_stream(stream);
  cull_count_kernel<<<grid, kCullThreads, 0, s>>>(p);
  TGS_LAUNCH_CHECK();
  cull_write_kernel<<<grid, kCullThreads, 0, s>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}
