// Owner-side reduction of exchanged per-block gradient tiles.
//
// After the all-to-all of block gradients (owner = block_id mod world), the
// owner holds, for each of its visible blocks, one [block_size, 59] tile per
// sender that saw the block. This kernel sums those tiles in sender order and
// writes the result as the six compact SoA gradient components the resident
// Adam step consumes, in the owner's row order. The summation order is fixed
// (sender 0 first), so the result equals a single-GPU sum in rank order bit for
// bit. No counterpart in the reference (it is single-GPU).
#include "tgs_common.cuh"

namespace tgs {
namespace {

constexpr int kSumThreads = 256;
constexpr int kSumTileRows = 64;

struct BlockSumParams {
  const float* recv;               // [n_recv_blocks * B, 59] AoS, UNIFIED order
  const int64_t* contrib_offsets;  // [n_out + 1]
  const int64_t* contrib_blocks;   // recv tile index per contribution
  int n_out;
  int64_t block_size;
  int64_t n_recv_blocks;
  float* out[kNumComp];            // [n_out * B, W_c]
  int32_t* err;
};

// Grid (row tile, output block). Each thread owns elements of the 64-row x
// 59-column tile in AoS order; contributions are added in sender order, then
// the tile is written to the component arrays through shared memory so both
// the AoS reads and the SoA writes are coalesced.
__global__ void __launch_bounds__(kSumThreads) block_sum_kernel(const BlockSumParams a) {
  __shared__ float tile[kSumTileRows * kRowWidth];
  for (int k = blockIdx.y; k < a.n_out; k += gridDim.y) {
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kSumTileRows;
    if (r0 >= a.block_size) continue;
    const int rows = static_cast<int>(min64(kSumTileRows, a.block_size - r0));
    const int64_t c0 = a.contrib_offsets[k];
    const int64_t c1 = a.contrib_offsets[k + 1];
    const int n = rows * kRowWidth;
    for (int e = threadIdx.x; e < n; e += kSumThreads) {
      float acc = 0.0f;
      for (int64_t c = c0; c < c1; ++c) {
        const int64_t blk = a.contrib_blocks[c];
        if (blk < 0 || blk >= a.n_recv_blocks) {
          report_error(a.err, TGS_DEV_BAD_SLICE, c);
          continue;
        }
        const float* src = a.recv + (blk * a.block_size + r0) * kRowWidth;
        acc = (c == c0) ? src[e] : fadd(acc, src[e]);
      }
      tile[e] = acc;
    }
    __syncthreads();
#pragma unroll
    for (int comp = 0; comp < kNumComp; ++comp) {
      const int w = comp_width(comp);
      const int col = unified_offset(comp);
      float* dst = a.out[comp] + (static_cast<int64_t>(k) * a.block_size + r0) * w;
      for (int e = threadIdx.x; e < rows * w; e += kSumThreads) {
        const int r = e / w;
        dst[e] = tile[r * kRowWidth + col + (e - r * w)];
      }
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_block_grad_sum(const TgsBlockSumArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_block_grad_sum: args is NULL");
  TGS_CHECK_ARG(a->n_out >= 0 && a->block_size >= 1 && a->n_recv_blocks >= 0,
                "tgs_block_grad_sum: bad sizes");
  if (a->n_out == 0) return TGS_OK;
  TGS_CHECK_ARG(a->recv && a->contrib_offsets && a->contrib_blocks,
                "tgs_block_grad_sum: NULL plan");
  BlockSumParams p;
  p.recv = a->recv;
  p.contrib_offsets = a->contrib_offsets;
  p.contrib_blocks = a->contrib_blocks;
  p.n_out = a->n_out;
  p.block_size = a->block_size;
  p.n_recv_blocks = a->n_recv_blocks;
  p.err = a->err;
  for (int c = 0; c < kNumComp; ++c) {
    TGS_CHECK_ARG(a->out[c] != nullptr, "tgs_block_grad_sum: output component %d is NULL", c);
    p.out[c] = a->out[c];
  }
  const int64_t tiles = ceil_div<int64_t>(a->block_size, kSumTileRows);
  TGS_CHECK_ARG(tiles < (1ll << 31), "tgs_block_grad_sum: block_size too large");
  dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(std::min(a->n_out, 65535)));
  block_sum_kernel<<<grid, kSumThreads, 0, as_stream(stream)>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}
