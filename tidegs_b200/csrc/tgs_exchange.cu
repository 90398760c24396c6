// Owner-side reduction of exchanged per-block gradient tiles.
//
// After the all-to-all of block gradients (owner = block_id mod world), the
// owner holds, for each of its visible blocks, one [block_size, 59] tile per
// sender that saw the block. This kernel sums those tiles in sender order and
// writes the result as the six compact SoA gradient components the resident
// Adam step consumes, in the owner's row order. The summation order is fixed
// (sender 0 first), so the result equals a single-GPU sum in rank order bit for
// bit. No counterpart in the reference (it is single-GPU).
//
// The tiles reach the owners either through an all-to-all (after
// tgs_pack_rows) or through tgs_grad_push below, which gathers each tile and
// stores it straight into the owner's receive buffer over NVLink (a CUDA IPC
// mapping of the owner's buffer), so the pack pass, the send buffer and the
// collective's own copy disappear.
#include <cuda.h>

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

// ---------------------------------------------------------------------------
// Direct push: grid (64-row tile, sent block). The CTA gathers its tile of
// the sender's SoA gradient components into an AoS UNIFIED tile in shared
// memory (coalesced component reads), then stores the tile into the owner's
// receive buffer with 16-byte stores when the destination rows allow it.
// Remote stores are plain st.global through the peer mapping: no TMA or bulk
// copy touches another GPU's memory.
// ---------------------------------------------------------------------------
constexpr int kPushThreads = 256;
constexpr int kPushTileRows = 64;

struct PushParams {
  const float* comp[kNumComp];
  const int64_t* src_start;
  const int64_t* row_count;
  const int32_t* dst_rank;
  const int64_t* dst_row;
  int n_tiles;
  float* recv[TGS_MAX_PEERS];
  int64_t recv_rows[TGS_MAX_PEERS];
  int n_ranks;
  int32_t* err;
};

__global__ void __launch_bounds__(kPushThreads) grad_push_kernel(const PushParams a) {
  __shared__ __align__(16) float tile[kPushTileRows * kRowWidth];
  __shared__ float* s_dst;
  for (int k = blockIdx.y; k < a.n_tiles; k += gridDim.y) {
    const int64_t rows_total = a.row_count[k];
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kPushTileRows;
    if (r0 >= rows_total) continue;
    const int rows = static_cast<int>(min64(kPushTileRows, rows_total - r0));
    if (threadIdx.x == 0) {
      const int d = a.dst_rank[k];
      const int64_t row = a.dst_row[k];
      float* dst = nullptr;
      if (d >= 0 && d < a.n_ranks && row >= 0 && rows_total <= a.recv_rows[d] &&
          row <= a.recv_rows[d] - rows_total && a.recv[d] != nullptr)
        dst = a.recv[d] + (row + r0) * kRowWidth;
      else if (blockIdx.x == 0)
        report_error(a.err, TGS_DEV_BAD_SLICE, k, d);
      s_dst = dst;
    }
    const int64_t src = a.src_start[k] + r0;
#pragma unroll
    for (int c = 0; c < kNumComp; ++c) {
      const int w = comp_width(c);
      const int col = unified_offset(c);
      const float* __restrict__ s = a.comp[c] + src * w;
      for (int e = threadIdx.x; e < rows * w; e += kPushThreads) {
        const int r = e / w;
        tile[r * kRowWidth + col + (e - r * w)] = s[e];
      }
    }
    __syncthreads();
    float* dst = s_dst;
    if (dst != nullptr) {
      const int n = rows * kRowWidth;
      if (aligned16(dst) && (n & 3) == 0) {
        float4* d4 = reinterpret_cast<float4*>(dst);
        const float4* t4 = reinterpret_cast<const float4*>(tile);
        for (int e = threadIdx.x; e < (n >> 2); e += kPushThreads) d4[e] = t4[e];
      } else {
        for (int e = threadIdx.x; e < n; e += kPushThreads) dst[e] = tile[e];
      }
    }
    __syncthreads();
  }
  // Order this thread's remote stores before anything the owner is told
  // later (the barrier collective that follows on the stream).
  __threadfence_system();
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

extern "C" int tgs_grad_push(const TgsGradPushArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_grad_push: args is NULL");
  TGS_CHECK_ARG(a->n_tiles >= 0 && a->max_rows >= 0, "tgs_grad_push: bad sizes");
  TGS_CHECK_ARG(a->n_ranks >= 1 && a->n_ranks <= TGS_MAX_PEERS,
                "tgs_grad_push: n_ranks=%d outside [1, %d]", a->n_ranks, TGS_MAX_PEERS);
  if (a->n_tiles == 0 || a->max_rows == 0) return TGS_OK;
  TGS_CHECK_ARG(a->src_start && a->row_count && a->dst_rank && a->dst_row,
                "tgs_grad_push: NULL plan");
  PushParams p;
  for (int c = 0; c < kNumComp; ++c) {
    TGS_CHECK_ARG(a->comp[c] != nullptr, "tgs_grad_push: component %d is NULL", c);
    p.comp[c] = a->comp[c];
  }
  for (int r = 0; r < TGS_MAX_PEERS; ++r) {
    const bool used = r < a->n_ranks;
    TGS_CHECK_ARG(!used || (a->recv[r] != nullptr && a->recv_rows[r] >= 0),
                  "tgs_grad_push: receive buffer of rank %d is missing", r);
    p.recv[r] = used ? a->recv[r] : nullptr;
    p.recv_rows[r] = used ? a->recv_rows[r] : 0;
  }
  p.src_start = a->src_start;
  p.row_count = a->row_count;
  p.dst_rank = a->dst_rank;
  p.dst_row = a->dst_row;
  p.n_tiles = a->n_tiles;
  p.n_ranks = a->n_ranks;
  p.err = a->err;
  const int64_t tiles = ceil_div<int64_t>(a->max_rows, kPushTileRows);
  TGS_CHECK_ARG(tiles < (1ll << 31), "tgs_grad_push: max_rows too large");
  dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(std::min(a->n_tiles, 65535)));
  grad_push_kernel<<<grid, kPushThreads, 0, as_stream(stream)>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

static_assert(sizeof(cudaIpcMemHandle_t) == TGS_PEER_HANDLE_BYTES,
              "TgsPeerHandle must hold a cudaIpcMemHandle_t");

extern "C" int tgs_peer_buffer_alloc(int64_t bytes, void** dev_ptr, TgsPeerHandle* handle) {
  TGS_CHECK_ARG(bytes > 0 && dev_ptr != nullptr && handle != nullptr,
                "tgs_peer_buffer_alloc: bad arguments (bytes=%lld)", (long long)bytes);
  void* p = nullptr;
  TGS_CUDA(cudaMalloc(&p, static_cast<size_t>(bytes)));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    set_error("cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
    return TGS_ERR_CUDA;
  }
  memcpy(handle->bytes, &h, sizeof(h));
  *dev_ptr = p;
  return TGS_OK;
}

extern "C" int tgs_peer_buffer_free(void* dev_ptr) {
  if (dev_ptr == nullptr) return TGS_OK;
  TGS_CUDA(cudaFree(dev_ptr));
  return TGS_OK;
}

extern "C" int tgs_peer_buffer_open(const TgsPeerHandle* handle, void** dev_ptr) {
  TGS_CHECK_ARG(handle != nullptr && dev_ptr != nullptr, "tgs_peer_buffer_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  void* p = nullptr;
  TGS_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *dev_ptr = p;
  return TGS_OK;
}

extern "C" int tgs_peer_buffer_close(void* dev_ptr) {
  if (dev_ptr == nullptr) return TGS_OK;
  TGS_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return TGS_OK;
}

extern "C" int tgs_peer_export(const void* dev_ptr, TgsPeerHandle* handle, int64_t* offset) {
  TGS_CHECK_ARG(dev_ptr != nullptr && handle != nullptr && offset != nullptr,
                "tgs_peer_export: NULL argument");
  // The allocation base comes from the driver (no libcuda link: the entry
  // point is resolved through the runtime).
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  if (get_range == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    TGS_CUDA(cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000,
                                              cudaEnableDefault, &q));
    TGS_CHECK_ARG(q == cudaDriverEntryPointSuccess && fn != nullptr,
                  "tgs_peer_export: cuMemGetAddressRange not available");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = get_range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
  TGS_CHECK_ARG(r == CUDA_SUCCESS, "tgs_peer_export: %p is not device memory (driver error %d)",
                dev_ptr, static_cast<int>(r));
  cudaIpcMemHandle_t h;
  TGS_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle->bytes, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return TGS_OK;
}

extern "C" int tgs_peer_access_enable(int32_t peer_device) {
  int dev = 0;
  TGS_CUDA(cudaGetDevice(&dev));
  if (peer_device == dev) return TGS_OK;
  int can = 0;
  TGS_CUDA(cudaDeviceCanAccessPeer(&can, dev, peer_device));
  TGS_CHECK_ARG(can != 0, "tgs_peer_access_enable: device %d cannot access device %d", dev,
                peer_device);
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // reset the last-error state this call left behind
    return TGS_OK;
  }
  TGS_CUDA(e);
  return TGS_OK;
}
