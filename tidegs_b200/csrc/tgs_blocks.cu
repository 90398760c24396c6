// Block data movement: streamed-row unpack, slot-remap copies, global-id maps,
// write-back pack and per-block bounds.
//
// Reference behaviour followed:
//   strategies/tide_engine/double_buffer_gpu.py:40-128   _copy_resident_rows_kernel
//   strategies/tide_engine/double_buffer_gpu.py:130-148  _fill_cold_global_ids_kernel
//   strategies/tide_engine/double_buffer_gpu.py:150-209  _unpack_streamed_rows_kernel
//   strategies/tide_engine/double_buffer_gpu.py:212-256  block starts / global->local
//   strategies/tide_engine/gpu_working_set.py:35-115     pack + bounds kernels
#include <mutex>

#include "tgs_common.cuh"
#include "tgs_scan.cuh"

namespace tgs {
namespace {

struct Comp6 {
  float* p[kNumComp];
};
struct ConstComp6 {
  const float* p[kNumComp];
};

// ---------------------------------------------------------------------------
// Unpack: packed [rows, 59] -> six SoA components (+ global ids).
// Persistent CTAs walk 64-row tiles; one thread keeps kUnpackStages tiles in
// flight with bulk (TMA) copies into a shared-memory ring, while all threads
// scatter the oldest tile's columns into the component arrays with coalesced
// stores.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 64;
constexpr int kTileFloats = kTileRows * kRowWidth;  // 3776 floats = 15104 B (multiple of 16)
constexpr int kUnpackThreads = 256;
constexpr int kUnpackStages = 4;
constexpr int kUnpackCtasPerSm = 3;

struct UnpackParams {
  const float* packed;
  int64_t n_rows;
  int layout;
  Comp6 comp;
  int64_t target_offset;
  int64_t* gids;
  const int64_t* block_ids;
  int64_t block_size;
  int use_bulk;  // packed is 16-byte aligned
  int32_t* err;
  const int64_t* block_dst;  // first target row per block, or null (contiguous)
  int block_shift;           // block_size == 1 << block_shift, or -1
};

struct UnpackSmem {
  float tile[kUnpackStages][kTileFloats];
  uint64_t bar[kUnpackStages];
};
constexpr size_t kUnpackSmemBytes = sizeof(UnpackSmem);

// Writes a staged tile's rows into the six components. A component range
// that starts on a 16-byte boundary and holds a multiple of 4 floats (every
// full tile of a 16-byte aligned component whose first row is a multiple of
// 4) goes out as float4 stores, each thread gathering 4 consecutive floats of
// the range from the staged rows; other ranges use one float per thread.
template <int kLayout>
__device__ __forceinline__ void scatter_tile(const float* __restrict__ tile, int rows,
                                             int64_t dst_row0, const Comp6& comp) {
#pragma unroll
  for (int c = 0; c < kNumComp; ++c) {
    const int w = comp_width(c);
    const int src_col = layout_offset(kLayout, c);
    float* __restrict__ dst = comp.p[c] + dst_row0 * w;
    const int n = rows * w;
    if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
      for (int e4 = threadIdx.x; e4 < (n >> 2); e4 += kUnpackThreads) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int e = 4 * e4 + j;
          const int r = e / w;
          v[j] = tile[r * kRowWidth + src_col + (e - r * w)];
        }
        *reinterpret_cast<float4*>(dst + 4 * e4) = make_float4(v[0], v[1], v[2], v[3]);
      }
      continue;
    }
    for (int e = threadIdx.x; e < n; e += kUnpackThreads) {
      const int r = e / w;
      const int k = e - r * w;
      dst[e] = tile[r * kRowWidth + src_col + k];
    }
  }
}

template <int kLayout>
__global__ void __launch_bounds__(kUnpackThreads, kUnpackCtasPerSm) unpack_kernel(const UnpackParams a) {
  extern __shared__ __align__(128) unsigned char unpack_smem_raw[];
  UnpackSmem& sm = *reinterpret_cast<UnpackSmem*>(unpack_smem_raw);
  const int64_t n_tiles = ceil_div<int64_t>(a.n_rows, kTileRows);
  const int tid = threadIdx.x;

  // Rows of a tile the bulk engine can move: a multiple of 4 rows keeps the
  // byte count a multiple of 16; the (< 4) leftover rows use plain loads.
  auto tile_rows = [&](int64_t t) -> int {
    return static_cast<int>(min64(kTileRows, a.n_rows - t * kTileRows));
  };
  auto bulk_rows = [&](int rows) -> int { return a.use_bulk ? (rows & ~3) : 0; };

  if (tid == 0) {
    for (int q = 0; q < kUnpackStages; ++q) mbar_init(&sm.bar[q], 1);
    fence_mbar_init();
  }
  __syncthreads();

  uint32_t pending = 0;  // stages with a bulk copy in flight (thread 0)
  auto issue = [&](int64_t t, int q) {
    if (t >= n_tiles) return;
    const int br = bulk_rows(tile_rows(t));
    if (br > 0) {
      const uint32_t bytes = static_cast<uint32_t>(br) * kRowWidth * sizeof(float);
      mbar_arrive_expect_tx(&sm.bar[q], bytes);
      bulk_g2s(sm.tile[q], a.packed + t * kTileFloats, bytes, &sm.bar[q]);
      pending |= 1u << q;
    }
  };

  if (tid == 0)
    for (int q = 0; q < kUnpackStages; ++q) issue(blockIdx.x + static_cast<int64_t>(q) * gridDim.x, q);
  uint32_t phase = 0;  // bit q: parity of stage q's next completion
  int q = 0;
  for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    const int rows = tile_rows(t);
    const int br = bulk_rows(rows);
    float* tile = sm.tile[q];
    // Plain loads for rows the bulk copy does not cover (disjoint bytes).
    for (int e = br * kRowWidth + tid; e < rows * kRowWidth; e += kUnpackThreads)
      tile[e] = a.packed[t * kTileFloats + e];
    bool ok = true;
    if (br > 0) {
      ok = mbar_wait_bounded(&sm.bar[q], (phase >> q) & 1u);
      phase ^= 1u << q;
      if (tid == 0) pending &= ~(1u << q);
    }
    if (__syncthreads_or(!ok)) {
      report_error(a.err, TGS_DEV_WAIT_TIMEOUT, t);
      // Wait (bounded) for the copies still in flight before the shared
      // memory they target is released.
      if (tid == 0) {
        for (int k = 0; k < kUnpackStages; ++k)
          if (pending & (1u << k)) mbar_wait_bounded(&sm.bar[k], (phase >> k) & 1u);
      }
      __syncthreads();
      return;
    }
    // a tile never straddles two blocks in the scatter mode (block_size is a
    // multiple of the tile), so its target rows stay contiguous
    const int64_t row0 = t * kTileRows;
    int64_t dst_row0 = a.target_offset + row0;
    if (a.block_dst != nullptr) {  // block_size >= kTileRows here
      const int64_t blk0 = a.block_shift >= 0 ? row0 >> a.block_shift : row0 / a.block_size;
      dst_row0 = a.block_dst[blk0] + (row0 - blk0 * a.block_size);
    }
    scatter_tile<kLayout>(tile, rows, dst_row0, a.comp);
    if (a.gids != nullptr) {
      for (int r = tid; r < rows; r += kUnpackThreads) {
        const int64_t row = row0 + r;
        const int64_t pos = a.block_shift >= 0 ? row >> a.block_shift : row / a.block_size;
        a.gids[dst_row0 + r] = a.block_ids[pos] * a.block_size + (row - pos * a.block_size);
      }
    }
    // This stage's generic-proxy reads/writes precede the bulk copy that
    // refills it.
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) issue(t + static_cast<int64_t>(kUnpackStages) * gridDim.x, q);
    q = (q + 1 == kUnpackStages) ? 0 : q + 1;
  }
}

// ---------------------------------------------------------------------------
// Slot-remap copy. Grid (row chunk, block). For each block the CTA copies its
// chunk of rows of the six components and of the int64 global ids. When both
// slices start at a multiple of 4 rows the 16-byte rule holds for every
// segment, and one thread drives a 4-stage bulk pipeline
// (global -> shared -> global, mbarrier completion, bulk groups for stores);
// the other rows go through plain coalesced copies.
// ---------------------------------------------------------------------------
constexpr int kCopyThreads = 128;
constexpr int kCopyStages = 4;
constexpr uint32_t kCopyPiece = 16384;
constexpr int64_t kCopyChunkRows = 2048;  // multiple of 4

struct CopyParams {
  ConstComp6 src;
  Comp6 dst;
  const int64_t* src_gids;
  int64_t* dst_gids;
  const int64_t* src_start;
  const int64_t* dst_start;
  const int64_t* row_count;
  int n_blocks;
  int bases_aligned;  // every component / id base pointer is 16-byte aligned
  int32_t* err;
};

struct Segment {
  const char* src;
  char* dst;
  uint32_t bytes;
};

// Runs the bulk pipeline over `segs` (thread 0 only): pieces of at most
// kCopyPiece bytes go global -> stage slot -> global. Piece i uses slot
// i % kCopyStages. After piece i is stored, the slot of piece i-1 is refilled
// once at most one store group (piece i's) still reads shared memory.
// Returns false on a timed-out wait, after a bounded drain of the loads it
// started.
// `phase_bits` (bit k = parity to wait for on bars[k]) and `slot_base` (slot
// of this call's first piece) carry the barrier state across calls of one CTA.
__device__ bool bulk_copy_segments(const Segment* segs, int n_segs, unsigned char* stage,
                                   uint64_t* bars, uint32_t& phase_bits, uint32_t& slot_base) {
  int ls = 0, ss = 0;             // segment cursors: next load / next store
  uint32_t loff = 0, soff = 0;    // byte offsets inside those segments
  int64_t issued = 0, stored = 0;

  auto advance = [&](int& seg, uint32_t& off) {
    while (seg < n_segs && off >= segs[seg].bytes) {
      ++seg;
      off = 0;
    }
  };
  auto try_load = [&]() -> bool {
    advance(ls, loff);
    if (ls >= n_segs) return false;
    const uint32_t bytes = min(kCopyPiece, segs[ls].bytes - loff);
    const int slot = static_cast<int>((slot_base + issued) % kCopyStages);
    mbar_arrive_expect_tx(&bars[slot], bytes);
    bulk_g2s(stage + slot * kCopyPiece, segs[ls].src + loff, bytes, &bars[slot]);
    loff += bytes;
    ++issued;
    return true;
  };

  for (int k = 0; k < kCopyStages; ++k)
    if (!try_load()) break;
  bool ok = true;
  while (stored < issued) {
    const int slot = static_cast<int>((slot_base + stored) % kCopyStages);
    if (!mbar_wait_bounded(&bars[slot], (phase_bits >> slot) & 1u)) {
      ok = false;
      break;
    }
    phase_bits ^= 1u << slot;
    advance(ss, soff);
    const uint32_t bytes = min(kCopyPiece, segs[ss].bytes - soff);
    bulk_s2g(segs[ss].dst + soff, stage + slot * kCopyPiece, bytes);
    bulk_commit();
    soff += bytes;
    ++stored;
    if (stored >= 2) {
      bulk_wait_read<1>();
      try_load();
    }
  }
  if (!ok) {
    for (int64_t k = stored; k < issued; ++k) {
      const int slot = static_cast<int>((slot_base + k) % kCopyStages);
      if (!mbar_wait_bounded(&bars[slot], (phase_bits >> slot) & 1u)) break;
      phase_bits ^= 1u << slot;
    }
  }
  bulk_wait_all();
  slot_base = static_cast<uint32_t>((slot_base + issued) % kCopyStages);
  return ok;
}

__global__ void __launch_bounds__(kCopyThreads) copy_blocks_kernel(const CopyParams a) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kCopyStages * kCopyPiece);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kCopyStages; ++i) mbar_init(&bars[i], 1);
    fence_proxy_async_smem();
  }
  __syncthreads();
  if (load_error(a.err) != 0) return;
  uint32_t phase_bits = 0, slot_base = 0;  // thread 0's barrier state

  for (int k = blockIdx.y; k < a.n_blocks; k += gridDim.y) {
    const int64_t rows = a.row_count[k];
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kCopyChunkRows;
    if (r0 >= rows) continue;
    const int64_t r1 = min64(rows, r0 + kCopyChunkRows);
    const int64_t ss = a.src_start[k] + r0;
    const int64_t ds = a.dst_start[k] + r0;
    const bool bulk = a.bases_aligned && ((a.src_start[k] | a.dst_start[k]) & 3) == 0;
    const int64_t bulk_rows = bulk ? ((r1 - r0) & ~int64_t(3)) : 0;

    if (bulk_rows > 0 && threadIdx.x == 0) {
      Segment segs[kNumComp + 1];
      int n = 0;
#pragma unroll
      for (int c = 0; c < kNumComp; ++c) {
        const int w = comp_width(c);
        segs[n++] = {reinterpret_cast<const char*>(a.src.p[c] + ss * w),
                     reinterpret_cast<char*>(a.dst.p[c] + ds * w),
                     static_cast<uint32_t>(bulk_rows * w * sizeof(float))};
      }
      if (a.src_gids != nullptr && a.dst_gids != nullptr) {
        segs[n++] = {reinterpret_cast<const char*>(a.src_gids + ss),
                     reinterpret_cast<char*>(a.dst_gids + ds),
                     static_cast<uint32_t>(bulk_rows * sizeof(int64_t))};
      }
      if (!bulk_copy_segments(segs, n, smem, bars, phase_bits, slot_base))
        report_error(a.err, TGS_DEV_WAIT_TIMEOUT, k);
    }
    // Plain copies for the rows the bulk path did not take.
    const int64_t pr0 = bulk_rows;
    const int64_t prows = (r1 - r0) - pr0;
    if (prows > 0) {
#pragma unroll
      for (int c = 0; c < kNumComp; ++c) {
        const int w = comp_width(c);
        const float* __restrict__ s = a.src.p[c] + (ss + pr0) * w;
        float* __restrict__ d = a.dst.p[c] + (ds + pr0) * w;
        for (int64_t e = threadIdx.x; e < prows * w; e += kCopyThreads) d[e] = s[e];
      }
      if (a.src_gids != nullptr && a.dst_gids != nullptr) {
        for (int64_t e = threadIdx.x; e < prows; e += kCopyThreads)
          a.dst_gids[ds + pr0 + e] = a.src_gids[ss + pr0 + e];
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Global ids and block-start tables.
// ---------------------------------------------------------------------------
// shift >= 0: block_size == 1 << shift (a shift and a mask instead of a
// 64-bit division per row).
__global__ void fill_gids_kernel(int64_t* __restrict__ dst, int64_t offset,
                                 const int64_t* __restrict__ block_ids, int64_t n,
                                 int64_t block_size, int shift) {
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < n;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t pos = shift >= 0 ? r >> shift : r / block_size;
    const int64_t in_block = shift >= 0 ? r & (block_size - 1) : r - pos * block_size;
    dst[offset + r] = __ldg(block_ids + pos) * block_size + in_block;
  }
}

__global__ void scatter_block_starts_kernel(int64_t* __restrict__ block_starts, int64_t num_blocks,
                                            const int64_t* __restrict__ ids,
                                            const int64_t* __restrict__ starts, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) {
    const int64_t b = ids[i];
    if (b >= 0 && b < num_blocks) block_starts[b] = starts[i];
  }
}

__device__ __forceinline__ int64_t g2l(int64_t g, const int64_t* __restrict__ block_starts,
                                       int64_t num_blocks, int64_t block_size) {
  // floor division (ids may be negative)
  int64_t b = g / block_size;
  if ((g % block_size != 0) && ((g < 0) != (block_size < 0))) --b;
  if (b < 0 || b >= num_blocks) return -1;
  const int64_t s = block_starts[b];
  if (s < 0) return -1;
  return s + (g - b * block_size);
}

__global__ void g2l_kernel(int64_t* __restrict__ out, const int64_t* __restrict__ gids, int64_t n,
                           const int64_t* __restrict__ block_starts, int64_t num_blocks,
                           int64_t block_size) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = g2l(gids[i], block_starts, num_blocks, block_size);
}

// Ordered compaction of global->local, three phases over tiles of
// kCompactTile ids: (1) per-tile valid counts, (2) exclusive scan of the
// counts in one CTA, (3) per-tile warp-ballot ranks + tile offset -> output.
constexpr int kCompactThreads = 256;
constexpr int kCompactPerThread = 8;
constexpr int kCompactTile = kCompactThreads * kCompactPerThread;

__global__ void __launch_bounds__(kCompactThreads) g2l_count_kernel(
    const int64_t* __restrict__ gids, int64_t n, const int64_t* __restrict__ block_starts,
    int64_t num_blocks, int64_t block_size, int64_t* __restrict__ tile_counts) {
  __shared__ int warp_sums[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kCompactTile;
  int cnt = 0;
#pragma unroll
  for (int j = 0; j < kCompactPerThread; ++j) {
    const int64_t i = base + j * kCompactThreads + threadIdx.x;
    if (i < n && g2l(gids[i], block_starts, num_blocks, block_size) >= 0) ++cnt;
  }
  int total;
  block_exclusive_scan(cnt, warp_sums, total);
  if (threadIdx.x == 0) tile_counts[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kCompactThreads) g2l_write_kernel(
    int64_t* __restrict__ out, const int64_t* __restrict__ gids, int64_t n,
    const int64_t* __restrict__ block_starts, int64_t num_blocks, int64_t block_size,
    const int64_t* __restrict__ tile_offsets) {
  __shared__ int warp_sums[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kCompactTile;
  int64_t offset = tile_offsets[blockIdx.x];
  // Row-major over the tile: element base + j*threads + tid keeps each pass
  // coalesced; passes are ranked in order.
  for (int j = 0; j < kCompactPerThread; ++j) {
    const int64_t i = base + j * kCompactThreads + threadIdx.x;
    int64_t l = -1;
    if (i < n) l = g2l(gids[i], block_starts, num_blocks, block_size);
    const int flag = l >= 0 ? 1 : 0;
    int total;
    const int rank = block_exclusive_scan(flag, warp_sums, total);
    if (flag) out[offset + rank] = l;
    offset += total;
  }
}

// ---------------------------------------------------------------------------
// Write-back pack: SoA components -> packed rows (CACHE order by default).
// Persistent CTAs walk (plan, 64-row tile) pairs. A tile's rows of one
// component are contiguous in the SoA arrays, so one thread streams the six
// ranges into a shared-memory stage with bulk (TMA) copies, kPackStages tiles
// ahead of the consumer; all threads then write the tile's packed rows with
// coalesced stores, each element read from its component's range. Tiles whose
// ranges are not 16-byte aligned are read with plain loads instead.
// ---------------------------------------------------------------------------
constexpr int kPackThreads = 256;
constexpr int kPackStages = 4;
constexpr int kPackCtasPerSm = 3;

// First float of component c inside a staged tile (component order; every
// offset is a multiple of 64 floats, so each range starts 16-byte aligned).
__host__ __device__ constexpr int staged_offset(int c) {
  return kTileRows * unified_offset(c);
}

struct PackParams {
  ConstComp6 comp;
  const int64_t* src_start;
  const int64_t* row_count;
  const int64_t* out_start;
  int64_t n_tiles;     // n_plans * tiles_per_plan
  int tiles_per_plan;
  float* out;
  int comp_aligned;    // all six component bases are 16-byte aligned
  int32_t* err;
};

struct PackSmem {
  float stage[kPackStages][kTileFloats];
  uint64_t bar[kPackStages];
  // Output column j: staged offset of its component (low 16 bits) + column
  // within the component, and the component width (high 16 bits).
  uint32_t col[kRowWidth];
};
constexpr size_t kPackSmemBytes = sizeof(PackSmem);

struct PackTile {
  int rows;       // <= 0: nothing to do
  int64_t src;    // first source row
  int64_t dst;    // first output row
  bool bulk;
};

__device__ __forceinline__ PackTile pack_tile(const PackParams& a, int64_t t) {
  PackTile d;
  const int64_t k = t / a.tiles_per_plan;
  const int64_t r0 = (t - k * a.tiles_per_plan) * kTileRows;
  d.rows = static_cast<int>(min64(kTileRows, a.row_count[k] - r0));
  d.src = a.src_start[k] + r0;
  d.dst = a.out_start[k] + r0;
  d.bulk = a.comp_aligned && (d.src & 3) == 0 && (d.rows & 3) == 0;
  return d;
}

template <int kLayout>
__global__ void __launch_bounds__(kPackThreads, kPackCtasPerSm) pack_kernel(const PackParams a) {
  extern __shared__ __align__(128) unsigned char pack_smem_raw[];
  PackSmem& sm = *reinterpret_cast<PackSmem*>(pack_smem_raw);
  const int tid = threadIdx.x;
  if (tid < kRowWidth) {
    const int c = layout_comp_of(kLayout, tid);
    const int k = tid - layout_offset(kLayout, c);
    sm.col[tid] = static_cast<uint32_t>(staged_offset(c) + k) |
                  (static_cast<uint32_t>(comp_width(c)) << 16);
  }
  if (tid == 0) {
    for (int s = 0; s < kPackStages; ++s) mbar_init(&sm.bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  uint32_t pending = 0;  // stages with a bulk copy in flight (thread 0)
  auto issue = [&](int64_t t, int s) {
    if (t >= a.n_tiles) return;
    const PackTile d = pack_tile(a, t);
    if (d.rows <= 0 || !d.bulk) return;
    mbar_arrive_expect_tx(&sm.bar[s], static_cast<uint32_t>(d.rows) * kRowWidth * sizeof(float));
#pragma unroll
    for (int c = 0; c < kNumComp; ++c) {
      const int w = comp_width(c);
      bulk_g2s(&sm.stage[s][staged_offset(c)], a.comp.p[c] + d.src * w,
               static_cast<uint32_t>(d.rows * w) * sizeof(float), &sm.bar[s]);
    }
    pending |= 1u << s;
  };

  if (tid == 0) {
    for (int s = 0; s < kPackStages; ++s) issue(blockIdx.x + static_cast<int64_t>(s) * gridDim.x, s);
  }
  uint32_t phase = 0;  // bit s: parity of stage s's next completion
  int s = 0;
  for (int64_t t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
    const PackTile d = pack_tile(a, t);
    if (d.rows > 0) {
      bool ok = true;
      if (d.bulk) {
        ok = mbar_wait_bounded(&sm.bar[s], (phase >> s) & 1u);
        phase ^= 1u << s;
        if (tid == 0) pending &= ~(1u << s);
      }
      if (__syncthreads_or(!ok)) {
        report_error(a.err, TGS_DEV_WAIT_TIMEOUT, t);
        // Wait (bounded) for the copies still in flight before the shared
        // memory they target is released.
        if (tid == 0) {
          for (int q = 0; q < kPackStages; ++q)
            if (pending & (1u << q)) mbar_wait_bounded(&sm.bar[q], (phase >> q) & 1u);
        }
        __syncthreads();
        return;
      }
      float* __restrict__ out = a.out + d.dst * kRowWidth;
      const int n = d.rows * kRowWidth;
      if (d.bulk) {
        const float* __restrict__ tile = sm.stage[s];
#pragma unroll 4
        for (int e = tid; e < n; e += kPackThreads) {
          const int r = e / kRowWidth;
          const uint32_t cw = sm.col[e - r * kRowWidth];
          out[e] = tile[(cw & 0xffffu) + r * (cw >> 16)];
        }
      } else {
        for (int e = tid; e < n; e += kPackThreads) {
          const int r = e / kRowWidth;
          const int j = e - r * kRowWidth;
          const int c = layout_comp_of(kLayout, j);
          const int w = comp_width(c);
          out[e] = pick6(a.comp.p, c)[(d.src + r) * w + (j - layout_offset(kLayout, c))];
        }
      }
    }
    // Every thread's reads of this stage precede the bulk copy that refills it.
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) issue(t + static_cast<int64_t>(kPackStages) * gridDim.x, s);
    s = (s + 1 == kPackStages) ? 0 : s + 1;
  }
}

// ---------------------------------------------------------------------------
// Per-block xyz bounds (min/max are order independent, so exact).
// ---------------------------------------------------------------------------
constexpr int kBoundsThreads = 256;

__global__ void __launch_bounds__(kBoundsThreads) bounds_kernel(const float* __restrict__ xyz,
                                                                const int64_t* __restrict__ start,
                                                                const int64_t* __restrict__ count,
                                                                int n_plans,
                                                                float* __restrict__ bounds) {
  __shared__ float red[6][kBoundsThreads / 32];
  for (int k = blockIdx.x; k < n_plans; k += gridDim.x) {
    const int64_t s = start[k];
    const int64_t n = count[k];
    float lo[3] = {INFINITY, INFINITY, INFINITY};
    float hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    auto take = [&](int ax, float x) {
      lo[ax] = fminf(lo[ax], x);
      hi[ax] = fmaxf(hi[ax], x);
    };
    int64_t r0 = 0;
    if ((s & 3) == 0 && (reinterpret_cast<uintptr_t>(xyz) & 15u) == 0) {
      // 4 rows = 12 floats = 3 float4 whose lanes hold axes x y z x | y z x y
      // | z x y z: a thread takes whole 4-row groups, so every lane of each
      // of its vector loads has a fixed axis
      const float4* g4 = reinterpret_cast<const float4*>(xyz + s * 3);
      const int64_t groups = n / 4;
      for (int64_t q = threadIdx.x; q < groups; q += kBoundsThreads) {
        const float4 a = __ldg(g4 + 3 * q);
        const float4 b = __ldg(g4 + 3 * q + 1);
        const float4 c = __ldg(g4 + 3 * q + 2);
        take(0, a.x); take(1, a.y); take(2, a.z); take(0, a.w);
        take(1, b.x); take(2, b.y); take(0, b.z); take(1, b.w);
        take(2, c.x); take(0, c.y); take(1, c.z); take(2, c.w);
      }
      r0 = groups * 4;
    }
    for (int64_t r = r0 + threadIdx.x; r < n; r += kBoundsThreads) {
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) take(ax, xyz[(s + r) * 3 + ax]);
    }
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        lo[ax] = fminf(lo[ax], __shfl_xor_sync(0xffffffffu, lo[ax], o));
        hi[ax] = fmaxf(hi[ax], __shfl_xor_sync(0xffffffffu, hi[ax], o));
      }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        red[ax][warp] = lo[ax];
        red[3 + ax][warp] = hi[ax];
      }
    }
    __syncthreads();
    if (threadIdx.x < 6) {
      const int q = threadIdx.x;
      float v = red[q][0];
      for (int w = 1; w < kBoundsThreads / 32; ++w)
        v = q < 3 ? fminf(v, red[q][w]) : fmaxf(v, red[q][w]);
      bounds[static_cast<int64_t>(k) * 6 + q] = v;
    }
    __syncthreads();
  }
}

int grid_for(int64_t n, int threads, int per_sm = 8) {
  const int64_t need = ceil_div<int64_t>(std::max<int64_t>(n, 1), threads);
  return static_cast<int>(std::min<int64_t>(need, static_cast<int64_t>(sm_count()) * per_sm));
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_unpack_rows(const TgsUnpackArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_unpack_rows: args is NULL");
  TGS_CHECK_ARG(a->n_rows >= 0 && a->target_offset >= 0, "tgs_unpack_rows: bad sizes");
  TGS_CHECK_ARG(a->layout == TGS_LAYOUT_CACHE || a->layout == TGS_LAYOUT_UNIFIED,
                "tgs_unpack_rows: unsupported layout %d", a->layout);
  if (a->n_rows == 0) return TGS_OK;
  TGS_CHECK_ARG(a->packed != nullptr, "tgs_unpack_rows: packed is NULL");
  for (int c = 0; c < kNumComp; ++c)
    TGS_CHECK_ARG(a->comp[c] != nullptr, "tgs_unpack_rows: component %d is NULL", c);
  TGS_CHECK_ARG(a->global_ids == nullptr || (a->block_ids != nullptr && a->block_size >= 1),
                "tgs_unpack_rows: global id fill needs block_ids and block_size");
  TGS_CHECK_ARG(a->block_dst == nullptr || (a->block_size >= kTileRows &&
                                            a->block_size % kTileRows == 0),
                "tgs_unpack_rows: block_dst needs block_size a multiple of %d", kTileRows);
  UnpackParams p;
  p.packed = a->packed;
  p.n_rows = a->n_rows;
  p.layout = a->layout;
  for (int c = 0; c < kNumComp; ++c) p.comp.p[c] = a->comp[c];
  p.target_offset = a->target_offset;
  p.gids = a->global_ids;
  p.block_ids = a->block_ids;
  p.block_size = a->block_size;
  p.use_bulk = aligned16(a->packed) ? 1 : 0;
  p.err = a->err;
  p.block_dst = a->block_dst;
  p.block_shift = a->block_size >= 1 && (a->block_size & (a->block_size - 1)) == 0
                      ? __builtin_ctzll(a->block_size) : -1;
  const int64_t n_tiles = ceil_div<int64_t>(a->n_rows, kTileRows);
  const int grid = static_cast<int>(
      std::min<int64_t>(n_tiles, static_cast<int64_t>(sm_count()) * kUnpackCtasPerSm));
  static bool unpack_configured[64] = {};
  static std::mutex unpack_mu;
  int dev = 0;
  TGS_CUDA(cudaGetDevice(&dev));
  TGS_CHECK_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(unpack_mu);
    if (!unpack_configured[dev]) {
      TGS_CUDA(cudaFuncSetAttribute(unpack_kernel<TGS_LAYOUT_UNIFIED>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kUnpackSmemBytes));
      TGS_CUDA(cudaFuncSetAttribute(unpack_kernel<TGS_LAYOUT_CACHE>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kUnpackSmemBytes));
      unpack_configured[dev] = true;
    }
  }
  cudaStream_t s = as_stream(stream);
  if (a->layout == TGS_LAYOUT_UNIFIED)
    unpack_kernel<TGS_LAYOUT_UNIFIED><<<grid, kUnpackThreads, kUnpackSmemBytes, s>>>(p);
  else
    unpack_kernel<TGS_LAYOUT_CACHE><<<grid, kUnpackThreads, kUnpackSmemBytes, s>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_copy_blocks(const TgsCopyBlocksArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_copy_blocks: args is NULL");
  TGS_CHECK_ARG(a->n_blocks >= 0 && a->max_rows >= 0, "tgs_copy_blocks: bad sizes");
  if (a->n_blocks == 0 || a->max_rows == 0) return TGS_OK;
  TGS_CHECK_ARG(a->src_start && a->dst_start && a->row_count, "tgs_copy_blocks: NULL plan");
  CopyParams p;
  bool aligned = true;
  for (int c = 0; c < kNumComp; ++c) {
    TGS_CHECK_ARG(a->src_comp[c] && a->dst_comp[c], "tgs_copy_blocks: component %d is NULL", c);
    p.src.p[c] = a->src_comp[c];
    p.dst.p[c] = a->dst_comp[c];
    aligned = aligned && aligned16(a->src_comp[c]) && aligned16(a->dst_comp[c]);
  }
  p.src_gids = a->src_global_ids;
  p.dst_gids = a->dst_global_ids;
  if (p.src_gids && p.dst_gids) aligned = aligned && aligned16(p.src_gids) && aligned16(p.dst_gids);
  p.src_start = a->src_start;
  p.dst_start = a->dst_start;
  p.row_count = a->row_count;
  p.n_blocks = a->n_blocks;
  p.bases_aligned = aligned ? 1 : 0;
  p.err = a->err;
  const int64_t chunks = ceil_div<int64_t>(a->max_rows, kCopyChunkRows);
  TGS_CHECK_ARG(chunks < (1ll << 31), "tgs_copy_blocks: max_rows too large");
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(std::min(a->n_blocks, 65535)));
  const size_t smem = kCopyStages * kCopyPiece + kCopyStages * sizeof(uint64_t);
  static_assert(kCopyStages * kCopyPiece + kCopyStages * 8 <= 227 * 1024, "smem");
  TGS_CUDA(cudaFuncSetAttribute(copy_blocks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  copy_blocks_kernel<<<grid, kCopyThreads, smem, as_stream(stream)>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_fill_global_ids(int64_t* dst, int64_t offset, const int64_t* block_ids,
                                   int64_t n_rows, int64_t block_size, void* stream) {
  TGS_CHECK_ARG(n_rows >= 0 && offset >= 0 && block_size >= 1, "tgs_fill_global_ids: bad sizes");
  if (n_rows == 0) return TGS_OK;
  TGS_CHECK_ARG(dst && block_ids, "tgs_fill_global_ids: NULL pointer");
  const int shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctzll(block_size) : -1;
  fill_gids_kernel<<<grid_for(n_rows, 256), 256, 0, as_stream(stream)>>>(dst, offset, block_ids,
                                                                        n_rows, block_size, shift);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_build_block_starts(int64_t* block_starts, int64_t num_blocks, const int64_t* ids,
                                      const int64_t* starts, int64_t n, void* stream) {
  TGS_CHECK_ARG(num_blocks >= 0 && n >= 0, "tgs_build_block_starts: bad sizes");
  if (num_blocks == 0) return TGS_OK;
  TGS_CHECK_ARG(block_starts != nullptr, "tgs_build_block_starts: block_starts is NULL");
  cudaStream_t s = as_stream(stream);
  TGS_CUDA(cudaMemsetAsync(block_starts, 0xff, sizeof(int64_t) * num_blocks, s));  // all -1
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(ids && starts, "tgs_build_block_starts: NULL ids/starts");
  scatter_block_starts_kernel<<<static_cast<unsigned>(ceil_div<int64_t>(n, 256)), 256, 0, s>>>(
      block_starts, num_blocks, ids, starts, n);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_global_to_local(int64_t* out, const int64_t* global_ids, int64_t n,
                                   const int64_t* block_starts, int64_t num_blocks,
                                   int64_t block_size, void* stream) {
  TGS_CHECK_ARG(n >= 0 && num_blocks >= 1 && block_size >= 1, "tgs_global_to_local: bad sizes");
  if (n == 0) return TGS_OK;
  TGS_CHECK_ARG(out && global_ids && block_starts, "tgs_global_to_local: NULL pointer");
  g2l_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(out, global_ids, n, block_starts,
                                                              num_blocks, block_size);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int64_t tgs_compact_scratch_words(int64_t n) {
  return ceil_div<int64_t>(std::max<int64_t>(n, 0), kCompactTile) + 1;
}

extern "C" int tgs_global_to_local_compact(int64_t* out, int64_t* dev_count,
                                           const int64_t* global_ids, int64_t n,
                                           const int64_t* block_starts, int64_t num_blocks,
                                           int64_t block_size, int64_t* scratch, void* stream) {
  TGS_CHECK_ARG(n >= 0 && num_blocks >= 1 && block_size >= 1,
                "tgs_global_to_local_compact: bad sizes");
  TGS_CHECK_ARG(dev_count != nullptr, "tgs_global_to_local_compact: dev_count is NULL");
  cudaStream_t s = as_stream(stream);
  if (n == 0) {
    TGS_CUDA(cudaMemsetAsync(dev_count, 0, sizeof(int64_t), s));
    return TGS_OK;
  }
  TGS_CHECK_ARG(out && global_ids && block_starts && scratch,
                "tgs_global_to_local_compact: NULL pointer");
  const int64_t tiles = ceil_div<int64_t>(n, kCompactTile);
  TGS_CHECK_ARG(tiles < (1ll << 31), "tgs_global_to_local_compact: n too large");
  g2l_count_kernel<<<static_cast<unsigned>(tiles), kCompactThreads, 0, s>>>(
      global_ids, n, block_starts, num_blocks, block_size, scratch);
  TGS_LAUNCH_CHECK();
  scan_counts_kernel<<<1, 1024, 0, s>>>(scratch, tiles, dev_count);
  TGS_LAUNCH_CHECK();
  g2l_write_kernel<<<static_cast<unsigned>(tiles), kCompactThreads, 0, s>>>(
      out, global_ids, n, block_starts, num_blocks, block_size, scratch);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free global->local compaction.
//
// Some callers cannot hand us scratch memory: an engine whose device memory is
// laid out once at start-up has no allocator left to call, and allocating or
// freeing on the fly (cudaMalloc / cudaFree) would synchronize the whole
// device in the middle of a pipeline that overlaps copies and kernels. This
// variant of tgs_global_to_local_compact keeps its per-tile scratch in a fixed
// array compiled into the library instead: one int64 word per 2048-id tile,
// for at most kNoAllocMaxIds ids (16,385 words = 128 KiB). Every GPU that
// loads the library holds that array until the process exits.
//
// The array is shared by every call on a device and keeps the previous call's
// contents. Nothing in it has to start at zero: each call writes every tile
// count it later reads, then their prefix sums. Calls whose work overlaps on
// the GPU (two streams, or two host threads) race on the array and must be
// serialized by the caller.
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kNoAllocMaxIds = int64_t(1) << 25;  // 33,554,432 ids
constexpr int64_t kNoAllocScratchWords = kNoAllocMaxIds / kCompactTile + 1;
}  // namespace

static __device__ __align__(256) int64_t g_noalloc_compact_scratch[kNoAllocScratchWords];

namespace {
std::mutex g_noalloc_mutex;
int64_t* g_noalloc_scratch_ptr[64] = {nullptr};

// Device address of the fixed scratch array on the current device. Host code
// must not use the array's name as a device pointer: it is only a host-side
// stand-in, so the address is looked up once per device, with that device
// current, and kept for the life of the process. A cudaDeviceReset (or any
// new primary context on the device) invalidates it; the entry point's
// contract rules calls after one out.
int noalloc_scratch(int64_t** out) {
  int dev = -1;
  TGS_CUDA(cudaGetDevice(&dev));
  TGS_CHECK_ARG(dev >= 0 && dev < 64, "tgs_global_to_local_compact_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    TGS_CUDA(cudaGetSymbolAddress(&p, g_noalloc_compact_scratch));
    g_noalloc_scratch_ptr[dev] = static_cast<int64_t*>(p);
  }
  *out = g_noalloc_scratch_ptr[dev];
  return TGS_OK;
}
}  // namespace

extern "C" int tgs_global_to_local_compact_noalloc(int64_t* out, int64_t* dev_count,
                                                   const int64_t* global_ids, int64_t n,
                                                   const int64_t* block_starts,
                                                   int64_t num_blocks, int64_t block_size,
                                                   void* stream) {
  TGS_CHECK_ARG(n >= 0 && num_blocks >= 1 && block_size >= 1,
                "tgs_global_to_local_compact_noalloc: bad sizes");
  TGS_CHECK_ARG(n <= kNoAllocMaxIds,
                "tgs_global_to_local_compact_noalloc: n=%lld ids exceeds the fixed scratch "
                "limit of %lld ids; use tgs_global_to_local_compact with caller scratch",
                (long long)n, (long long)kNoAllocMaxIds);
  TGS_CHECK_ARG(dev_count != nullptr, "tgs_global_to_local_compact_noalloc: dev_count is NULL");
  TGS_CHECK_ARG(n == 0 || (out && global_ids && block_starts),
                "tgs_global_to_local_compact_noalloc: NULL pointer");
  int64_t* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != TGS_OK) return rc;
  cudaStream_t s = as_stream(stream);
  if (n == 0) {
    TGS_CUDA(cudaMemsetAsync(dev_count, 0, sizeof(int64_t), s));
    return TGS_OK;
  }
  const int64_t tiles = ceil_div<int64_t>(n, kCompactTile);
  g2l_count_kernel<<<static_cast<unsigned>(tiles), kCompactThreads, 0, s>>>(
      global_ids, n, block_starts, num_blocks, block_size, scratch);
  TGS_LAUNCH_CHECK();
  scan_counts_kernel<<<1, 1024, 0, s>>>(scratch, tiles, dev_count);
  TGS_LAUNCH_CHECK();
  g2l_write_kernel<<<static_cast<unsigned>(tiles), kCompactThreads, 0, s>>>(
      out, global_ids, n, block_starts, num_blocks, block_size, scratch);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_pack_rows(const TgsPackArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_pack_rows: args is NULL");
  TGS_CHECK_ARG(a->n_plans >= 0 && a->max_rows >= 0, "tgs_pack_rows: bad sizes");
  TGS_CHECK_ARG(a->layout == TGS_LAYOUT_CACHE || a->layout == TGS_LAYOUT_UNIFIED,
                "tgs_pack_rows: unsupported layout %d", a->layout);
  if (a->n_plans == 0 || a->max_rows == 0) return TGS_OK;
  TGS_CHECK_ARG(a->src_start && a->row_count && a->out_start && a->out, "tgs_pack_rows: NULL plan");
  PackParams p;
  p.comp_aligned = 1;
  for (int c = 0; c < kNumComp; ++c) {
    TGS_CHECK_ARG(a->comp[c] != nullptr, "tgs_pack_rows: component %d is NULL", c);
    p.comp.p[c] = a->comp[c];
    if (!aligned16(a->comp[c])) p.comp_aligned = 0;
  }
  p.src_start = a->src_start;
  p.row_count = a->row_count;
  p.out_start = a->out_start;
  p.out = a->out;
  p.err = a->err;
  const int64_t tiles = ceil_div<int64_t>(a->max_rows, kTileRows);
  TGS_CHECK_ARG(tiles < (1ll << 31), "tgs_pack_rows: max_rows too large");
  p.tiles_per_plan = static_cast<int>(tiles);
  p.n_tiles = tiles * a->n_plans;
  const int grid = static_cast<int>(
      std::min<int64_t>(p.n_tiles, static_cast<int64_t>(sm_count()) * kPackCtasPerSm));
  static bool configured[64] = {};
  static std::mutex mu;
  int dev = 0;
  TGS_CUDA(cudaGetDevice(&dev));
  TGS_CHECK_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      TGS_CUDA(cudaFuncSetAttribute(pack_kernel<TGS_LAYOUT_CACHE>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kPackSmemBytes));
      TGS_CUDA(cudaFuncSetAttribute(pack_kernel<TGS_LAYOUT_UNIFIED>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kPackSmemBytes));
      configured[dev] = true;
    }
  }
  cudaStream_t s = as_stream(stream);
  if (a->layout == TGS_LAYOUT_CACHE)
    pack_kernel<TGS_LAYOUT_CACHE><<<grid, kPackThreads, kPackSmemBytes, s>>>(p);
  else
    pack_kernel<TGS_LAYOUT_UNIFIED><<<grid, kPackThreads, kPackSmemBytes, s>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

extern "C" int tgs_block_bounds(const float* xyz, const int64_t* start, const int64_t* count,
                                int32_t n_plans, float* bounds, void* stream) {
  TGS_CHECK_ARG(n_plans >= 0, "tgs_block_bounds: n_plans < 0");
  if (n_plans == 0) return TGS_OK;
  TGS_CHECK_ARG(xyz && start && count && bounds, "tgs_block_bounds: NULL pointer");
  const int grid = std::min(n_plans, sm_count() * 8);
  bounds_kernel<<<grid, kBoundsThreads, 0, as_stream(stream)>>>(xyz, start, count, n_plans, bounds);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}
