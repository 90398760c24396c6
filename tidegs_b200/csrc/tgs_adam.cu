// Optimizer kernels: GPU-resident Adam over resident block slots, and the
// dense masked SelectiveAdam / SelectiveSophia steps.
//
// Reference behaviour followed:
//   strategies/tide_engine/gpu_resident_optimizer.py:16-70   (per-element Adam math)
//   strategies/tide_engine/gpu_resident_optimizer.py:266-337 (row->slot, step tables)
//   submodules/clm_kernels/adam.cu:12-41                     (SelectiveAdam math)
#include <math.h>

#include <mutex>

#include "tgs_common.cuh"

namespace tgs {
namespace {

// First index p in [0, n) with a[p] > x (n if none).
__device__ __forceinline__ int upper_bound_i64(const int64_t* __restrict__ a, int n, int64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(a + mid) > x) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// Position of the working-set row `id` (pos_start[p] <= id < pos_end[p]), or
// the upper bound when no position holds it. Positions are the block slices
// in slice order; when they are whole blocks from row 0 (the persistent-slot
// layout) position id / block_size holds the row, so the search only runs
// when that guess misses (a short tail block earlier in the working set).
__device__ __forceinline__ int find_position(const int64_t* __restrict__ pos_start,
                                             const int64_t* __restrict__ pos_end, int n_pos,
                                             int64_t block_size, int64_t id) {
  const int64_t q = (block_size & (block_size - 1)) == 0 ? (id >> (__ffsll(block_size) - 1))
                                                          : id / block_size;
  const int g = static_cast<int>(q < n_pos - 1 ? q : n_pos - 1);
  if (__ldg(pos_start + g) <= id && id < __ldg(pos_end + g)) return g;
  return upper_bound_i64(pos_end, n_pos, id);
}

// ---------------------------------------------------------------------------
// Kernel A: validate the ids (in range, strictly ascending, inside a resident
// position) and count touched rows per position.
// ---------------------------------------------------------------------------
constexpr int kCountThreads = 256;
constexpr int kCountRows = 4;  // consecutive rows per thread: a warp covers four 32-row chunks

__global__ void __launch_bounds__(kCountThreads) resident_count_kernel(
    const int64_t* __restrict__ ids, int64_t n, int64_t param_rows,
    const int64_t* __restrict__ pos_start, const int64_t* __restrict__ pos_end,
    const int32_t* __restrict__ pos_slot, int n_pos, int64_t block_size,
    int32_t* __restrict__ pos_count, int64_t* __restrict__ chunk_table,
    int32_t* __restrict__ err) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int64_t i0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * kCountRows;
  // The thread's rows i0 .. i0+3 (-1 past the end), two 16-byte loads when
  // the array allows.
  int64_t id[kCountRows];
  if (i0 + kCountRows <= n && (reinterpret_cast<uintptr_t>(ids) & 15) == 0) {
    const longlong2 a = __ldg(reinterpret_cast<const longlong2*>(ids + i0));
    const longlong2 b = __ldg(reinterpret_cast<const longlong2*>(ids + i0) + 1);
    id[0] = a.x; id[1] = a.y; id[2] = b.x; id[3] = b.y;
  } else {
#pragma unroll
    for (int k = 0; k < kCountRows; ++k) id[k] = i0 + k < n ? __ldg(ids + i0 + k) : -1;
  }
  // The rows on either side of the thread's four: the neighbouring lanes'
  // ids, or loads at the warp's ends.
  int64_t before = __shfl_up_sync(full, id[kCountRows - 1], 1);
  int64_t after = __shfl_down_sync(full, id[0], 1);
  if (lane == 0) before = i0 > 0 && i0 <= n ? __ldg(ids + i0 - 1) : -1;
  if (lane == 31) after = i0 + kCountRows < n ? __ldg(ids + i0 + kCountRows) : -1;

  // One position lookup per row that leaves the previous row's position:
  // position (and state row) of each row, or an error code.
  int p[kCountRows];
  int64_t sr[kCountRows];
  int cp = -1;
  int64_t cps = 0, cpe = 0, cslot = 0;
#pragma unroll
  for (int k = 0; k < kCountRows; ++k) {
    p[k] = -1;
    sr[k] = -1;
    const int64_t i = i0 + k;
    if (i >= n) continue;
    const int64_t x = id[k];
    const int64_t prev = k == 0 ? before : id[k - 1];
    int code = TGS_DEV_OK;
    if (x < 0 || x >= param_rows) {
      code = TGS_DEV_ID_OUT_OF_RANGE;
    } else if (i > 0 && prev >= x) {
      code = TGS_DEV_ID_NOT_SORTED;
    } else {
      if (!(cp >= 0 && x >= cps && x < cpe)) {
        cp = find_position(pos_start, pos_end, n_pos, block_size, x);
        if (cp < n_pos) {
          cps = __ldg(pos_start + cp);
          cpe = __ldg(pos_end + cp);
          cslot = __ldg(pos_slot + cp);
        }
        if (cp >= n_pos || cps > x) cp = -1;
      }
      if (cp < 0) {
        code = TGS_DEV_ID_NOT_RESIDENT;
      } else {
        p[k] = cp;
        sr[k] = cslot * block_size + (x - cps);
      }
    }
    if (code != TGS_DEV_OK) report_error(err, code, i);
  }

  // Lanes 8j .. 8j+7 cover one 32-row chunk: the chunk table records whether
  // the chunk can be streamed by bulk copies -- all 32 rows valid, ids and
  // state rows both consecutive (every row checked), first id a multiple of 4.
  if (chunk_table != nullptr) {
    bool ok = true;
#pragma unroll
    for (int k = 0; k < kCountRows; ++k)
      ok = ok && sr[k] >= 0 && id[k] == id[0] + k && sr[k] == sr[0] + k;
    const int64_t last_id = __shfl_up_sync(full, id[kCountRows - 1], 1);
    const int64_t last_sr = __shfl_up_sync(full, sr[kCountRows - 1], 1);
    if ((lane & 7) != 0) ok = ok && id[0] == last_id + 1 && sr[0] == last_sr + 1;
    const unsigned votes = __ballot_sync(full, ok);
    const bool stream = ((votes >> (lane & ~7)) & 0xffu) == 0xffu && (id[0] & 3) == 0;
    if ((lane & 7) == 0 && i0 < n) {
      const int64_t chunk = i0 >> 5;
      chunk_table[2 * chunk] = stream ? id[0] : -1;
      chunk_table[2 * chunk + 1] = stream ? sr[0] : -1;
    }
  }

  // Rows of a position are consecutive (ids ascending): its first row
  // subtracts its index and its last row adds its index + 1, so the count
  // costs two uncontended additions per position (an addition per row or per
  // warp serializes on one counter while a block's rows are counted). int32
  // wrap-around keeps the difference exact. Counts are only used when no row
  // reported an error.
#pragma unroll
  for (int k = 0; k < kCountRows; ++k) {
    if (p[k] < 0) continue;
    const int64_t i = i0 + k;
    const int64_t prev = k == 0 ? before : id[k - 1];
    const int64_t next = k == kCountRows - 1 ? after : id[k + 1];
    if (i == 0 || prev < __ldg(pos_start + p[k]))
      atomicSub(pos_count + p[k], static_cast<int32_t>(static_cast<uint32_t>(i)));
    if (i == n - 1 || next >= __ldg(pos_end + p[k]))
      atomicAdd(pos_count + p[k], static_cast<int32_t>(static_cast<uint32_t>(i + 1)));
  }
}

// ---------------------------------------------------------------------------
// Kernel B: per touched position, advance its slot's step and publish the
// bias-correction pair of that step (table precomputed on the host in double
// precision exactly as gpu_resident_optimizer.py:325-328 does). The slot keeps
// (1 / (1-b1^t), sqrt(1-b2^t)): the reference's `lr / bias` is evaluated as
// reciprocal(bias) * lr, so the reciprocal is shared by all rows of the slot.
// ---------------------------------------------------------------------------
__global__ void resident_slot_kernel(const int32_t* __restrict__ pos_count,
                                     const int32_t* __restrict__ pos_slot, int n_pos,
                                     int32_t* __restrict__ slot_step, float2* __restrict__ slot_bias,
                                     const float2* __restrict__ table, int table_len,
                                     const int32_t* __restrict__ err) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n_pos || load_error(err) != 0) return;
  if (pos_count[p] > 0) {
    const int s = pos_slot[p];
    const int t = slot_step[s] + 1;
    slot_step[s] = t;
    const float2 e = table[t < table_len ? t : table_len - 1];
    slot_bias[s] = make_float2(fdiv(1.0f, e.x), e.y);
  }
}

// ---------------------------------------------------------------------------
// Kernel C: fused 59-column resident Adam. One warp updates one row at a time:
// lane l owns UNIFIED columns 2l and 2l+1, so the row's 512-byte (m,v) state
// row is one fully coalesced float4 access per lane. A warp takes 32 rows,
// resolves their slot/state row once (one row per lane, binary search over
// the resident layout) into a per-warp shared-memory table, then streams the
// rows U at a time, all loads of the U rows issued before any store. The
// update itself is branch-free: every lane computes both columns and only
// the stores are predicated.
// ---------------------------------------------------------------------------
struct ResidentApplyParams {
  float* param[kNumComp];
  const float* grad[kNumComp];
  float lr[kNumComp];
  float beta1, beta2, omb1, omb2, eps, batch_size, inv_batch_size;
  const int64_t* pos_start;
  const int64_t* pos_end;
  const int32_t* pos_slot;
  int n_pos;
  int64_t block_size;
  const int64_t* ids;
  int64_t n;
  float4* state;
  const uint32_t* slot_stamp;
  const float2* slot_bias;  // (1/(1-b1^t), sqrt(1-b2^t)) per slot
  const int32_t* err;
  // [chunks][2] from the count kernel, or null: chunks marked kChunkDone
  // were updated by the streaming kernel and are skipped
  int64_t* chunk_table;
};

// Chunk-table entry (second word) of a chunk the streaming kernel updated.
constexpr int64_t kChunkDone = -2;

// Occupancy target (CTAs per SM) and rows in flight per warp of the update
// kernel; overridable at build time for tuning sweeps.
#ifndef TGS_APPLY_MIN_BLOCKS
#define TGS_APPLY_MIN_BLOCKS 2
#endif
#ifndef TGS_APPLY_UNROLL
#define TGS_APPLY_UNROLL 4
#endif
constexpr int kApplyThreads = 256;
constexpr int kApplyWarps = kApplyThreads / 32;
constexpr int kApplyUnroll = TGS_APPLY_UNROLL;
constexpr int kApplyMinBlocks = TGS_APPLY_MIN_BLOCKS;
// The pulling variant (kernel C') waits on remote reads: its own knobs.
#ifndef TGS_SUM_MIN_BLOCKS
#define TGS_SUM_MIN_BLOCKS 2
#endif
#ifndef TGS_SUM_UNROLL
#define TGS_SUM_UNROLL 4
#endif
#ifndef TGS_SUM_FAST_UNROLL
#define TGS_SUM_FAST_UNROLL 2
#endif
constexpr int kSumUnroll = TGS_SUM_UNROLL;
constexpr int kSumFastUnroll = TGS_SUM_FAST_UNROLL;  // rows per batch, one-segment chunks
constexpr int kStagedContribs = 2;  // contributions loaded with the batch (more: per row)
constexpr int kSumMinBlocks = TGS_SUM_MIN_BLOCKS;

struct AdamScalars {
  float beta1, beta2, omb1, omb2, eps, batch_size, inv_batch_size;
};

// Reference torch-fallback order (gpu_resident_optimizer.py:355-364), one
// rounding per operation; step_scale = (1/bias1) * lr. With a power-of-two
// batch size grad/bs and grad*(1/bs) are the same exactly rounded value.
template <bool kPow2Batch>
__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float graw,
                                          const AdamScalars& h, float step_scale,
                                          float denom_scale) {
  const float g = kPow2Batch ? fmul(graw, h.inv_batch_size) : fdiv(graw, h.batch_size);
  m = fadd(fmul(h.beta1, m), fmul(h.omb1, g));
  v = fadd(fmul(h.beta2, v), fmul(fmul(h.omb2, g), g));
  const float denom = fadd(fdiv(fsqrt(v), denom_scale), h.eps);
  p = fsub(p, fmul(fdiv(m, denom), step_scale));
}

// Per-row metadata shared by the lanes of a warp (two 16-byte halves, each
// read with one broadcast shared-memory load).
struct __align__(16) RowAddr {
  int64_t id;  // local row
  int64_t sr;  // state row
};
struct __align__(16) RowScale {
  float rb1;      // 1 / (1 - b1^t) of the row's slot
  float ds;       // sqrt(1 - b2^t)
  uint32_t stamp; // admission stamp of the slot
  uint32_t pad;
};

// Resolves the chunk's rows (lane l: row row0 + l) into the warp's tables and
// returns, uniformly across the warp, whether the chunk is contiguous: 32 rows
// whose ids AND state rows both advance by one from lane to lane. Every lane
// checks its own row; ends alone do not decide it, because with blocks
// shorter than 32 rows consecutive ids can sit in slots out of order (slots
// 0,5,2,.. of 4-row blocks) while the first and last rows still line up.
__device__ __forceinline__ bool resolve_chunk_rows(const ResidentApplyParams& a, int64_t row0,
                                                   int nr, int lane, RowAddr* addr,
                                                   RowScale* scale) {
  int64_t id = 0, sr = 0;
  if (lane < nr) {
    id = a.ids[row0 + lane];
    const int p = find_position(a.pos_start, a.pos_end, a.n_pos, a.block_size, id);
    const int s = __ldg(a.pos_slot + p);
    const float2 bb = a.slot_bias[s];
    sr = static_cast<int64_t>(s) * a.block_size + (id - __ldg(a.pos_start + p));
    addr[lane] = {id, sr};
    scale[lane] = {bb.x, bb.y, __ldg(a.slot_stamp + s), 0u};
  }
  const unsigned full = 0xffffffffu;
  const int64_t id0 = __shfl_sync(full, id, 0);
  const int64_t sr0 = __shfl_sync(full, sr, 0);
  __syncwarp();
  return __all_sync(full, nr == 32 && id == id0 + lane && sr == sr0 + lane) != 0;
}

// Contiguous chunks (32 consecutive ids whose state rows are consecutive,
// e.g. all rows of visible blocks) take a staged path: lane 0 copies the state
// rows of the warp's next kStateBatch-row batches with one non-multicast bulk
// copy each into a two-stage ring in shared memory, so that only parameters
// and gradients travel through registers and twice as many rows are in
// flight per warp. Waits are bounded; on timeout the warp records
// TGS_DEV_WAIT_TIMEOUT, waits (bounded) for its copies in flight and exits.
#ifndef TGS_STATE_BATCH
#define TGS_STATE_BATCH 4
#endif
#ifndef TGS_STATE_STAGES
#define TGS_STATE_STAGES 3
#endif
#ifndef TGS_STATE_PG_AHEAD
#define TGS_STATE_PG_AHEAD 1
#endif
constexpr int kStateBatch = TGS_STATE_BATCH;
constexpr int kStateStages = TGS_STATE_STAGES;
constexpr int kStateStageBytes = kStateBatch * TGS_STATE_ROW_FLOATS * 4;  // 4 KB
struct __align__(16) ApplyWarpSmem {
  float4 stage[kStateStages][kStateBatch][32];
  uint64_t bar[kStateStages];
};
constexpr int kApplySmemBytes = kApplyWarps * static_cast<int>(sizeof(ApplyWarpSmem));

template <bool kPow2Batch>
__global__ void __launch_bounds__(kApplyThreads, kApplyMinBlocks) resident_adam_kernel(const ResidentApplyParams a) {
  __shared__ RowAddr s_addr[kApplyWarps][32];
  __shared__ RowScale s_scale[kApplyWarps][32];
  extern __shared__ __align__(16) unsigned char apply_smem[];
  if (load_error(a.err) != 0) return;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const unsigned full = 0xffffffffu;
  ApplyWarpSmem& ws = reinterpret_cast<ApplyWarpSmem*>(apply_smem)[warp];
  if (lane == 0) {
    for (int st = 0; st < kStateStages; ++st) mbar_init(&ws.bar[st], 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t phase = 0;  // bit st: parity of stage st's next completion
  const AdamScalars hp = {a.beta1, a.beta2, a.omb1, a.omb2, a.eps, a.batch_size, a.inv_batch_size};

  // Per-lane column bindings (fixed for the whole kernel). Lanes past column
  // 58 bind to column 0 of xyz: they load and compute but never store.
  const float* gbase[2];
  float* pbase[2];
  int width[2];
  float lr[2];
  bool act[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = 2 * lane + e;
    act[e] = j < kRowWidth;
    const int c = act[e] ? unified_comp_of(j) : 0;
    const int k = act[e] ? j - unified_offset(c) : 0;
    gbase[e] = pick6(a.grad, c) + k;
    pbase[e] = pick6(a.param, c) + k;
    width[e] = comp_width(c);
    lr[e] = pick6(a.lr, c);
  }
  // State float4 lanes: pair 2l in .xy (valid for l <= 29), pair 2l+1 in .zw
  // (valid for l <= 28); lane 31's .x carries the row stamp.
  const bool keep_lo = lane < 30;
  const bool keep_hi = lane < 29;
  const bool stamp_lane = lane == 31;

  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * kApplyWarps + warp;
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kApplyWarps;

  for (int64_t base = warp_id; base * 32 < a.n; base += 32 * warp_stride) {
   // lane l looks at chunk base + l * warp_stride; the warp then updates the
   // chunks the streaming kernel left
   const int64_t mine = base + lane * warp_stride;
   const bool todo = mine * 32 < a.n &&
                     !(a.chunk_table != nullptr && a.chunk_table[2 * mine + 1] == kChunkDone);
   uint32_t pending_chunks = __ballot_sync(full, todo);
   while (pending_chunks != 0) {
    const int pick = __ffs(pending_chunks) - 1;
    pending_chunks &= pending_chunks - 1;
    const int64_t chunk = base + pick * warp_stride;
    const int64_t row0 = chunk * 32;
    const int nr = static_cast<int>(min64(32, a.n - row0));

    const bool contiguous = resolve_chunk_rows(a, row0, nr, lane, s_addr[warp], s_scale[warp]);
    __syncwarp();

    const float* gptr0 = gbase[0] + row0 * width[0];
    const float* gptr1 = gbase[1] + row0 * width[1];
    const RowAddr first = s_addr[warp][0];
    if (contiguous) {
      // staged path: state rows first.sr .. first.sr + 31 are contiguous
      const float4* src = a.state + first.sr * 32;
      if (lane == 0) {
        for (int st = 0; st < kStateStages; ++st) {
          mbar_arrive_expect_tx(&ws.bar[st], kStateStageBytes);
          bulk_g2s(&ws.stage[st][0][0], src + st * kStateBatch * 32, kStateStageBytes,
                   &ws.bar[st]);
        }
      }
      uint32_t pending = (1u << kStateStages) - 1u;
      bool timed_out = false;
#if TGS_STATE_PG_AHEAD
      float ng0[kStateBatch], ng1[kStateBatch], np0[kStateBatch], np1[kStateBatch];
#pragma unroll
      for (int u = 0; u < kStateBatch; ++u) {
        ng0[u] = gptr0[u * width[0]];
        ng1[u] = gptr1[u * width[1]];
        np0[u] = pbase[0][(first.id + u) * width[0]];
        np1[u] = pbase[1][(first.id + u) * width[1]];
      }
#endif
#pragma unroll 1
      for (int q = 0; q < 32 / kStateBatch; ++q) {
        const int st = q % kStateStages;
        float g0[kStateBatch], g1[kStateBatch], p0[kStateBatch], p1[kStateBatch];
#if TGS_STATE_PG_AHEAD
#pragma unroll
        for (int u = 0; u < kStateBatch; ++u) {
          g0[u] = ng0[u];
          g1[u] = ng1[u];
          p0[u] = np0[u];
          p1[u] = np1[u];
        }
        if (q + 1 < 32 / kStateBatch) {
#pragma unroll
          for (int u = 0; u < kStateBatch; ++u) {
            const int rr = (q + 1) * kStateBatch + u;
            const int64_t id = first.id + rr;
            ng0[u] = gptr0[rr * width[0]];
            ng1[u] = gptr1[rr * width[1]];
            np0[u] = pbase[0][id * width[0]];
            np1[u] = pbase[1][id * width[1]];
          }
        }
#else
#pragma unroll
        for (int u = 0; u < kStateBatch; ++u) {
          const int rr = q * kStateBatch + u;
          const int64_t id = first.id + rr;
          g0[u] = gptr0[rr * width[0]];
          g1[u] = gptr1[rr * width[1]];
          p0[u] = pbase[0][id * width[0]];
          p1[u] = pbase[1][id * width[1]];
        }
#endif
        if (!mbar_wait_bounded(&ws.bar[st], (phase >> st) & 1u)) {
          report_error(const_cast<int32_t*>(a.err), TGS_DEV_WAIT_TIMEOUT, row0);
          timed_out = true;
          break;
        }
        phase ^= 1u << st;
        pending &= ~(1u << st);
#pragma unroll
        for (int u = 0; u < kStateBatch; ++u) {
          const int rr = q * kStateBatch + u;
          const RowScale rs = s_scale[warp][rr];
          const float4 sv = ws.stage[st][u][lane];
          const bool fresh = __shfl_sync(full, __float_as_uint(sv.x) == rs.stamp ? 1 : 0, 31) != 0;
          float m0 = fresh ? sv.x : 0.f, v0 = fresh ? sv.y : 0.f;
          float m1 = fresh ? sv.z : 0.f, v1 = fresh ? sv.w : 0.f;
          adam_elem<kPow2Batch>(p0[u], m0, v0, g0[u], hp, fmul(rs.rb1, lr[0]), rs.ds);
          adam_elem<kPow2Batch>(p1[u], m1, v1, g1[u], hp, fmul(rs.rb1, lr[1]), rs.ds);
          float4 out;
          out.x = stamp_lane ? __uint_as_float(rs.stamp) : (keep_lo ? m0 : 0.f);
          out.y = keep_lo ? v0 : 0.f;
          out.z = keep_hi ? m1 : 0.f;
          out.w = keep_hi ? v1 : 0.f;
          a.state[(first.sr + rr) * 32 + lane] = out;
          const int64_t id = first.id + rr;
          if (act[0]) pbase[0][id * width[0]] = p0[u];
          if (act[1]) pbase[1][id * width[1]] = p1[u];
        }
        __syncwarp();  // every lane is done with the stage
        const int qn = q + kStateStages;
        if (qn < 32 / kStateBatch) {
          if (lane == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&ws.bar[st], kStateStageBytes);
            bulk_g2s(&ws.stage[st][0][0], src + qn * kStateBatch * 32, kStateStageBytes,
                     &ws.bar[st]);
          }
          pending |= 1u << st;
        }
      }
      if (timed_out) {
        for (int st = 0; st < kStateStages; ++st)
          if ((pending >> st) & 1u) (void)mbar_wait_bounded(&ws.bar[st], (phase >> st) & 1u);
        return;
      }
      __syncwarp();  // the tables are rewritten by the next chunk
      continue;
    }
    for (int r = 0; r < nr; r += kApplyUnroll) {
      float4 st[kApplyUnroll];
      float g0[kApplyUnroll], g1[kApplyUnroll], p0[kApplyUnroll], p1[kApplyUnroll];
#pragma unroll
      for (int u = 0; u < kApplyUnroll; ++u) {
        const int rr = r + u;  // warp-uniform
        st[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        g0[u] = g1[u] = p0[u] = p1[u] = 0.f;
        if (rr < nr) {
          const RowAddr ra = s_addr[warp][rr];
          st[u] = a.state[ra.sr * 32 + lane];
          g0[u] = gptr0[rr * width[0]];
          g1[u] = gptr1[rr * width[1]];
          p0[u] = pbase[0][ra.id * width[0]];
          p1[u] = pbase[1][ra.id * width[1]];
        }
      }
#pragma unroll
      for (int u = 0; u < kApplyUnroll; ++u) {
        const int rr = r + u;
        if (rr >= nr) break;  // warp-uniform
        const RowAddr ra = s_addr[warp][rr];
        const RowScale rs = s_scale[warp][rr];
        // A row whose stamp is not its slot's current stamp has not been
        // touched since the block was (re)admitted: its moments are zero.
        const bool fresh =
            __shfl_sync(full, __float_as_uint(st[u].x) == rs.stamp ? 1 : 0, 31) != 0;
        float m0 = fresh ? st[u].x : 0.f, v0 = fresh ? st[u].y : 0.f;
        float m1 = fresh ? st[u].z : 0.f, v1 = fresh ? st[u].w : 0.f;
        adam_elem<kPow2Batch>(p0[u], m0, v0, g0[u], hp, fmul(rs.rb1, lr[0]), rs.ds);
        adam_elem<kPow2Batch>(p1[u], m1, v1, g1[u], hp, fmul(rs.rb1, lr[1]), rs.ds);
        float4 out;
        out.x = stamp_lane ? __uint_as_float(rs.stamp) : (keep_lo ? m0 : 0.f);
        out.y = keep_lo ? v0 : 0.f;
        out.z = keep_hi ? m1 : 0.f;
        out.w = keep_hi ? v1 : 0.f;
        a.state[ra.sr * 32 + lane] = out;
        if (act[0]) pbase[0][ra.id * width[0]] = p0[u];
        if (act[1]) pbase[1][ra.id * width[1]] = p1[u];
      }
    }
    __syncwarp();  // the table is rewritten by the next chunk
   }
  }
}

// ---------------------------------------------------------------------------
// Kernel C': the same update with the owner-side gradient reduction fused in
// ("pull"). A row's gradient is the sum, in listed (rank) order, of its
// contributions read straight from the senders' gradient components (peer
// memory through IPC mappings for other ranks): plain loads, issued together
// with the row's state and parameter loads, so the NVLink reads overlap the
// HBM traffic of the update. The first two contributions of the U rows in
// flight load in one round; further ones (rare) follow one by one.
// ---------------------------------------------------------------------------
struct ResidentSumParams {
  ResidentApplyParams a;            // a.grad unused
  const float* const* grad_src;     // [n_ranks * kNumComp]
  const int64_t* grad_rows;         // [n_ranks]
  int n_ranks;
  const int64_t* seg_begin;         // [n_seg + 1]
  int n_seg;
  const int64_t* contrib_offsets;   // [n_seg + 1]
  const int32_t* contrib_rank;
  const int64_t* contrib_row;
  int64_t rotate_chunks;            // first 32-row chunk walked
  int32_t* err;
};

struct __align__(16) RowSeg {
  int64_t off;  // row offset inside its segment
  int32_t cb;   // first contribution
  int32_t cn;   // contributions
};

struct LaneCols {
  int comp[2];
  int col[2];
  int width[2];
};

__device__ __forceinline__ void load_contrib(const ResidentSumParams& q, const LaneCols& lc, int j,
                                             int64_t off, float& x0, float& x1) {
  const int r = __ldg(q.contrib_rank + j);
  const int64_t srow = __ldg(q.contrib_row + j) + off;
  if (r < 0 || r >= q.n_ranks || srow < 0 || srow >= __ldg(q.grad_rows + r)) {
    report_error(q.err, TGS_DEV_BAD_SLICE, j, r);
    x0 = x1 = 0.f;
    return;
  }
  const float* b0 = q.grad_src[r * kNumComp + lc.comp[0]];
  const float* b1 = q.grad_src[r * kNumComp + lc.comp[1]];
  x0 = b0[srow * lc.width[0] + lc.col[0]];
  x1 = b1[srow * lc.width[1] + lc.col[1]];
}

template <bool kPow2Batch>
__global__ void __launch_bounds__(kApplyThreads, kSumMinBlocks)
    resident_adam_sum_kernel(const ResidentSumParams q) {
  __shared__ RowAddr s_addr[kApplyWarps][32];
  __shared__ RowScale s_scale[kApplyWarps][32];
  __shared__ RowSeg s_seg[kApplyWarps][32];
  extern __shared__ __align__(16) unsigned char apply_smem[];
  const ResidentApplyParams& a = q.a;
  if (load_error(a.err) != 0) return;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const unsigned full = 0xffffffffu;
  ApplyWarpSmem& ws = reinterpret_cast<ApplyWarpSmem*>(apply_smem)[warp];
  if (lane == 0) {
    for (int st = 0; st < kStateStages; ++st) mbar_init(&ws.bar[st], 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t phase = 0;  // bit st: parity of stage st's next completion
  const AdamScalars hp = {a.beta1, a.beta2, a.omb1, a.omb2, a.eps, a.batch_size, a.inv_batch_size};

  LaneCols lc;
  float* pbase[2];
  int width[2];
  float lr[2];
  bool act[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = 2 * lane + e;
    act[e] = j < kRowWidth;
    const int c = act[e] ? unified_comp_of(j) : 0;
    const int k = act[e] ? j - unified_offset(c) : 0;
    lc.comp[e] = c;
    lc.col[e] = k;
    lc.width[e] = comp_width(c);
    pbase[e] = pick6(a.param, c) + k;
    width[e] = comp_width(c);
    lr[e] = pick6(a.lr, c);
  }
  const bool keep_lo = lane < 30;
  const bool keep_hi = lane < 29;
  const bool stamp_lane = lane == 31;

  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * kApplyWarps + warp;
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kApplyWarps;

  const int64_t n_chunks = (a.n + 31) / 32;
  for (int64_t base = warp_id; base < n_chunks; base += 32 * warp_stride) {
   const int64_t cl = base + lane * warp_stride;
   int64_t mine = cl + q.rotate_chunks;
   if (mine >= n_chunks) mine -= n_chunks;
   const bool todo = cl < n_chunks &&
                     !(a.chunk_table != nullptr && a.chunk_table[2 * mine + 1] == kChunkDone);
   uint32_t pending_chunks = __ballot_sync(full, todo);
   while (pending_chunks != 0) {
    const int pick = __ffs(pending_chunks) - 1;
    pending_chunks &= pending_chunks - 1;
    int64_t chunk = base + pick * warp_stride + q.rotate_chunks;
    if (chunk >= n_chunks) chunk -= n_chunks;
    const int64_t row0 = chunk * 32;
    const int nr = static_cast<int>(min64(32, a.n - row0));

    const bool contiguous = resolve_chunk_rows(a, row0, nr, lane, s_addr[warp], s_scale[warp]);
    // Segment of the chunk's first row (first s with seg_begin[s + 1] > row0),
    // resolved by lane 0; the chunk takes the fast path when its last row is
    // in the same segment.
    int sg_cb = 0, sg_cn = 0, uniform = 0;
    int64_t sg_off = 0;
    if (lane == 0) {
      const int sg = upper_bound_i64(q.seg_begin + 1, q.n_seg, row0);
      if (sg < q.n_seg && __ldg(q.seg_begin + sg) <= row0) {
        sg_cb = static_cast<int>(__ldg(q.contrib_offsets + sg));
        sg_cn = static_cast<int>(__ldg(q.contrib_offsets + sg + 1)) - sg_cb;
        sg_off = row0 - __ldg(q.seg_begin + sg);
        uniform = row0 + nr <= __ldg(q.seg_begin + sg + 1) ? 1 : 0;
      }
    }
    uniform = __shfl_sync(full, uniform, 0);
    __syncwarp();

    if (uniform) {
      sg_cb = __shfl_sync(full, sg_cb, 0);
      sg_cn = __shfl_sync(full, sg_cn, 0);
      sg_off = __shfl_sync(full, sg_off, 0);
      // This lane's columns of the first two contributions at the chunk's
      // first row: a row's gradient is then one load per contribution, as
      // in the single-GPU kernel. Out-of-range contributions read as zero.
      const int ns = sg_cn < kStagedContribs ? sg_cn : kStagedContribs;
      const float* gb[kStagedContribs][2] = {{nullptr, nullptr}, {nullptr, nullptr}};
#pragma unroll
      for (int jj = 0; jj < kStagedContribs; ++jj) {
        if (jj < ns) {
          const int r = __ldg(q.contrib_rank + sg_cb + jj);
          const int64_t srow = __ldg(q.contrib_row + sg_cb + jj) + sg_off;
          if (r >= 0 && r < q.n_ranks && srow >= 0 && srow + nr <= __ldg(q.grad_rows + r)) {
#pragma unroll
            for (int e = 0; e < 2; ++e)
              gb[jj][e] = q.grad_src[r * kNumComp + lc.comp[e]] + srow * lc.width[e] + lc.col[e];
          } else if (lane == 0) {
            report_error(q.err, TGS_DEV_BAD_SLICE, sg_cb + jj, r);
          }
        }
      }
      auto load_grads = [&](int rr, float& x0, float& x1, float& y0, float& y1) {
        x0 = x1 = y0 = y1 = 0.f;
        if (rr < nr) {
          if (gb[0][0] != nullptr) {
            x0 = gb[0][0][rr * width[0]];
            x1 = gb[0][1][rr * width[1]];
          }
          if (gb[1][0] != nullptr) {
            y0 = gb[1][0][rr * width[0]];
            y1 = gb[1][1][rr * width[1]];
          }
        }
      };
      const RowAddr first = s_addr[warp][0];
      if (contiguous) {
        // Contiguous chunk: state rows staged by bulk copies as in kernel C;
        // the next batch's parameters and contributions load into registers
        // while the current batch updates.
        const float4* src = a.state + first.sr * 32;
        if (lane == 0) {
          for (int st = 0; st < kStateStages; ++st) {
            mbar_arrive_expect_tx(&ws.bar[st], kStateStageBytes);
            bulk_g2s(&ws.stage[st][0][0], src + st * kStateBatch * 32, kStateStageBytes,
                     &ws.bar[st]);
          }
        }
        uint32_t pending = (1u << kStateStages) - 1u;
        bool timed_out = false;
        float nx0[kStateBatch], nx1[kStateBatch], ny0[kStateBatch], ny1[kStateBatch];
        float np0[kStateBatch], np1[kStateBatch];
#pragma unroll
        for (int u = 0; u < kStateBatch; ++u) {
          load_grads(u, nx0[u], nx1[u], ny0[u], ny1[u]);
          np0[u] = pbase[0][(first.id + u) * width[0]];
          np1[u] = pbase[1][(first.id + u) * width[1]];
        }
#pragma unroll 1
        for (int qb = 0; qb < 32 / kStateBatch; ++qb) {
          const int st = qb % kStateStages;
          float x0[kStateBatch], x1[kStateBatch], y0[kStateBatch], y1[kStateBatch];
          float p0[kStateBatch], p1[kStateBatch];
#pragma unroll
          for (int u = 0; u < kStateBatch; ++u) {
            x0[u] = nx0[u];
            x1[u] = nx1[u];
            y0[u] = ny0[u];
            y1[u] = ny1[u];
            p0[u] = np0[u];
            p1[u] = np1[u];
          }
          if (qb + 1 < 32 / kStateBatch) {
#pragma unroll
            for (int u = 0; u < kStateBatch; ++u) {
              const int rr = (qb + 1) * kStateBatch + u;
              load_grads(rr, nx0[u], nx1[u], ny0[u], ny1[u]);
              np0[u] = pbase[0][(first.id + rr) * width[0]];
              np1[u] = pbase[1][(first.id + rr) * width[1]];
            }
          }
          if (!mbar_wait_bounded(&ws.bar[st], (phase >> st) & 1u)) {
            report_error(q.err, TGS_DEV_WAIT_TIMEOUT, row0);
            timed_out = true;
            break;
          }
          phase ^= 1u << st;
          pending &= ~(1u << st);
#pragma unroll
          for (int u = 0; u < kStateBatch; ++u) {
            const int rr = qb * kStateBatch + u;
            const RowScale rs = s_scale[warp][rr];
            const float4 sv = ws.stage[st][u][lane];
            float g0 = x0[u], g1 = x1[u];
            if (ns > 1) {
              g0 = fadd(g0, y0[u]);
              g1 = fadd(g1, y1[u]);
            }
#pragma unroll 1
            for (int jj = kStagedContribs; jj < sg_cn; ++jj) {
              float z0, z1;
              load_contrib(q, lc, sg_cb + jj, sg_off + rr, z0, z1);
              g0 = fadd(g0, z0);
              g1 = fadd(g1, z1);
            }
            const bool fresh =
                __shfl_sync(full, __float_as_uint(sv.x) == rs.stamp ? 1 : 0, 31) != 0;
            float m0 = fresh ? sv.x : 0.f, v0 = fresh ? sv.y : 0.f;
            float m1 = fresh ? sv.z : 0.f, v1 = fresh ? sv.w : 0.f;
            adam_elem<kPow2Batch>(p0[u], m0, v0, g0, hp, fmul(rs.rb1, lr[0]), rs.ds);
            adam_elem<kPow2Batch>(p1[u], m1, v1, g1, hp, fmul(rs.rb1, lr[1]), rs.ds);
            float4 out;
            out.x = stamp_lane ? __uint_as_float(rs.stamp) : (keep_lo ? m0 : 0.f);
            out.y = keep_lo ? v0 : 0.f;
            out.z = keep_hi ? m1 : 0.f;
            out.w = keep_hi ? v1 : 0.f;
            a.state[(first.sr + rr) * 32 + lane] = out;
            if (act[0]) pbase[0][(first.id + rr) * width[0]] = p0[u];
            if (act[1]) pbase[1][(first.id + rr) * width[1]] = p1[u];
          }
          __syncwarp();  // every lane is done with the stage
          const int qn = qb + kStateStages;
          if (qn < 32 / kStateBatch) {
            if (lane == 0) {
              fence_proxy_async_smem();
              mbar_arrive_expect_tx(&ws.bar[st], kStateStageBytes);
              bulk_g2s(&ws.stage[st][0][0], src + qn * kStateBatch * 32, kStateStageBytes,
                       &ws.bar[st]);
            }
            pending |= 1u << st;
          }
        }
        if (timed_out) {
          for (int st = 0; st < kStateStages; ++st)
            if ((pending >> st) & 1u) (void)mbar_wait_bounded(&ws.bar[st], (phase >> st) & 1u);
          return;
        }
        __syncwarp();
        continue;
      }
      // gradients of the next batch load while the current one updates
      float n0[kSumFastUnroll], n1[kSumFastUnroll], m0n[kSumFastUnroll], m1n[kSumFastUnroll];
#pragma unroll
      for (int u = 0; u < kSumFastUnroll; ++u) load_grads(u, n0[u], n1[u], m0n[u], m1n[u]);
      for (int r = 0; r < nr; r += kSumFastUnroll) {
        float4 st[kSumFastUnroll];
        float g0[kSumFastUnroll], g1[kSumFastUnroll], h0[kSumFastUnroll], h1[kSumFastUnroll];
        float p0[kSumFastUnroll], p1[kSumFastUnroll];
#pragma unroll
        for (int u = 0; u < kSumFastUnroll; ++u) {
          const int rr = r + u;  // warp-uniform
          g0[u] = n0[u];
          g1[u] = n1[u];
          h0[u] = m0n[u];
          h1[u] = m1n[u];
          st[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          p0[u] = p1[u] = 0.f;
          if (rr < nr) {
            const RowAddr ra = s_addr[warp][rr];
            st[u] = a.state[ra.sr * 32 + lane];
            p0[u] = pbase[0][ra.id * width[0]];
            p1[u] = pbase[1][ra.id * width[1]];
          }
        }
#pragma unroll
        for (int u = 0; u < kSumFastUnroll; ++u)
          load_grads(r + kSumFastUnroll + u, n0[u], n1[u], m0n[u], m1n[u]);
#pragma unroll
        for (int u = 0; u < kSumFastUnroll; ++u) {
          const int rr = r + u;
          if (rr >= nr) break;  // warp-uniform
          const RowAddr ra = s_addr[warp][rr];
          const RowScale rs = s_scale[warp][rr];
          if (ns > 1) {
            g0[u] = fadd(g0[u], h0[u]);
            g1[u] = fadd(g1[u], h1[u]);
          }
#pragma unroll 1
          for (int jj = kStagedContribs; jj < sg_cn; ++jj) {
            float x0, x1;
            load_contrib(q, lc, sg_cb + jj, sg_off + rr, x0, x1);
            g0[u] = fadd(g0[u], x0);
            g1[u] = fadd(g1[u], x1);
          }
          const bool fresh =
              __shfl_sync(full, __float_as_uint(st[u].x) == rs.stamp ? 1 : 0, 31) != 0;
          float m0 = fresh ? st[u].x : 0.f, v0 = fresh ? st[u].y : 0.f;
          float m1 = fresh ? st[u].z : 0.f, v1 = fresh ? st[u].w : 0.f;
          adam_elem<kPow2Batch>(p0[u], m0, v0, g0[u], hp, fmul(rs.rb1, lr[0]), rs.ds);
          adam_elem<kPow2Batch>(p1[u], m1, v1, g1[u], hp, fmul(rs.rb1, lr[1]), rs.ds);
          float4 out;
          out.x = stamp_lane ? __uint_as_float(rs.stamp) : (keep_lo ? m0 : 0.f);
          out.y = keep_lo ? v0 : 0.f;
          out.z = keep_hi ? m1 : 0.f;
          out.w = keep_hi ? v1 : 0.f;
          a.state[ra.sr * 32 + lane] = out;
          if (act[0]) pbase[0][ra.id * width[0]] = p0[u];
          if (act[1]) pbase[1][ra.id * width[1]] = p1[u];
        }
      }
      __syncwarp();
      continue;
    }

    // Chunk straddling segments: each row resolves its own segment.
    if (lane < nr) {
      const int64_t row = row0 + lane;
      const int sg = upper_bound_i64(q.seg_begin + 1, q.n_seg, row);
      RowSeg rs = {0, 0, 0};
      if (sg < q.n_seg && __ldg(q.seg_begin + sg) <= row) {
        rs.cb = static_cast<int32_t>(__ldg(q.contrib_offsets + sg));
        rs.cn = static_cast<int32_t>(__ldg(q.contrib_offsets + sg + 1)) - rs.cb;
        rs.off = row - __ldg(q.seg_begin + sg);
      } else {
        report_error(q.err, TGS_DEV_BAD_SLICE, row);
      }
      s_seg[warp][lane] = rs;
    }
    __syncwarp();

    for (int r = 0; r < nr; r += kSumUnroll) {
      float4 st[kSumUnroll];
      float g0[kSumUnroll], g1[kSumUnroll], h0[kSumUnroll], h1[kSumUnroll];
      float p0[kSumUnroll], p1[kSumUnroll];
#pragma unroll
      for (int u = 0; u < kSumUnroll; ++u) {
        const int rr = r + u;  // warp-uniform
        st[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        g0[u] = g1[u] = h0[u] = h1[u] = p0[u] = p1[u] = 0.f;
        if (rr < nr) {
          const RowAddr ra = s_addr[warp][rr];
          const RowSeg sg = s_seg[warp][rr];
          st[u] = a.state[ra.sr * 32 + lane];
          if (sg.cn > 0) load_contrib(q, lc, sg.cb, sg.off, g0[u], g1[u]);
          if (sg.cn > 1) load_contrib(q, lc, sg.cb + 1, sg.off, h0[u], h1[u]);
          p0[u] = pbase[0][ra.id * width[0]];
          p1[u] = pbase[1][ra.id * width[1]];
        }
      }
#pragma unroll
      for (int u = 0; u < kSumUnroll; ++u) {
        const int rr = r + u;
        if (rr >= nr) break;  // warp-uniform
        const RowAddr ra = s_addr[warp][rr];
        const RowScale rs = s_scale[warp][rr];
        const RowSeg sg = s_seg[warp][rr];
        if (sg.cn > 1) {
          g0[u] = fadd(g0[u], h0[u]);
          g1[u] = fadd(g1[u], h1[u]);
        }
#pragma unroll 1
        for (int jj = 2; jj < sg.cn; ++jj) {
          float x0, x1;
          load_contrib(q, lc, sg.cb + jj, sg.off, x0, x1);
          g0[u] = fadd(g0[u], x0);
          g1[u] = fadd(g1[u], x1);
        }
        const bool fresh =
            __shfl_sync(full, __float_as_uint(st[u].x) == rs.stamp ? 1 : 0, 31) != 0;
        float m0 = fresh ? st[u].x : 0.f, v0 = fresh ? st[u].y : 0.f;
        float m1 = fresh ? st[u].z : 0.f, v1 = fresh ? st[u].w : 0.f;
        adam_elem<kPow2Batch>(p0[u], m0, v0, g0[u], hp, fmul(rs.rb1, lr[0]), rs.ds);
        adam_elem<kPow2Batch>(p1[u], m1, v1, g1[u], hp, fmul(rs.rb1, lr[1]), rs.ds);
        float4 out;
        out.x = stamp_lane ? __uint_as_float(rs.stamp) : (keep_lo ? m0 : 0.f);
        out.y = keep_lo ? v0 : 0.f;
        out.z = keep_hi ? m1 : 0.f;
        out.w = keep_hi ? v1 : 0.f;
        a.state[ra.sr * 32 + lane] = out;
        if (act[0]) pbase[0][ra.id * width[0]] = p0[u];
        if (act[1]) pbase[1][ra.id * width[1]] = p1[u];
      }
    }
    __syncwarp();
   }
  }
}

// ---------------------------------------------------------------------------
// Kernels D / D': the update of streamable chunks as a bulk-copy pipeline.
// A chunk streams when its 32 ids and its 32 state rows both run
// consecutively and its first id is a multiple of 4 (the count kernel's
// chunk table): every chunk of a step that updates whole visible blocks. One
// CTA per SM walks a contiguous range of chunks with three warp roles (two
// loaders and two storers, each taking every other chunk):
//   loader    brings a chunk's 32 state rows (16 KB), six parameter segments
//             and six gradient segments (7.4 KB each; D': the first two
//             contributions' segments, read from the senders' memory) into a
//             shared-memory stage with non-multicast bulk copies, S stages
//             ahead, plus the rows' slot scales;
//   consumers update the stage in shared memory (16 warps, 2 rows each;
//             lane l: UNIFIED columns l and l + 32 of a row);
//   storer    writes the stage's parameters and state rows back with bulk
//             stores once the consumers are done, and frees the stage for
//             the loader when the stores have read it.
// A chunk costs a few large copies instead of 32 rows of per-lane loads
// whose latency the warps would have to hide. Chunks it updates are marked
// kChunkDone in the chunk table; kernels C / C' take the rest. Every wait is
// bounded: on a timeout the kernel records TGS_DEV_WAIT_TIMEOUT, waits
// (bounded) for its copies in flight and exits.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 32;
constexpr int kStreamConsumerWarps = 16;
// two loader and two storer warps: each takes every other chunk, so the
// per-chunk latency of issuing copies (and of waiting for the stores to
// read a stage) is spread over two warps
constexpr int kStreamLoaders = 2;
constexpr int kStreamStorers = 2;
constexpr int kFirstLoaderWarp = kStreamConsumerWarps;
constexpr int kFirstStorerWarp = kStreamConsumerWarps + kStreamLoaders;
constexpr int kStreamThreads = (kStreamConsumerWarps + kStreamLoaders + kStreamStorers) * 32;
constexpr int kRowsPerConsumer = kTileRows / kStreamConsumerWarps;
#ifndef TGS_STREAM_STAGES
#define TGS_STREAM_STAGES 4
#endif
#ifndef TGS_SUM_STREAM_STAGES
#define TGS_SUM_STREAM_STAGES 4
#endif
// contributions of a segment D' stages in shared memory; further ones are
// read from the senders' memory element by element
#ifndef TGS_SUM_STAGED_CONTRIBS
#define TGS_SUM_STAGED_CONTRIBS 4
#endif
// CTAs per SM of the streaming kernels (the stages of all of them share the
// SM's shared memory)
#ifndef TGS_STREAM_CTAS
#define TGS_STREAM_CTAS 1
#endif
#ifndef TGS_SUM_STREAM_CTAS
#define TGS_SUM_STREAM_CTAS 1
#endif
constexpr int kStateTileBytes = kTileRows * TGS_STATE_ROW_FLOATS * 4;  // 16 KB
constexpr int kRowTileBytes = kTileRows * kRowWidth * 4;                // 7552 B

struct __align__(16) StreamDesc {
  int64_t chunk;     // < 0: the CTA has no further chunk
  int64_t first_id;  // local row of the chunk's first row
  int64_t first_sr;  // state row of the chunk's first row
  int64_t seg_off;   // D': offset of the chunk's first row in its segment
  int32_t cb, cn;    // D': first contribution and contribution count of the segment
  int32_t ns;        // D': contributions staged in shared memory (<= kGrads)
  int32_t pad;
};

// One pipeline stage: a chunk's state rows, parameters (component c at
// kTileRows * unified_offset(c), rows contiguous) and kGrads gradient tiles
// of the same layout, plus the chunk's per-row slot scales.
template <int kGrads>
struct __align__(128) StreamStage {
  float state[kTileRows * TGS_STATE_ROW_FLOATS];
  float param[kTileRows * kRowWidth];
  float grad[kGrads][kTileRows * kRowWidth];
  RowScale scale[kTileRows];
  StreamDesc desc;
};

template <int kGrads, int kStages>
constexpr int stream_smem_bytes() {
  return kStages * static_cast<int>(sizeof(StreamStage<kGrads>)) + 3 * kStages * 8;
}

// Bulk loads of the six component segments of a chunk into a row tile:
// component c's kTileRows rows at kTileRows * unified_offset(c).
template <typename Src>
__device__ __forceinline__ void load_row_tile(float* dst, const Src (&src)[kNumComp], int64_t row,
                                              uint64_t* bar) {
#pragma unroll
  for (int c = 0; c < kNumComp; ++c)
    bulk_g2s(dst + kTileRows * unified_offset(c), src[c] + row * comp_width(c),
             kTileRows * comp_width(c) * 4, bar);
}

template <int kGrads>
__device__ __forceinline__ void store_tile(const ResidentApplyParams& a, StreamStage<kGrads>& st) {
  const int64_t fid = st.desc.first_id;
  bulk_s2g(a.state + st.desc.first_sr * (TGS_STATE_ROW_FLOATS / 4), st.state, kStateTileBytes);
#pragma unroll
  for (int c = 0; c < kNumComp; ++c)
    bulk_s2g(a.param[c] + fid * comp_width(c), st.param + kTileRows * unified_offset(c),
             kTileRows * comp_width(c) * 4);
}

// Per-lane column binding of the consumer warps: UNIFIED column j.
struct StreamCol {
  int base;   // kTileRows * unified_offset(c) + k
  int width;  // w_c
  int comp;
  int col;    // k
  float lr;
};

__device__ __forceinline__ StreamCol stream_col(const float (&lrs)[kNumComp], int j) {
  StreamCol sc;
  const int c = unified_comp_of(j);
  sc.comp = c;
  sc.col = j - unified_offset(c);
  sc.width = comp_width(c);
  sc.base = kTileRows * unified_offset(c) + sc.col;
  sc.lr = pick6(lrs, c);
  return sc;
}

// The loader's scan of its CTA's chunk range: the next chunk whose table
// entry marks it streamable (32 entries examined per load, lane-parallel).
struct ChunkScan {
  int64_t next, end, base;
  uint32_t mask;
  int64_t id, sr;  // this lane's entry of the current window
};

__device__ __forceinline__ int64_t scan_next(ChunkScan& cs, const int64_t* table, int lane,
                                             int64_t& fid, int64_t& fsr) {
  const unsigned full = 0xffffffffu;
  while (true) {
    if (cs.mask == 0) {
      if (cs.next >= cs.end) return -1;
      const int64_t c = cs.next + lane;
      cs.id = -1;
      cs.sr = -1;
      if (c < cs.end) {
        cs.id = table[2 * c];
        cs.sr = table[2 * c + 1];
      }
      cs.mask = __ballot_sync(full, cs.sr >= 0);
      cs.base = cs.next;
      cs.next += 32;
      continue;
    }
    const int b = __ffs(cs.mask) - 1;
    cs.mask &= cs.mask - 1;
    fid = __shfl_sync(full, cs.id, b);
    fsr = __shfl_sync(full, cs.sr, b);
    return cs.base + b;
  }
}

// Consumer update of UNIFIED column j of stage row r: the gradient is the
// first staged tile (D: the chunk's gradient; D': contribution 0), plus, for
// D', the second staged contribution and then any further ones read from the
// senders' memory one by one, in the segment's (rank) order.
template <bool kPow2Batch, bool kSum, int kGrads>
__device__ __forceinline__ void stream_update_col(float* param,
                                                  const float (*grads)[kTileRows * kRowWidth],
                                                  const StreamDesc& d, const ResidentSumParams* q,
                                                  float2* srow, const StreamCol& sc, int r, int j,
                                                  bool fresh, const RowScale& rs,
                                                  const AdamScalars& hp) {
  const int idx = sc.base + r * sc.width;
  float p = param[idx];
  float g = grads[0][idx];
  if constexpr (kSum) {
#pragma unroll
    for (int jj = 1; jj < kGrads; ++jj)
      if (jj < d.ns) g = fadd(g, grads[jj][idx]);
    for (int jj = d.ns; jj < d.cn; ++jj) {
      const int k = d.cb + jj;
      const int rk = __ldg(q->contrib_rank + k);
      const int64_t srow_src = __ldg(q->contrib_row + k) + d.seg_off + r;
      float x = 0.f;
      if (rk < 0 || rk >= q->n_ranks || srow_src < 0 || srow_src >= __ldg(q->grad_rows + rk))
        report_error(q->err, TGS_DEV_BAD_SLICE, k, rk);
      else
        x = q->grad_src[rk * kNumComp + sc.comp][srow_src * sc.width + sc.col];
      g = fadd(g, x);
    }
  }
  const float2 mv = srow[j];
  float m = fresh ? mv.x : 0.f, v = fresh ? mv.y : 0.f;
  adam_elem<kPow2Batch>(p, m, v, g, hp, fmul(rs.rb1, sc.lr), rs.ds);
  param[idx] = p;
  srow[j] = make_float2(m, v);
}

template <bool kPow2Batch, bool kSum>
__device__ void stream_kernel_body(const ResidentApplyParams& a, const ResidentSumParams* q) {
  constexpr int kGrads = kSum ? TGS_SUM_STAGED_CONTRIBS : 1;
  constexpr int kStages = kSum ? TGS_SUM_STREAM_STAGES : TGS_STREAM_STAGES;
  using Stage = StreamStage<kGrads>;
  extern __shared__ __align__(128) unsigned char stream_smem[];
  Stage* stages = reinterpret_cast<Stage*>(stream_smem);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(stages + kStages);  // loader -> all
  uint64_t* done_bar = full_bar + kStages;                              // consumers -> storer
  uint64_t* empty_bar = done_bar + kStages;                             // storer -> loader
  __shared__ int s_skip;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  int32_t* err = const_cast<int32_t*>(a.err);
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full_bar[st], 32);
      mbar_init(&done_bar[st], kStreamConsumerWarps);
      mbar_init(&empty_bar[st], 1);
    }
    fence_mbar_init();
    s_skip = load_error(a.err);
  }
  __syncthreads();
  if (s_skip != 0) return;

  static_assert(kStages % kStreamLoaders == 0 && kStages % kStreamStorers == 0,
                "a stage must always be filled by the same loader and drained by the same storer");
  if (warp >= kFirstLoaderWarp && warp < kFirstStorerWarp) {
    // ------------------------------- loaders ------------------------------
    // Loader w fills the chunks t = w, w + 2, ... of the CTA's sequence of
    // accepted chunks (both loaders walk the same sequence).
    const int w = warp - kFirstLoaderWarp;
    const int64_t n_chunks = a.n / kTileRows;  // only full chunks stream
    ChunkScan cs;
    cs.next = n_chunks * blockIdx.x / gridDim.x;
    cs.end = n_chunks * (blockIdx.x + 1) / gridDim.x;
    cs.base = 0;
    cs.mask = 0;
    cs.id = cs.sr = -1;
    const int64_t B = a.block_size;
    const bool pow2B = (B & (B - 1)) == 0;
    const int shiftB = __ffsll(B) - 1;
    // D': the segment of the last chunk looked at, cached per loader: its
    // row range, its contributions, and (shared memory) the base pointers
    // and source rows of the staged ones. Every check of a staged
    // contribution (rank in range, base pointers 16-byte aligned, the
    // segment's rows inside the sender's gradient rows, row offsets a
    // multiple of 4) is made once per segment.
    __shared__ const float* s_src[kStreamLoaders][kGrads][kNumComp];
    __shared__ int64_t s_row[kStreamLoaders][kGrads];
    int64_t seg_lo = 0, seg_hi = -1;
    int32_t seg_cb = 0, seg_cn = 0, seg_ns = 0;
    bool seg_ok = false;
    bool failed = false;
    int64_t accepted = 0;  // chunks of the sequence seen so far (both loaders')
    int64_t t = w;
    for (;; t += kStreamLoaders) {
      const int st = static_cast<int>(t % kStages);
      const uint32_t use = static_cast<uint32_t>(t / kStages);
      Stage& S = stages[st];
      int64_t chunk = -1, fid = 0, fsr = 0;
      // the t-th accepted chunk of the sequence
      while (true) {
        chunk = scan_next(cs, a.chunk_table, lane, fid, fsr);
        if (chunk < 0) break;
        if constexpr (kSum) {
          const int64_t row0 = chunk * kTileRows;
          if (row0 < seg_lo || row0 >= seg_hi) {
            if (lane == 0) {
              const int sg = upper_bound_i64(q->seg_begin + 1, q->n_seg, row0);
              seg_ok = false;
              seg_hi = -1;
              if (sg < q->n_seg && __ldg(q->seg_begin + sg) <= row0) {
                seg_lo = __ldg(q->seg_begin + sg);
                seg_hi = __ldg(q->seg_begin + sg + 1);
                seg_cb = static_cast<int32_t>(__ldg(q->contrib_offsets + sg));
                seg_cn = static_cast<int32_t>(__ldg(q->contrib_offsets + sg + 1)) - seg_cb;
                seg_ns = seg_cn < kGrads ? seg_cn : kGrads;
                seg_ok = seg_cn >= 1;
#pragma unroll
                for (int jj = 0; jj < kGrads; ++jj) {
                  if (jj >= seg_ns) break;
                  const int r = __ldg(q->contrib_rank + seg_cb + jj);
                  const int64_t row = __ldg(q->contrib_row + seg_cb + jj);
                  s_row[w][jj] = row;
                  if (r < 0 || r >= q->n_ranks || row < 0 || ((row - seg_lo) & 3) != 0 ||
                      row + (seg_hi - seg_lo) > __ldg(q->grad_rows + r)) {
                    seg_ok = false;
                    continue;
                  }
                  for (int c = 0; c < kNumComp; ++c) {
                    const float* ptr = q->grad_src[r * kNumComp + c];
                    if (!aligned16(ptr)) seg_ok = false;
                    s_src[w][jj][c] = ptr;
                  }
                }
              }
            }
            seg_lo = __shfl_sync(full, seg_lo, 0);
            seg_hi = __shfl_sync(full, seg_hi, 0);
            seg_ok = __shfl_sync(full, seg_ok ? 1 : 0, 0) != 0;
            seg_cb = __shfl_sync(full, seg_cb, 0);
            seg_cn = __shfl_sync(full, seg_cn, 0);
            seg_ns = __shfl_sync(full, seg_ns, 0);
          }
          if (!(seg_ok && row0 + kTileRows <= seg_hi)) continue;  // not streamable
        }
        if (accepted++ == t) break;  // the other loader's chunks are skipped
      }
      // the chunk's row scales start loading before the wait for the stage
      float2 bb = make_float2(0.f, 0.f);
      uint32_t stamp = 0;
      if (chunk >= 0) {
        const int64_t sr = fsr + lane;
        const int64_t slot = pow2B ? (sr >> shiftB) : sr / B;
        bb = a.slot_bias[slot];
        stamp = __ldg(a.slot_stamp + slot);
      }
      if (t >= kStages) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait_bounded(&empty_bar[st], (use - 1) & 1u) ? 1 : 0;
        if (__shfl_sync(full, ok, 0) == 0) {
          failed = true;
          break;
        }
      }
      if (chunk < 0) {
        if (lane == 0) S.desc.chunk = -1;
        __syncwarp();
        mbar_arrive(&full_bar[st]);  // completes the phase without bytes
        break;
      }
      const int ns = kSum ? seg_ns : 1;
      const int64_t seg_off = kSum ? chunk * kTileRows - seg_lo : 0;
      if (lane == 0) {
        S.desc.chunk = chunk;
        S.desc.first_id = fid;
        S.desc.first_sr = fsr;
        S.desc.ns = ns;
        S.desc.cb = seg_cb;
        S.desc.cn = seg_cn;
        S.desc.seg_off = seg_off;
        mbar_expect_tx(&full_bar[st], kStateTileBytes + kRowTileBytes * (1 + ns));
        bulk_g2s(S.state, a.state + fsr * (TGS_STATE_ROW_FLOATS / 4), kStateTileBytes,
                 &full_bar[st]);
        load_row_tile(S.param, a.param, fid, &full_bar[st]);
        if constexpr (kSum) {
#pragma unroll
          for (int jj = 0; jj < kGrads; ++jj) {
            if (jj >= ns) break;
            const int64_t srow = s_row[w][jj] + seg_off;
#pragma unroll
            for (int c = 0; c < kNumComp; ++c)
              bulk_g2s(S.grad[jj] + kTileRows * unified_offset(c),
                       s_src[w][jj][c] + srow * comp_width(c), kTileRows * comp_width(c) * 4,
                       &full_bar[st]);
          }
        } else {
          load_row_tile(S.grad[0], a.grad, chunk * kTileRows, &full_bar[st]);
        }
        a.chunk_table[2 * chunk + 1] = kChunkDone;
      }
      S.scale[lane] = {bb.x, bb.y, stamp, 0u};
      // the 32 arrivals publish the descriptor and the row scales; the phase
      // completes when the copies' bytes have landed as well
      mbar_arrive(&full_bar[st]);
      __syncwarp();
    }
    if (failed && lane == 0) {
      report_error(err, TGS_DEV_WAIT_TIMEOUT, t);
      // this loader's loads still in flight land before the CTA may exit
      for (int64_t j = t - kStages; j < t; j += kStreamLoaders)
        if (j >= 0)
          (void)mbar_wait_bounded(&full_bar[j % kStages], static_cast<uint32_t>(j / kStages) & 1u);
    }
    return;
  }

  if (warp >= kFirstStorerWarp) {
    // ------------------------------- storers ------------------------------
    // Storer w drains the chunks t = w, w + 2, ...
    const int w = warp - kFirstStorerWarp;
    for (int64_t t = w;; t += kStreamStorers) {
      const int st = static_cast<int>(t % kStages);
      const uint32_t par = static_cast<uint32_t>(t / kStages) & 1u;
      Stage& S = stages[st];
      int ok = 1;
      if (lane == 0) {
        ok = mbar_wait_bounded(&full_bar[st], par) ? 1 : 0;
        if (ok && S.desc.chunk < 0) ok = 2;  // no further chunk
        if (ok == 1) ok = mbar_wait_bounded(&done_bar[st], par) ? 1 : 0;
        if (ok == 1) {
          store_tile(a, S);
          bulk_commit();
          bulk_wait_read<0>();  // the stage may be overwritten from here on
          mbar_arrive(&empty_bar[st]);
        }
        if (ok == 0) report_error(err, TGS_DEV_WAIT_TIMEOUT, t);
      }
      if (__shfl_sync(full, ok, 0) != 1) break;
    }
    if (lane == 0) bulk_wait_all();
    return;
  }

  // ------------------------------ consumers ------------------------------
  const AdamScalars hp = {a.beta1, a.beta2, a.omb1, a.omb2, a.eps, a.batch_size, a.inv_batch_size};
  const StreamCol c0 = stream_col(a.lr, lane);
  const bool has1 = lane + 32 < kRowWidth;
  const StreamCol c1 = stream_col(a.lr, has1 ? lane + 32 : 0);
  for (int64_t t = 0;; ++t) {
    const int st = static_cast<int>(t % kStages);
    Stage& S = stages[st];
    if (!mbar_wait_bounded(&full_bar[st], static_cast<uint32_t>(t / kStages) & 1u)) {
      if (lane == 0) report_error(err, TGS_DEV_WAIT_TIMEOUT, t);
      break;
    }
    if (S.desc.chunk < 0) break;
    const StreamDesc d = S.desc;
#pragma unroll
    for (int u = 0; u < kRowsPerConsumer; ++u) {
      const int r = warp * kRowsPerConsumer + u;
      const RowScale rs = S.scale[r];
      float* srow_f = S.state + r * TGS_STATE_ROW_FLOATS;
      float2* srow = reinterpret_cast<float2*>(srow_f);
      // a row whose stamp is not its slot's current stamp has not been
      // touched since the block was (re)admitted: its moments are zero
      const bool fresh = __float_as_uint(srow_f[124]) == rs.stamp;
      stream_update_col<kPow2Batch, kSum, kGrads>(S.param, S.grad, d, q, srow, c0, r, lane,
                                                  fresh, rs, hp);
      if (has1)
        stream_update_col<kPow2Batch, kSum, kGrads>(S.param, S.grad, d, q, srow, c1, r,
                                                    lane + 32, fresh, rs, hp);
      __syncwarp();  // every lane has read the stamp
      if (lane == 30) srow_f[124] = __uint_as_float(rs.stamp);
    }
    fence_proxy_async_smem();  // this warp's writes, before the bulk stores read them
    __syncwarp();
    if (lane == 0) mbar_arrive(&done_bar[st]);
  }
}

template <bool kPow2Batch>
__global__ void __launch_bounds__(kStreamThreads, TGS_STREAM_CTAS)
    resident_adam_stream_kernel(const ResidentApplyParams a) {
  stream_kernel_body<kPow2Batch, false>(a, nullptr);
}

template <bool kPow2Batch>
__global__ void __launch_bounds__(kStreamThreads, TGS_SUM_STREAM_CTAS)
    resident_adam_sum_stream_kernel(const ResidentSumParams q) {
  stream_kernel_body<kPow2Batch, true>(q.a, &q);
}

// ---------------------------------------------------------------------------
// Dense masked optimizers (SelectiveAdam, SelectiveSophia). All groups run in
// one launch: CTAs [cta_begin[g], cta_begin[g+1]) serve group g. A thread
// handles 4 consecutive elements (one float4 when the group is 16-byte
// aligned); the row of the first element comes from a multiply-high by a
// precomputed reciprocal, the others by increment.
// ---------------------------------------------------------------------------
struct DenseGroupParams {
  float* param;
  const float* grad;
  float* m;
  float* v;
  const float* noise;
  int64_t width;
  uint64_t magic;  // floor(2^64 / width) + 1, valid for width >= 2
  int64_t total;   // N * width
  float lr, beta1, beta2, omb1, omb2, eps, rho, wd;
  int vec_ok;
};

struct DenseParams {
  DenseGroupParams g[TGS_MAX_GROUPS];
  int cta_begin[TGS_MAX_GROUPS + 1];
  int n_groups;
  const uint8_t* vis;
  int hessian_step;
};

constexpr int kDenseThreads = 256;
constexpr int kDenseVecPerThread = 4;

__device__ __forceinline__ void selective_adam_elem(float& p, float& m, float& v, float g,
                                                    const DenseGroupParams& G) {
  m = fadd(fmul(G.beta1, m), fmul(G.omb1, g));
  v = fadd(fmul(G.beta2, v), fmul(fmul(G.omb2, g), g));
  const float step = fdiv(fmul(-G.lr, m), fadd(fsqrt(v), G.eps));
  p = fadd(p, step);
}

__device__ __forceinline__ void sophia_elem(float& p, float& m, float& h, float g, float u,
                                            bool hess, const DenseGroupParams& G) {
  m = fadd(fmul(G.beta1, m), fmul(G.omb1, g));
  if (hess) {
    const float q = fmul(u, g);
    h = fadd(fmul(G.beta2, h), fmul(G.omb2, fmul(q, q)));
  }
  if (G.wd != 0.f) p = fsub(p, fmul(fmul(G.lr, G.wd), p));
  float ratio = fdiv(m, fmaxf(fmul(G.rho, h), G.eps));
  ratio = fminf(fmaxf(ratio, -1.f), 1.f);
  p = fsub(p, fmul(G.lr, ratio));
}

// Eight CTAs of 256 threads fill every warp slot of an SM: the kernel is
// bound by load latency (one float4 per array in flight per thread), so the
// 32-register cap (20 bytes of spill in the SelectiveAdam variant) buys more
// loads in flight than it costs: 0.178 / 1.29 ms per SelectiveAdam / Sophia
// step against 0.187 / 1.47 ms at six CTAs per SM.
template <bool kSophia>
__global__ void __launch_bounds__(kDenseThreads, 8) dense_kernel(const DenseParams a) {
  int gi = 0;
#pragma unroll 1
  while (gi + 1 < a.n_groups && static_cast<int>(blockIdx.x) >= a.cta_begin[gi + 1]) ++gi;
  const DenseGroupParams& G = a.g[gi];
  const int64_t local_cta = static_cast<int64_t>(blockIdx.x) - a.cta_begin[gi];
  const int64_t ctas = a.cta_begin[gi + 1] - a.cta_begin[gi];
  const int64_t nvec = (G.total + 3) / 4;
  const bool hess = kSophia && a.hessian_step != 0;

  for (int64_t q = local_cta * kDenseThreads + threadIdx.x; q < nvec;
       q += ctas * kDenseThreads) {
    const int64_t e0 = q * 4;
    int64_t row = G.width == 1 ? e0 : static_cast<int64_t>(__umul64hi(static_cast<uint64_t>(e0), G.magic));
    int64_t col = e0 - row * G.width;
    bool vis[4];
    bool any = false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const bool in = e0 + k < G.total;
      vis[k] = in && a.vis[row] != 0;
      any |= vis[k];
      if (++col == G.width) {
        col = 0;
        ++row;
      }
    }
    if (!any) continue;
    float pv[4], gv[4], mv[4], vv[4], uv[4] = {0.f, 0.f, 0.f, 0.f};
    const bool full_vec = G.vec_ok && e0 + 4 <= G.total;
    if (full_vec) {
      const float4 p4 = *reinterpret_cast<const float4*>(G.param + e0);
      const float4 g4 = *reinterpret_cast<const float4*>(G.grad + e0);
      const float4 m4 = *reinterpret_cast<const float4*>(G.m + e0);
      const float4 v4 = *reinterpret_cast<const float4*>(G.v + e0);
      pv[0] = p4.x; pv[1] = p4.y; pv[2] = p4.z; pv[3] = p4.w;
      gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
      mv[0] = m4.x; mv[1] = m4.y; mv[2] = m4.z; mv[3] = m4.w;
      vv[0] = v4.x; vv[1] = v4.y; vv[2] = v4.z; vv[3] = v4.w;
      if (hess) {
        const float4 u4 = *reinterpret_cast<const float4*>(G.noise + e0);
        uv[0] = u4.x; uv[1] = u4.y; uv[2] = u4.z; uv[3] = u4.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        pv[k] = gv[k] = mv[k] = vv[k] = 0.f;
        if (vis[k]) {
          pv[k] = G.param[e0 + k];
          gv[k] = G.grad[e0 + k];
          mv[k] = G.m[e0 + k];
          vv[k] = G.v[e0 + k];
          if (hess) uv[k] = G.noise[e0 + k];
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (!vis[k]) continue;
      if (kSophia) sophia_elem(pv[k], mv[k], vv[k], gv[k], uv[k], hess, G);
      else selective_adam_elem(pv[k], mv[k], vv[k], gv[k], G);
    }
    if (full_vec) {
      // Invisible lanes carry their unchanged values back.
      *reinterpret_cast<float4*>(G.param + e0) = make_float4(pv[0], pv[1], pv[2], pv[3]);
      *reinterpret_cast<float4*>(G.m + e0) = make_float4(mv[0], mv[1], mv[2], mv[3]);
      *reinterpret_cast<float4*>(G.v + e0) = make_float4(vv[0], vv[1], vv[2], vv[3]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (!vis[k]) continue;
        G.param[e0 + k] = pv[k];
        G.m[e0 + k] = mv[k];
        G.v[e0 + k] = vv[k];
      }
    }
  }
}

int launch_dense(const TgsDenseArgs* args, void* stream, bool sophia) {
  const char* who = sophia ? "tgs_sophia_step" : "tgs_selective_adam";
  TGS_CHECK_ARG(args != nullptr, "%s: args is NULL", who);
  TGS_CHECK_ARG(args->n_groups >= 0 && args->n_groups <= TGS_MAX_GROUPS,
                "%s: n_groups=%d outside [0, %d]", who, args->n_groups, TGS_MAX_GROUPS);
  TGS_CHECK_ARG(args->n_rows >= 0, "%s: n_rows=%lld < 0", who, (long long)args->n_rows);
  if (args->n_rows == 0 || args->n_groups == 0) return TGS_OK;
  TGS_CHECK_ARG(args->visibility != nullptr, "%s: visibility is NULL", who);

  DenseParams p;
  memset(&p, 0, sizeof(p));
  p.n_groups = args->n_groups;
  p.vis = args->visibility;
  p.hessian_step = args->hessian_step;
  int64_t cta_total = 0;
  for (int gi = 0; gi < args->n_groups; ++gi) {
    const TgsDenseGroup& in = args->groups[gi];
    DenseGroupParams& G = p.g[gi];
    TGS_CHECK_ARG(in.param && in.grad && in.exp_avg && in.exp_avg_sq,
                  "%s: group %d has a NULL tensor", who, gi);
    TGS_CHECK_ARG(in.width >= 1 && in.width <= (1 << 20), "%s: group %d width=%lld invalid", who,
                  gi, (long long)in.width);
    TGS_CHECK_ARG(!(sophia && args->hessian_step && in.noise == nullptr),
                  "%s: group %d needs a noise tensor on a Hessian step", who, gi);
    G.param = in.param;
    G.grad = in.grad;
    G.m = in.exp_avg;
    G.v = in.exp_avg_sq;
    G.noise = in.noise;
    G.width = in.width;
    G.magic = in.width >= 2 ? (~0ull / static_cast<uint64_t>(in.width)) + 1ull : 0ull;
    G.total = args->n_rows * in.width;
    TGS_CHECK_ARG(G.total < (1ll << 44), "%s: group %d too large", who, gi);
    G.lr = in.lr;
    G.beta1 = in.beta1;
    G.beta2 = in.beta2;
    // (1 - b) rounded in fp32, as the reference computes it in device fp32.
    G.omb1 = 1.0f - in.beta1;
    G.omb2 = 1.0f - in.beta2;
    G.eps = in.eps;
    G.rho = in.rho;
    G.wd = in.weight_decay;
    G.vec_ok = aligned16(in.param) && aligned16(in.grad) && aligned16(in.exp_avg) &&
               aligned16(in.exp_avg_sq) && (!sophia || in.noise == nullptr || aligned16(in.noise));
    const int64_t nvec = (G.total + 3) / 4;
    const int64_t ctas = std::max<int64_t>(
        1, ceil_div<int64_t>(nvec, static_cast<int64_t>(kDenseThreads) * kDenseVecPerThread));
    p.cta_begin[gi] = static_cast<int>(cta_total);
    cta_total += ctas;
  }
  TGS_CHECK_ARG(cta_total < (1ll << 31), "%s: grid too large", who);
  p.cta_begin[args->n_groups] = static_cast<int>(cta_total);
  cudaStream_t s = as_stream(stream);
  if (sophia) dense_kernel<true><<<static_cast<unsigned>(cta_total), kDenseThreads, 0, s>>>(p);
  else dense_kernel<false><<<static_cast<unsigned>(cta_total), kDenseThreads, 0, s>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_resident_adam_count(const TgsResidentCountArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_resident_adam_count: args is NULL");
  TGS_CHECK_ARG(a->n_positions >= 1, "tgs_resident_adam_count: working set contains no resident blocks");
  TGS_CHECK_ARG(a->n_rows >= 0 && a->block_size >= 1 && a->param_rows >= 0,
                "tgs_resident_adam_count: bad sizes n=%lld block=%lld rows=%lld",
                (long long)a->n_rows, (long long)a->block_size, (long long)a->param_rows);
  TGS_CHECK_ARG(a->pos_start && a->pos_end && a->pos_slot && a->pos_count && a->err &&
                    a->slot_step && a->slot_bias && a->step_table && a->step_table_len >= 2,
                "tgs_resident_adam_count: NULL table or step_table_len < 2");
  TGS_CHECK_ARG(a->n_rows == 0 || a->local_ids != nullptr, "tgs_resident_adam_count: local_ids is NULL");
  cudaStream_t s = as_stream(stream);
  TGS_CUDA(cudaMemsetAsync(a->pos_count, 0, sizeof(int32_t) * a->n_positions, s));
  TGS_CUDA(cudaMemsetAsync(a->err, 0, sizeof(int32_t) * 4, s));
  if (a->n_rows == 0) return TGS_OK;
  const int64_t blocks = ceil_div<int64_t>(a->n_rows, int64_t(kCountThreads) * kCountRows);
  TGS_CHECK_ARG(blocks < (1ll << 31), "tgs_resident_adam_count: n_rows too large");
  resident_count_kernel<<<static_cast<unsigned>(blocks), kCountThreads, 0, s>>>(
      a->local_ids, a->n_rows, a->param_rows, a->pos_start, a->pos_end, a->pos_slot,
      a->n_positions, a->block_size, a->pos_count, a->chunk_table, a->err);
  TGS_LAUNCH_CHECK();
  resident_slot_kernel<<<ceil_div(a->n_positions, 256), 256, 0, s>>>(
      a->pos_count, a->pos_slot, a->n_positions, a->slot_step,
      reinterpret_cast<float2*>(a->slot_bias), reinterpret_cast<const float2*>(a->step_table),
      a->step_table_len, a->err);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

namespace {

// Checks the update arguments shared by both apply entry points and fills the
// kernel parameters; *pow2 tells whether the batch divide is a multiply.
int fill_apply_params(const TgsResidentAdamArgs* a, bool need_grad, const char* who,
                      ResidentApplyParams* p, bool* pow2) {
  TGS_CHECK_ARG(a->n_rows > 0 && a->n_positions >= 1 && a->block_size >= 1, "%s: bad sizes", who);
  TGS_CHECK_ARG(a->local_ids && a->pos_start && a->pos_end && a->pos_slot && a->state &&
                    a->slot_stamp && a->slot_bias && a->err,
                "%s: NULL pointer", who);
  TGS_CHECK_ARG(aligned16(a->state), "%s: state must be 16-byte aligned", who);
  TGS_CHECK_ARG(a->batch_size != 0.0f, "%s: batch_size is 0", who);
  for (int c = 0; c < kNumComp; ++c) {
    TGS_CHECK_ARG(a->param[c] && (a->grad[c] || !need_grad), "%s: component %d is NULL", who, c);
    p->param[c] = a->param[c];
    p->grad[c] = a->grad[c];
    p->lr[c] = a->lr[c];
  }
  p->beta1 = a->beta1;
  p->beta2 = a->beta2;
  p->omb1 = a->one_minus_beta1;
  p->omb2 = a->one_minus_beta2;
  p->eps = a->eps;
  p->batch_size = a->batch_size;
  // A power-of-two batch size with a normal reciprocal divides exactly by a
  // multiply (same exactly rounded result as the division).
  int exp2 = 0;
  const float mant = frexpf(a->batch_size, &exp2);
  *pow2 = mant == 0.5f && exp2 > -125 && exp2 < 126;
  p->inv_batch_size = *pow2 ? 1.0f / a->batch_size : 0.0f;
  p->pos_start = a->pos_start;
  p->pos_end = a->pos_end;
  p->pos_slot = a->pos_slot;
  p->n_pos = a->n_positions;
  p->block_size = a->block_size;
  p->ids = a->local_ids;
  p->n = a->n_rows;
  p->state = reinterpret_cast<float4*>(a->state);
  p->slot_stamp = a->slot_stamp;
  p->slot_bias = reinterpret_cast<const float2*>(a->slot_bias);
  p->err = a->err;
  p->chunk_table = a->chunk_table;
  return TGS_OK;
}

// Whether the bulk-copy pipeline may run: a chunk table, at least one full
// chunk, and 16-byte aligned parameter (and, for the single-GPU update,
// gradient) components.
bool can_stream(const ResidentApplyParams& p, bool need_grad) {
  if (p.chunk_table == nullptr || p.n < kTileRows) return false;
  for (int c = 0; c < kNumComp; ++c) {
    if (!aligned16(p.param[c])) return false;
    if (need_grad && !aligned16(p.grad[c])) return false;
  }
  return true;
}

int stream_grid(int64_t n_rows, int ctas_per_sm) {
  const int64_t chunks = n_rows / kTileRows;
  return static_cast<int>(std::min<int64_t>(chunks, int64_t(sm_count()) * ctas_per_sm));
}

// Launches a streaming kernel, raising its dynamic shared-memory limit on
// first use on the current device.
template <typename Kernel, typename Params>
int launch_stream(Kernel kernel, const Params& p, int smem, int grid, cudaStream_t s,
                  bool* configured) {
  static std::mutex mu;
  int dev = 0;
  TGS_CUDA(cudaGetDevice(&dev));
  TGS_CHECK_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      TGS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      configured[dev] = true;
    }
  }
  kernel<<<grid, kStreamThreads, smem, s>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

int apply_grid(int64_t n_rows, int ctas_per_sm = kApplyMinBlocks) {
  const int64_t warps_needed = ceil_div<int64_t>(n_rows, 32);
  const int64_t ctas_needed = ceil_div<int64_t>(warps_needed, kApplyThreads / 32);
  const int64_t cap = static_cast<int64_t>(sm_count()) * ctas_per_sm;
  return static_cast<int>(std::min<int64_t>(ctas_needed, cap));
}

// Launches resident_adam_kernel, raising its dynamic shared-memory limit on
// first use on the current device.
template <bool kPow2>
int launch_apply(const ResidentApplyParams& p, int grid, cudaStream_t s) {
  static bool configured[64] = {false};
  static std::mutex mu;
  int dev = 0;
  TGS_CUDA(cudaGetDevice(&dev));
  TGS_CHECK_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      TGS_CUDA(cudaFuncSetAttribute(resident_adam_kernel<kPow2>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kApplySmemBytes));
      configured[dev] = true;
    }
  }
  resident_adam_kernel<kPow2><<<grid, kApplyThreads, kApplySmemBytes, s>>>(p);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

// Launches resident_adam_sum_kernel, raising its dynamic shared-memory limit
// on first use on the current device.
template <bool kPow2>
int launch_sum(const ResidentSumParams& q, int grid, cudaStream_t s) {
  static bool configured[64] = {false};
  static std::mutex mu;
  int dev = 0;
  TGS_CUDA(cudaGetDevice(&dev));
  TGS_CHECK_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      TGS_CUDA(cudaFuncSetAttribute(resident_adam_sum_kernel<kPow2>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kApplySmemBytes));
      configured[dev] = true;
    }
  }
  resident_adam_sum_kernel<kPow2><<<grid, kApplyThreads, kApplySmemBytes, s>>>(q);
  TGS_LAUNCH_CHECK();
  return TGS_OK;
}

}  // namespace

extern "C" int tgs_resident_adam_apply(const TgsResidentAdamArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_resident_adam_apply: args is NULL");
  if (a->n_rows == 0) return TGS_OK;
  ResidentApplyParams p;
  bool pow2 = false;
  const int rc = fill_apply_params(a, true, "tgs_resident_adam_apply", &p, &pow2);
  if (rc != TGS_OK) return rc;
  cudaStream_t s = as_stream(stream);
  if (can_stream(p, true)) {
    static bool configured[2][64] = {};
    constexpr int smem = stream_smem_bytes<1, TGS_STREAM_STAGES>();
    const int sgrid = stream_grid(a->n_rows, TGS_STREAM_CTAS);
    const int rc2 = pow2 ? launch_stream(resident_adam_stream_kernel<true>, p, smem, sgrid, s,
                                         configured[1])
                         : launch_stream(resident_adam_stream_kernel<false>, p, smem, sgrid, s,
                                         configured[0]);
    if (rc2 != TGS_OK) return rc2;
  }
  const int grid = apply_grid(a->n_rows);
  return pow2 ? launch_apply<true>(p, grid, s) : launch_apply<false>(p, grid, s);
}

extern "C" int tgs_resident_adam_apply_sum(const TgsResidentAdamSumArgs* a, void* stream) {
  TGS_CHECK_ARG(a != nullptr, "tgs_resident_adam_apply_sum: args is NULL");
  if (a->adam.n_rows == 0) return TGS_OK;
  ResidentSumParams q;
  bool pow2 = false;
  const int rc = fill_apply_params(&a->adam, false, "tgs_resident_adam_apply_sum", &q.a, &pow2);
  if (rc != TGS_OK) return rc;
  TGS_CHECK_ARG(a->n_ranks >= 1 && a->n_segments >= 1,
                "tgs_resident_adam_apply_sum: n_ranks=%d n_segments=%d", a->n_ranks,
                a->n_segments);
  TGS_CHECK_ARG(a->grad_src && a->grad_rows && a->seg_begin && a->contrib_offsets &&
                    a->contrib_rank && a->contrib_row && a->err,
                "tgs_resident_adam_apply_sum: NULL table");
  TGS_CHECK_ARG(a->err == a->adam.err, "tgs_resident_adam_apply_sum: err must be adam.err");
  q.grad_src = a->grad_src;
  q.grad_rows = a->grad_rows;
  q.n_ranks = a->n_ranks;
  q.seg_begin = a->seg_begin;
  q.n_seg = a->n_segments;
  q.contrib_offsets = a->contrib_offsets;
  q.contrib_rank = a->contrib_rank;
  q.contrib_row = a->contrib_row;
  const int64_t n_chunks = ceil_div<int64_t>(a->adam.n_rows, 32);
  TGS_CHECK_ARG(a->rotate_rows >= 0, "tgs_resident_adam_apply_sum: rotate_rows < 0");
  q.rotate_chunks = (a->rotate_rows / 32) % n_chunks;
  q.err = a->err;
  cudaStream_t s = as_stream(stream);
  if (can_stream(q.a, false)) {
    static bool configured[2][64] = {};
    constexpr int smem = stream_smem_bytes<TGS_SUM_STAGED_CONTRIBS, TGS_SUM_STREAM_STAGES>();
    TGS_CHECK_ARG(a->max_ctas >= 0, "tgs_resident_adam_apply_sum: max_ctas < 0");
    int sgrid = stream_grid(a->adam.n_rows, TGS_SUM_STREAM_CTAS);
    if (a->max_ctas > 0) sgrid = std::min(sgrid, static_cast<int>(a->max_ctas));
    const int rc2 = pow2 ? launch_stream(resident_adam_sum_stream_kernel<true>, q, smem, sgrid, s,
                                         configured[1])
                         : launch_stream(resident_adam_sum_stream_kernel<false>, q, smem, sgrid,
                                         s, configured[0]);
    if (rc2 != TGS_OK) return rc2;
  }
  const int grid = apply_grid(a->adam.n_rows, kSumMinBlocks);
  return pow2 ? launch_sum<true>(q, grid, s) : launch_sum<false>(q, grid, s);
}

extern "C" int tgs_selective_adam(const TgsDenseArgs* args, void* stream) {
  return launch_dense(args, stream, false);
}

extern "C" int tgs_sophia_step(const TgsDenseArgs* args, void* stream) {
  return launch_dense(args, stream, true);
}
