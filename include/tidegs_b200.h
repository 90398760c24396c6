/*
 * tidegs_b200.h -- C ABI of libtidegs_b200.so, the sm_100a implementation of
 * TideGS's resident-block optimizer / materialization / write-back hot path,
 * and of the steps either side of it: touched-only gradient accumulation,
 * per-block host DMAs, block frustum culling, and the gsplat render kernels
 * (projection, SH colors, tile intersection, rasterization).
 *
 * Conventions shared by every entry point:
 *   - Plain pointers and sizes only. Every pointer named dev_* / inside an args
 *     struct is a DEVICE pointer unless its comment says "host".
 *   - The library allocates nothing and keeps no per-call state: every buffer,
 *     including scratch words, is owned by the caller. Calls are re-entrant and
 *     may come from several host threads on different streams. Two
 *     exceptions: tgs_peer_buffer_alloc allocates the exportable buffer its
 *     caller asks for and hands its ownership to that caller, and
 *     tgs_global_to_local_compact_noalloc keeps fixed per-device scratch
 *     inside the library (see its declaration).
 *   - `stream` is a cudaStream_t passed as void* (0 = legacy default stream).
 *     All work is enqueued on it; no entry point synchronizes the device.
 *   - Return value: 0 (TGS_OK) or a TGS_ERR_* code. The message of the last
 *     failure on the calling host thread is returned by tgs_last_error().
 *   - Device-side errors (bad index, unsorted ids, wait that timed out) are
 *     written to a caller-owned int32[4] "error word" on the device:
 *       err[0] = error code (0 = none), err[1] = first offending index (low 32),
 *       err[2] = first offending index (high 32), err[3] = auxiliary value.
 *     A kernel that finds err[0] != 0 at entry does nothing, so a failed
 *     validation never leaves the optimizer state half-updated.
 *
 * Row layout: one Gaussian = 59 fp32 columns split into six components, in the
 * reference's COMPONENT_SPECS order (strategies/tide_engine/
 * gpu_resident_optimizer.py:82-89):
 *   component  0 xyz(3)  1 opacity(1)  2 scaling(3)  3 rotation(4)
 *              4 features_dc(3)  5 features_rest(45)
 * Packed [rows, 59] host/SSD blocks use one of the two reference column orders
 * (storage/block_reader.py:43-44):
 *   TGS_LAYOUT_UNIFIED = xyz|opacity|scaling|rotation|dc|rest
 *   TGS_LAYOUT_CACHE   = xyz|scaling|rotation|opacity|dc|rest
 */
#ifndef TIDEGS_B200_H
#define TIDEGS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TGS_ABI_VERSION 1

#if defined(__GNUC__)
#define TGS_API __attribute__((visibility("default")))
#else
#define TGS_API
#endif

#define TGS_NUM_COMPONENTS 6
#define TGS_ROW_WIDTH 59
/* Resident-Adam state row: 64 (m, v) fp32 pairs = 512 bytes. Pairs 0..58 hold
 * the 59 columns in UNIFIED order, float 124 (pair 62's first word) holds the
 * admission stamp of the row as uint32 bits, the rest is padding. */
#define TGS_STATE_ROW_FLOATS 128

enum {
  TGS_OK = 0,
  TGS_ERR_INVALID_ARG = 1,
  TGS_ERR_CUDA = 2,
  TGS_ERR_UNSUPPORTED = 3
};

/* Device error codes written to err[0]. */
enum {
  TGS_DEV_OK = 0,
  TGS_DEV_ID_OUT_OF_RANGE = 1,   /* a local row id is < 0 or >= param_rows */
  TGS_DEV_ID_NOT_SORTED = 2,     /* local row ids are not strictly ascending */
  TGS_DEV_ID_NOT_RESIDENT = 3,   /* a local row id lies in no resident block */
  TGS_DEV_WAIT_TIMEOUT = 4,      /* a bounded mbarrier wait gave up */
  TGS_DEV_BAD_SLICE = 5,         /* a copy segment/plan is inconsistent */
  TGS_DEV_ID_NOT_TOUCHED = 6     /* a filter id is missing from the touched rows */
};

enum { TGS_LAYOUT_CACHE = 0, TGS_LAYOUT_UNIFIED = 1 };

/* ------------------------------------------------------------------------ */
/* Library information                                                       */
/* ------------------------------------------------------------------------ */

/* ABI version (TGS_ABI_VERSION of the build). */
TGS_API int tgs_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to len). Returns the full message length. */
TGS_API int tgs_last_error(char* buf, size_t len);

/* ------------------------------------------------------------------------ */
/* GPU-resident Adam                                                         */
/* Replaces: strategies/tide_engine/gpu_resident_optimizer.py                */
/*   _working_set_state_rows   :266-300  (row -> block position -> state row) */
/*   _update_touched_slot_metadata :302-337 (per-slot step, bias tables)     */
/*   _fused_resident_adam_kernel   :16-70, called 6x by step :420-509        */
/* ------------------------------------------------------------------------ */

typedef struct {
  /* Working-set layout: P resident block positions sorted by slice start.
   * Position p covers local rows [pos_start[p], pos_end[p]) and owns optimizer
   * slot pos_slot[p]; its state rows are pos_slot[p]*block_size + row-start. */
  const int64_t* pos_start;   /* [P] */
  const int64_t* pos_end;     /* [P] */
  const int32_t* pos_slot;    /* [P] */
  int32_t n_positions;        /* P */
  int64_t block_size;
  int64_t param_rows;         /* M: rows of every parameter component */

  /* Touched rows: the compacted gradient's row i belongs to local row
   * local_ids[i]; ids must be strictly ascending (torch.nonzero order). */
  const int64_t* local_ids;   /* [n] */
  int64_t n_rows;             /* n */

  /* Per-slot device tables (slots = n_slots). */
  int32_t* slot_step;         /* [slots] steps taken since admission */
  const uint32_t* slot_stamp; /* [slots] admission stamp of the slot (>=1) */
  float* slot_bias;           /* [slots][2] (1-b1^t, sqrt(1-b2^t)) of this step */
  const float* step_table;    /* [table_len][2] (1-b1^t, sqrt(1-b2^t)) for t */
  int32_t step_table_len;     /* t >= len uses entry len-1 (saturated) */
  int32_t n_slots;

  int32_t* pos_count;         /* [P] out: touched rows per position */
  int32_t* err;               /* [4] device error word (zeroed by the call) */

  /* Optional [ceil(n/32)][2] out, or NULL: per 32-row chunk of local_ids,
   * (first local row, first state row) when the chunk's rows and state rows
   * both run consecutively and its first row is a multiple of 4 (the update
   * then streams it by bulk copies), else (-1, -1). */
  int64_t* chunk_table;
} TgsResidentCountArgs;

/* Validates local_ids (range, strict order, residency), counts touched rows
 * per position (from each position's first and last row), and for every
 * touched position increments its slot's step counter and fills slot_bias
 * from step_table. Enqueues: memsets of pos_count and err, 2 kernels.
 * Replaces gpu_resident_optimizer.py:266-337. */
TGS_API int tgs_resident_adam_count(const TgsResidentCountArgs* args, void* stream);

typedef struct {
  float* param[TGS_NUM_COMPONENTS];       /* [M, W_c] contiguous */
  const float* grad[TGS_NUM_COMPONENTS];  /* [n, W_c] contiguous */
  float lr[TGS_NUM_COMPONENTS];           /* learning rate per component */
  float beta1, beta2, eps;
  /* 1 - beta evaluated in double precision by the caller, then rounded to
   * fp32 (as the reference's torch step does with its Python-float betas). */
  float one_minus_beta1, one_minus_beta2;
  float batch_size;                       /* grad is divided by it */

  const int64_t* pos_start;               /* as in TgsResidentCountArgs */
  const int64_t* pos_end;
  const int32_t* pos_slot;
  int32_t n_positions;
  int64_t block_size;
  const int64_t* local_ids;
  int64_t n_rows;

  float* state;                           /* [slots*block_size, 128] 16B-aligned */
  const uint32_t* slot_stamp;             /* [slots] */
  const float* slot_bias;                 /* [slots][2] from tgs_resident_adam_count */
  const int32_t* err;                     /* [4] skip everything when err[0]!=0 */

  /* The chunk table tgs_resident_adam_count wrote for these local_ids, or
   * NULL. With it, streamable chunks are updated by a bulk-copy pipeline
   * (one CTA per SM) and marked done in the table (which the call rewrites),
   * then the other chunks by the per-row kernel; without it, one per-row
   * launch. Both give the same result bit for bit. */
  int64_t* chunk_table;
} TgsResidentAdamArgs;

/* One fused launch updating all 59 columns of every touched row, in the op
 * order of the reference's torch step (gpu_resident_optimizer.py:355-364):
 *   g = grad / batch_size
 *   m = b1*m + (1-b1)*g ;  v = b2*v + ((1-b2)*g)*g
 *   p = p - (m / (sqrt(v) / denom_scale[slot] + eps)) * ((1 / bias1[slot]) * lr_c)
 * with every operation rounded separately (no FMA contraction). A state row
 * whose stamp differs from its slot's stamp is read as m = v = 0 (cold
 * restart after re-admission, gpu_resident_optimizer.py:249-261).
 * Replaces the six _fused_resident_adam_kernel launches of step :474-499. */
TGS_API int tgs_resident_adam_apply(const TgsResidentAdamArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* SelectiveAdam / SelectiveSophia (dense [N, W] groups + per-row mask)      */
/* Replaces: optimizer.py:46-87 SelectiveAdam.step and                       */
/*   submodules/clm_kernels/adam.cu:12-77 selective_adam_update (one launch  */
/*   per group there, one launch for all groups here).                       */
/* ------------------------------------------------------------------------ */

#define TGS_MAX_GROUPS 16

typedef struct {
  float* param;        /* [N * width] contiguous */
  const float* grad;   /* [N * width] */
  float* exp_avg;      /* [N * width] (Sophia: m) */
  float* exp_avg_sq;   /* [N * width] (Sophia: h, the Hessian-diagonal EMA) */
  const float* noise;  /* Sophia only: [N * width] u ~ N(0,1) for the estimator */
  int64_t width;       /* elements per row, = numel / N */
  float lr, beta1, beta2, eps;
  float rho;           /* Sophia clip scale */
  float weight_decay;  /* Sophia decoupled weight decay (0 = off) */
} TgsDenseGroup;

typedef struct {
  TgsDenseGroup groups[TGS_MAX_GROUPS];
  int32_t n_groups;
  const uint8_t* visibility;  /* [N] bool: row r is updated iff visibility[r] */
  int64_t n_rows;             /* N */
  int32_t hessian_step;       /* Sophia: 1 = update h from the estimator */
} TgsDenseArgs;

/* Reference arithmetic (adam.cu:33-37), no bias correction, no FMA:
 *   m = b1*m + (1-b1)*g ; v = b2*v + ((1-b2)*g)*g ; p = p + ((-lr)*m)/(sqrt(v)+eps) */
TGS_API int tgs_selective_adam(const TgsDenseArgs* args, void* stream);

/* Sophia (Liu et al. 2023, Algorithm 3) on visible rows; no reference
 * counterpart exists in TideGS:
 *   m = b1*m + (1-b1)*g
 *   if hessian_step: q = u*g ; h = b2*h + (1-b2)*(q*q)
 *   if wd != 0: p = p - (lr*wd)*p
 *   p = p - lr * clamp(m / max(rho*h, eps), -1, 1)                         */
TGS_API int tgs_sophia_step(const TgsDenseArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Materialization                                                           */
/* ------------------------------------------------------------------------ */

typedef struct {
  const float* packed;                 /* [n_rows, 59] device, TGS_LAYOUT_* */
  int64_t n_rows;
  int32_t layout;
  float* comp[TGS_NUM_COMPONENTS];     /* [*, W_c] SoA targets */
  int64_t target_offset;               /* first target row */
  /* Optional global-id fill (global_ids == NULL to skip): row r of the batch
   * gets block_ids[r / block_size] * block_size + r % block_size. */
  int64_t* global_ids;                 /* [*] written at target_offset + r */
  const int64_t* block_ids;            /* [ceil(n_rows / block_size)] */
  int64_t block_size;
  int32_t* err;                        /* [4] device error word (may be NULL) */
  /* Optional scatter by block (NULL: the batch lands contiguously at
   * target_offset): [ceil(n_rows / block_size)] first target row of each
   * block of the batch, e.g. a free slot of a slot arena, so that incoming
   * blocks need no later slot-remap copy. Needs block_size a multiple of 64;
   * target_offset is then ignored. */
  const int64_t* block_dst;
} TgsUnpackArgs;

/* Packed [rows,59] -> six SoA components (+ global ids), TMA bulk tile loads.
 * Replaces double_buffer_gpu.py:150-209 _unpack_streamed_rows_kernel and
 * :130-148 _fill_cold_global_ids_kernel (fused). */
TGS_API int tgs_unpack_rows(const TgsUnpackArgs* args, void* stream);

typedef struct {
  const float* src_comp[TGS_NUM_COMPONENTS]; /* source SoA components */
  const int64_t* src_global_ids;             /* may be NULL (then not copied) */
  float* dst_comp[TGS_NUM_COMPONENTS];
  int64_t* dst_global_ids;                   /* may be NULL */
  const int64_t* src_start;   /* [n_blocks] first source row of block k */
  const int64_t* dst_start;   /* [n_blocks] first target row of block k */
  const int64_t* row_count;   /* [n_blocks] rows of block k */
  int32_t n_blocks;
  int64_t max_rows;           /* max(row_count) (grid sizing) */
  int32_t* err;               /* [4] device error word (may be NULL) */
} TgsCopyBlocksArgs;

/* Block-granular slot remap: for each block, copies its rows of all six
 * components and its global ids from source slice to target slice with TMA
 * bulk copies (cp.async.bulk global->shared->global, no multicast) where the
 * segment is 16-byte aligned, vector copies elsewhere.
 * Replaces double_buffer_gpu.py:40-128 _copy_resident_rows_kernel /
 * :811-872 _copy_resident_blocks. */
TGS_API int tgs_copy_blocks(const TgsCopyBlocksArgs* args, void* stream);

/* dst[offset + r] = block_ids[r / block_size] * block_size + r % block_size
 * for r < n_rows. Replaces double_buffer_gpu.py:130-148 / :924-961. */
TGS_API int tgs_fill_global_ids(int64_t* dst, int64_t offset, const int64_t* block_ids,
                        int64_t n_rows, int64_t block_size, void* stream);

/* block_starts[k] = -1 for all k < num_blocks, then block_starts[ids[i]] =
 * starts[i] for ids in range. Replaces double_buffer_gpu.py:212-234. */
TGS_API int tgs_build_block_starts(int64_t* block_starts, int64_t num_blocks,
                           const int64_t* ids, const int64_t* starts,
                           int64_t n, void* stream);

/* out[i] = block_starts[b] + (g - b*block_size) with b = floor(g/block_size)
 * when 0 <= b < num_blocks and block_starts[b] >= 0, else -1.
 * Replaces double_buffer_gpu.py:237-256 _global_ids_to_local and
 * gpu_working_set.py:312-333 global_to_local. */
TGS_API int tgs_global_to_local(int64_t* out, const int64_t* global_ids, int64_t n,
                        const int64_t* block_starts, int64_t num_blocks,
                        int64_t block_size, void* stream);

/* Order-preserving compaction of global_to_local: writes only the ids that
 * map to a resident row (>= 0), in input order, to out; *dev_count receives
 * their number. scratch must hold tgs_compact_scratch_words(n) int64 words.
 * Replaces `filter_local[filter_local >= 0]` at double_buffer_gpu.py:1145-1157. */
TGS_API int64_t tgs_compact_scratch_words(int64_t n);
TGS_API int tgs_global_to_local_compact(int64_t* out, int64_t* dev_count,
                                const int64_t* global_ids, int64_t n,
                                const int64_t* block_starts, int64_t num_blocks,
                                int64_t block_size, int64_t* scratch,
                                void* stream);

/* Same result as tgs_global_to_local_compact, but the call allocates nothing
 * and takes no scratch argument. It has no counterpart in the reference.
 * It serves callers that cannot provide scratch device memory when they call:
 * an engine that lays out all of its device memory once at start-up has no
 * allocator to call, and cudaMalloc/cudaFree on the fly would synchronize the
 * device in the middle of an overlapped pipeline. The scratch lives in a
 * fixed array inside the library (128 KiB per device, held until the process
 * exits), which bounds n to 33,554,432 ids; larger n is rejected with
 * TGS_ERR_INVALID_ARG and a message. The first call on a device looks up the
 * array's device address (with that device current); make that first call
 * before any stream capture. The address is kept per device index for the
 * rest of the process: it does not survive cudaDeviceReset (or a new primary
 * context on that device), after which this entry point must not be called.
 * All calls on a device share the array, so calls that overlap on the GPU
 * race: serialize them. */
TGS_API int tgs_global_to_local_compact_noalloc(int64_t* out, int64_t* dev_count,
                                                const int64_t* global_ids, int64_t n,
                                                const int64_t* block_starts, int64_t num_blocks,
                                                int64_t block_size, void* stream);

/* Copies `bytes` from src to dst with a kernel on `stream` (src/dst: device
 * memory or page-locked host memory, which the device reads directly). Used
 * for the small per-step tables (row ids, plans, layouts): as kernels they are
 * ordered on the compute stream and never wait behind multi-GB block DMA
 * queued on the copy engines by the prefetch stream. Addresses must be
 * 4-byte aligned (16-byte aligned pairs take 16-byte accesses). No reference
 * counterpart (the reference uploads such tables with torch.tensor(...,
 * device=...) copies). */
TGS_API int tgs_copy_small(void* dst, const void* src, int64_t bytes, void* stream);

/* Issues one cudaMemcpyAsync per block (host -> device) so pinned host blocks
 * reach the device staging buffer without a CPU-side pack. host_src[k] is a
 * host pointer, dev_dst[k] a device pointer, bytes[k] the size (all host
 * arrays). Replaces the torch.cat pack of storage/block_reader.py:55-87 +
 * the single H2D at double_buffer_gpu.py:1053 when blocks are pinned. */
TGS_API int tgs_h2d_blocks(void* const* dev_dst, const void* const* host_src,
                   const int64_t* bytes, int32_t n, void* stream);

/* Issues one cudaMemcpyAsync per block (device -> host): the write-back
 * payload lands in page-locked host-cache entries, host_dst[k] <- dev_src[k].
 * Replaces the pinned staging copy of gpu_working_set.py:960-967 followed by
 * the CPU copy into the cache's slab in
 * storage/tiered_cache_manager.py:524-599 (upsert_dirty_block_batch). */
TGS_API int tgs_d2h_blocks(void* const* host_dst, const void* const* dev_src,
                   const int64_t* bytes, int32_t n, void* stream);

/* ------------------------------------------------------------------------ */
/* Dirty tracking and write-back                                             */
/* ------------------------------------------------------------------------ */

/* Bit-packed dirty bitmap of num_blocks blocks: bit (id & 31) of word id >> 5.
 * value != 0 sets the bits of ids, value == 0 clears them; ids outside
 * [0, num_blocks) are ignored (the reference range-filters them).
 * Replaces double_buffer_gpu.py:494-508 / :530-543 (bool bitmap index_fill_). */
TGS_API int tgs_dirty_mark(uint32_t* bitmap, int64_t num_blocks, const int64_t* ids, int64_t n,
                   int32_t value, void* stream);

/* Order-preserving warp-ballot compaction: out_ids = [ids[i] for i if bit set],
 * *dev_count = its length; ids outside [0, num_blocks) count as clean.
 * Single CTA; n up to ~1M.
 * Replaces double_buffer_gpu.py:510-523 dirty_blocks_for_eviction. */
TGS_API int tgs_dirty_select(const uint32_t* bitmap, int64_t num_blocks, const int64_t* ids,
                     int64_t n, int64_t* out_ids, int64_t* dev_count, void* stream);

/* All set bits of the first num_blocks bits, ascending.
 * Replaces double_buffer_gpu.py:525-528 dirty_blocks (nonzero). */
TGS_API int tgs_dirty_list(const uint32_t* bitmap, int64_t num_blocks, int64_t* out_ids,
                   int64_t* dev_count, void* stream);

typedef struct {
  const float* comp[TGS_NUM_COMPONENTS]; /* source SoA components */
  const int64_t* src_start;   /* [n_plans] first source row of plan k */
  const int64_t* row_count;   /* [n_plans] */
  const int64_t* out_start;   /* [n_plans] first output row (exclusive cumsum) */
  int32_t n_plans;
  int64_t max_rows;           /* max(row_count) */
  float* out;                 /* [sum rows, 59] CACHE layout */
  int32_t layout;             /* output column order, normally TGS_LAYOUT_CACHE */
  int32_t* err;               /* [4] device error word (may be NULL) */
} TgsPackArgs;

/* SoA -> packed CACHE rows for write-back: each 64-row tile's component ranges
 * are streamed into shared memory with TMA bulk copies (plain loads where a
 * range is not 16-byte aligned), then stored as packed rows.
 * Replaces gpu_working_set.py:35-86 _pack_resident_rows_kernel (:948-967). */
TGS_API int tgs_pack_rows(const TgsPackArgs* args, void* stream);

/* bounds[k] = (min x, min y, min z, max x, max y, max z) over xyz rows
 * [start[k], start[k]+count[k]). Replaces gpu_working_set.py:88-115
 * _resident_block_bounds_kernel (:990-1061). */
TGS_API int tgs_block_bounds(const float* xyz, const int64_t* start, const int64_t* count,
                     int32_t n_plans, float* bounds, void* stream);

/* ------------------------------------------------------------------------ */
/* Touched-only gradient accumulation of a camera batch                      */
/* Replaces: strategies/tide_engine/engine.py                                */
/*   :1801-1826  touched mask (zeros + scatter_ True) -> nonzero ids,        */
/*               local_to_global gather, zero-filled compact components      */
/*   :2434-2471  per camera: searchsorted + six scatter_add_                 */
/* ------------------------------------------------------------------------ */

/* Sets bit ids[i] of a bitmap of num_bits bits for every i; ids outside
 * [0, num_bits) are skipped and reported in err (TGS_DEV_ID_OUT_OF_RANGE).
 * The touched-row mask of engine.py:1803-1806 (scatter_ True per filter). */
TGS_API int tgs_bitmap_set(uint32_t* bitmap, int64_t num_bits, const int64_t* ids, int64_t n,
                   int32_t* err, void* stream);

/* Scratch words tgs_bitmap_list needs for num_bits bits. */
TGS_API int64_t tgs_bitmap_list_scratch_words(int64_t num_bits);

/* Ascending positions of the set bits among the first num_bits bits of
 * bitmap (bit i = word i/32, bit i%32), *dev_count = how many. Multi-CTA,
 * order preserving (tile counts, one-CTA scan, ranked writes). With
 * tgs_bitmap_set setting the bits of every camera's filter, this is the
 * touched-row list (torch.nonzero of the mask, engine.py:1803-1807).
 * pos_map (optional, [num_bits] int32, filled with -1 by the caller; fewer
 * than 2^31 set bits): pos_map[b] = rank of set bit b, so that a later
 * lookup of a row's position is one load instead of a binary search. */
TGS_API int tgs_bitmap_list(const uint32_t* bitmap, int64_t num_bits, int64_t* out_ids,
                    int64_t* dev_count, int64_t* scratch, int32_t* pos_map, void* stream);

/* out[i] = src[idx[i]] (int64), e.g. local_to_global[touched ids]
 * (engine.py:1815). Indices outside [0, n_src) are reported in err. */
TGS_API int tgs_gather_i64(int64_t* out, const int64_t* src, int64_t n_src, const int64_t* idx,
                   int64_t n, int32_t* err, void* stream);

typedef struct {
  const int64_t* touched;   /* [n_touched] ascending touched local ids */
  int64_t n_touched;
  /* optional: the pos_map of tgs_bitmap_list for these touched rows; a row's
   * position is then pos_map[id] (-1: not touched) instead of a binary
   * search of touched */
  const int32_t* pos_map;
  int64_t pos_map_len;
  const int64_t* filter;    /* [n_filter] this camera's local ids */
  int64_t n_filter;
  /* The camera's gradients per component (xyz, opacity, scaling, rotation,
   * features_dc, features_rest), row r of component c at
   * src[c] + r * src_stride[c] (floats); a NULL component is skipped (the
   * reference skips the SH components when they have no gradient). The SH
   * gradient [n, 48] passes as dc = shs (stride 48), rest = shs + 3. */
  const float* src[TGS_NUM_COMPONENTS];
  int64_t src_stride[TGS_NUM_COMPONENTS];
  float* acc[TGS_NUM_COMPONENTS];  /* [n_touched, W_c] compact gradients */
  /* 1: no id repeats inside filter (true of projection filters): each sum
   * is one exactly rounded addition. 0: atomic additions (order of repeated
   * ids unspecified, as in torch's scatter_add_ on a GPU). */
  int32_t unique_filter;
  int32_t* err;             /* [4] TGS_DEV_ID_NOT_TOUCHED for a missing id */
} TgsSparseAccumArgs;

/* acc[c][searchsorted(touched, filter[r])] += src row r of component c, all
 * six components in one launch. */
TGS_API int tgs_sparse_grad_accumulate(const TgsSparseAccumArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Multi-GPU gradient exchange (no counterpart in the reference, which is    */
/* single-GPU). Blocks are owned by rank block_id mod world; each rank packs */
/* the gradient tiles of the blocks it rendered by owner (tgs_pack_rows,     */
/* UNIFIED order), one all-to-all moves them to their owners, and the owner  */
/* sums the tiles of each block here.                                        */
/* ------------------------------------------------------------------------ */

typedef struct {
  const float* recv;              /* [n_recv_blocks * block_size, 59] tiles, UNIFIED order */
  int64_t n_recv_blocks;
  const int64_t* contrib_offsets; /* [n_out + 1] CSR offsets into contrib_blocks */
  const int64_t* contrib_blocks;  /* recv tile index of each contribution, sender order */
  int32_t n_out;                  /* output blocks (the owner's visible blocks, row order) */
  int64_t block_size;
  float* out[TGS_NUM_COMPONENTS]; /* [n_out * block_size, W_c] compact gradients */
  int32_t* err;                   /* [4] device error word (may be NULL) */
} TgsBlockSumArgs;

/* out block k = sum of its contributions, added in listed (sender) order with
 * one rounding per addition, written as the six SoA gradient components. */
TGS_API int tgs_block_grad_sum(const TgsBlockSumArgs* args, void* stream);

/* Direct push over peer memory: the pack and the all-to-all above in one
 * kernel. Each rank writes its UNIFIED tiles straight into the owners'
 * receive buffers (NVLink stores through CUDA IPC mappings), at the rows an
 * all-to-all would have put them, so tgs_block_grad_sum runs unchanged on the
 * owner. The caller orders the push before the owners' sums with a barrier
 * across ranks (a collective on the same stream) and double-buffers the
 * receive buffers, so that a push never overwrites tiles an owner still sums. */

#define TGS_MAX_PEERS 64
#define TGS_PEER_HANDLE_BYTES 64

typedef struct {
  unsigned char bytes[TGS_PEER_HANDLE_BYTES]; /* a cudaIpcMemHandle_t */
} TgsPeerHandle;

/* Device buffer of `bytes` (cudaMalloc, so that it can be exported) and its
 * IPC handle. Free with tgs_peer_buffer_free after every peer closed it. */
TGS_API int tgs_peer_buffer_alloc(int64_t bytes, void** dev_ptr, TgsPeerHandle* handle);
TGS_API int tgs_peer_buffer_free(void* dev_ptr);
/* Maps another process's buffer into the current device's address space
 * (peer access enabled on first use). Unmap with tgs_peer_buffer_close. */
TGS_API int tgs_peer_buffer_open(const TgsPeerHandle* handle, void** dev_ptr);
TGS_API int tgs_peer_buffer_close(void* dev_ptr);

typedef struct {
  const float* comp[TGS_NUM_COMPONENTS]; /* this rank's gradients, SoA components */
  const int64_t* src_start;       /* [n_tiles] first source row of each sent block */
  const int64_t* row_count;       /* [n_tiles] rows of each sent block */
  const int32_t* dst_rank;        /* [n_tiles] owner rank of each sent block */
  const int64_t* dst_row;         /* [n_tiles] first row in the owner's receive buffer */
  int32_t n_tiles;
  int64_t max_rows;               /* max(row_count) */
  float* recv[TGS_MAX_PEERS];     /* each rank's receive buffer as mapped here (own included) */
  int64_t recv_rows[TGS_MAX_PEERS]; /* capacity of each receive buffer, rows */
  int32_t n_ranks;
  int32_t* err;                   /* [4] device error word (may be NULL) */
} TgsGradPushArgs;

/* recv[dst_rank[k]][dst_row[k] + i] = UNIFIED row src_start[k] + i of comp,
 * i < row_count[k]. A tile that would land outside its receive buffer is
 * skipped and reported in err (TGS_DEV_BAD_SLICE). */
TGS_API int tgs_grad_push(const TgsGradPushArgs* args, void* stream);

/* Lets kernels on the current device read and write peer_device's memory
 * directly (one process driving several GPUs; processes use IPC mappings).
 * Already enabled counts as success. */
TGS_API int tgs_peer_access_enable(int32_t peer_device);

/* IPC handle of the allocation that contains dev_ptr (any device pointer,
 * for example a tensor inside a caching allocator's segment) and dev_ptr's
 * byte offset from that allocation's base. A peer maps the allocation with
 * tgs_peer_buffer_open and adds the offset. */
TGS_API int tgs_peer_export(const void* dev_ptr, TgsPeerHandle* handle, int64_t* offset);

/* Owner-side reduction fused into the resident Adam step ("pull"): the
 * gradient of compact row i is read from the senders' own gradient buffers
 * (this rank's and peers' through IPC mappings, over NVLink: non-multicast
 * bulk copies into shared memory for streamable 32-row chunks inside one
 * segment when adam.chunk_table is given, plain loads elsewhere) and summed
 * in listed (rank) order, one rounding per addition, then the update of
 * tgs_resident_adam_apply runs on it. Equal, bit for bit, to
 * tgs_grad_push / all-to-all + tgs_block_grad_sum + tgs_resident_adam_apply,
 * without the receive buffers, the push and the sum pass.
 * Compact rows are split into segments (normally one per visible block);
 * row i of segment s (seg_begin[s] <= i < seg_begin[s+1]) receives, for each
 * contribution j of s, row contrib_row[j] + (i - seg_begin[s]) of rank
 * contrib_rank[j]'s gradient components. The caller orders the senders'
 * gradient writes before this kernel and this kernel before the senders'
 * next writes (barriers across ranks on the stream). */
typedef struct {
  TgsResidentAdamArgs adam;         /* grad[] is not read (may be NULL) */
  const float* const* grad_src;     /* [n_ranks * 6] rank r's component c at r*6+c, as mapped here */
  const int64_t* grad_rows;         /* [n_ranks] rows of each rank's gradient components */
  int32_t n_ranks;
  const int64_t* seg_begin;         /* [n_segments + 1] ascending, 0 .. adam.n_rows */
  int32_t n_segments;
  const int64_t* contrib_offsets;   /* [n_segments + 1] CSR into contrib_rank / contrib_row */
  const int32_t* contrib_rank;      /* [n_contrib] summation order inside a segment */
  const int64_t* contrib_row;       /* [n_contrib] source row of the segment's first row */
  /* The kernel walks the compact rows starting at this one (wrapping around).
   * Owners that start at different senders' rows read from every sender at
   * once instead of all reading the same sender first; 0 = natural order. */
  int64_t rotate_rows;
  int32_t* err;                     /* [4] the error word of adam.err, writable */
  /* Most CTAs the streamed kernel may use (it runs at most one per SM);
   * 0 = one per SM. A smaller grid leaves SMs to kernels that run at the same
   * time on another stream, which pays when NVLink, not HBM, bounds the
   * update (many ranks, many remote contributions). */
  int32_t max_ctas;
} TgsResidentAdamSumArgs;

TGS_API int tgs_resident_adam_apply_sum(const TgsResidentAdamSumArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Block frustum culling                                                     */
/* Replaces: storage/gaussian_block.py                                       */
/*   :264-312  FrustumCuller bounding spheres (center, radius * 1.15)        */
/*   :318-340  update_block_bounds                                           */
/*   :359-406  cull_subset, :408-465 cull (6-plane test); the planes        */
/*             (:145-228) are extracted on the host                          */
/* ------------------------------------------------------------------------ */

/* centers[b] = (min+max)/2 and radii[b] = |max-min|/2 * 1.15f from
 * bounds[b] = (min x, min y, min z, max x, max y, max z), in float32 with
 * every operation rounded once, sums left to right (the reference's numpy
 * evaluation). */
TGS_API int tgs_block_spheres(const float* bounds, int64_t n_blocks, float* centers,
                      float* radii, void* stream);

typedef struct {
  const float* centers;   /* [n_blocks, 3] device */
  const float* radii;     /* [n_blocks] device */
  int64_t n_blocks;
  const int64_t* subset;  /* [n_items] candidate block ids (device), or NULL = all blocks */
  int64_t n_items;
  const float* planes;    /* [n_cameras, 6, 4] normalized planes (device) */
  int32_t n_cameras;      /* 0 .. 65535 */
  int64_t* out_ids;       /* [n_cameras, out_stride] visible ids, in candidate order */
  int64_t out_stride;     /* >= n_items */
  int64_t* out_counts;    /* [n_cameras] visible blocks per camera */
  int64_t* slice_counts;  /* [n_cameras * tgs_frustum_cull_slices(n_items)] device scratch */
  int32_t* err;           /* [4] TGS_DEV_ID_OUT_OF_RANGE for a subset id (skipped) */
} TgsCullArgs;

/* Slices of 4096 candidates each camera's candidates are split into (the
 * scratch size per camera of tgs_frustum_cull). */
TGS_API int64_t tgs_frustum_cull_slices(int64_t n_items);

/* For every camera, the candidates whose sphere has signed distance >= -radius
 * to all six planes (gaussian_block.py:429-465): a counting pass and an
 * ordered writing pass, each a grid of (slice, camera) CTAs. */
TGS_API int tgs_frustum_cull(const TgsCullArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Render path before the optimizer (the engine's gsplat 1.0.0 calls,        */
/* strategies/tide_engine/engine.py:481-561)                                 */
/* Replaces: submodules/gsplat/gsplat/cuda/csrc                              */
/*   fully_fused_projection_fwd.cu:19-121, fully_fused_projection_bwd.cu     */
/*   isect_tiles.cu:15-280, rasterize_to_pixels_fwd.cu:15-158,               */
/*   rasterize_to_pixels_bwd.cu:15-250                                       */
/* Layouts are gsplat's non-packed ones: per camera c and Gaussian n the      */
/* flat index c * N + n.                                                      */
/* ------------------------------------------------------------------------ */

typedef struct {
  const float* means;     /* [N, 3] world positions */
  const float* quats;     /* [N, 4] (w, x, y, z), normalized in the kernel */
  const float* scales;    /* [N, 3] */
  const float* viewmats;  /* [C, 4, 4] row-major world-to-camera */
  const float* Ks;        /* [C, 3, 3] row-major intrinsics */
  int32_t n_cameras;
  int64_t n_gaussians;
  int32_t image_width;
  int32_t image_height;
  float eps2d;            /* added to the 2D covariance diagonal */
  float near_plane;
  float far_plane;
  float radius_clip;      /* radii <= this are culled */
  int32_t* radii;         /* [C, N] 0 = culled */
  float* means2d;         /* [C, N, 2] */
  float* depths;          /* [C, N] */
  float* conics;          /* [C, N, 3] inverse 2D covariance (xx, xy, yy) */
  float* compensations;   /* [C, N] sqrt(det / det_blurred), or NULL */
} TgsProjectArgs;

/* Projection of every Gaussian into every camera
 * (fully_fused_projection_fwd.cu:19-121); culled entries get radius 0 and
 * zero outputs. */
TGS_API int tgs_project_fwd(const TgsProjectArgs* args, void* stream);

typedef struct {
  TgsProjectArgs fwd;              /* forward inputs; radii, conics, compensations read */
  const float* v_means2d;          /* [C, N, 2] */
  const float* v_depths;           /* [C, N] */
  const float* v_conics;           /* [C, N, 3] */
  const float* v_compensations;    /* [C, N] or NULL */
  float* v_means;                  /* [N, 3] accumulated (caller zeroes) */
  float* v_quats;                  /* [N, 4] accumulated */
  float* v_scales;                 /* [N, 3] accumulated */
} TgsProjectBwdArgs;

/* Gradients of the projection with respect to means, quats and scales
 * (fully_fused_projection_bwd.cu:19-190; camera gradients not computed). */
TGS_API int tgs_project_bwd(const TgsProjectBwdArgs* args, void* stream);

/* Tiles each projected Gaussian overlaps (isect_tiles.cu first pass). */
TGS_API int tgs_isect_count(const float* means2d, const int32_t* radii, int64_t n,
                    int32_t tile_size, int32_t tile_width, int32_t tile_height,
                    int32_t* tiles_per_gauss, void* stream);
/* floor(log2(n_tiles)) + 1: bits of the tile id in an intersection key. */
TGS_API int32_t tgs_isect_tile_bits(int32_t n_tiles);
/* Keys camera << (32 + tile_bits) | tile << 32 | depth bits and flat
 * Gaussian ids, written at the inclusive prefix sums cum_tiles of the
 * counts (isect_tiles.cu second pass; the caller sorts them, stably). */
TGS_API int tgs_isect_write(const float* means2d, const int32_t* radii, const float* depths,
                    int64_t n, int64_t n_per_camera, int32_t tile_size, int32_t tile_width,
                    int32_t tile_height, const int64_t* cum_tiles, int64_t* isect_ids,
                    int32_t* flatten_ids, void* stream);
/* The sorted keys of isect_tiles.cu:170-224 (cub sort of the keys' low
 * 32 + tile_bits + camera_bits bits, stable) without a 64-bit key sort:
 *   tgs_isect_depth_order   order[] = the n = C*N Gaussians stably sorted
 *                           by their depth bits (unsigned), and cum_tiles[]
 *                           = inclusive prefix sums of
 *                           tiles_per_gauss[order[]] (int64);
 *   tgs_isect_write_ordered each Gaussian's tiles in that order as keys
 *                           camera << tile_bits | tile (all ones for a
 *                           negative depth, as the sign-extended reference
 *                           key has) and flat Gaussian ids;
 *   tgs_isect_sort_tiles    stable sort of those keys (tile_bits +
 *                           camera_bits bits);
 *   tgs_isect_expand_ids    the reference's 64-bit keys from the sorted
 *                           keys and the depths.
 * Keys are tgs_isect_key_bytes(...) wide: 2 (uint16) when tile_bits +
 * camera_bits <= 16, else 4 (uint32); 0 means the ids need more than 32
 * bits. Keys, flatten ids and their order equal the reference's. Scratch
 * is the caller's device memory of the size the *_scratch_bytes calls
 * return; expand wants its arrays on 16-byte boundaries. */
TGS_API int32_t tgs_isect_key_bytes(int32_t n_cameras, int32_t tile_width, int32_t tile_height);
TGS_API int tgs_isect_depth_order_scratch_bytes(int64_t n, size_t* bytes);
TGS_API int tgs_isect_depth_order(const float* depths, const int32_t* tiles_per_gauss, int64_t n,
                          int32_t* order, int64_t* cum_tiles, void* scratch,
                          size_t scratch_bytes, void* stream);
TGS_API int tgs_isect_write_ordered(const float* means2d, const int32_t* radii,
                            const float* depths, const int32_t* order, int64_t n,
                            int64_t n_per_camera, int32_t tile_size, int32_t tile_width,
                            int32_t tile_height, const int64_t* cum_tiles, void* tile_keys,
                            int32_t* flatten_ids, void* stream);
TGS_API int tgs_isect_sort_tiles_scratch_bytes(int64_t n_isects, int32_t n_cameras,
                                       int32_t tile_width, int32_t tile_height,
                                       size_t* bytes);
TGS_API int tgs_isect_sort_tiles(const void* tile_keys_in, const int32_t* flatten_in,
                         int64_t n_isects, int32_t n_cameras, int32_t tile_width,
                         int32_t tile_height, void* tile_keys_out, int32_t* flatten_out,
                         void* scratch, size_t scratch_bytes, void* stream);
TGS_API int tgs_isect_expand_ids(const void* tile_keys, int32_t key_bytes,
                         const int32_t* flatten_ids, const float* depths, int64_t n_isects,
                         int64_t* isect_ids, void* stream);
/* offsets[c, tile] = index of the first sorted key of (c, tile)
 * (isect_offset_encode, isect_tiles.cu:227-280). */
TGS_API int tgs_isect_offsets(const int64_t* isect_ids, int64_t n_isects, int32_t n_cameras,
                      int32_t tile_width, int32_t tile_height, int32_t* offsets, void* stream);

typedef struct {
  const float* means2d;       /* [C, N, 2] */
  const float* conics;        /* [C, N, 3] */
  const float* colors;        /* [C, N, channels] */
  const float* opacities;     /* [C, N] */
  const float* backgrounds;   /* [C, channels] or NULL */
  int32_t n_cameras;
  int64_t n_gaussians;        /* N */
  int32_t channels;           /* 1 .. 4 */
  int32_t image_width;
  int32_t image_height;
  int32_t tile_size;          /* tile_size^2 threads per CTA: a multiple of 32, <= 1024 */
  int32_t tile_width;
  int32_t tile_height;
  const int32_t* tile_offsets; /* [C, tile_height, tile_width] */
  const int32_t* flatten_ids;  /* [n_isects] sorted */
  int64_t n_isects;
  float* render_colors;       /* [C, H, W, channels] */
  float* render_alphas;       /* [C, H, W] */
  int32_t* last_ids;          /* [C, H, W] index of the last contributing intersection */
} TgsRasterArgs;

/* Front-to-back alpha compositing per 16x16 tile (rasterize_to_pixels_fwd.cu). */
TGS_API int tgs_rasterize_fwd(const TgsRasterArgs* args, void* stream);

typedef struct {
  TgsRasterArgs fwd;              /* render_alphas, last_ids read */
  const float* v_render_colors;   /* [C, H, W, channels] */
  const float* v_render_alphas;   /* [C, H, W] */
  float* v_means2d_abs;           /* [C, N, 2] or NULL; accumulated */
  float* v_means2d;               /* [C, N, 2] accumulated (caller zeroes) */
  float* v_conics;                /* [C, N, 3] accumulated */
  float* v_colors;                /* [C, N, channels] accumulated */
  float* v_opacities;             /* [C, N] accumulated */
} TgsRasterBwdArgs;

/* Back-to-front gradient of the compositing (rasterize_to_pixels_bwd.cu);
 * per Gaussian and tile, one set of global additions. */
TGS_API int tgs_rasterize_bwd(const TgsRasterBwdArgs* args, void* stream);

/* Spherical-harmonics colors (gsplat compute_sh_fwd.cu / compute_sh_bwd.cu,
 * spherical_harmonics.cuh; the engine's call engine.py:508-520):
 * colors[n] = sum_{k < (degree+1)^2} coeffs[n, k, :] Y_k(dirs[n] / |dirs[n]|),
 * real SH of degree <= 4 in 3D Gaussian splatting's order and signs. */
typedef struct {
  const float* dirs;          /* [n, 3] (need not be unit length) */
  const float* coeffs;        /* [n, K, 3] */
  const uint8_t* masks;       /* [n] bool, or NULL: masked rows give 0 */
  int64_t n;
  int32_t K;                  /* coefficients per row, 1..25 */
  int32_t degree;             /* degrees_to_use, (degree + 1)^2 <= K */
  float* colors;              /* [n, 3] out (forward) */
} TgsShArgs;

TGS_API int tgs_sh_fwd(const TgsShArgs* args, void* stream);

typedef struct {
  TgsShArgs fwd;              /* colors unused */
  const float* v_colors;      /* [n, 3] */
  float* v_coeffs;            /* [n, K, 3] out, every entry written */
  float* v_dirs;              /* [n, 3] out, or NULL (not computed) */
} TgsShBwdArgs;

/* dL/dcoeffs[n, k, c] = v_colors[n, c] Y_k; dL/ddirs through the
 * normalization (compute_sh_bwd.cu; v_dirs only when not NULL). */
TGS_API int tgs_sh_bwd(const TgsShBwdArgs* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TIDEGS_B200_H */
