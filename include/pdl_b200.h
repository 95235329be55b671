/*
 * pdl_b200.h -- C ABI of the B200 (sm_100a) paged decode-attention operator.
 *
 * One query token per sequence attends over a paged KV cache:
 *   q        bf16 [batch, num_heads, head_dim]          (innermost stride 1)
 *   k_cache  bf16 [num_pages, 256, num_kv_heads, head_dim]  contiguous NHD pages
 *   v_cache  bf16 same shape as k_cache
 *   table    int32 [batch, table_width]   logical page j of row b -> physical page
 *   lengths  int32 [batch]                live tokens of row b
 * Logical token t of row b is read from page table[b][t / 256], slot t % 256,
 * KV head h / (num_heads / num_kv_heads).  Table entries past
 * ceil(lengths[b] / 256) are padding (may be -1) and are never read.
 *
 * All launch entry points take raw device pointers and sizes, enqueue work on
 * the given stream, never allocate, never synchronise and never read device
 * memory from the host, so they may be captured in a CUDA graph (warm up
 * once per device/geometry before capture).  The pdl_peer_buffer_* set-up
 * calls are the exception: they allocate, map and synchronise.  Every entry
 * point returns PDL_OK or a PdlStatus; no C++ exception crosses this boundary.
 */
#ifndef PDL_B200_H
#define PDL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *pdl_stream_t; /* same handle as cudaStream_t */

#define PDL_ABI_VERSION 5
#define PDL_PAGE_SIZE 256

typedef enum PdlStatus {
  PDL_OK = 0,
  PDL_ERR_NULL = 1,        /* a required pointer is NULL                      */
  PDL_ERR_GEOMETRY = 2,    /* head_dim / page size / head grouping unsupported */
  PDL_ERR_SHAPE = 3,       /* batch, table width, pages or strides invalid     */
  PDL_ERR_WORKSPACE = 4,   /* split workspace missing or too small             */
  PDL_ERR_SCALE = 5,       /* scale not finite (or not positive where needed)  */
  PDL_ERR_ALIGNMENT = 6,   /* pointer or stride not aligned for vector access  */
  PDL_ERR_SPLITS = 7,      /* split count / size inconsistent with capacity    */
  PDL_ERR_CUDA = 8,        /* a CUDA runtime or driver call failed             */
  PDL_ERR_DEVICE = 9,      /* no usable sm_100 device                          */
  PDL_ERR_KERNEL = 10,     /* requested kernel variant cannot run this shape   */
  PDL_ERR_TIMEOUT = 11     /* a bounded device-side wait gave up (see fault)   */
} PdlStatus;

/* Which partial protocol the split workspace uses. */
typedef enum PdlProtocol {
  /* Normalised partial [B,Hq,S,D] + LSE [B,Hq,S] (natural log, scaled
   * scores); empty partitions store partial 0 and LSE -inf. */
  PDL_PROTOCOL_LSE = 0,
  /* Unnormalised maxima / denominators [B,Hq,S] and accumulators [B,Hq,S,D];
   * maxima are in scaled-score units, empty partitions store -inf / 0 / 0. */
  PDL_PROTOCOL_MLA = 1
} PdlProtocol;

/* Which partition kernel runs. AUTO picks the CUDA-core kernel when a KV head
 * serves 1 or 2 query heads and the tensor-core kernel from 3 (measured:
 * the CUDA-core kernel turns issue-bound at 4 heads per KV head). */
typedef enum PdlKernel {
  PDL_KERNEL_AUTO = 0,
  PDL_KERNEL_SIMT = 1, /* FP32 CUDA-core kernel, warp-shuffle reductions      */
  PDL_KERNEL_MMA = 2   /* BF16 tensor-core kernel (mma.sync), FP32 softmax    */
} PdlKernel;

/* Optional behaviour bits for PdlDecodeArgs.flags (0 = reference behaviour);
 * other bits are rejected with PDL_ERR_SHAPE. */
typedef enum PdlFlags {
  /* Do not store empty partitions; the merge then reads only the
   * ceil(len / tokens_per_split) live partitions of each row. */
  PDL_FLAG_SKIP_EMPTY = 1,
  /* With splits == 1, pdl_paged_decode writes the output directly from the
   * partition kernel and leaves the workspace untouched. */
  PDL_FLAG_DIRECT_SINGLE = 2,
  /* Work items are handed to the persistent CTAs from an atomic counter
   * (each CTA's first item is its index; later ones are claimed) instead of
   * a static stride: balances batches of very different lengths.  Uses
   * counters[0] and counters[1] (zero-initialised once; the kernel leaves
   * them zeroed).  The counter is touched only when a launch has more live
   * work items than CTAs.  Outputs are bit-identical to static scheduling. */
  PDL_FLAG_DYNAMIC = 8,
  /* Partition bounds follow each row's length (no counterpart in the
   * reference, whose partitions are fixed tokens_per_split ranges): with
   * L = min(max(len, 0), table_width * 256) and G = tokens_per_split (> 0,
   * the granule), partition p of the row covers [p*c, min((p+1)*c, L)) with
   * c = G * ceil(ceil(L / splits) / G), so a row's live partitions are equal
   * up to the last one; ceil(L / c) of them are live.  The merge derives the
   * same bounds.  For single-wave launches whose rows are shorter than the
   * table capacity the split plan was made for (pdl_b200_plan sets it). */
  PDL_FLAG_BALANCED = 16
} PdlFlags;

/* Geometry contract; mirrors DecodeSpec (reference src/paged_decode/spec.py:11-30). */
typedef struct PdlSpec {
  int32_t max_batch;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;        /* 64, 128 or 256 */
  int32_t max_context_len;
  int32_t page_size;       /* must be 256 */
} PdlSpec;

/* Static split-KV plan; mirrors SplitKVPlan (reference src/paged_decode/splitkv_plan.py:15-23). */
typedef struct PdlPlan {
  int32_t splits;
  int32_t tile_tokens;
  int32_t tokens_per_split;
  int32_t table_capacity_tokens;
  int32_t lse_lanes;
  int32_t sm_count;
  int32_t explicit_splits;  /* 1: policy "explicit", 0: "pinned_geometry" */
  int32_t balanced;         /* pdl_b200_plan only: 1 when the plan recommends launching
                               with PDL_FLAG_BALANCED and tokens_per_split = tile_tokens
                               (the granule); tokens_per_split above stays the fixed-bounds
                               plan.  0 in reference plans. */
} PdlPlan;

/* Arguments of one decode launch.  Element strides, not bytes. */
typedef struct PdlDecodeArgs {
  const void *q;              /* bf16 [batch, num_heads, head_dim]            */
  int64_t q_stride_batch;
  int64_t q_stride_head;
  const void *k_cache;        /* bf16 [num_pages, 256, num_kv_heads, head_dim] */
  const void *v_cache;
  int64_t num_pages;
  const int32_t *block_table; /* [batch, table_width], row stride below       */
  int64_t table_stride;
  int32_t table_width;
  const int32_t *lengths;     /* [batch]                                      */
  int32_t batch;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float scale;                /* softmax scale applied to q.k                 */
  int32_t tokens_per_split;   /* partition size; 0 = one partition per row   */
  int32_t splits;             /* partitions per row held by the workspace     */
  int32_t protocol;           /* PdlProtocol                                  */
  int32_t kernel;             /* PdlKernel                                    */
  int32_t flags;              /* PdlFlags bits                                */
  void *out;                  /* bf16 [batch, num_heads, head_dim] contiguous */
  float *partial;             /* LSE protocol: [batch, num_heads, splits, head_dim] */
  float *lse;                 /*               [batch, num_heads, splits]          */
  float *maxima;              /* MLA protocol: [batch, num_heads, splits]          */
  float *denoms;              /*               [batch, num_heads, splits]          */
  float *accums;              /*               [batch, num_heads, splits, head_dim] */
  int32_t *counters;          /* PDL_FLAG_DYNAMIC: int32 [2] scheduler words, zeroed once   */
} PdlDecodeArgs;

/* Partition kernel: per (row, KV head, partition) online softmax over the
 * partition's tokens for every query head of the group; writes the split
 * workspace in args->protocol.  Only partitions holding live tokens are
 * computed; empty ones are stored as such (unless PDL_FLAG_SKIP_EMPTY).
 * With tokens_per_split == 0 and splits == 1 it writes the normalised output
 * to args->out directly and needs no workspace.
 * Replaces _normalized_partition (reference src/paged_decode/matched_splitkv.py:52-98),
 * _split (src/paged_decode/kernels.py:44-80), _tc_partition
 * (src/paged_decode/tc_splitk.py:13-60), _base (src/paged_decode/kernels.py:10-41)
 * and _tensorcore (src/paged_decode/experimental_precision.py:46-107). */
int pdl_partition(const PdlDecodeArgs *args, pdl_stream_t stream);

/* Merge kernel: combines args->splits partitions per (row, query head) into
 * bf16 args->out.  LSE protocol replaces _lse_merge
 * (reference src/paged_decode/matched_splitkv.py:101-127); MLA protocol replaces
 * _merge (src/paged_decode/kernels.py:83-100). */
int pdl_merge(const PdlDecodeArgs *args, pdl_stream_t stream);

/* Strided LSE merge: rows r = 0..rows-1, partitions p = 0..parts-1 with
 *   partial row at partial[r*row_stride + p*part_stride]   (head_dim floats)
 *   lse         at lse[r*lse_row_stride + p*lse_part_stride].
 * Covers the split workspace (row_stride = parts*D, part_stride = D) and the
 * rank-major buffer of an all-gather (row_stride = D, part_stride = the
 * per-rank block).  Strides are in floats. */
typedef struct PdlMergeArgs {
  const float *partial;
  const float *lse;
  int64_t row_stride;
  int64_t part_stride;
  int64_t lse_row_stride;
  int64_t lse_part_stride;
  int32_t rows;               /* batch * num_heads */
  int32_t parts;
  int32_t head_dim;
  void *out;                  /* bf16 [rows, head_dim], or NULL                  */
  float *out_partial;         /* f32 [rows, head_dim] merged partial, or NULL    */
  float *out_lse;             /* f32 [rows] merged LSE (-inf if empty), or NULL  */
} PdlMergeArgs;

/* Stable LSE merge of arbitrary-strided partitions into a BF16 output and/or
 * an FP32 (partial, LSE) pair that can feed a further merge (the
 * context-parallel combine after an all-gather).  Same arithmetic as
 * _lse_merge (reference src/paged_decode/matched_splitkv.py:101-127); the
 * strided layout and the (partial, LSE) output have no counterpart in the
 * reference, which has no multi-GPU path. */
int pdl_lse_merge(const PdlMergeArgs *args, pdl_stream_t stream);

/* Partition + merge (or the single-pass kernel when tokens_per_split == 0).
 * Replaces the launch sequence of paged_decode (reference
 * src/paged_decode/runtime.py:87-117), matched_decode
 * (src/paged_decode/matched_splitkv.py:130-150) and tc_splitk_decode
 * (src/paged_decode/tc_splitk.py:63-79). */
int pdl_paged_decode(const PdlDecodeArgs *args, pdl_stream_t stream);

/* Capacity of the device array used by pdl_paged_decode_static_scratch. */
#define PDL_STATIC_SCRATCH_BYTES (4u << 20)

/* pdl_paged_decode without a caller-provided workspace, for callers that
 * cannot allocate device memory: an engine that has reserved nearly all HBM
 * for its KV page pool, a host behind an FFI that only holds pointers the
 * engine gave it, or a path that must not call cudaMalloc/cudaFree because
 * they can synchronise the device.  No counterpart in the reference.
 * The partial + LSE workspace is a file-scope __device__ array of
 * PDL_STATIC_SCRATCH_BYTES (4 MiB) that every GPU loading the library holds
 * until exit; calls needing batch*num_heads*splits*(head_dim+1)*4 bytes
 * beyond that are rejected with PDL_ERR_WORKSPACE (pdl_last_error says how
 * much was needed).  The workspace pointers and protocol in `args` are
 * ignored (LSE protocol); the flags mean what they mean for
 * pdl_paged_decode, PDL_FLAG_DYNAMIC using the caller's `counters` (two
 * zeroed int32, rejected if NULL).  The first call on a device looks up the array's
 * device address with that device current; make that first call before any
 * stream capture.  All calls on a device share the array and it keeps the
 * last call's contents (nothing in it needs to start at zero), so calls
 * that overlap on the GPU race.  Nothing is allocated. */
int pdl_paged_decode_static_scratch(const PdlDecodeArgs *args, pdl_stream_t stream);

/* New K/V rows to append to the paged cache (element strides). */
typedef struct PdlAppendArgs {
  const void *key;            /* bf16 [n_tokens, num_kv_heads, head_dim], head_dim contiguous */
  const void *value;
  int64_t key_stride_token;
  int64_t key_stride_head;
  int64_t value_stride_token;
  int64_t value_stride_head;
  void *k_cache;              /* bf16 [num_pages, 256, num_kv_heads, head_dim] contiguous */
  void *v_cache;
  int64_t num_pages;
  int32_t n_tokens;
  int32_t num_kv_heads;
  int32_t head_dim;
  /* Slot mode: physical slot (page * 256 + offset) per token; -1 skips it. */
  const int32_t *slot_mapping;
  /* Table mode (slot_mapping == NULL): token b is row b's next position. */
  const int32_t *block_table; /* [n_tokens, table_width], row stride below */
  int64_t table_stride;
  int32_t table_width;
  int32_t *lengths;           /* [n_tokens]; read as the write position */
  int32_t increment_lengths;  /* 1: lengths[b] += 1 after its slot is resolved */
} PdlAppendArgs;

/* Copy each new token's K and V rows into its cache slot.  Slot mode
 * replaces store_kvcache (reference overlays/nano-vllm/nanovllm/layers/
 * attention.py:10-40); table mode replaces the paged write of
 * PagedHybridCache.update (reference src/paged_decode/hybrid.py:63-72) for a
 * decode position, with the length update done on the device so a decode
 * loop can be captured in a CUDA graph.  Slots outside the pool and rows
 * whose table is full are skipped. */
int pdl_append_kv(const PdlAppendArgs *args, pdl_stream_t stream);

/* ------------------------------------------------------------------------
 * Context-parallel combine over peer memory (no counterpart in the
 * reference, which has no multi-GPU path).  One process per GPU; every rank
 * owns one exchange buffer, created with pdl_peer_buffer_create and mapped
 * into every other rank's process with pdl_peer_buffer_open (CUDA IPC; the
 * 64-byte handles travel over the host process group).  pdl_exchange_merge
 * then replaces "local merge -> all-gather -> merge" with ONE kernel: each
 * rank merges its local partitions, stores the merged FP32 partial + LSE
 * into every rank's buffer over NVLink, each value tagged with the call's
 * sequence number, waits (bounded) until every rank's values of its rows
 * carry that sequence and merges the `world` blocks into its BF16 output.
 * Output bits equal the two-kernel path's.
 * ---------------------------------------------------------------------- */
#define PDL_MAX_PEERS 8

typedef struct PdlIpcHandle {
  unsigned char bytes[64];    /* cudaIpcMemHandle_t */
} PdlIpcHandle;

/* Geometry of the exchange for `rows` (= batch * num_heads) rows. */
typedef struct PdlExchangePlan {
  int32_t ctas;               /* CTAs per rank (identical on identical GPUs)   */
  int32_t reserved;
  int64_t block_words;        /* 8-byte words per rank block: rows*D partials, rows LSEs
                               * padded to an even count (value | sequence << 32)    */
  int64_t data_offset;        /* bytes of per-warp sequence words before the data   */
  int64_t buffer_bytes;       /* bytes each rank's exchange buffer needs        */
} PdlExchangePlan;

/* Pure arithmetic (no device access).  emulate_ranks: plan the single-GPU
 * emulation launch of pdl_exchange_merge instead. */
int pdl_exchange_plan(int32_t rows, int32_t head_dim, int32_t world, int32_t sm_count,
                      int32_t emulate_ranks, PdlExchangePlan *plan);

/* Allocate `bytes` of zeroed device memory on the current device (synchronises)
 * and, if `handle` is not NULL, export it for other processes. */
int pdl_peer_buffer_create(int64_t bytes, void **dev_ptr, PdlIpcHandle *handle);
/* Map another process's buffer into this one (peer access over NVLink). */
int pdl_peer_buffer_open(const PdlIpcHandle *handle, void **dev_ptr);
/* Unmap a buffer opened with pdl_peer_buffer_open. */
int pdl_peer_buffer_close(void *dev_ptr);
/* Free a buffer made by pdl_peer_buffer_create (after every peer closed it). */
int pdl_peer_buffer_free(void *dev_ptr);

typedef struct PdlExchangeArgs {
  const float *partial;       /* f32 [rows, parts, head_dim]: this rank's split workspace */
  const float *lse;           /* f32 [rows, parts]                                        */
  const int32_t *lengths;     /* optional int32 [rows / num_heads] tokens of each row in this
                               * rank's range: only ceil(len / tokens_per_split) partitions
                               * are read (fixed bounds: a workspace written with
                               * PDL_FLAG_BALANCED needs lengths NULL); NULL reads all
                               * `parts`                                                  */
  int32_t num_heads;
  int32_t tokens_per_split;
  int32_t rows;
  int32_t parts;
  int32_t head_dim;
  int32_t rank;
  int32_t world;              /* 1 .. PDL_MAX_PEERS                                       */
  /* 1: ONE cooperative launch on this GPU runs all `world` ranks (testing):
   * partial, lse, lengths and out then hold `world` consecutive rank slices
   * and every buffer is local.  `rank` is ignored. */
  int32_t emulate_ranks;
  uint32_t timeout_us;        /* bound on the wait for peers; 0 = 1 s, at most 10 s      */
  void *buffers[PDL_MAX_PEERS]; /* rank q's exchange buffer as mapped here (buffer_bytes) */
  void *out;                  /* bf16 [rows, head_dim]                                    */
} PdlExchangeArgs;

/* Every rank must call this with the same rows/parts/head_dim/world, in the
 * same order as its other exchanges on the same buffers.  A wait that runs
 * out sets a bit (16) in the fault word (pdl_read_fault) and leaves the
 * waiting warp's remaining output rows unwritten; the buffers are then out
 * of step and must be re-created on every rank. */
int pdl_exchange_merge(const PdlExchangeArgs *args, pdl_stream_t stream);

/* Static plan for `spec` on `sm_count` SMs; num_splits 0 = heuristic.
 * Replaces make_splitkv_plan (reference src/paged_decode/splitkv_plan.py:26-56). */
int pdl_splitkv_plan(const PdlSpec *spec, int32_t sm_count, int32_t num_splits,
                     PdlPlan *plan);

/* Split plan for this library's persistent, dynamically scheduled kernels on
 * `sm_count` SMs (two CTA slots per SM): at most one wave of work items, or
 * (head_dim <= 128, items longer than 1024 tokens) two full waves; items of
 * at most 4096 tokens; partitions a multiple of the reference plan's tile.  No counterpart
 * in the reference (its plan, pdl_splitkv_plan, is tuned for one CTA per
 * partition on A100). */
int pdl_b200_plan(const PdlSpec *spec, int32_t sm_count, PdlPlan *plan);

/* partitions = ceil(max_context_len/1024), table_width = ceil(max_context_len/256),
 * split workspace bytes = max_batch*num_heads*partitions*(head_dim+2)*4.
 * Replaces DecodeSpec.partitions / table_width / split_workspace_bytes
 * (reference src/paged_decode/spec.py:32-42) and the checks of
 * DecodeSpec.__post_init__ (spec.py:20-30). */
int pdl_spec_geometry(const PdlSpec *spec, int32_t *partitions, int32_t *table_width,
                      int64_t *split_workspace_bytes);

/* Human-readable name of a PdlStatus. */
const char *pdl_status_string(int status);

/* What the last failing call on this host thread tried and why (the CUDA
 * error string, or the CUresult of descriptor encoding); "" if none. */
const char *pdl_last_error(void);

/* PDL_ABI_VERSION of the loaded library. */
int pdl_abi_version(void);

/* Sticky device-side fault word of the current device (0 = none); a
 * non-zero value records which bounded wait gave up (bits: 1 producer
 * waiting for a free stage, 2 consumer waiting for a tile, 4 draining copies
 * at exit, 8 misaligned shared memory, 16 exchange peer).  The outputs and
 * workspaces of every launch since the word was last cleared are then
 * undefined: a CTA that gives up stops processing, and an item it had
 * already claimed is processed by nobody.  Synchronises the device; for
 * diagnostics only, never on a hot path. */
int pdl_read_fault(uint32_t *fault, int clear);

#ifdef __cplusplus
}
#endif
#endif /* PDL_B200_H */
