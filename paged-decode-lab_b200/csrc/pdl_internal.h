// pdl_internal.h -- parameter blocks shared by the C-ABI layer and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pdl {

constexpr int kMaxDevices = 64;

// What the partition kernel stores per (row, query head, partition).
enum OutMode : int {
  MODE_LSE = 0,     // normalised partial + LSE
  MODE_MLA = 1,     // unnormalised maxima / denominators / accumulators
  MODE_DIRECT = 2,  // one partition per row: normalised BF16 output
};

// Work item = (row b, KV head, head sub-group, partition).  The producer warp
// of every persistent CTA enumerates the live items from the lengths and
// hands them out round-robin over the CTAs, or from an atomic counter
// (dynamic scheduling, `sched`).
struct PartitionParams {
  const __nv_bfloat16 *q;
  int64_t q_stride_batch;   // elements
  int64_t q_stride_head;    // elements
  const int32_t *table;
  int64_t table_stride;     // elements
  int32_t table_width;      // live tokens are clamped to table_width * 256
  const int32_t *lengths;
  int32_t batch;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t group;            // num_heads / num_kv_heads
  int32_t nsub;             // head sub-groups per KV head
  int32_t tokens_per_split; // > 0
  int32_t splits;
  int32_t n_items;          // splits * num_kv_heads * nsub * batch (live or not)
  float log2_scale;         // scale * log2(e)
  int32_t mode;             // OutMode
  int32_t q_vec16;          // q rows 16-byte aligned (vector loads)
  int32_t write_empty;      // store -inf/0 for empty partitions
  int32_t fill_splits;      // empty partitions (all heads of one row) per fill item
  __nv_bfloat16 *out;
  float *partial;
  float *lse;
  float *maxima;
  float *denoms;
  float *accums;
  uint32_t *fault;          // per-device fault word
  int32_t *sched;           // dynamic scheduling: [items claimed, finished CTAs], or null (static)
  int32_t live;             // enumerate live items only (set by the launcher: multi-wave
                            // launches of batches up to 512 rows)
  int32_t balanced;         // partition bounds from each row's length (balanced_span);
                            // tokens_per_split is then the granule
};

// Partition p of row r: rows at partial/accums[r*row_stride + p*part_stride],
// weights at lse/maxima/denoms[r*w_row_stride + p*w_part_stride].
struct MergeParams {
  const float *partial;     // LSE protocol
  const float *lse;
  const float *maxima;      // MLA protocol
  const float *denoms;
  const float *accums;
  int64_t row_stride;
  int64_t part_stride;
  int64_t w_row_stride;
  int64_t w_part_stride;
  __nv_bfloat16 *out;       // BF16 [rows, D], or null
  float *out_partial;       // FP32 [rows, D] merged partial, or null (LSE protocol)
  float *out_lse;           // FP32 [rows] merged LSE (-inf if empty), or null
  const int32_t *lengths;   // optional: bound the partitions read per row
  int32_t early_lengths;    // launched right after the partition kernel: read lengths
                            // before the dependency wait
  int32_t balanced;         // partitions follow the row lengths (balanced_span)
  int32_t cap_tokens;       // table_width * 256: lengths are clamped to it like the
                            // partition kernel clamps them
  int32_t num_heads;
  int32_t tokens_per_split;
  int32_t rows;             // batch * num_heads
  int32_t splits;
  int32_t protocol;         // MODE_LSE or MODE_MLA
};

// New K/V rows -> paged cache (pdl_append.cu).
struct AppendParams {
  const __nv_bfloat16 *key;
  const __nv_bfloat16 *value;
  int64_t key_stride_token, key_stride_head;      // elements
  int64_t value_stride_token, value_stride_head;  // elements
  __nv_bfloat16 *k_cache;
  __nv_bfloat16 *v_cache;
  int64_t num_pages;
  int32_t n_tokens;
  int32_t num_kv_heads;
  int32_t head_dim;
  const int32_t *slot_mapping;  // slot mode, or null for table mode
  const int32_t *table;         // table mode
  int64_t table_stride;
  int32_t table_width;
  int32_t *lengths;             // table mode: write position, incremented when `increment`
  int32_t increment;
  int32_t key_vec16;            // 16-byte vector copies allowed
  int32_t value_vec16;
};

cudaError_t launch_append(const AppendParams &params, cudaStream_t stream);

// Peer exchange of the context-parallel merge (pdl_exchange.cu).
// Every rank's exchange buffer has the same layout:
//   uint32 seq[kMaxExchangeWarps]    calls completed by warp w of this rank (local only)
//   uint64 data[2][world][block]     at kExchangeHeaderBytes; half = sequence & 1
// where a rank block holds rows*D merged partial words, then rows LSE words
// (padded to an even count).  A word is (float bits) | (sequence << 32):
// the reader knows a value is current when its sequence matches.
constexpr int kMaxPeers = 8;
constexpr int kMaxExchangeCtas = 1024;
constexpr int kExchangeWarps = 4;  // warps per exchange CTA
constexpr int kMaxExchangeWarps = kMaxExchangeCtas * kExchangeWarps;
constexpr int64_t kExchangeHeaderBytes = int64_t(kMaxExchangeWarps) * 4;
constexpr int kExchangeCtasPerSm = 4;  // occupancy the exchange kernel is built for

struct ExchangeParams {
  const float *partial;     // [rows, splits, D] local split workspace (LSE protocol)
  const float *lse;         // [rows, splits]
  const int32_t *lengths;   // optional local lengths [rows / num_heads]
  int32_t num_heads;
  int32_t tokens_per_split;
  int32_t rows;
  int32_t splits;
  int32_t rank;
  int32_t world;
  int32_t emulate;          // 1: blockIdx.y is the rank, every rank's slices and buffers on this GPU
  int32_t ctas;             // CTAs per rank; the same on every rank
  int64_t block;            // 8-byte words per rank block
  unsigned char *buffers[kMaxPeers];
  __nv_bfloat16 *out;       // [rows, D]
  uint64_t timeout_ns;
  uint32_t *fault;
};

cudaError_t launch_exchange(const ExchangeParams &params, int head_dim, cudaStream_t stream);
// CTAs per rank of an exchange launch (a function of the shape and SM count
// only, so every rank of a node computes the same grid).
int exchange_ctas(int rows, int head_dim, int world, int sm_count, bool emulate);

struct KernelLaunch {
  const CUtensorMap *k_map;
  const CUtensorMap *v_map;
  PartitionParams params;
  int head_dim;
  int group_per_cta;        // query heads handled by one CTA
  int sm_count;
};

// Launchers (return a cudaError_t).  Each configures its kernel's shared
// memory on first use and sizes a persistent grid from the occupancy query.
cudaError_t launch_partition_simt(const KernelLaunch &launch, cudaStream_t stream);
cudaError_t launch_partition_mma(const KernelLaunch &launch, cudaStream_t stream);
cudaError_t launch_merge(const MergeParams &params, int head_dim, cudaStream_t stream);

// Query heads per CTA each kernel supports for a given group size.
int simt_heads_per_cta(int group);
int mma_heads_per_cta(int group, int head_dim);

// Tokens per pipeline stage (TMA box height) of each kernel for a head dim.
int simt_tile_tokens(int head_dim);
int mma_tile_tokens(int head_dim);

}  // namespace pdl
