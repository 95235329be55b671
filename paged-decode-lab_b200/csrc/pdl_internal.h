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

// Work item = (row b, KV head, head sub-group, partition); items are
// enumerated partition-fastest and handed to persistent CTAs round-robin.
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
  int32_t n_items;          // splits * num_kv_heads * nsub * batch
  float log2_scale;         // scale * log2(e)
  int32_t mode;             // OutMode
  int32_t q_vec16;          // q rows 16-byte aligned (vector loads)
  int32_t write_empty;      // store -inf/0 for empty partitions
  __nv_bfloat16 *out;
  float *partial;
  float *lse;
  float *maxima;
  float *denoms;
  float *accums;
  uint32_t *fault;          // per-device fault word
  int32_t *counters;        // fused merge: finished items per (row, KV head, sub-group), or null
  int32_t *sched;           // dynamic scheduling: [next item, finished CTAs], or null (static)
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
