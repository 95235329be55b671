// pdl_merge.cu -- stable merge of split-K partitions.
//
// One warp per (row, query head, column slice of at most 128 floats); lane l
// owns 4 (or D/32 for D = 64) contiguous FP32 columns of the slice.  The
// rows of up to min(splits, 48) partitions are copied into shared memory
// asynchronously (one 16- or 8-byte cp.async per lane and partition) while
// the weights are loaded and reduced, so a merge costs about one memory
// round trip.  The kernel is launched with
// programmatic stream serialization: its CTAs may be scheduled while the
// partition kernel still runs and wait (griddepcontrol.wait) for it to
// complete before reading anything.
// Partition p of row r is read at  rows_src[r * row_stride + p * part_stride]
// and its weight at  weights_src[r * w_row_stride + p * w_part_stride], so
// the same kernel merges the split workspace ([B,Hq,S,D], S contiguous) and
// the rank-major buffer an all-gather produces ([N][B*Hq][D]).
//
// The arithmetic (LSE and MLA protocols) is merge_slice in
// pdl_merge_core.cuh.  Optionally the merged row is stored as an FP32
// partial plus its LSE (logsum, or -inf for an empty row), so a merge can
// feed another merge.
// When `lengths` is given, only the ceil(len / tokens_per_split) live
// partitions of a row are read (the others hold no tokens and their weights
// are exactly 0), so empty partitions need not be stored at all; with
// balanced partitions, ceil(len / balanced_span(len)).
#include "pdl_merge_core.cuh"

namespace pdl {
namespace {

constexpr int MERGE_WARPS = 4;
// Partitions staged per round trip: rows of up to 48 live partitions arrive
// in one (config 3 at B = 1 has 33 at ctx 2064).  At 96 KB a CTA still fits
// beside one partition CTA of about 113 KB on an SM, so the merge CTAs are
// scheduled, and read the lengths, while the partition kernel runs.
constexpr int kMergeStageParts = 48;

template <int D>
__global__ void __launch_bounds__(32 * MERGE_WARPS)
    merge_kernel(const MergeParams p) {
  constexpr int CW = D < 128 ? D : 128;  // columns per warp
  constexpr int SLICES = D / CW;
  constexpr int E = CW / 32;
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x * MERGE_WARPS + (threadIdx.x >> 5);
  const int row = unit / SLICES, col0 = (unit % SLICES) * CW;
  // The next decode step's partition kernel may be scheduled now; it waits
  // for this grid to complete before touching the workspace.
  allow_dependent_launch();
  // The lengths are an input of the decode.  Launched right after this
  // library's partition kernel (`early_lengths`), every kernel that may
  // write them completed before that kernel let this one be scheduled (it
  // triggers after its own dependency wait), so they are read before waiting
  // for it; the workspace is always read after.
  int len = 0;
  if (p.early_lengths && p.lengths != nullptr && row < p.rows)
    len = __ldg(p.lengths + row / p.num_heads);
  grid_dependency_wait();
  if (row >= p.rows) return;
  int live = p.splits;
  if (p.lengths != nullptr) {
    if (!p.early_lengths) len = __ldg(p.lengths + row / p.num_heads);
    if (p.balanced) {
      const int clamped = min(max(len, 0), p.cap_tokens);
      const int64_t span = balanced_span(clamped, p.splits, p.tokens_per_split);
      live = span > 0 ? (int)min((int64_t)live, (clamped + span - 1) / span) : 0;
    } else {
      live = min(live, (int)((max(len, 0) + (int64_t)p.tokens_per_split - 1) / p.tokens_per_split));
    }
  }
  const bool lse_protocol = p.protocol == MODE_LSE;
  const float *w_src = (lse_protocol ? p.lse : p.maxima) + (int64_t)row * p.w_row_stride;
  const float *r_src = (lse_protocol ? p.partial : p.accums) + (int64_t)row * p.row_stride + col0;
  const float *l_src = lse_protocol ? nullptr : p.denoms + (int64_t)row * p.w_row_stride;
  extern __shared__ __align__(16) float merge_stage[];
  const int cap = min(p.splits, kMergeStageParts);
  float acc[E], shift, tot;
  merge_slice<E>(lse_protocol, w_src, p.w_part_stride, l_src, r_src, p.part_stride, live,
                        lane, merge_stage + (threadIdx.x >> 5) * cap * 32 * E, cap, acc, shift,
                        tot);
  if (p.out != nullptr) {
    __nv_bfloat16 *dst = p.out + (int64_t)row * D + col0 + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2)
      *reinterpret_cast<__nv_bfloat162 *>(dst + e) = __floats2bfloat162_rn(acc[e], acc[e + 1]);
  }
  if (p.out_partial != nullptr)
    merge_store_cols<E>(p.out_partial + (int64_t)row * D + col0 + lane * E, acc);
  if (p.out_lse != nullptr && lane == 0 && col0 == 0)
    p.out_lse[row] = tot > 0.f ? shift : -INFINITY;
}

template <int D>
cudaError_t launch_merge_t(const MergeParams &params, cudaStream_t stream) {
  constexpr int CW = D < 128 ? D : 128;
  constexpr int SLICES = D / CW;
  // Up to kMergeStageParts staged partition rows of CW floats per warp.
  constexpr int max_smem = MERGE_WARPS * kMergeStageParts * CW * 4;
  const int smem = MERGE_WARPS * min(params.splits, kMergeStageParts) * CW * 4;
  static bool configured[kMaxDevices] = {false};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    err = cudaFuncSetAttribute(merge_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               max_smem);
    if (err != cudaSuccess) return err;
    configured[dev] = true;
  }
  const int64_t units = (int64_t)params.rows * SLICES;
  const int grid = (int)((units + MERGE_WARPS - 1) / MERGE_WARPS);
  if (grid <= 0) return cudaSuccess;
  return launch_programmatic(merge_kernel<D>, dim3(grid), dim3(32 * MERGE_WARPS), smem, stream,
                             params);
}

}  // namespace

cudaError_t launch_merge(const MergeParams &params, int head_dim, cudaStream_t stream) {
  switch (head_dim) {
    case 64: return launch_merge_t<64>(params, stream);
    case 128: return launch_merge_t<128>(params, stream);
    case 256: return launch_merge_t<256>(params, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pdl
