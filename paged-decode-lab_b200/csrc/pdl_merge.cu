// pdl_merge.cu -- stable merge of split-K partitions.
//
// One warp per (row, query head, column slice of at most 128 floats); lane l
// owns 4 (or D/32 for D = 64) contiguous FP32 columns of the slice, so each
// partition row is read with one coalesced vector load per lane, and rows of
// eight partitions are in flight at once.  The kernel is launched with
// programmatic stream serialization: its CTAs may be scheduled while the
// partition kernel still runs and wait (griddepcontrol.wait) for it to
// complete before reading anything.
// Partition p of row r is read at  rows_src[r * row_stride + p * part_stride]
// and its weight at  weights_src[r * w_row_stride + p * w_part_stride], so
// the same kernel merges the split workspace ([B,Hq,S,D], S contiguous) and
// the rank-major buffer an all-gather produces ([N][B*Hq][D]).
//
// LSE protocol (reference src/paged_decode/matched_splitkv.py:101-127):
//   M = max_p lse_p (an all -inf row uses 0); total = sum_p exp(lse_p - M);
//   logsum = ln(total) + M, or +inf when total = 0;
//   out = sum_p exp(lse_p - logsum) * partial_p.
// Optionally the merged row is stored as an FP32 partial plus its LSE
// (logsum, or -inf for an empty row), so a merge can feed another merge.
// MLA protocol (reference src/paged_decode/kernels.py:83-100):
//   M = max_p m_p (-inf -> 0); f_p = exp(m_p - M);
//   out = sum_p f_p * acc_p / (sum_p f_p * l_p, or 1 when that is 0).
// When `lengths` is given, only the ceil(len / tokens_per_split) live
// partitions of a row are read (the others hold no tokens and their weights
// are exactly 0), so empty partitions need not be stored at all.
#include "pdl_device.cuh"

namespace pdl {
namespace {

constexpr int MERGE_WARPS = 4;

template <int E>
__device__ __forceinline__ void load_cols(const float *src, float (&v)[E]) {
  if constexpr (E == 2) {
    const float2 a = *reinterpret_cast<const float2 *>(src);
    v[0] = a.x; v[1] = a.y;
  } else {
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      const float4 a = *reinterpret_cast<const float4 *>(src + i);
      v[i] = a.x; v[i + 1] = a.y; v[i + 2] = a.z; v[i + 3] = a.w;
    }
  }
}

template <int E>
__device__ __forceinline__ void store_cols(float *dst, const float (&v)[E]) {
  if constexpr (E == 2) {
    *reinterpret_cast<float2 *>(dst) = make_float2(v[0], v[1]);
  } else {
#pragma unroll
    for (int i = 0; i < E; i += 4)
      *reinterpret_cast<float4 *>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}

template <int D>
__global__ void __launch_bounds__(32 * MERGE_WARPS)
    merge_kernel(const MergeParams p) {
  constexpr int CW = D < 128 ? D : 128;  // columns per warp
  constexpr int SLICES = D / CW;
  constexpr int E = CW / 32;
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x * MERGE_WARPS + (threadIdx.x >> 5);
  const int row = unit / SLICES, col0 = (unit % SLICES) * CW;
  // Lengths are an input of the decode, not an output of the partition
  // kernel, so they are read before waiting for it.
  int live = p.splits;
  if (p.lengths != nullptr && row < p.rows) {
    const int len = __ldg(p.lengths + row / p.num_heads);
    live = min(live, (int)((len + (int64_t)p.tokens_per_split - 1) / p.tokens_per_split));
  }
  grid_dependency_wait();
  if (row >= p.rows) return;
  const bool lse_protocol = p.protocol == MODE_LSE;
  const float *w_src = (lse_protocol ? p.lse : p.maxima) + (int64_t)row * p.w_row_stride;
  const float *r_src = (lse_protocol ? p.partial : p.accums) + (int64_t)row * p.row_stride + col0;

  // Weights of partitions lane, lane+32, ... stay in registers (up to 128
  // partitions; more are re-read).
  constexpr int WR = 4;
  float wreg[WR];
#pragma unroll
  for (int i = 0; i < WR; ++i)
    wreg[i] = lane + 32 * i < live ? __ldcg(w_src + (lane + 32 * i) * p.w_part_stride) : -INFINITY;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < WR; ++i) mx = fmaxf(mx, wreg[i]);
  for (int s = lane + 32 * WR; s < live; s += 32) mx = fmaxf(mx, __ldcg(w_src + s * p.w_part_stride));
  mx = warp_max(mx);
  if (mx == -INFINITY) mx = 0.f;

  float shift = mx;   // exponent subtracted from every weight
  float scale = 1.f;  // final multiplier
  float tot = 0.f;
  if (lse_protocol) {
#pragma unroll
    for (int i = 0; i < WR; ++i) tot += lane + 32 * i < live ? expf(wreg[i] - mx) : 0.f;
    for (int s = lane + 32 * WR; s < live; s += 32) tot += expf(__ldcg(w_src + s * p.w_part_stride) - mx);
    tot = warp_sum(tot);
    shift = tot > 0.f ? logf(tot) + mx : INFINITY;
  } else {
    const float *l_src = p.denoms + (int64_t)row * p.w_row_stride;
    for (int s = lane; s < live; s += 32)
      tot += __ldcg(l_src + s * p.w_part_stride) * expf(__ldcg(w_src + s * p.w_part_stride) - mx);
    tot = warp_sum(tot);
    scale = 1.f / (tot > 0.f ? tot : 1.f);
  }

  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int s0 = 0; s0 < live; s0 += 32) {
    const int wi = s0 / 32;
    // Register select (a dynamic index would put wreg in local memory).
    const float wsrc = wi == 0 ? wreg[0] : wi == 1 ? wreg[1] : wi == 2 ? wreg[2]
                     : wi == 3 ? wreg[3]
                     : (s0 + lane < live ? __ldcg(w_src + (s0 + lane) * p.w_part_stride)
                                         : -INFINITY);
    const float wl = (s0 + lane < live) ? expf(wsrc - shift) : 0.f;
    const int n = min(32, live - s0);
    // Rows of up to BATCH partitions are loaded before any is consumed, so
    // the memory round trips overlap instead of serialising per partition.
    constexpr int BATCH = E <= 4 ? 16 : 8;
    for (int k0 = 0; k0 < n; k0 += BATCH) {
      float v[BATCH][E];
#pragma unroll
      for (int j = 0; j < BATCH; ++j)
        load_cols<E>(r_src + (int64_t)(s0 + min(k0 + j, n - 1)) * p.part_stride + lane * E, v[j]);
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        const float wk = __shfl_sync(FULL_MASK, wl, min(k0 + j, 31));
        if (k0 + j < n) {
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = fmaf(wk, v[j][e], acc[e]);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] *= scale;
  if (p.out != nullptr) {
    __nv_bfloat16 *dst = p.out + (int64_t)row * D + col0 + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2)
      *reinterpret_cast<__nv_bfloat162 *>(dst + e) = __floats2bfloat162_rn(acc[e], acc[e + 1]);
  }
  if (p.out_partial != nullptr)
    store_cols<E>(p.out_partial + (int64_t)row * D + col0 + lane * E, acc);
  if (p.out_lse != nullptr && lane == 0 && col0 == 0)
    p.out_lse[row] = tot > 0.f ? shift : -INFINITY;
}

template <int D>
cudaError_t launch_merge_t(const MergeParams &params, cudaStream_t stream) {
  constexpr int SLICES = D / (D < 128 ? D : 128);
  const int64_t units = (int64_t)params.rows * SLICES;
  const int grid = (int)((units + MERGE_WARPS - 1) / MERGE_WARPS);
  if (grid <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(32 * MERGE_WARPS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, merge_kernel<D>, params);
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
