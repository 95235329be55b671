// pdl_merge_core.cuh -- the merge arithmetic of one warp over one (row,
// column slice), shared by the merge kernel (pdl_merge.cu) and the
// peer-exchange kernel (pdl_exchange.cu) so both produce identical bits.
//
// Lane l owns E contiguous FP32 columns of the slice.  Partition p's row is
// read at r_src[p * part_stride] and its weight at w_src[p * w_part_stride].
//
// LSE protocol (reference src/paged_decode/matched_splitkv.py:101-127):
//   M = max_p lse_p (an all -inf row uses 0); total = sum_p exp(lse_p - M);
//   logsum = ln(total) + M, or +inf when total = 0;
//   out = sum_p exp(lse_p - logsum) * partial_p.
// MLA protocol (reference src/paged_decode/kernels.py:83-100):
//   M = max_p m_p (-inf -> 0); f_p = exp(m_p - M);
//   out = sum_p f_p * acc_p / (sum_p f_p * l_p, or 1 when that is 0).
// Partitions are accumulated in index order with one fused multiply-add per
// partition, whatever the staging of the loads; the exchange kernel's merge
// across ranks keeps the same order, so both give the same bits.
#pragma once

#include "pdl_device.cuh"

namespace pdl {

template <int E>
__device__ __forceinline__ void merge_store_cols(float *dst, const float (&v)[E]) {
  if constexpr (E == 2) {
    *reinterpret_cast<float2 *>(dst) = make_float2(v[0], v[1]);
  } else {
#pragma unroll
    for (int i = 0; i < E; i += 4)
      *reinterpret_cast<float4 *>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  }
}

__device__ __forceinline__ float warp_max_all(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum_all(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// The partition rows are staged through shared memory: every lane issues one
// asynchronous copy (cp.async, L2 only) per partition for up to `cap`
// partitions right after the weights are requested, so the rows arrive in
// one round trip that overlaps the weights'.  `stage` is this warp's
// cap * 32 * E floats of shared memory.
template <int E>
__device__ __forceinline__ void stage_rows(float *stage, const float *r_src, int64_t part_stride,
                                           int first, int n, int lane) {
  const uint32_t dst0 = static_cast<uint32_t>(__cvta_generic_to_shared(stage + lane * E));
#pragma unroll 4
  for (int j = 0; j < n; ++j) {
    const float *src = r_src + (int64_t)(first + j) * part_stride + lane * E;
    const uint32_t dst = dst0 + j * 32 * E * 4;
    if constexpr (E == 4) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    } else {
      static_assert(E == 2, "two or four columns per lane");
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void wait_staged_rows() {
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
}

// Merges `live` partitions into acc (already scaled).  `shift` is the
// exponent subtracted from every weight (the LSE protocol's logsum), `tot`
// the weight total, so the merged LSE is (tot > 0 ? shift : -inf).  Rows are
// staged `cap` partitions at a time (one round trip when live <= cap).
template <int E>
__device__ __forceinline__ void merge_slice(bool lse_protocol, const float *w_src,
                                                   int64_t w_part_stride, const float *l_src,
                                                   const float *r_src, int64_t part_stride,
                                                   int live, int lane, float *stage, int cap,
                                                   float (&acc)[E], float &shift, float &tot) {
  // The weights are requested first: the copies' asm statements are ordered
  // memory operations, so loads issued after them would wait behind their
  // issue instead of overlapping it.
  constexpr int WR = 4;
  float wreg[WR];
#pragma unroll
  for (int i = 0; i < WR; ++i)
    wreg[i] = lane + 32 * i < live ? __ldcg(w_src + (lane + 32 * i) * w_part_stride) : -INFINITY;
  stage_rows<E>(stage, r_src, part_stride, 0, min(live, cap), lane);
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < WR; ++i) mx = fmaxf(mx, wreg[i]);
  for (int s = lane + 32 * WR; s < live; s += 32) mx = fmaxf(mx, __ldcg(w_src + s * w_part_stride));
  mx = warp_max_all(mx);
  if (mx == -INFINITY) mx = 0.f;

  shift = mx;
  float scale = 1.f;
  tot = 0.f;
  if (lse_protocol) {
#pragma unroll
    for (int i = 0; i < WR; ++i) tot += lane + 32 * i < live ? expf(wreg[i] - mx) : 0.f;
    for (int s = lane + 32 * WR; s < live; s += 32) tot += expf(__ldcg(w_src + s * w_part_stride) - mx);
    tot = warp_sum_all(tot);
    shift = tot > 0.f ? logf(tot) + mx : INFINITY;
  } else {
    for (int s = lane; s < live; s += 32)
      tot += __ldcg(l_src + s * w_part_stride) * expf(__ldcg(w_src + s * w_part_stride) - mx);
    tot = warp_sum_all(tot);
    scale = 1.f / (tot > 0.f ? tot : 1.f);
  }

#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  int staged0 = 0;      // first partition held by the stage (chunks of cap partitions)
  bool waited = false;  // the current chunk has landed
  for (int s0 = 0; s0 < live; s0 += 32) {
    const int n = min(32, live - s0);
    const int wi = s0 / 32;
    // Register select (a dynamic index would put wreg in local memory).
    const float wsrc = wi == 0 ? wreg[0] : wi == 1 ? wreg[1] : wi == 2 ? wreg[2]
                     : wi == 3 ? wreg[3]
                     : (s0 + lane < live ? __ldcg(w_src + (s0 + lane) * w_part_stride)
                                         : -INFINITY);
    const float wl = (s0 + lane < live) ? expf(wsrc - shift) : 0.f;
    for (int c = 0; c < n;) {
      const int s = s0 + c;
      if (s >= staged0 + cap) {
        __syncwarp();  // every lane is done with the previous chunk
        staged0 = s;
        stage_rows<E>(stage, r_src, part_stride, s, min(cap, live - s), lane);
        waited = false;
      }
      if (!waited) {
        wait_staged_rows();
        waited = true;
      }
      const int m = min(n - c, staged0 + cap - s);
      const float *rows = stage + (s - staged0) * 32 * E + lane * E;
      // Partition order, 8 rows per step: their weights and rows are read
      // before their multiply-adds, so only the adds form a dependent chain.
      int j = 0;
      for (; j + 8 <= m; j += 8) {
        float wk[8], rv[8][E];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          wk[u] = __shfl_sync(FULL_MASK, wl, c + j + u);
#pragma unroll
          for (int e = 0; e < E; ++e) rv[u][e] = rows[(j + u) * 32 * E + e];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = fmaf(wk[u], rv[u][e], acc[e]);
      }
      for (; j < m; ++j) {
        const float wk = __shfl_sync(FULL_MASK, wl, c + j);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] = fmaf(wk, rows[j * 32 * E + e], acc[e]);
      }
      c += m;
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] *= scale;
}

}  // namespace pdl
