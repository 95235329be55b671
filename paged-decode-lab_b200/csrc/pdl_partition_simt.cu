// pdl_partition_simt.cu -- FP32 CUDA-core split-K partition kernel (sm_100a).
//
// One work item is (row b, KV head, query-head sub-group, partition).  A CTA
// is persistent: it walks items blockIdx.x, +gridDim.x, ... and keeps one
// TMA pipeline running across item boundaries.
//
//   warp 0      producer (run_producer): live block-table entries -> 5-D TMA
//               loads of T-token K and V tiles of one KV head into a 3-stage
//               shared-memory ring (128-byte swizzle, L2 evict-first).
//   warps 1..4  consumers: each owns T/4 rows of every tile.  D/8 lanes share
//               a row (one 16-byte chunk each); q of the head group lives in
//               registers as FP32 pairs.  Scores use packed FP32 FMAs and an
//               xor-shuffle all-reduce, the online softmax keeps a per-warp
//               running max (one rescale per tile), and P*V reuses the same
//               lane layout, so no probability goes through memory.  At the
//               end of an item the warp states are merged through shared
//               memory (combine_and_store).
//
// Replaces the reference's CUDA-core kernels _base and _split
// (src/paged_decode/kernels.py:10-80) and, for groups below 8, the GQA
// partition of _normalized_partition (src/paged_decode/matched_splitkv.py:52-98).
#include "pdl_pipeline.cuh"

namespace pdl {
namespace {

constexpr int NC = 4;                  // consumer warps
constexpr int NS = 3;                  // pipeline stages
constexpr int NTHREADS = 32 * (NC + 1);

template <int D>
struct SimtShape {
  static constexpr int T = D == 64 ? 128 : (D == 128 ? 64 : 32);  // tokens per stage
  static constexpr int TW = T / NC;                               // rows per warp per stage
  static constexpr int LPT = D / 8;                               // lanes per row
  static constexpr int TPS = 32 / LPT;                            // rows per warp step
  static constexpr int STEPS = TW / TPS;                          // 8 for every D
  static constexpr int SUB_BYTES = T * 128;
  static constexpr int TILE_BYTES = T * D * 2;                    // one of K or V
};

template <int D, int GC>
__global__ void __launch_bounds__(NTHREADS, 2)
    simt_partition_kernel(const __grid_constant__ CUtensorMap k_map,
                          const __grid_constant__ CUtensorMap v_map,
                          const PartitionParams p) {
  using S = SimtShape<D>;
  using L = PartitionSmem<D, S::T, NS, NC, GC>;
  constexpr int T = S::T, TW = S::TW, LPT = S::LPT, TPS = S::TPS, STEPS = S::STEPS;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *kbuf = smem;
  uint8_t *vbuf = smem + NS * S::TILE_BYTES;
  float *comb_acc = reinterpret_cast<float *>(smem + L::KV_BYTES);
  float *comb_ml = comb_acc + L::ACC_FLOATS;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFFSET);
  uint64_t *empty = full + NS;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG_OFFSET);
  const ItemRing ring = item_ring<L>(smem);
  static_assert(L::BYTES <= kTwoCtaSmemBytes, "two CTAs per SM");
  if (!smem_base_aligned(smem, p.fault)) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    ring_init(ring);
    *abort_flag = 0;
    mbar_init_fence();
  }
  __syncthreads();
  // Launched with programmatic stream serialization: the set-up above may
  // overlap the previous kernel; its outputs (q, lengths, block table, the
  // workspace and scheduler words it may still read) are touched only after
  // it has completed.  Only then may the merge kernel that follows be
  // scheduled: everything before this kernel has completed and is visible,
  // so the merge can read the lengths before its own wait (it waits for this
  // grid only to read the workspace).
  grid_dependency_wait();
  allow_dependent_launch();

  if (warp == 0) {
    run_producer<D, T, NS>(&k_map, &v_map, p, kbuf, vbuf, full, empty, abort_flag, ring, lane);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int tg = lane / LPT;          // row within a warp step
  const int j = lane % LPT;           // 16-byte chunk of the row
  const int jsub = j >> 3, jc = j & 7;
  const uint32_t kbase = smem_u32(kbuf) + jsub * S::SUB_BYTES;
  const uint32_t vbase = smem_u32(vbuf) + jsub * S::SUB_BYTES;
  const int tid = cw * 32 + lane;
  uint32_t it = 0;

  uint32_t ik = 0;
  while (true) {
    const WorkItem w = consumer_next<NC>(ring, ik, cw, lane, p.fault, abort_flag);
    if (w.kind == ITEM_STOP) break;
    int h0, rows;
    item_heads<GC>(p, w.hs, h0, rows);
    if (w.kind == ITEM_FILL) {
      store_fill<D>(p, w, h0, rows, tid, NC * 32);
      if (w.last) break;
      continue;
    }
    // q chunk j of every head of the sub-group, as FP32 pairs.
    float2 q2[GC][4];
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      uint32_t raw[4] = {0u, 0u, 0u, 0u};
      if (g < rows) {
        const __nv_bfloat16 *src =
            p.q + (int64_t)w.b * p.q_stride_batch + (int64_t)(h0 + g) * p.q_stride_head + j * 8;
        if (p.q_vec16) {
          const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src));
          raw[0] = v.x; raw[1] = v.y; raw[2] = v.z; raw[3] = v.w;
        } else {
          const unsigned short *s16 = reinterpret_cast<const unsigned short *>(src);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            raw[e] = (uint32_t)__ldg(s16 + 2 * e) | ((uint32_t)__ldg(s16 + 2 * e + 1) << 16);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) q2[g][e] = bf16x2_to_float2(raw[e]);
    }

    float m[GC], l[GC];
    float2 acc[GC][4];
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] = make_float2(0.f, 0.f);
    }

    const int t0 = w.start / T * T;
    const int ntiles = (w.stop - t0 + T - 1) / T;
    const int r0 = cw * TW;
    for (int i = 0; i < ntiles; ++i, ++it) {
      const int s = it % NS;
      // On a failed wait the tile is garbage but the warp keeps going, so
      // all consumer warps still meet at the named barriers below; the
      // fault word tells the host the results are invalid.
      pipeline_wait(&full[s], (it / NS) & 1, p.fault, FAULT_CONSUMER_FULL_WAIT, abort_flag);
      const int tile_tok = t0 + i * T;
      const int lo = max(w.start - tile_tok, 0);
      const int hi = min(w.stop - tile_tok, T);
      if (r0 < hi && r0 + TW > lo) {
        const uint32_t ks = kbase + s * S::TILE_BYTES;
        const uint32_t vs = vbase + s * S::TILE_BYTES;
        float sc[STEPS][GC];
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
          const int r = r0 + st * TPS + tg;
          const uint4 raw = lds128(ks + swizzle128(r, jc));
          const float2 k0 = bf16x2_to_float2(raw.x), k1 = bf16x2_to_float2(raw.y);
          const float2 k2 = bf16x2_to_float2(raw.z), k3 = bf16x2_to_float2(raw.w);
          float part[GC];
#pragma unroll
          for (int g = 0; g < GC; ++g) {
            float2 a = __fmul2_rn(q2[g][0], k0);
            a = __ffma2_rn(q2[g][1], k1, a);
            a = __ffma2_rn(q2[g][2], k2, a);
            a = __ffma2_rn(q2[g][3], k3, a);
            part[g] = a.x + a.y;
          }
#pragma unroll
          for (int o = LPT / 2; o >= 1; o >>= 1) {
#pragma unroll
            for (int g = 0; g < GC; ++g) part[g] += __shfl_xor_sync(FULL_MASK, part[g], o);
          }
          const bool valid = r >= lo && r < hi;
#pragma unroll
          for (int g = 0; g < GC; ++g) sc[st][g] = valid ? part[g] * p.log2_scale : -INFINITY;
        }
        // One running max per warp and head: tile max, then a single rescale.
#pragma unroll
        for (int g = 0; g < GC; ++g) {
          float mt = sc[0][g];
#pragma unroll
          for (int st = 1; st < STEPS; ++st) mt = fmaxf(mt, sc[st][g]);
#pragma unroll
          for (int o = LPT; o < 32; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(FULL_MASK, mt, o));
          const float mn = fmaxf(m[g], mt);
          const float alpha = fast_exp2(m[g] - mn);
          m[g] = mn;
          l[g] *= alpha;
          const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[g][e] = __fmul2_rn(acc[g][e], a2);
        }
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
          const int r = r0 + st * TPS + tg;
          const bool valid = r >= lo && r < hi;
          uint4 raw = lds128(vs + swizzle128(r, jc));
          if (!valid) raw = make_uint4(0u, 0u, 0u, 0u);  // dead slots may hold NaN
          const float2 v0 = bf16x2_to_float2(raw.x), v1 = bf16x2_to_float2(raw.y);
          const float2 v2 = bf16x2_to_float2(raw.z), v3 = bf16x2_to_float2(raw.w);
#pragma unroll
          for (int g = 0; g < GC; ++g) {
            const float pr = fast_exp2(sc[st][g] - m[g]);
            l[g] += pr;
            const float2 p2 = make_float2(pr, pr);
            acc[g][0] = __ffma2_rn(p2, v0, acc[g][0]);
            acc[g][1] = __ffma2_rn(p2, v1, acc[g][1]);
            acc[g][2] = __ffma2_rn(p2, v2, acc[g][2]);
            acc[g][3] = __ffma2_rn(p2, v3, acc[g][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- merge the rows of this warp (same max), then the warps.
#pragma unroll
    for (int o = LPT; o < 32; o <<= 1) {
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        l[g] += __shfl_xor_sync(FULL_MASK, l[g], o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[g][e].x += __shfl_xor_sync(FULL_MASK, acc[g][e].x, o);
          acc[g][e].y += __shfl_xor_sync(FULL_MASK, acc[g][e].y, o);
        }
      }
    }
    float *mine = comb_acc + cw * GC * D;
    if (tg == 0) {
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        float4 *dst = reinterpret_cast<float4 *>(mine + g * D + comb_col(g, j * 8));
        dst[0] = make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
        dst[1] = make_float4(acc[g][2].x, acc[g][2].y, acc[g][3].x, acc[g][3].y);
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        comb_ml[cw * 2 * GC + g] = m[g];
        comb_ml[cw * 2 * GC + GC + g] = l[g];
      }
    }
    if (!w.last) ring_peek(ring, ik, cw == 0 && lane == 0);
    named_barrier(1, NC * 32);
    if (!w.last) {  // a CTA's last item has no next one to prepare
      // The next item's q chunks into L1 while this one is combined.
      const WorkItem nx = peeked_item(ring, ik);
      if (nx.kind == ITEM_COMPUTE) {
        int nh0, nrows;
        item_heads<GC>(p, nx.hs, nh0, nrows);
#pragma unroll
        for (int g = 0; g < GC; ++g)
          if (g < nrows)
            prefetch_l1(p.q + (int64_t)nx.b * p.q_stride_batch +
                        (int64_t)(nh0 + g) * p.q_stride_head + j * 8);
      }
    }
    combine_and_store<D, GC, NC>(p, w, h0, rows, comb_acc, comb_ml, tid);
    if (w.last) break;
    named_barrier(1, NC * 32);  // the combine area is rewritten by the next item
  }
}

template <int D, int GC>
cudaError_t launch_simt_t(const KernelLaunch &L, cudaStream_t stream) {
  auto kernel = simt_partition_kernel<D, GC>;
  constexpr int smem = PartitionSmem<D, SimtShape<D>::T, NS, NC, GC>::BYTES;
  static int blocks_per_sm[kMaxDevices] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (blocks_per_sm[dev] == 0) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    int n = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, NTHREADS, smem);
    if (err != cudaSuccess) return err;
    blocks_per_sm[dev] = n < 1 ? 1 : n;
  }
  const int grid = min(L.params.n_items, blocks_per_sm[dev] * L.sm_count);
  if (grid <= 0) return cudaSuccess;
  PartitionParams params = L.params;
  params.live = live_schedule(params, grid);
  return launch_programmatic(kernel, dim3(grid), dim3(NTHREADS), smem, stream, *L.k_map, *L.v_map, params);
}

template <int D>
cudaError_t launch_simt_d(const KernelLaunch &L, cudaStream_t stream) {
  switch (L.group_per_cta) {
    case 1: return launch_simt_t<D, 1>(L, stream);
    case 2: return launch_simt_t<D, 2>(L, stream);
    case 4: return launch_simt_t<D, 4>(L, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int simt_heads_per_cta(int group) { return group >= 3 ? 4 : group; }

int simt_tile_tokens(int head_dim) {
  return head_dim == 64 ? SimtShape<64>::T : (head_dim == 128 ? SimtShape<128>::T
                                                              : SimtShape<256>::T);
}

cudaError_t launch_partition_simt(const KernelLaunch &L, cudaStream_t stream) {
  switch (L.head_dim) {
    case 64: return launch_simt_d<64>(L, stream);
    case 128: return launch_simt_d<128>(L, stream);
    case 256: return launch_simt_d<256>(L, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pdl
