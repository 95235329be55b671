// pdl_partition_mma.cu -- BF16 tensor-core split-K partition kernel (sm_100a).
//
// Same work items, persistent CTAs and TMA producer warp as the CUDA-core
// kernel; the consumers use warp-level mma.sync.m16n8k16 (BF16 in, FP32
// accumulate) with the head group as the N dimension, so 8 query heads that
// share a KV head form one dense N=8 tile:
//
//   S^T[16 tokens, 8 heads] = K[16 tokens, D] . Q^T[D, 8 heads]
//       A = K rows from the swizzled tile (ldmatrix), B = q in registers.
//   online softmax on S^T in FP32 (per-head max over a warp's tokens via
//       three xor shuffles; exp2 with the scale folded in).
//   O^T[D, 8 heads] += V^T[D, 16 tokens] . P^T[16 tokens, 8 heads]
//       A = V rows loaded transposed (ldmatrix.trans), B = P^T obtained from
//       the S^T accumulator registers with movmatrix.trans.  P is split into
//       BF16 hi + lo parts (two MMAs) so P.V keeps FP32-level accuracy.
//
// Consumer warps come in NG token groups of DS warps.  Each group owns 16*MT
// rows of every T-token tile and its own running (m, l, O).  At D = 256 the
// two warps of a group (DS = 2) split D: each multiplies its half of D for
// the scores, the two halves are exchanged through shared memory and added
// (s_a + s_b in one warp, s_b + s_a in the other: the same bits), so both
// warps hold identical scores, m, l and P; each then keeps the O columns of
// its half of D.  The q.k and P.V work per warp are both halved.  The groups are merged at the end of an item
// through shared memory (combine_and_store).  Rows outside the partition or beyond
// the live length are masked: scores to -inf, V fragment halves to zero
// (dead page slots may hold NaN).
//
// Replaces the reference's tensor-core kernels _tc_partition
// (src/paged_decode/tc_splitk.py:13-60), _tensorcore
// (src/paged_decode/experimental_precision.py:46-107) and, for groups >= 8,
// _normalized_partition (src/paged_decode/matched_splitkv.py:52-98).
#include "pdl_pipeline.cuh"

namespace pdl {
namespace {

template <int D>
struct MmaShape {
  static constexpr int NG = D == 256 ? 2 : 4;                      // token groups
  static constexpr int DS = D == 256 ? 2 : 1;                      // warps per group (D split)
  static constexpr int NC = NG * DS;                               // consumer warps
  static constexpr int T = D == 64 ? 128 : (D == 128 ? 64 : 32);   // tokens per stage
  static constexpr int TW = T / NG;                                // rows per group per stage
  static constexpr int MT = TW / 16;                               // 16-row MMA tiles per warp
  static constexpr int KS = D / 16;                                // 16-column slices of D
  static constexpr int KSW = KS / DS;                              // slices of O per warp
  static constexpr int KQ = KS / DS;                               // slices of q.k per warp
  static constexpr int SUB_BYTES = T * 128;
  static constexpr int TILE_BYTES = T * D * 2;
  static constexpr int NTHREADS = 32 * (NC + 1);
};

// Stages: 3 when two CTAs still fit one SM, else 2.  The combine area holds
// one partial state per token group.
template <int D, int GC>
struct MmaStages {
  static constexpr int NG = MmaShape<D>::NG, T = MmaShape<D>::T;
  static constexpr int NS = PartitionSmem<D, T, 3, NG, GC>::BYTES <= kTwoCtaSmemBytes ? 3 : 2;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// d += a . b  (m16n8k16, BF16 inputs, FP32 accumulators)
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

// Two consecutive BF16 of a q row (4-byte aligned when `vec`).
__device__ __forceinline__ uint32_t load_q_pair(const __nv_bfloat16 *src, bool vec) {
  if (vec) return __ldg(reinterpret_cast<const uint32_t *>(src));
  const unsigned short *s16 = reinterpret_cast<const unsigned short *>(src);
  return (uint32_t)__ldg(s16) | ((uint32_t)__ldg(s16 + 1) << 16);
}

template <int D, int NT, bool PRECISE>
__global__ void __launch_bounds__(MmaShape<D>::NTHREADS, 2)
    mma_partition_kernel(const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map,
                         const PartitionParams p) {
  using S = MmaShape<D>;
  constexpr int GC = 8 * NT;
  constexpr int NS = MmaStages<D, GC>::NS;
  using L = PartitionSmem<D, S::T, NS, S::NG, GC>;
  constexpr int NC = S::NC, NG = S::NG, DS = S::DS, T = S::T, TW = S::TW, MT = S::MT;
  constexpr int KSW = S::KSW, KQ = S::KQ;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *kbuf = smem;
  uint8_t *vbuf = smem + NS * S::TILE_BYTES;
  float *comb_acc = reinterpret_cast<float *>(smem + L::KV_BYTES);
  float *comb_ml = comb_acc + L::ACC_FLOATS;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFFSET);
  uint64_t *empty = full + NS;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG_OFFSET);
  const ItemRing ring = item_ring<L>(smem);
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
  const int tg = cw / DS, dh = cw % DS;  // token group, half of D (DS = 2)
  const int tid = cw * 32 + lane;
  const int quad = lane & 3, grp = lane >> 2;  // MMA fragment coordinates
  // ldmatrix row providers: lane -> (matrix mi, row rr).
  const int mi = lane >> 3, rr = lane & 7;
  const int k_row = rr + (mi & 1) * 8, k_chunk = mi >> 1;  // K: A[token][dim]
  const int v_row = rr + (mi >> 1) * 8, v_chunk = mi & 1;  // V: A = V^T via .trans
  const uint32_t kbase = smem_u32(kbuf), vbase = smem_u32(vbuf);
  const bool q_vec = p.q_vec16 != 0;
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
    // q of head (nt*8 + grp) as B fragments for this warp's slices of D
    // (kk = dh * KQ + kq): dims kk*16 + quad*2 + {0,1} and +8.
    uint32_t qf[NT][KQ][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int hl = nt * 8 + grp;
      const bool valid = hl < rows;
      const __nv_bfloat16 *qrow =
          p.q + (int64_t)w.b * p.q_stride_batch + (int64_t)(h0 + (valid ? hl : 0)) * p.q_stride_head;
#pragma unroll
      for (int kq = 0; kq < KQ; ++kq) {
        const int kk = dh * KQ + kq;
        qf[nt][kq][0] = valid ? load_q_pair(qrow + kk * 16 + quad * 2, q_vec) : 0u;
        qf[nt][kq][1] = valid ? load_q_pair(qrow + kk * 16 + quad * 2 + 8, q_vec) : 0u;
      }
    }

    // Running state for heads nt*8 + quad*2 + {0,1}; acc[nt][j] holds O^T
    // rows (dh*KSW + j)*16 + grp (+8) for those two heads.
    float m[NT][2], l[NT][2], acc[NT][KSW][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int dm = 0; dm < KSW; ++dm) acc[nt][dm][0] = acc[nt][dm][1] = acc[nt][dm][2] = acc[nt][dm][3] = 0.f;
    }

    const int t0 = w.start / T * T;
    const int ntiles = (w.stop - t0 + T - 1) / T;
    const int r0 = tg * TW;
    for (int i = 0; i < ntiles; ++i, ++it) {
      const int s = it % NS;
      pipeline_wait(&full[s], (it / NS) & 1, p.fault, FAULT_CONSUMER_FULL_WAIT, abort_flag);
      const int tile_tok = t0 + i * T;
      const int lo = max(w.start - tile_tok, 0);
      const int hi = min(w.stop - tile_tok, T);
      if (r0 < hi && r0 + TW > lo) {
        const uint32_t ks = kbase + s * S::TILE_BYTES;
        const uint32_t vs = vbase + s * S::TILE_BYTES;
        // ---- S^T = K . Q^T over this warp's slices of D, accumulated in CH
        // independent chains (slices interleaved) so consecutive MMAs do not
        // wait on each other.
        constexpr int CH = KQ >= 16 ? 4 : 2;
        float part[CH][MT][NT][4];
#pragma unroll
        for (int c = 0; c < CH; ++c)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              part[c][mt][nt][0] = part[c][mt][nt][1] = part[c][mt][nt][2] = part[c][mt][nt][3] = 0.f;
#pragma unroll
        for (int kq = 0; kq < KQ; ++kq) {
          const int chunk = (dh * KQ + kq) * 2 + k_chunk;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            uint32_t a[4];
            ldsm_x4(ks + (chunk >> 3) * S::SUB_BYTES + swizzle128(r0 + mt * 16 + k_row, chunk & 7), a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              mma_bf16(part[kq % CH][mt][nt], a, qf[nt][kq][0], qf[nt][kq][1]);
          }
        }
        float sc[MT][NT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float v = part[0][mt][nt][e];
#pragma unroll
              for (int c = 1; c < CH; ++c) v += part[c][mt][nt][e];
              sc[mt][nt][e] = v;
            }
        if constexpr (DS == 2) {
          // Exchange the halves with the other warp of the pair through a
          // slot of the combine area (unused during the tiles), double
          // buffered by tile parity so a warp one tile ahead never overwrites
          // what its partner still reads.
          constexpr int E = MT * NT * 4;
          static_assert(NG * 2 * 2 * 32 * E <= NG * GC * D, "exchange slots fit the combine area");
          float *xmine = comb_acc + ((((tg * 2 + dh) * 2 + (i & 1)) * 32) + lane) * E;
          const float *xpeer = comb_acc + ((((tg * 2 + (dh ^ 1)) * 2 + (i & 1)) * 32) + lane) * E;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              *reinterpret_cast<float4 *>(xmine + (mt * NT + nt) * 4) =
                  make_float4(sc[mt][nt][0], sc[mt][nt][1], sc[mt][nt][2], sc[mt][nt][3]);
          // One named barrier per pair (ids 2, 3: compile-time constants, so
          // the kernel reserves 4 barriers, not all 16).
          static_assert(NG == 2, "pair barriers 2 and 3");
          if (tg == 0)
            named_barrier(2, 64);
          else
            named_barrier(3, 64);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const float4 o = *reinterpret_cast<const float4 *>(xpeer + (mt * NT + nt) * 4);
              sc[mt][nt][0] += o.x;
              sc[mt][nt][1] += o.y;
              sc[mt][nt][2] += o.z;
              sc[mt][nt][3] += o.w;
            }
        }
        // ---- mask rows outside [lo, hi) and fold in the scale (base 2)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int ta = r0 + mt * 16 + grp, tb = ta + 8;
          const bool va = ta >= lo && ta < hi, vb = tb >= lo && tb < hi;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            sc[mt][nt][0] = va ? sc[mt][nt][0] * p.log2_scale : -INFINITY;
            sc[mt][nt][1] = va ? sc[mt][nt][1] * p.log2_scale : -INFINITY;
            sc[mt][nt][2] = vb ? sc[mt][nt][2] * p.log2_scale : -INFINITY;
            sc[mt][nt][3] = vb ? sc[mt][nt][3] * p.log2_scale : -INFINITY;
          }
        }
        // ---- per-head tile max over the warp's rows, one rescale per tile
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float mx = fmaxf(sc[0][nt][j], sc[0][nt][j + 2]);
#pragma unroll
            for (int mt = 1; mt < MT; ++mt) mx = fmaxf(mx, fmaxf(sc[mt][nt][j], sc[mt][nt][j + 2]));
            mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, 16));
            const float mn = fmaxf(m[nt][j], mx);
            const float alpha = fast_exp2(m[nt][j] - mn);
            m[nt][j] = mn;
            l[nt][j] *= alpha;
#pragma unroll
            for (int dm = 0; dm < KSW; ++dm) {
              acc[nt][dm][j] *= alpha;
              acc[nt][dm][j + 2] *= alpha;
            }
          }
        }
        // ---- probabilities -> B fragments of P^T (hi and lo BF16 parts)
        uint32_t bh[MT][NT][2], bl[MT][NT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float p0 = fast_exp2(sc[mt][nt][0] - m[nt][0]);
            const float p1 = fast_exp2(sc[mt][nt][1] - m[nt][1]);
            const float p2 = fast_exp2(sc[mt][nt][2] - m[nt][0]);
            const float p3 = fast_exp2(sc[mt][nt][3] - m[nt][1]);
            l[nt][0] += p0 + p2;
            l[nt][1] += p1 + p3;
            const uint32_t x0 = pack_bf16(p0, p1), x1 = pack_bf16(p2, p3);
            bh[mt][nt][0] = movmatrix_trans(x0);
            bh[mt][nt][1] = movmatrix_trans(x1);
            if (PRECISE) {
              bl[mt][nt][0] = movmatrix_trans(pack_bf16(p0 - bf16_lo(x0), p1 - bf16_hi(x0)));
              bl[mt][nt][1] = movmatrix_trans(pack_bf16(p2 - bf16_lo(x1), p3 - bf16_hi(x1)));
            }
          }
        }
        // ---- O^T += V^T . P^T (this warp's half of D when DS = 2)
        const bool edge = r0 < lo || r0 + TW > hi;
#pragma unroll
        for (int dw = 0; dw < KSW; ++dw) {
          const int chunk = (dh * KSW + dw) * 2 + v_chunk;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            uint32_t a[4];
            ldsm_x4_trans(vs + (chunk >> 3) * S::SUB_BYTES + swizzle128(r0 + mt * 16 + v_row, chunk & 7), a);
            if (edge) {
              // a[0], a[1]: rows quad*2 + {0,1}; a[2], a[3]: rows 8 + quad*2 + {0,1}
              const int t = r0 + mt * 16 + quad * 2;
              const uint32_t m01 = ((t >= lo && t < hi) ? 0x0000ffffu : 0u) |
                                   ((t + 1 >= lo && t + 1 < hi) ? 0xffff0000u : 0u);
              const uint32_t m23 = ((t + 8 >= lo && t + 8 < hi) ? 0x0000ffffu : 0u) |
                                   ((t + 9 >= lo && t + 9 < hi) ? 0xffff0000u : 0u);
              a[0] &= m01;
              a[1] &= m01;
              a[2] &= m23;
              a[3] &= m23;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma_bf16(acc[nt][dw], a, bh[mt][nt][0], bh[mt][nt][1]);
              if (PRECISE) mma_bf16(acc[nt][dw], a, bl[mt][nt][0], bl[mt][nt][1]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- per-warp state -> shared memory, then merge the warps
    // (at D = 256 the combine area held the score exchange: every pair is
    // done with it first)
    if constexpr (DS == 2) named_barrier(1, NC * 32);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float v = l[nt][j];
        v += __shfl_xor_sync(FULL_MASK, v, 4);
        v += __shfl_xor_sync(FULL_MASK, v, 8);
        v += __shfl_xor_sync(FULL_MASK, v, 16);
        l[nt][j] = v;
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int g = nt * 8 + quad * 2 + j;
        float *dst = comb_acc + (tg * GC + g) * D;
        const int c0 = dh * KSW * 16 + grp;
#pragma unroll
        for (int dm = 0; dm < KSW; ++dm) {
          dst[comb_col(g, c0 + dm * 16)] = acc[nt][dm][j];
          dst[comb_col(g, c0 + dm * 16 + 8)] = acc[nt][dm][j + 2];
        }
        if (grp == 0 && dh == 0) {
          comb_ml[tg * 2 * GC + nt * 8 + quad * 2 + j] = m[nt][j];
          comb_ml[tg * 2 * GC + GC + nt * 8 + quad * 2 + j] = l[nt][j];
        }
      }
    }
    if (!w.last) ring_peek(ring, ik, cw == 0 && lane == 0);
    named_barrier(1, NC * 32);
    if (!w.last) {  // a CTA's last item has no next one to prepare
      // The next item's q rows into L1 while this one is combined (each of a
      // row's D/64 lines by one of the four lanes that load it).
      const WorkItem nx = peeked_item(ring, ik);
      if (nx.kind == ITEM_COMPUTE) {
        int nh0, nrows;
        item_heads<GC>(p, nx.hs, nh0, nrows);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          if (nt * 8 + grp < nrows)
            prefetch_l1(p.q + (int64_t)nx.b * p.q_stride_batch +
                        (int64_t)(nh0 + nt * 8 + grp) * p.q_stride_head + (quad % (D / 64)) * 64);
      }
    }
    combine_and_store<D, GC, NG, NC>(p, w, h0, rows, comb_acc, comb_ml, tid);
    if (w.last) break;
    named_barrier(1, NC * 32);  // the combine area is rewritten by the next item
  }
}

template <int D, int NT>
cudaError_t launch_mma_t(const KernelLaunch &L, cudaStream_t stream) {
  using S = MmaShape<D>;
  constexpr int GC = 8 * NT;
  auto kernel = mma_partition_kernel<D, NT, true>;
  constexpr int smem = PartitionSmem<D, S::T, MmaStages<D, GC>::NS, S::NG, GC>::BYTES;
  static int blocks_per_sm[kMaxDevices] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (blocks_per_sm[dev] == 0) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    int n = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, S::NTHREADS, smem);
    if (err != cudaSuccess) return err;
    blocks_per_sm[dev] = n < 1 ? 1 : n;
  }
  const int grid = min(L.params.n_items, blocks_per_sm[dev] * L.sm_count);
  if (grid <= 0) return cudaSuccess;
  PartitionParams params = L.params;
  params.live = live_schedule(params, grid);
  return launch_programmatic(kernel, dim3(grid), dim3(S::NTHREADS), smem, stream, *L.k_map, *L.v_map, params);
}

template <int D>
cudaError_t launch_mma_d(const KernelLaunch &L, cudaStream_t stream) {
  switch (L.group_per_cta) {
    case 8: return launch_mma_t<D, 1>(L, stream);
    case 16:
      if constexpr (D != 256) return launch_mma_t<D, 2>(L, stream);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int mma_heads_per_cta(int group, int head_dim) {
  if (group <= 8 || head_dim == 256) return 8;
  return 16;
}

int mma_tile_tokens(int head_dim) {
  return head_dim == 64 ? MmaShape<64>::T : (head_dim == 128 ? MmaShape<128>::T
                                                             : MmaShape<256>::T);
}

cudaError_t launch_partition_mma(const KernelLaunch &L, cudaStream_t stream) {
  switch (L.head_dim) {
    case 64: return launch_mma_d<64>(L, stream);
    case 128: return launch_mma_d<128>(L, stream);
    case 256: return launch_mma_d<256>(L, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pdl
