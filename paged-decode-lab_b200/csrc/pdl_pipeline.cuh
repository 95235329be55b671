// pdl_pipeline.cuh -- pieces shared by the partition kernels: work-item
// decoding, the TMA producer warp, stores for empty partitions, and the
// merge of the consumer warps' softmax states into the stored outputs.
#pragma once

#include "pdl_device.cuh"

namespace pdl {

struct Item {
  int b, kvh, sub, split;
};

// Static order:  item = ((b * num_kv_heads + kvh) * nsub + sub) * splits + split
// (a CTA's consecutive items are neighbouring partitions of one row).
// Dynamic order: item = split * (batch * num_kv_heads * nsub) + group, so every
// row's first partition is handed out before any row's second one and the
// last items are the tail partitions of the longest rows.
__device__ __forceinline__ Item decode_item(const PartitionParams &p, int item) {
  Item it;
  const int per_row = p.num_kv_heads * p.nsub;
  int rest;
  if (p.sched != nullptr) {
    const int groups = p.batch * per_row;
    it.split = item / groups;
    rest = item % groups;
  } else {
    it.split = item % p.splits;
    rest = item / p.splits;
  }
  it.b = rest / per_row;
  const int r = rest % per_row;
  it.kvh = r / p.nsub;
  it.sub = r % p.nsub;
  return it;
}

// Token range [start, stop) of an item; empty when start >= stop.  Lengths
// beyond the table capacity are clamped to it, so no table entry past the
// row's width is ever read.
struct Range {
  int start, stop;
};

__device__ __forceinline__ Range item_range(const PartitionParams &p, const Item &w) {
  const int len = min(__ldg(p.lengths + w.b), p.table_width * 256);
  const int64_t start = (int64_t)w.split * p.tokens_per_split;
  const int64_t stop = min((int64_t)len, start + p.tokens_per_split);
  Range r;
  r.start = start >= stop ? 0 : (int)start;
  r.stop = start >= stop ? 0 : (int)stop;
  return r;
}

// Stores for a partition with no live tokens: partial 0 / LSE -inf,
// (m, l, acc) = (-inf, 0, 0), or a zero output row.
template <int D>
__device__ void store_empty(const PartitionParams &p, int b, int h0, int rows, int split,
                            int tid, int nthreads) {
  for (int e = tid; e < rows * D; e += nthreads) {
    const int g = e / D, d = e % D;
    const int64_t row = (int64_t)b * p.num_heads + h0 + g;
    const int64_t idx = row * p.splits + split;
    if (p.mode == MODE_LSE) {
      p.partial[idx * D + d] = 0.f;
      if (d == 0) p.lse[idx] = -INFINITY;
    } else if (p.mode == MODE_MLA) {
      p.accums[idx * D + d] = 0.f;
      if (d == 0) {
        p.maxima[idx] = -INFINITY;
        p.denoms[idx] = 0.f;
      }
    } else {
      p.out[row * D + d] = __float2bfloat16_rn(0.f);
    }
  }
}

// ------------------------------------------------------------- work items
// Static scheduling: CTA c takes items c, c + gridDim.x, ...  Dynamic
// scheduling (p.sched != null): the producer warp takes the next item from a
// global atomic counter and publishes it in an IR-deep shared-memory ring;
// one consumer thread (the leader) takes it from the ring and hands it to all
// consumer warps through a named barrier, so every warp processes the same
// sequence even if a bounded wait gives up (the leader then hands out "stop").
constexpr int IR = 8;

struct ItemRing {
  uint64_t *full;       // [IR] producer -> consumers, count 1
  uint64_t *empty;      // [IR] consumers -> producer, count 1 (the leader)
  volatile int *slot;   // [IR] item indices (-1 = no more items)
  volatile int *shared; // item handed to the consumer warps
};

__device__ __forceinline__ void ring_init(const ItemRing &r) {
  for (int i = 0; i < IR; ++i) {
    mbar_init(&r.full[i], 1);
    mbar_init(&r.empty[i], 1);
  }
}

// Next item of the producer warp (all lanes return it); -1 when done.
__device__ __forceinline__ int producer_next(const PartitionParams &p, const ItemRing &r,
                                             uint32_t &k, int &static_next, int lane,
                                             volatile int *abort_flag) {
  if (p.sched == nullptr) {
    const int item = static_next;
    static_next += gridDim.x;
    return item < p.n_items ? item : -1;
  }
  int item = -1;
  if (lane == 0) {
    item = atomicAdd(p.sched, 1);
    if (item >= p.n_items) item = -1;
    const int s = k % IR;
    if (k >= IR)
      pipeline_wait(&r.empty[s], ((k / IR) & 1) ^ 1, p.fault, FAULT_PRODUCER_EMPTY_WAIT, abort_flag);
    r.slot[s] = item;
    mbar_arrive(&r.full[s]);
  }
  ++k;
  return __shfl_sync(FULL_MASK, item, 0);
}

// The producer's exit: count this CTA as finished; the last one resets the
// scheduler words for the next launch (every CTA's final fetch precedes its
// count, and no fetch follows the last count).
__device__ __forceinline__ void producer_finish(const PartitionParams &p, int lane) {
  if (p.sched == nullptr || lane != 0) return;
  __threadfence();
  if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
    atomicExch(p.sched, 0);
    atomicExch(p.sched + 1, 0);
  }
}

// Next item of the consumer warps (identical in every consumer warp); -1 when done.
template <int NC>
__device__ __forceinline__ int consumer_next(const PartitionParams &p, const ItemRing &r,
                                             uint32_t &k, int &static_next, int cw, int lane,
                                             volatile int *abort_flag) {
  if (p.sched == nullptr) {
    const int item = static_next;
    static_next += gridDim.x;
    return item < p.n_items ? item : -1;
  }
  if (cw == 0 && lane == 0) {
    const int s = k % IR;
    int item = -1;
    if (pipeline_wait(&r.full[s], (k / IR) & 1, p.fault, FAULT_CONSUMER_FULL_WAIT, abort_flag))
      item = r.slot[s];
    *r.shared = (item >= 0 && item < p.n_items) ? item : -1;
    mbar_arrive(&r.empty[s]);
  }
  ++k;
  named_barrier(1, NC * 32);
  const int item = *r.shared;
  named_barrier(1, NC * 32);  // all warps read it before the leader writes the next one
  return item;
}

// Producer warp: for every item of this CTA, in the consumers' order, read
// the partition's block-table entries (32 per load, one per lane, never past
// the table width; only entries of live pages are used) and issue one
// T-token tile of K and V per stage as D/64 TMA boxes each.  T divides 256,
// so a tile never spans two pages.
template <int D, int T, int NS>
__device__ void run_producer(const CUtensorMap *k_map, const CUtensorMap *v_map,
                             const PartitionParams &p, uint8_t *kbuf, uint8_t *vbuf,
                             uint64_t *full, uint64_t *empty, volatile int *abort_flag,
                             const ItemRing &ring, int lane) {
  constexpr int SUBTILES = D / 64;
  constexpr int SUB_BYTES = T * 128;
  constexpr int TILE_BYTES = T * D * 2;
  const uint64_t policy = l2_evict_first_policy();
  if (lane == 0) {
    prefetch_tensormap(k_map);
    prefetch_tensormap(v_map);
  }
  uint32_t it = 0, k = 0;
  int static_next = blockIdx.x;
  bool ok = true;
  while (ok) {
    const int item = producer_next(p, ring, k, static_next, lane, abort_flag);
    if (item < 0) break;
    const Item w = decode_item(p, item);
    // The first 32 table entries of the partition are read together with the
    // row length (speculatively, but never past the table's width), so the
    // two round trips overlap; entries past the live pages are never used.
    const int32_t *trow = p.table + (int64_t)w.b * p.table_stride;
    const int64_t first_tok = (int64_t)w.split * p.tokens_per_split;
    int base = first_tok < (int64_t)p.table_width * 256 ? (int)(first_tok >> 8) : -64;
    int my_page = (base >= 0 && base + lane < p.table_width) ? __ldg(trow + base + lane) : 0;
    const Range r = item_range(p, w);
    if (r.start >= r.stop) continue;
    const int t0 = r.start / T * T;
    const int ntiles = (r.stop - t0 + T - 1) / T;
    for (int i = 0; i < ntiles; ++i, ++it) {
      const int tok = t0 + i * T;
      const int pg = tok >> 8;
      if (base < 0 || pg >= base + 32) {
        base = pg;
        my_page = (pg + lane < p.table_width) ? __ldg(trow + pg + lane) : 0;
      }
      const int page = __shfl_sync(FULL_MASK, my_page, pg - base);
      if (lane == 0) {
        const int s = it % NS;
        if (it >= NS && !pipeline_wait(&empty[s], ((it / NS) & 1) ^ 1, p.fault,
                                       FAULT_PRODUCER_EMPTY_WAIT, abort_flag)) {
          ok = false;
        } else {
          mbar_arrive_expect_tx(&full[s], 2 * TILE_BYTES);
#pragma unroll
          for (int st = 0; st < SUBTILES; ++st) {
            tma_load_4d(kbuf + s * TILE_BYTES + st * SUB_BYTES, k_map, st * 64, w.kvh, tok & 255,
                        page, &full[s], policy);
            tma_load_4d(vbuf + s * TILE_BYTES + st * SUB_BYTES, v_map, st * 64, w.kvh, tok & 255,
                        page, &full[s], policy);
          }
        }
      }
      ok = __shfl_sync(FULL_MASK, ok, 0);
      if (!ok) break;
    }
  }
  if (!ok && lane == 0) {
    // Let the copies already issued land before the CTA exits, and tell the
    // consumers there is nothing more.
    const uint32_t first = it > NS ? it - NS : 0;
    for (uint32_t j = first; j < it; ++j)
      mbar_wait_bounded(&full[j % NS], (j / NS) & 1, p.fault, FAULT_DRAIN_WAIT);
  }
  if (!ok && p.sched != nullptr && lane == 0) {
    while (true) {  // publish "stop" so the consumer leader need not time out
      const int s = k % IR;
      if (k >= IR && !mbar_wait_bounded(&ring.empty[s], ((k / IR) & 1) ^ 1, p.fault,
                                        FAULT_PRODUCER_EMPTY_WAIT))
        break;
      ring.slot[s] = -1;
      mbar_arrive(&ring.full[s]);
      break;
    }
  }
  producer_finish(p, lane);
}

// Merge NC per-warp (or per-group) softmax states of one item and store the
// outputs, with the NW consumer warps' threads (tid < NW * 32).
//   comb_acc [NC][GC][D]  unnormalised accumulators (relative to each state's max)
//   comb_ml  [NC][2][GC]  per-state running max (base-2 scaled units) and sum
// M = max_w m_w; f_w = 2^(m_w - M); L = sum f_w l_w; O = sum f_w acc_w.
// Stores O/L + LSE (natural log), (M ln2, L, O), or BF16 O/L.
template <int D, int GC, int NC, int NW = NC>
__device__ void combine_and_store(const PartitionParams &p, const Item &w, int h0, int rows,
                                  const float *comb_acc, const float *comb_ml, int tid) {
  for (int e = tid * 4; e < rows * D; e += NW * 32 * 4) {
    const int g = e / D, d = e % D;
    float mx = -INFINITY;
#pragma unroll
    for (int wi = 0; wi < NC; ++wi) mx = fmaxf(mx, comb_ml[wi * 2 * GC + g]);
    float den = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int wi = 0; wi < NC; ++wi) {
      const float mw = comb_ml[wi * 2 * GC + g];
      const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - mx);
      den += f * comb_ml[wi * 2 * GC + GC + g];
      const float4 a = *reinterpret_cast<const float4 *>(comb_acc + (wi * GC + g) * D + d);
      o.x += f * a.x;
      o.y += f * a.y;
      o.z += f * a.z;
      o.w += f * a.w;
    }
    const int64_t row = (int64_t)w.b * p.num_heads + h0 + g;
    const int64_t idx = row * p.splits + w.split;
    if (p.mode == MODE_MLA) {
      *reinterpret_cast<float4 *>(p.accums + idx * D + d) = o;
      if (d == 0) {
        p.maxima[idx] = mx * LN2;
        p.denoms[idx] = den;
      }
    } else {
      const float inv = 1.f / den;
      o.x *= inv;
      o.y *= inv;
      o.z *= inv;
      o.w *= inv;
      if (p.mode == MODE_LSE) {
        *reinterpret_cast<float4 *>(p.partial + idx * D + d) = o;
        if (d == 0) p.lse[idx] = (mx + log2f(den)) * LN2;
      } else {
        __nv_bfloat162 lo2 = __floats2bfloat162_rn(o.x, o.y);
        __nv_bfloat162 hi2 = __floats2bfloat162_rn(o.z, o.w);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t *>(&lo2);
        packed.y = *reinterpret_cast<uint32_t *>(&hi2);
        *reinterpret_cast<uint2 *>(p.out + row * D + d) = packed;
      }
    }
  }
}

// Fused merge of one (row, KV head, sub-group): the consumer warps of the CTA
// that finished the group's last partition combine its partitions (stored by
// any CTA of this launch, so read through L2 with ld.global.cg) into the BF16
// output, with the arithmetic of merge_kernel (pdl_merge.cu).  Warp w takes
// heads w, w+NC, ...; lane l owns D/32 contiguous columns.
template <int D, int NC>
__device__ void merge_group(const PartitionParams &p, const Item &w, int h0, int rows, int live,
                            int cw, int lane) {
  constexpr int E = D / 32;
  for (int g = cw; g < rows; g += NC) {
    const int64_t row = (int64_t)w.b * p.num_heads + h0 + g;
    const int64_t base = row * p.splits;
    const bool lse_protocol = p.mode == MODE_LSE;
    const float *wsrc = (lse_protocol ? p.lse : p.maxima) + base;
    float mx = -INFINITY;
    for (int s = lane; s < live; s += 32) mx = fmaxf(mx, __ldcg(wsrc + s));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, o));
    if (mx == -INFINITY) mx = 0.f;
    float tot = 0.f;
    for (int s = lane; s < live; s += 32) {
      const float e = expf(__ldcg(wsrc + s) - mx);
      tot += lse_protocol ? e : e * __ldcg(p.denoms + base + s);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) tot += __shfl_xor_sync(FULL_MASK, tot, o);
    const float shift = lse_protocol ? (tot > 0.f ? logf(tot) + mx : INFINITY) : mx;
    const float scale = lse_protocol ? 1.f : 1.f / (tot > 0.f ? tot : 1.f);
    const float *rsrc = (lse_protocol ? p.partial : p.accums) + base * D + lane * E;
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    for (int s0 = 0; s0 < live; s0 += 32) {
      const float wl = s0 + lane < live ? expf(__ldcg(wsrc + s0 + lane) - shift) : 0.f;
      const int n = min(32, live - s0);
      // Rows of up to 8 partitions are loaded before any is consumed, so the
      // L2 round trips overlap instead of serialising per partition.
      for (int k0 = 0; k0 < n; k0 += 8) {
        float2 v[8][E / 2];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float *src = rsrc + (int64_t)(s0 + min(k0 + j, n - 1)) * D;
#pragma unroll
          for (int e = 0; e < E; e += 2) v[j][e / 2] = __ldcg(reinterpret_cast<const float2 *>(src + e));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float wk = __shfl_sync(FULL_MASK, wl, min(k0 + j, 31));
          if (k0 + j < n) {
#pragma unroll
            for (int e = 0; e < E; e += 2) {
              acc[e] = fmaf(wk, v[j][e / 2].x, acc[e]);
              acc[e + 1] = fmaf(wk, v[j][e / 2].y, acc[e + 1]);
            }
          }
        }
      }
    }
    __nv_bfloat16 *dst = p.out + row * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2)
      *reinterpret_cast<__nv_bfloat162 *>(dst + e) =
          __floats2bfloat162_rn(acc[e] * scale, acc[e + 1] * scale);
  }
}

// End of every item (empty or not).  With the fused merge enabled, count the
// item against its (row, KV head, sub-group); the CTA whose count completes
// the group's `splits` items merges the group and resets the counter for the
// next launch.  Release: a CTA barrier orders all consumers' stores before
// one thread's fence + atomic; acquire: the merging CTA fences after
// observing the count.
template <int D, int NC>
__device__ void finish_item(const PartitionParams &p, const Item &w, int h0, int rows, int cw,
                            int lane, volatile int *merge_flag) {
  if (p.counters == nullptr || p.mode == MODE_DIRECT) return;
  named_barrier(1, NC * 32);  // every consumer's partition stores precede the fence below
  if (cw == 0 && lane == 0) {
    const int64_t g = ((int64_t)w.b * p.num_kv_heads + w.kvh) * p.nsub + w.sub;
    __threadfence();          // release (cumulative over the CTA's stores ordered by the barrier)
    const int prev = atomicAdd(p.counters + g, 1);
    const int last = prev == p.splits - 1;
    if (last) atomicExch(p.counters + g, 0);
    *merge_flag = last;
  }
  named_barrier(1, NC * 32);
  if (*merge_flag) {
    __threadfence();
    // Only the ceil(len / tokens_per_split) live partitions carry weight; the
    // others are empty (weight exactly 0), so skipping them changes no bit.
    const int len = min(__ldg(p.lengths + w.b), p.table_width * 256);
    const int live =
        min(p.splits, (int)((len + (int64_t)p.tokens_per_split - 1) / p.tokens_per_split));
    merge_group<D, NC>(p, w, h0, rows, live, cw, lane);
  }
}

// Dynamic shared memory one CTA may use so that two CTAs share an SM
// (228 KB per SM, 1 KB reserved per CTA).
constexpr int kTwoCtaSmemBytes = 233472 / 2 - 1024;

// The swizzle arithmetic assumes the dynamic shared-memory base is 1024-byte
// aligned (it is when a kernel has no static shared memory).  If it ever is
// not, the CTA records FAULT_SMEM_ALIGN and returns without touching memory.
__device__ __forceinline__ bool smem_base_aligned(const void *smem, uint32_t *fault) {
  if ((smem_u32(smem) & 1023u) == 0) return true;
  if (threadIdx.x == 0 && fault) atomicOr(fault, FAULT_SMEM_ALIGN);
  return false;
}

// Shared-memory plan of a partition kernel: K ring | V ring | per-warp
// accumulators [NC][GC][D] | per-warp (m, l) [NC][2][GC] | mbarriers | flag.
// Tail after the mbarriers: item ring barriers [2][IR], item slots [IR],
// then abort flag, merge flag and the handed-out item (16 bytes).
template <int D, int T, int NS, int NC, int GC>
struct PartitionSmem {
  static constexpr int TILE_BYTES = T * D * 2;
  static constexpr int KV_BYTES = 2 * NS * TILE_BYTES;
  static constexpr int ACC_FLOATS = NC * GC * D;
  static constexpr int ML_FLOATS = NC * 2 * GC;
  static constexpr int BAR_OFFSET = KV_BYTES + (ACC_FLOATS + ML_FLOATS) * 4;
  static constexpr int RING_OFFSET = BAR_OFFSET + 2 * NS * 8;
  static constexpr int FLAG_OFFSET = RING_OFFSET + 2 * IR * 8 + IR * 4;
  static constexpr int BYTES = FLAG_OFFSET + 16;
  static_assert(TILE_BYTES % 1024 == 0, "swizzled tiles need 1024-byte alignment");
  static_assert((T * 128) % 1024 == 0, "swizzled sub-tiles need 1024-byte alignment");
  static_assert((GC * D * 4) % 16 == 0, "per-warp accumulators are accessed as float4");
  static_assert(BAR_OFFSET % 8 == 0, "mbarriers need 8-byte alignment");
};

}  // namespace pdl
