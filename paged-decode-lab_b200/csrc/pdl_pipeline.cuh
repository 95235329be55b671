// pdl_pipeline.cuh -- pieces shared by the partition kernels: the work
// schedule, the TMA producer warp, the hand-off of work items to the
// consumer warps, stores for empty partitions, and the merge of the
// consumer warps' softmax states into the stored outputs.
#pragma once

#include "pdl_device.cuh"

namespace pdl {

// ------------------------------------------------------------- work items
// A work item handed from the producer warp to the consumer warps is one of
//   COMPUTE  tokens [start, stop) of partition `split` of row b, for KV head
//            and head sub-group hs = kvh * nsub + sub;
//   FILL     the stores that mark row b's partitions [split, split_end) empty
//            (partial 0 and LSE -inf, or (-inf, 0, 0)) for all query heads
//            (hs < 0) or for the heads of sub-group hs, or, in direct mode,
//            the zero output rows of a zero-length row;
//   STOP     this CTA has no more items.
enum ItemKind : int { ITEM_STOP = 0, ITEM_COMPUTE = 1, ITEM_FILL = 2 };

struct WorkItem {
  int kind, b, split, split_end, hs, start, stop;
};

__device__ __forceinline__ WorkItem stop_item() {
  WorkItem w;
  w.kind = ITEM_STOP;
  w.b = w.split = w.split_end = w.hs = w.start = w.stop = 0;
  return w;
}

// Lengths are clamped to the table capacity, so no table entry past a row's
// width is ever read.
__device__ __forceinline__ int row_capacity(const PartitionParams &p) {
  return p.table_width * 256;  // the host checks table_width * 256 fits in int32
}

__device__ __forceinline__ int clamp_length(const PartitionParams &p, int b) {
  return min(max(__ldg(p.lengths + b), 0), row_capacity(p));
}

// Position of the k-th (0-based) set bit of m; m has more than k set bits.
__device__ __forceinline__ int nth_set_bit(uint32_t m, int k) {
  int base = 0;
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const uint32_t low = m & ((1u << w) - 1u);
    const int c = __popc(low);
    if (k >= c) {
      k -= c;
      m >>= w;
      base += w;
    } else {
      m = low;
    }
  }
  return base;
}

// ------------------------------------------------- the live-item schedule
// Every CTA's producer warp derives the same schedule from the lengths (held
// in registers: lane l owns rows l, l + 32, ...), so only work that exists is
// ever handed out -- partitions past a row's length cost nothing -- and the
// order is good for balance under dynamic scheduling, like longest-first:
//   1. every FULL partition (tokens_per_split tokens), row-major;
//   2. every row's last, PARTIAL partition, in four size classes, largest
//      first (in direct mode each row is one partial partition);
//   3. one FILL item per row with empty partitions to store (or, in direct
//      mode, per zero-length row).
// Items 1 and 2 are expanded over the (KV head, sub-group) pairs, which vary
// fastest, so concurrent CTAs read neighbouring bytes of the same pages.
constexpr int RMAX = 16;  // rows per lane: batches up to 512 rows use this schedule

struct LiveSchedule {
  int len[RMAX];   // clamped length of row r * 32 + lane (0 past the batch)
  int fpre[RMAX];  // exclusive row-major prefix of full partitions
  int cls[RMAX];   // size class of the row's partial partition, -1 if none
  int kpre[5];     // partial partitions of classes < c
  int full;        // full partitions of the batch
  int compute;     // compute items = (full + partial) * heads-and-sub-groups
  int total;       // compute + fill items
};

__device__ __forceinline__ bool fill_row(const PartitionParams &p, int b, int len, int live) {
  if (b >= p.batch) return false;
  if (p.mode == MODE_DIRECT) return len == 0;
  return p.write_empty && live < p.splits;
}

__device__ __forceinline__ LiveSchedule build_schedule(const PartitionParams &p, int lane) {
  LiveSchedule s;
  const int tps = p.tokens_per_split;
  const int R = (p.batch + 31) >> 5;
  int maxlen = 0;
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    const int b = r * 32 + lane;
    s.len[r] = (r < R && b < p.batch) ? clamp_length(p, b) : 0;
    maxlen = max(maxlen, s.len[r]);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) maxlen = max(maxlen, __shfl_xor_sync(FULL_MASK, maxlen, o));
  // Size classes are quarters of the largest possible partial partition.
  const int span = max(1, min(tps, maxlen));
  int carry = 0;
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    const int f = s.len[r] / tps;
    const int rem = s.len[r] - f * tps;
    int x = f;  // inclusive scan over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(FULL_MASK, x, o);
      if (lane >= o) x += y;
    }
    s.fpre[r] = carry + x - f;
    carry += __shfl_sync(FULL_MASK, x, 31);
    s.cls[r] = rem > 0 ? min(3, (int)(((int64_t)(span - rem) * 4) / span)) : -1;
  }
  s.full = carry;
  s.kpre[0] = 0;
  int fills = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    int n = 0;
#pragma unroll
    for (int r = 0; r < RMAX; ++r) n += __popc(__ballot_sync(FULL_MASK, s.cls[r] == c));
    s.kpre[c + 1] = s.kpre[c] + n;
  }
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    const int b = r * 32 + lane;
    const int live = s.len[r] / tps + (s.cls[r] >= 0 ? 1 : 0);
    fills += __popc(__ballot_sync(FULL_MASK, fill_row(p, b, s.len[r], live)));
  }
  const int heads = p.num_kv_heads * p.nsub;
  s.compute = (s.full + s.kpre[4]) * heads;  // <= the host-checked dense item count
  s.total = s.compute + fills;
  return s;
}

// Item `item` (< s.total) of the schedule; every lane returns the same item.
// COMPUTE items of a partial partition carry stop = the row's length.
__device__ __forceinline__ WorkItem decode_live(const PartitionParams &p, const LiveSchedule &s, int item,
                                int lane) {
  WorkItem w = stop_item();
  const int tps = p.tokens_per_split;
  if (item < s.compute) {
    const int heads = p.num_kv_heads * p.nsub;
    const int u = item / heads;
    w.kind = ITEM_COMPUTE;
    w.hs = item - u * heads;
    if (u < s.full) {
      // The row whose full partitions [fpre, fpre + f) hold u.  (Values of
      // the matching row are read inside the unrolled loops: an array
      // indexed by a run-time chunk would move to local memory.)
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        int next = __shfl_down_sync(FULL_MASK, s.fpre[r], 1);
        const int head_next = __shfl_sync(FULL_MASK, s.fpre[r + 1 < RMAX ? r + 1 : r], 0);
        if (lane == 31) next = r + 1 < RMAX ? head_next : s.full;
        const uint32_t m = __ballot_sync(FULL_MASK, s.fpre[r] <= u && u < next);
        if (m) {
          const int src = __ffs(m) - 1;
          w.b = r * 32 + src;
          w.split = u - __shfl_sync(FULL_MASK, s.fpre[r], src);
        }
      }
      w.start = w.split * tps;
      w.stop = w.start + tps;
    } else {
      int k = u - s.full, c = 0, first = 0;
#pragma unroll
      for (int j = 1; j < 4; ++j) {
        if (k >= s.kpre[j]) {
          c = j;
          first = s.kpre[j];
        }
      }
      k -= first;
      bool found = false;
      int len = 0;
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        const uint32_t m = __ballot_sync(FULL_MASK, s.cls[r] == c);
        const int n = __popc(m);
        if (!found && k < n) {
          const int src = nth_set_bit(m, k);
          w.b = r * 32 + src;
          len = __shfl_sync(FULL_MASK, s.len[r], src);
          found = true;
        } else if (!found) {
          k -= n;
        }
      }
      w.split = len / tps;
      w.start = w.split * tps;
      w.stop = len;
    }
  } else {
    int k = item - s.compute;
    bool found = false;
    int len = 0;
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      const int b = r * 32 + lane;
      const int live = s.len[r] / tps + (s.cls[r] >= 0 ? 1 : 0);
      const uint32_t m = __ballot_sync(FULL_MASK, fill_row(p, b, s.len[r], live));
      const int n = __popc(m);
      if (!found && k < n) {
        const int src = nth_set_bit(m, k);
        w.b = r * 32 + src;
        len = __shfl_sync(FULL_MASK, s.len[r], src);
        found = true;
      } else if (!found) {
        k -= n;
      }
    }
    w.kind = ITEM_FILL;
    w.hs = -1;
    w.split = (int)(((int64_t)len + tps - 1) / tps);
    w.split_end = p.splits;
  }
  return w;
}

// Batches above 32 * RMAX rows enumerate every (row, KV head, sub-group,
// partition) instead; empty ones become single-partition FILL items (or are
// skipped when empty partitions are not stored).
//   static:  item = ((b * num_kv_heads + kvh) * nsub + sub) * splits + split
//   dynamic: item = split * (batch * num_kv_heads * nsub) + group
__device__ __forceinline__ WorkItem decode_dense(const PartitionParams &p, int item, bool dynamic, bool &skip) {
  WorkItem w = stop_item();
  const int per_row = p.num_kv_heads * p.nsub;
  int rest;
  if (dynamic) {
    const int groups = p.batch * per_row;
    w.split = item / groups;
    rest = item % groups;
  } else {
    w.split = item % p.splits;
    rest = item / p.splits;
  }
  w.b = rest / per_row;
  w.hs = rest % per_row;
  const int len = clamp_length(p, w.b);
  const int64_t start = (int64_t)w.split * p.tokens_per_split;
  const int64_t stop = min((int64_t)len, start + p.tokens_per_split);
  skip = false;
  if (start < stop) {
    w.kind = ITEM_COMPUTE;
    w.start = (int)start;
    w.stop = (int)stop;
  } else if (p.write_empty || p.mode == MODE_DIRECT) {
    w.kind = ITEM_FILL;
    w.split_end = w.split + 1;
  } else {
    skip = true;
  }
  return w;
}

// ------------------------------------------------------------- hand-off
// The producer warp publishes every item (compute, fill, then stop) in an
// IR-deep shared-memory ring; one consumer thread (the leader) waits for it
// and all consumer warps read it between two named barriers, so every warp
// processes the same sequence even if a bounded wait gives up (the leader
// then hands out "stop").
constexpr int IR = 8;

struct ItemRing {
  uint64_t *full;        // [IR] producer -> consumers, count 1
  uint64_t *empty;       // [IR] consumers -> producer, count 1 (the leader)
  volatile int *slot;    // [IR][8] published items (WorkItem fields)
  volatile int *stop;    // the leader's "stop" decision for the current item
};

__device__ __forceinline__ void ring_init(const ItemRing &r) {
  for (int i = 0; i < IR; ++i) {
    mbar_init(&r.full[i], 1);
    mbar_init(&r.empty[i], 1);
  }
}

// Producer (lane 0 publishes, every lane returns whether the slot was free).
__device__ __forceinline__ bool publish(const ItemRing &r, uint32_t &k, const WorkItem &w,
                                        uint32_t *fault, volatile int *abort_flag, int lane) {
  bool ok = true;
  if (lane == 0) {
    const int s = k % IR;
    if (k >= IR)
      ok = pipeline_wait(&r.empty[s], ((k / IR) & 1) ^ 1, fault, FAULT_PRODUCER_EMPTY_WAIT,
                         abort_flag);
    if (ok) {
      volatile int *d = r.slot + 8 * s;
      d[0] = w.kind;
      d[1] = w.b;
      d[2] = w.split;
      d[3] = w.split_end;
      d[4] = w.hs;
      d[5] = w.start;
      d[6] = w.stop;
      mbar_arrive(&r.full[s]);
    }
  }
  ++k;
  return __shfl_sync(FULL_MASK, ok, 0);
}

// Next item of the consumer warps (identical in every consumer warp).
template <int NC>
__device__ __forceinline__ WorkItem consumer_next(const ItemRing &r, uint32_t &k, int cw,
                                                  int lane, uint32_t *fault,
                                                  volatile int *abort_flag) {
  const int s = k % IR;
  const bool leader = cw == 0 && lane == 0;
  if (leader)
    *r.stop = pipeline_wait(&r.full[s], (k / IR) & 1, fault, FAULT_CONSUMER_FULL_WAIT,
                            abort_flag) ? 0 : 1;
  named_barrier(1, NC * 32);
  WorkItem w = stop_item();
  if (!*r.stop) {
    const volatile int *src = r.slot + 8 * s;
    w.kind = src[0];
    w.b = src[1];
    w.split = src[2];
    w.split_end = src[3];
    w.hs = src[4];
    w.start = src[5];
    w.stop = src[6];
  }
  named_barrier(1, NC * 32);  // every warp has read the slot before it is released
  if (leader) mbar_arrive(&r.empty[s]);
  ++k;
  return w;
}

// ------------------------------------------------------------- producer
// Producer warp: walks this CTA's items -- blockIdx.x first, then (dynamic
// scheduling) gridDim.x + the next value of a global atomic counter, or
// (static) every gridDim.x-th item -- publishes each to the consumers and,
// for compute items, reads the partition's block-table entries (32 per load,
// one per lane, never past the table width) and issues one T-token tile of K
// and V per stage as D/64 TMA boxes each.  T divides 256, so a tile never
// spans two pages.  The next item is claimed before this one's copies are
// issued, so the atomic's round trip overlaps them.
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
  const bool live = p.batch <= 32 * RMAX;
  LiveSchedule sched;
  int total = p.n_items;
  if (live) {
    sched = build_schedule(p, lane);
    total = sched.total;
  }
  const bool dynamic = p.sched != nullptr && total > (int)gridDim.x;
  uint32_t it = 0, k = 0;
  bool ok = true;
  int item = blockIdx.x;
  while (ok) {
    if (item >= total) {
      publish(ring, k, stop_item(), p.fault, abort_flag, lane);
      break;
    }
    bool skip = false;
    const WorkItem w = live ? decode_live(p, sched, item, lane) : decode_dense(p, item, dynamic, skip);
    // Claim the next item now; its value is needed only after the copies.
    int claimed = 0;
    if (dynamic && lane == 0) claimed = atomicAdd(p.sched, 1);
    if (!skip && !publish(ring, k, w, p.fault, abort_flag, lane)) {
      ok = false;
      break;
    }
    if (w.kind == ITEM_COMPUTE) {
      const int32_t *trow = p.table + (int64_t)w.b * p.table_stride;
      const int kvh = w.hs / p.nsub;
      int base = w.start >> 8;
      int my_page = base + lane < p.table_width ? __ldg(trow + base + lane) : 0;
      const int t0 = w.start / T * T;
      const int ntiles = (w.stop - t0 + T - 1) / T;
      for (int i = 0; i < ntiles; ++i, ++it) {
        const int tok = t0 + i * T;
        const int pg = tok >> 8;
        if (pg >= base + 32) {
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
              tma_load_4d(kbuf + s * TILE_BYTES + st * SUB_BYTES, k_map, st * 64, kvh, tok & 255,
                          page, &full[s], policy);
              tma_load_4d(vbuf + s * TILE_BYTES + st * SUB_BYTES, v_map, st * 64, kvh, tok & 255,
                          page, &full[s], policy);
            }
          }
        }
        ok = __shfl_sync(FULL_MASK, ok, 0);
        if (!ok) break;
      }
    }
    item = dynamic ? (int)gridDim.x + __shfl_sync(FULL_MASK, claimed, 0) : item + (int)gridDim.x;
  }
  if (!ok && lane == 0) {
    // Let the copies already issued land before the CTA exits.
    const uint32_t first = it > NS ? it - NS : 0;
    for (uint32_t j = first; j < it; ++j)
      mbar_wait_bounded(&full[j % NS], (j / NS) & 1, p.fault, FAULT_DRAIN_WAIT);
  }
  // Count this CTA as finished; the last one resets the scheduler words for
  // the next launch (every CTA's final claim precedes its count, and no
  // claim follows the last count).  Every CTA computed the same `dynamic`.
  if (dynamic && lane == 0) {
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(p.sched, 0);
      atomicExch(p.sched + 1, 0);
    }
  }
}

// Stores of a FILL item by the consumer warps' threads (tid < nthreads):
// partitions [split, split_end) of heads [h0, h0 + rows) of row b, or the
// zero output rows in direct mode.
template <int D>
__device__ void store_fill(const PartitionParams &p, const WorkItem &w, int h0, int rows,
                           int tid, int nthreads) {
  const int nsplit = p.mode == MODE_DIRECT ? 1 : w.split_end - w.split;
  const int per_head = nsplit * (D / 4);
  for (int e = tid; e < rows * per_head; e += nthreads) {
    const int g = e / per_head, rest = e % per_head;
    const int split = w.split + rest / (D / 4), d = (rest % (D / 4)) * 4;
    const int64_t row = (int64_t)w.b * p.num_heads + h0 + g;
    const int64_t idx = row * p.splits + split;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.mode == MODE_LSE) {
      *reinterpret_cast<float4 *>(p.partial + idx * D + d) = zero;
      if (d == 0) p.lse[idx] = -INFINITY;
    } else if (p.mode == MODE_MLA) {
      *reinterpret_cast<float4 *>(p.accums + idx * D + d) = zero;
      if (d == 0) {
        p.maxima[idx] = -INFINITY;
        p.denoms[idx] = 0.f;
      }
    } else {
      *reinterpret_cast<uint2 *>(p.out + row * D + d) = make_uint2(0u, 0u);
    }
  }
}

// Heads [h0, h0 + rows) of an item for a kernel handling GC heads per sub-group.
template <int GC>
__device__ __forceinline__ void item_heads(const PartitionParams &p, int hs, int &h0, int &rows) {
  if (hs < 0) {
    h0 = 0;
    rows = p.num_heads;
    return;
  }
  const int kvh = hs / p.nsub, sub = hs - (hs / p.nsub) * p.nsub;
  h0 = kvh * p.group + sub * GC;
  rows = min(GC, p.group - sub * GC);
}

// Merge NC per-warp (or per-group) softmax states of one item and store the
// outputs, with the NW consumer warps' threads (tid < NW * 32).
//   comb_acc [NC][GC][D]  unnormalised accumulators (relative to each state's max)
//   comb_ml  [NC][2][GC]  per-state running max (base-2 scaled units) and sum
// M = max_w m_w; f_w = 2^(m_w - M); L = sum f_w l_w; O = sum f_w acc_w.
// Stores O/L + LSE (natural log), (M ln2, L, O), or BF16 O/L.
template <int D, int GC, int NC, int NW = NC>
__device__ void combine_and_store(const PartitionParams &p, const WorkItem &w, int h0, int rows,
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
// accumulators [NC][GC][D] | per-warp (m, l) [NC][2][GC] | mbarriers | item
// ring barriers [2][IR] | item slots [IR][32 bytes] | abort flag, stop word.
template <int D, int T, int NS, int NC, int GC>
struct PartitionSmem {
  static constexpr int TILE_BYTES = T * D * 2;
  static constexpr int KV_BYTES = 2 * NS * TILE_BYTES;
  static constexpr int ACC_FLOATS = NC * GC * D;
  static constexpr int ML_FLOATS = NC * 2 * GC;
  static constexpr int BAR_OFFSET = KV_BYTES + (ACC_FLOATS + ML_FLOATS) * 4;
  static constexpr int RING_OFFSET = BAR_OFFSET + 2 * NS * 8;
  static constexpr int SLOT_OFFSET = RING_OFFSET + 2 * IR * 8;
  static constexpr int FLAG_OFFSET = SLOT_OFFSET + IR * 32;
  static constexpr int BYTES = FLAG_OFFSET + 16;
  static_assert(TILE_BYTES % 1024 == 0, "swizzled tiles need 1024-byte alignment");
  static_assert((T * 128) % 1024 == 0, "swizzled sub-tiles need 1024-byte alignment");
  static_assert((GC * D * 4) % 16 == 0, "per-warp accumulators are accessed as float4");
  static_assert(BAR_OFFSET % 8 == 0, "mbarriers need 8-byte alignment");
};

// Pointers into a partition kernel's shared memory for layout L.
template <typename L>
__device__ __forceinline__ ItemRing item_ring(uint8_t *smem) {
  ItemRing r;
  r.full = reinterpret_cast<uint64_t *>(smem + L::RING_OFFSET);
  r.empty = r.full + IR;
  r.slot = reinterpret_cast<volatile int *>(smem + L::SLOT_OFFSET);
  r.stop = reinterpret_cast<volatile int *>(smem + L::FLAG_OFFSET) + 1;
  return r;
}

}  // namespace pdl
