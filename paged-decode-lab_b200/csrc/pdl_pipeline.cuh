// pdl_pipeline.cuh -- pieces shared by the partition kernels: the work
// schedule, the TMA producer warp, the hand-off of work items to the
// consumer warps, stores for empty partitions, and the merge of the
// consumer warps' softmax states into the stored outputs.
#pragma once

#include <climits>

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
  int last;  // the CTA's last item: its consumers exit after it without another hand-off
};

__device__ __forceinline__ WorkItem stop_item() {
  WorkItem w;
  w.kind = ITEM_STOP;
  w.b = w.split = w.split_end = w.hs = w.start = w.stop = w.last = 0;
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
// Launches with more work items than CTAs (and batches of at most 32 * RMAX
// rows) hand out only work that exists: every CTA's producer warp derives the
// same schedule from the row lengths, so partitions past a row's length cost
// no claim and no consumer round trip.  The order balances like
// longest-first under dynamic scheduling:
//   1. every FULL partition (tokens_per_split tokens), row-major;
//   2. every row's last, PARTIAL partition, in four size classes, largest
//      first (in direct mode each row is one partial partition);
//   3. FILL items storing the empty partitions, in chunks of fill_splits
//      partitions of all heads of one row (in direct mode, one per
//      zero-length row), last, so idle CTAs take them.
// Items of 1 and 2 are expanded over the (KV head, sub-group) pairs, which
// vary fastest, so concurrent CTAs read neighbouring bytes of the same
// pages.  One prefix sum over the rows' full-partition counts, at set-up,
// makes decoding any item a few warp ballots.  For rows that all hold
// full partitions only, the order is the dense row-major one, which lets the
// producer request the first item's block-table entries with the lengths.
//
// The code is kept small on purpose: the producer runs it once per item, so
// it is rarely in the instruction cache, and rolled loops over the batch's
// row chunks (the per-row arrays then live in L1-cached local memory) cost
// far less than fully unrolled ones -- measured on B200, unrolling all 16
// chunks added 4 to 40 us to short launches.  A partition-major order was
// tried as well: decoding its items needs one ballot pass per partition
// index, which made launches of many partitions the producer's bottleneck
// (config 4 in 1024-token partitions: 642 vs 505 us).
constexpr int RMAX = 16;  // rows per lane: batches up to 512 rows use this schedule

struct LiveSchedule {
  int len[RMAX];   // clamped length of row r * 32 + lane (0 past the batch)
  int full[RMAX];  // its full partitions
  int fpre[RMAX];  // exclusive row-major prefix of full partitions
  int cls[RMAX];   // size class of its partial partition, -1 if none
  int R;           // row chunks of the batch
  int nfull;       // full partitions of the batch
};

// The launch parameters the schedule depends on (passed by value, so the
// kernel's parameter block is not copied to local memory).
struct SchedParams {
  const int32_t *lengths;
  int batch, heads, tps, splits, cap, direct, write_empty, fill_splits;
};

__device__ __forceinline__ SchedParams sched_params(const PartitionParams &p) {
  SchedParams q;
  q.lengths = p.lengths;
  q.batch = p.batch;
  q.heads = p.num_kv_heads * p.nsub;
  q.tps = p.tokens_per_split;
  q.splits = p.splits;
  q.cap = row_capacity(p);
  q.direct = p.mode == MODE_DIRECT;
  q.write_empty = p.write_empty;
  q.fill_splits = p.fill_splits;
  return q;
}

// Fill chunks of row b.
__device__ __forceinline__ int fill_chunks(const SchedParams &p, int b, int len, int live) {
  if (b >= p.batch) return 0;
  if (p.direct) return len == 0 ? 1 : 0;
  if (!p.write_empty || live >= p.splits) return 0;
  return (p.splits - live + p.fill_splits - 1) / p.fill_splits;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}

// Inclusive prefix over the warp's lanes.
__device__ __forceinline__ int warp_scan(int x, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(FULL_MASK, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

static __device__ __noinline__ void build_schedule(const SchedParams p, int lane, LiveSchedule &s) {
  const int tps = p.tps;
  s.R = (p.batch + 31) >> 5;
  int maxlen = 0;
#pragma unroll 1
  for (int r = 0; r < s.R; ++r) {
    const int b = r * 32 + lane;
    s.len[r] = b < p.batch ? min(max(__ldg(p.lengths + b), 0), p.cap) : 0;
    maxlen = max(maxlen, s.len[r]);
  }
  // Size classes are quarters of the longest possible partial partition:
  // tokens_per_split, or in direct mode the longest row.
  int span = tps;
  if (p.direct) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) maxlen = max(maxlen, __shfl_xor_sync(FULL_MASK, maxlen, o));
    span = max(1, maxlen);
  }
  const float inv_span = 4.f / (float)span;
  int carry = 0;
#pragma unroll 1
  for (int r = 0; r < s.R; ++r) {
    const int f = s.len[r] / tps;
    const int rem = s.len[r] - f * tps;
    s.full[r] = f;
    const int x = warp_scan(f, lane);
    s.fpre[r] = carry + x - f;
    carry += __shfl_sync(FULL_MASK, x, 31);
    s.cls[r] = rem > 0 ? min(3, (int)((float)(span - rem) * inv_span)) : -1;
  }
  s.nfull = carry;
}

// Items of the schedule: (full + partial partitions) * heads + fill chunks.
static __device__ __noinline__ int schedule_total(const SchedParams p, const LiveSchedule &s,
                                                  int lane) {
  int partial = 0, fills = 0;
#pragma unroll 1
  for (int r = 0; r < s.R; ++r) {
    const int live = s.full[r] + (s.cls[r] >= 0 ? 1 : 0);
    partial += s.cls[r] >= 0 ? 1 : 0;
    fills += fill_chunks(p, r * 32 + lane, s.len[r], live);
  }
  return (s.nfull + warp_sum(partial)) * p.heads + warp_sum(fills);
}

// Item `item` of the schedule (every lane returns the same item); STOP past
// the last one.  Partial partitions carry stop = the row's length.
static __device__ __noinline__ WorkItem decode_live(const SchedParams p, const LiveSchedule &s,
                                                    int item, int lane) {
  WorkItem w = stop_item();
  const int tps = p.tps;
  const int heads = p.heads;
  const int u = item / heads;
  const int hs = item - u * heads;
  // 1. Full partitions, row-major: the row whose range [fpre, fpre + full) holds u.
  if (u < s.nfull) {
#pragma unroll 1
    for (int r = 0; r < s.R; ++r) {
      const uint32_t m =
          __ballot_sync(FULL_MASK, s.full[r] > 0 && s.fpre[r] <= u && u < s.fpre[r] + s.full[r]);
      if (m) {
        const int src = __ffs(m) - 1;
        w.kind = ITEM_COMPUTE;
        w.hs = hs;
        w.b = r * 32 + src;
        w.split = u - __shfl_sync(FULL_MASK, s.fpre[r], src);
        w.start = w.split * tps;
        w.stop = w.start + tps;
        return w;
      }
    }
    return w;  // not reached: u lies in some row's range
  }
  // 2. Partial partitions, largest class first.
  int before = s.nfull;
  for (int g = 0; g < 4; ++g) {
    int k = u - before, n_all = 0;
#pragma unroll 1
    for (int r = 0; r < s.R; ++r) {
      const uint32_t m = __ballot_sync(FULL_MASK, s.cls[r] == g);
      const int n = __popc(m);
      if (k < n) {
        const int src = nth_set_bit(m, k);
        const int len = __shfl_sync(FULL_MASK, s.len[r], src);
        w.kind = ITEM_COMPUTE;
        w.hs = hs;
        w.b = r * 32 + src;
        w.split = len / tps;
        w.start = w.split * tps;
        w.stop = len;
        return w;
      }
      k -= n;
      n_all += n;
    }
    before += n_all;
  }
  // 3. Fill chunks, row-major (a prefix sum over the rows' chunk counts).
  const int j = item - before * heads;
  int carry = 0;
#pragma unroll 1
  for (int r = 0; r < s.R; ++r) {
    const int live = s.full[r] + (s.cls[r] >= 0 ? 1 : 0);
    const int c = fill_chunks(p, r * 32 + lane, s.len[r], live);
    const int x = warp_scan(c, lane);
    const int pre = carry + x - c;
    const uint32_t m = __ballot_sync(FULL_MASK, c > 0 && pre <= j && j < pre + c);
    if (m) {
      const int src = __ffs(m) - 1;
      w.b = r * 32 + src;
      const int first = __shfl_sync(FULL_MASK, live, src) +
                        (j - __shfl_sync(FULL_MASK, pre, src)) * p.fill_splits;
      w.kind = ITEM_FILL;
      w.hs = -1;
      w.split = first;
      w.split_end = min(p.splits, first + p.fill_splits);
      return w;
    }
    carry += __shfl_sync(FULL_MASK, x, 31);
  }
  return w;
}

// Single-wave launches (at most one item per CTA), batches above 32 * RMAX
// rows and balanced partition bounds (derived per item from the row's
// length) enumerate every (row, KV head, sub-group, partition) instead;
// empty ones become single-partition FILL items (or are skipped when empty
// partitions are not stored).  The row length and the first 32
// block-table entries of the partition are requested together, so an item,
// and its first pages, are known after one round trip.
//   static:  item = ((b * num_kv_heads + kvh) * nsub + sub) * splits + split
//   dynamic: item = split * (batch * num_kv_heads * nsub) + group
__device__ __forceinline__ WorkItem decode_dense(const PartitionParams &p, int item, bool dynamic,
                                                 int lane, bool &skip, int &base, int &my_page) {
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
  // Fixed partitions start at split * tokens_per_split; balanced ones at
  // split * span with span >= tokens_per_split (the granule), so in both
  // cases the table window requested with the length starts at or before
  // the partition's first page (the tile loop moves it forward if needed).
  const int64_t lo = (int64_t)w.split * p.tokens_per_split;
  base = lo < (int64_t)row_capacity(p) ? (int)(lo >> 8) : -64;
  my_page = (base >= 0 && base + lane < p.table_width)
                ? __ldg(p.table + (int64_t)w.b * p.table_stride + base + lane) : 0;
  const int len = clamp_length(p, w.b);
  const int64_t span = p.balanced ? balanced_span(len, p.splits, p.tokens_per_split)
                                  : p.tokens_per_split;
  const int64_t start = (int64_t)w.split * span;
  const int64_t stop = min((int64_t)len, start + span);
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
  volatile int *peek;    // the leader's look at the next slot: published already?
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
      d[7] = w.last;
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
    w.last = src[7];
  }
  named_barrier(1, NC * 32);  // every warp has read the slot before it is released
  if (leader) mbar_arrive(&r.empty[s]);
  ++k;
  return w;
}

// While the consumers finish item k, the leader checks -- without waiting --
// whether item k + 1 is already published (it usually is: the producer runs
// ahead); after the next named barrier every consumer thread may read it and
// prefetch that item's q rows into L1, so the q loads at its start do not
// wait for L2.  `k` is the ring index consumer_next will use next.
__device__ __forceinline__ void ring_peek(const ItemRing &r, uint32_t k, bool leader) {
  if (leader) *r.peek = mbar_test_wait(&r.full[k % IR], (k / IR) & 1) ? 1 : 0;
}

__device__ __forceinline__ WorkItem peeked_item(const ItemRing &r, uint32_t k) {
  WorkItem w = stop_item();
  if (*r.peek) {
    const volatile int *src = r.slot + 8 * (k % IR);
    w.kind = src[0];
    w.b = src[1];
    w.hs = src[4];
  }
  return w;
}

// ------------------------------------------------------------- producer
// Producer warp: walks this CTA's items -- blockIdx.x first, then (dynamic
// scheduling) gridDim.x + the next value of a global atomic counter, or
// (static) every gridDim.x-th item -- publishes each to the consumers and,
// for compute items, reads the partition's block-table entries (32 per load,
// one per lane, never past the table width) and issues one T-token tile of K
// and V per stage, one TMA box each.  T divides 256, so a tile never
// spans two pages.  The next item is claimed once this one's first copies
// are issued, so the atomic's round trip overlaps them.
template <int D, int T, int NS>
__device__ void run_producer(const CUtensorMap *k_map, const CUtensorMap *v_map,
                             const PartitionParams &p, uint8_t *kbuf, uint8_t *vbuf,
                             uint64_t *full, uint64_t *empty, volatile int *abort_flag,
                             const ItemRing &ring, int lane) {
  constexpr int TILE_BYTES = T * D * 2;
  const uint64_t policy = l2_evict_first_policy();
  if (lane == 0) {
    prefetch_tensormap(k_map);
    prefetch_tensormap(v_map);
  }
  // The live schedule serves launches with more items than CTAs (set by the
  // launcher); a single wave is enumerated densely (decode_dense).
  const bool live = p.live != 0;
  const int heads = p.num_kv_heads * p.nsub;
  int item = blockIdx.x;
  const SchedParams sp = sched_params(p);
  LiveSchedule sched;
  // Live schedule: the first item's block-table entries are requested before
  // the lengths arrive, for the dense row-major guess (row u / splits,
  // partition u % splits with u = item / heads), which the live order equals
  // when every row fills the table's capacity with full partitions.
  int guess_row = -1, guess_base = -1, guess_page = 0;
  if (live) {
    const int u0 = item / heads;
    guess_row = min(u0 / p.splits, p.batch - 1);
    const int64_t first_tok = (int64_t)(u0 % p.splits) * p.tokens_per_split;
    guess_base = first_tok < (int64_t)row_capacity(p) ? (int)(first_tok >> 8) : -1;
    if (guess_base >= 0 && guess_base + lane < p.table_width)
      guess_page = __ldg(p.table + (int64_t)guess_row * p.table_stride + guess_base + lane);
    build_schedule(sp, lane, sched);
  }
  // Items of this launch: known at once when dense; for the live schedule
  // computed once the first item's copies are issued.
  int total = live ? -1 : p.n_items;
  int dynamic = -1;  // decided at the first claim: is there an item past the first wave?
  uint32_t it = 0, k = 0;
  bool ok = true, first = true;
  while (ok) {
    bool skip = false;
    int base = -64, my_page = 0;
    WorkItem w = stop_item();
    if (total < 0 || item < total) {
      if (live) {
        w = decode_live(sp, sched, item, lane);
        if (w.kind == ITEM_COMPUTE) {
          base = w.start >> 8;
          if (first && w.b == guess_row && base == guess_base)
            my_page = guess_page;
          else
            my_page = base + lane < p.table_width
                          ? __ldg(p.table + (int64_t)w.b * p.table_stride + base + lane) : 0;
        }
      } else {
        w = decode_dense(p, item, p.sched != nullptr, lane, skip, base, my_page);
      }
    }
    // Dense enumeration without claims past the first wave: the next item is
    // item + gridDim.x, so whether this one is the CTA's last is known now.
    if (!live && (p.sched == nullptr || total <= (int)gridDim.x) && item + (int)gridDim.x >= total)
      w.last = 1;
    // A skipped item (empty, its partition not stored) moves on to the next.
    if (w.kind == ITEM_STOP && !skip) {
      publish(ring, k, w, p.fault, abort_flag, lane);
      break;
    }
    if (!skip && !publish(ring, k, w, p.fault, abort_flag, lane)) {
      ok = false;
      break;
    }
    // The next item is claimed once this one's first copies are issued, so
    // the atomic's round trip (and the live schedule's total) overlaps them.
    int claimed = 0;
    bool claimed_yet = false;
    auto claim = [&]() {
      if (claimed_yet) return;
      claimed_yet = true;
      if (total < 0) total = schedule_total(sp, sched, lane);
      if (dynamic < 0) dynamic = p.sched != nullptr && total > (int)gridDim.x;
      if (dynamic && lane == 0) claimed = atomicAdd(p.sched, 1);
    };
    if (w.kind == ITEM_COMPUTE) {
      const int32_t *trow = p.table + (int64_t)w.b * p.table_stride;
      const int kvh = w.hs / p.nsub;
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
            tma_load_5d(kbuf + s * TILE_BYTES, k_map, 0, tok & 255, 0, kvh, page, &full[s], policy);
            tma_load_5d(vbuf + s * TILE_BYTES, v_map, 0, tok & 255, 0, kvh, page, &full[s], policy);
          }
        }
        ok = __shfl_sync(FULL_MASK, ok, 0);
        if (!ok) break;
        if (i + 1 == min(ntiles, NS)) claim();
      }
    }
    first = false;
    if (!ok) break;
    claim();
    item = dynamic ? (int)gridDim.x + __shfl_sync(FULL_MASK, claimed, 0) : item + (int)gridDim.x;
  }
  if (!ok && lane == 0) {
    // Let the copies already issued land before the CTA exits.
    const uint32_t j0 = it > NS ? it - NS : 0;
    for (uint32_t j = j0; j < it; ++j)
      mbar_wait_bounded(&full[j % NS], (j / NS) & 1, p.fault, FAULT_DRAIN_WAIT);
  }
  // Count this CTA as finished; the last one resets the scheduler words for
  // the next launch (every CTA's final claim precedes its count, and no
  // claim follows the last count).  Every CTA that claimed computed the same
  // `dynamic` (a CTA whose first item was past the end never claims, and
  // then the first wave held every item, so no CTA used the counter).
  if (dynamic > 0 && lane == 0) {
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

// Column of element (head g, column d) in a row of the combine area: bits 3-4
// of the column are XOR-ed with bits 1-2 of g, so the four head rows that an
// MMA fragment stores at once (g = quad * 2 + j) fall in four different
// groups of 8 banks instead of the same ones; 4 consecutive columns stay
// contiguous (float4 reads).
__device__ __forceinline__ int comb_col(int g, int d) { return d ^ (((g >> 1) & 3) << 3); }

// Merge NC per-warp (or per-group) softmax states of one item and store the
// outputs, with the NW consumer warps' threads (tid < NW * 32).
//   comb_acc [NC][GC][D]  unnormalised accumulators (relative to each state's max),
//                         columns placed by comb_col
//   comb_ml  [NC][2][GC]  per-state running max (base-2 scaled units) and sum
// M = max_w m_w; f_w = 2^(m_w - M); L = sum f_w l_w; O = sum f_w acc_w.
// Stores O/L + LSE (natural log), (M ln2, L, O), or BF16 O/L.
template <int D, int GC, int NC, int NW = NC>
__device__ void combine_and_store(const PartitionParams &p, const WorkItem &w, int h0, int rows,
                                  const float *comb_acc, const float *comb_ml, int tid) {
  // Each thread merges 8 consecutive columns of one head row per pass, so a
  // row's weights, 1/L and LSE are computed once for both of its float4s and
  // one pass covers 4 heads at D = 256 (8 at D = 128): measured on B200, the
  // second pass of 4-column chunks was ~0.27 us of a config 3 B=1 item.
  constexpr int V = 8;
#pragma unroll 1
  for (int e = tid * V; e < rows * D; e += NW * 32 * V) {
    const int g = e / D, d = e % D;
    float mx = -INFINITY;
#pragma unroll
    for (int wi = 0; wi < NC; ++wi) mx = fmaxf(mx, comb_ml[wi * 2 * GC + g]);
    float den = 0.f;
    float4 o0 = make_float4(0.f, 0.f, 0.f, 0.f), o1 = o0;
    const int c = comb_col(g, d);  // columns d + 4.. follow at c + 4 (bit 2 is not swizzled)
#pragma unroll
    for (int wi = 0; wi < NC; ++wi) {
      const float mw = comb_ml[wi * 2 * GC + g];
      const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - mx);
      den += f * comb_ml[wi * 2 * GC + GC + g];
      const float *src = comb_acc + (wi * GC + g) * D + c;
      const float4 a0 = *reinterpret_cast<const float4 *>(src);
      const float4 a1 = *reinterpret_cast<const float4 *>(src + 4);
      o0.x += f * a0.x;
      o0.y += f * a0.y;
      o0.z += f * a0.z;
      o0.w += f * a0.w;
      o1.x += f * a1.x;
      o1.y += f * a1.y;
      o1.z += f * a1.z;
      o1.w += f * a1.w;
    }
    const int64_t row = (int64_t)w.b * p.num_heads + h0 + g;
    const int64_t idx = row * p.splits + w.split;
    if (p.mode == MODE_MLA) {
      float4 *dst = reinterpret_cast<float4 *>(p.accums + idx * D + d);
      dst[0] = o0;
      dst[1] = o1;
      if (d == 0) {
        p.maxima[idx] = mx * LN2;
        p.denoms[idx] = den;
      }
    } else {
      const float inv = 1.f / den;
      o0.x *= inv;
      o0.y *= inv;
      o0.z *= inv;
      o0.w *= inv;
      o1.x *= inv;
      o1.y *= inv;
      o1.z *= inv;
      o1.w *= inv;
      if (p.mode == MODE_LSE) {
        float4 *dst = reinterpret_cast<float4 *>(p.partial + idx * D + d);
        dst[0] = o0;
        dst[1] = o1;
        if (d == 0) p.lse[idx] = (mx + log2f(den)) * LN2;
      } else {
        uint4 packed;
        __nv_bfloat162 b0 = __floats2bfloat162_rn(o0.x, o0.y), b1 = __floats2bfloat162_rn(o0.z, o0.w);
        __nv_bfloat162 b2 = __floats2bfloat162_rn(o1.x, o1.y), b3 = __floats2bfloat162_rn(o1.z, o1.w);
        packed.x = *reinterpret_cast<uint32_t *>(&b0);
        packed.y = *reinterpret_cast<uint32_t *>(&b1);
        packed.z = *reinterpret_cast<uint32_t *>(&b2);
        packed.w = *reinterpret_cast<uint32_t *>(&b3);
        *reinterpret_cast<uint4 *>(p.out + row * D + d) = packed;
      }
    }
  }
}

// Host: the live schedule pays when a launch has more (dense) items than CTAs
// -- partitions past the rows' lengths would otherwise cost claims -- and the
// lengths fit the producer's registers and local memory.  Balanced partition
// bounds are derived per item (dense enumeration only).
inline int live_schedule(const PartitionParams &p, int grid) {
  return !p.balanced && p.batch <= 32 * RMAX && p.n_items > grid ? 1 : 0;
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
  r.peek = reinterpret_cast<volatile int *>(smem + L::FLAG_OFFSET) + 2;
  return r;
}

}  // namespace pdl
