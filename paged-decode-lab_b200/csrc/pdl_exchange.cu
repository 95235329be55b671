// pdl_exchange.cu -- context-parallel combine over peer memory in one kernel.
//
// Context parallelism gives every rank a range of each row's pages; each rank
// has decoded its range into a split workspace (normalised partials + LSE).
// This kernel replaces "local merge -> all-gather -> merge" with one launch.
// Each warp owns a fixed list of units (row, column slice), the same list on
// every rank, and for each of them:
//
//   1. merges this rank's partitions (rows staged through shared memory with
//      cp.async, as in the merge kernel) and stores the merged FP32 partial
//      and LSE into block `rank` of EVERY rank's exchange buffer (peer stores
//      over NVLink), each float as one 8-byte word (float bits | sequence
//      << 32) written with a single-copy-atomic relaxed system-scope store;
//   2. reads the `world` blocks of the unit from this GPU's own buffer,
//      re-reading until every word carries this call's sequence number (for
//      at most the timeout; then it records FAULT_EXCHANGE_WAIT and leaves
//      that warp's remaining rows unwritten), and merges them into the BF16
//      output.
//
// The sequence travels inside every word, so no fence, flag or barrier is
// needed: a word whose sequence matches holds this call's value (measured on
// B200: a system-scope fence before a separate flag cost ~11 us per call; a
// round trip of relaxed stores over NVLink ~1.6 us).
//
// Sequence numbers live in the buffer (seq[w], advanced by warp w itself), so
// CUDA-graph replays need no host-side counter.  Data is double-buffered by
// sequence parity: a peer can run at most one call ahead (to finish call k+1
// it needs this rank's call-k+1 words, which this rank stores only after its
// call-k kernel completed), so a peer never overwrites a half still being read.
//
// Both merges compute exactly what merge_slice (pdl_merge_core.cuh) computes
// for the two-kernel path (pdl_lse_merge locally, an all-gather, pdl_lse_merge
// over the gathered blocks), so the output is bit-identical to it.
//
// Emulation (testing on one GPU): with `emulate`, blockIdx.y is the rank,
// every rank's workspace, lengths and output are consecutive slices and all
// buffers are on this GPU; the launch is cooperative, so every CTA of every
// emulated rank is resident and the waits between them can complete.
#include "pdl_merge_core.cuh"

namespace pdl {
namespace {

__device__ __forceinline__ uint64_t pack_word(float v, uint32_t seq) {
  return (uint64_t)__float_as_uint(v) | ((uint64_t)seq << 32);
}

__device__ __forceinline__ float word_value(uint64_t w) { return __uint_as_float((uint32_t)w); }

__device__ __forceinline__ uint32_t word_seq(uint64_t w) { return (uint32_t)(w >> 32); }

__device__ __forceinline__ void store_words(uint64_t *p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b)
               : "memory");
}

__device__ __forceinline__ void store_word(uint64_t *p, uint64_t a) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}

__device__ __forceinline__ void load_words(const uint64_t *p, uint64_t &a, uint64_t &b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p)
               : "memory");
}

__device__ __forceinline__ uint64_t load_word(const uint64_t *p) {
  uint64_t a;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}

constexpr int kExchangeStageParts = 16;

// Shared memory of one exchange CTA: each warp stages up to 16 partition
// rows of its column slice (at most 32 KB, so kExchangeCtasPerSm CTAs fit).
constexpr size_t exchange_smem_bytes(int head_dim, int splits) {
  return (size_t)kExchangeWarps * (splits < kExchangeStageParts ? splits : kExchangeStageParts) *
         (head_dim < 128 ? head_dim : 128) * 4;
}

__device__ __forceinline__ uint64_t *block_of(unsigned char *buffer, int64_t half, int rank,
                                              int64_t block) {
  return reinterpret_cast<uint64_t *>(buffer + kExchangeHeaderBytes) + half + rank * block;
}

template <int D>
__global__ void __launch_bounds__(32 * kExchangeWarps, kExchangeCtasPerSm)
    exchange_kernel(const ExchangeParams p) {
  constexpr int CW = D < 128 ? D : 128;  // columns per warp
  constexpr int SLICES = D / CW;
  constexpr int E = CW / 32;
  const int lane = threadIdx.x & 31;
  const int rank = p.emulate ? (int)blockIdx.y : p.rank;
  const int warp = blockIdx.x * kExchangeWarps + (threadIdx.x >> 5);
  const int units = p.rows * SLICES;
  const int stride = p.ctas * kExchangeWarps;
  const int64_t rank_slice = p.emulate ? rank : 0;
  const float *partial = p.partial + rank_slice * p.rows * p.splits * D;
  const float *lse = p.lse + rank_slice * p.rows * p.splits;
  const int32_t *lengths =
      p.lengths != nullptr ? p.lengths + rank_slice * (p.rows / p.num_heads) : nullptr;
  __nv_bfloat16 *out = p.out + rank_slice * p.rows * D;
  uint32_t *own_seq = reinterpret_cast<uint32_t *>(p.buffers[rank]);
  // Local partition rows are staged through shared memory, up to
  // kExchangeStageParts at a time per warp.
  extern __shared__ __align__(16) float stage[];
  const int stage_cap = min(p.splits, kExchangeStageParts);

  // The next step's partition kernel may be scheduled now (it waits for this
  // grid before touching anything).  The local partitions are the previous
  // kernel's output, and this rank's previous exchange may still read the
  // buffers until it completes.
  allow_dependent_launch();
  grid_dependency_wait();
  const uint32_t seq = __shfl_sync(FULL_MASK, lane == 0 ? own_seq[warp] + 1u : 0u, 0);
  const int64_t half = (int64_t)(seq & 1u) * p.world * p.block;

  // 1. Local merge; store the merged words into every rank's buffer.
  for (int unit = warp; unit < units; unit += stride) {
    const int row = unit / SLICES, col0 = (unit % SLICES) * CW;
    int live = p.splits;
    if (lengths != nullptr) {
      const int len = __ldg(lengths + row / p.num_heads);
      live = min(live, (int)((len + (int64_t)p.tokens_per_split - 1) / p.tokens_per_split));
    }
    float acc[E], shift, tot;
    merge_slice<E>(true, lse + (int64_t)row * p.splits, 1, nullptr,
                          partial + (int64_t)row * p.splits * D + col0, D, live, lane,
                          stage + (threadIdx.x >> 5) * stage_cap * 32 * E, stage_cap, acc, shift,
                          tot);
    const uint64_t lse_word = pack_word(tot > 0.f ? shift : -INFINITY, seq);
    for (int q = 0; q < p.world; ++q) {
      uint64_t *dst = block_of(p.buffers[q], half, rank, p.block);
#pragma unroll
      for (int e = 0; e < E; e += 2)
        store_words(dst + (int64_t)row * D + col0 + lane * E + e, pack_word(acc[e], seq),
                    pack_word(acc[e + 1], seq));
      if (lane == 0 && col0 == 0) store_word(dst + (int64_t)p.rows * D + row, lse_word);
    }
  }

  // 2. Wait for every rank's words of each unit, then merge the ranks.
  const uint64_t *g = block_of(p.buffers[rank], half, 0, p.block);
  bool gave_up = false;
  uint64_t t0 = 0;
  for (int unit = warp; unit < units && !gave_up; unit += stride) {
    const int row = unit / SLICES, col0 = (unit % SLICES) * CW;
    uint64_t v[kMaxPeers][E];
    uint64_t w = 0;
    while (true) {
      bool ok = true;
#pragma unroll
      for (int q = 0; q < kMaxPeers; ++q) {
        if (q < p.world) {
          const uint64_t *src = g + q * p.block + (int64_t)row * D + col0 + lane * E;
#pragma unroll
          for (int e = 0; e < E; e += 2) {
            load_words(src + e, v[q][e], v[q][e + 1]);
            ok = ok && word_seq(v[q][e]) == seq && word_seq(v[q][e + 1]) == seq;
          }
        }
      }
      if (lane < p.world) {
        w = load_word(g + lane * p.block + (int64_t)p.rows * D + row);
        ok = ok && word_seq(w) == seq;
      }
      if (__all_sync(FULL_MASK, ok)) break;
      // The timeout decision is lane 0's, so the warp leaves together.
      int expired = 0;
      if (lane == 0) {
        const uint64_t now = global_timer_ns();
        if (t0 == 0) t0 = now;
        expired = now - t0 > p.timeout_ns;
        if (expired) atomicOr(p.fault, FAULT_EXCHANGE_WAIT);
      }
      if (__shfl_sync(FULL_MASK, expired, 0)) {
        gave_up = true;
        break;
      }
      __nanosleep(64);
    }
    if (gave_up) break;

    // The arithmetic of merge_slice with live = world partitions held in
    // registers (lane q holds rank q's LSE).
    const float wr = lane < p.world ? word_value(w) : -INFINITY;
    float mx = warp_max_all(wr);
    if (mx == -INFINITY) mx = 0.f;
    const float tot = warp_sum_all(lane < p.world ? expf(wr - mx) : 0.f);
    const float shift = tot > 0.f ? logf(tot) + mx : INFINITY;
    const float wl = lane < p.world ? expf(wr - shift) : 0.f;
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxPeers; ++q) {
      const float wk = __shfl_sync(FULL_MASK, wl, q);
      if (q < p.world) {
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] = fmaf(wk, word_value(v[q][e]), acc[e]);
      }
    }
    __nv_bfloat16 *dst = out + (int64_t)row * D + col0 + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2)
      *reinterpret_cast<__nv_bfloat162 *>(dst + e) = __floats2bfloat162_rn(acc[e], acc[e + 1]);
  }
  if (lane == 0) own_seq[warp] = seq;
}

template <int D>
cudaError_t launch_exchange_t(const ExchangeParams &params, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(params.ctas, params.emulate ? params.world : 1);
  cfg.blockDim = dim3(32 * kExchangeWarps);
  cfg.dynamicSmemBytes = exchange_smem_bytes(D, params.splits);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (params.emulate) {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, exchange_kernel<D>, params);
}

}  // namespace

cudaError_t launch_exchange(const ExchangeParams &params, int head_dim, cudaStream_t stream) {
  switch (head_dim) {
    case 64: return launch_exchange_t<64>(params, stream);
    case 128: return launch_exchange_t<128>(params, stream);
    case 256: return launch_exchange_t<256>(params, stream);
    default: return cudaErrorInvalidValue;
  }
}

int exchange_ctas(int rows, int head_dim, int world, int sm_count, bool emulate) {
  const int slices = head_dim <= 128 ? 1 : head_dim / 128;
  const int64_t units = (int64_t)rows * slices;
  int64_t ctas = (units + kExchangeWarps - 1) / kExchangeWarps;
  int64_t cap = (int64_t)kExchangeCtasPerSm * sm_count;
  if (emulate) cap /= world;
  if (cap > kMaxExchangeCtas) cap = kMaxExchangeCtas;
  if (ctas > cap) ctas = cap;
  return ctas < 1 ? 1 : (int)ctas;
}

}  // namespace pdl
