// pdl_capi.cu -- extern "C" entry points declared in include/pdl_b200.h.
//
// Host-side only: argument validation (status codes, no exceptions), the
// static split-KV plan, TMA descriptor encoding for the paged K/V pools, the
// per-device state (SM count, fault word) and the launch sequence.  Nothing
// here allocates device memory, synchronises, or reads device memory, so every
// launch entry point can be captured in a CUDA graph.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "pdl_b200.h"
#include "pdl_internal.h"

// Sticky per-device fault word written by bounded device-side waits.
__device__ uint32_t g_pdl_fault_word;

namespace pdl {
namespace {

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  uint32_t *fault = nullptr;  // device address of g_pdl_fault_word
};

DeviceState g_devices[kMaxDevices];
std::mutex g_mutex;

// Description of the last failure on this host thread (pdl_last_error).
thread_local char g_last_error[256] = "";

int fail(int status, const char *where, const char *detail) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", where, detail ? detail : "");
  return status;
}

int cuda_fail(const char *where, cudaError_t e) {
  return fail(PDL_ERR_CUDA, where, cudaGetErrorString(e));
}

int current_device_state(DeviceState **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PDL_ERR_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return PDL_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState &st = g_devices[dev];
  if (!st.ready) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return PDL_ERR_DEVICE;
    if (major != 10) return PDL_ERR_DEVICE;  // built for sm_100a only
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return PDL_ERR_DEVICE;
    void *addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_pdl_fault_word);
    if (e != cudaSuccess) return cuda_fail("cudaGetSymbolAddress(fault word)", e);
    st.sm_count = sms;
    st.fault = static_cast<uint32_t *>(addr);
    st.ready = true;
  }
  *out = &st;
  return PDL_OK;
}

// cuTensorMapEncodeTiled from the driver, fetched through the runtime so the
// library does not link libcuda directly.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// View of a paged pool [pages, 256, Hkv, D] as a 5-D tensor
// (64 columns, 256 slots, D/64 column bands, Hkv, pages) with strides
// (2 B, Hkv*D*2, 128 B, D*2, 256*Hkv*D*2) and boxes of (64, box_tokens,
// D/64, 1, 1): one box is a whole T-token tile of one KV head inside one
// page, landed band after band -- [band][slot][128 bytes] with the 128-byte
// swizzle, the layout the kernels read -- so a tile of K (or V) is one copy
// instead of D/64.  Every coordinate stays inside its extent, so every byte
// read lies inside the pool.
int encode_pool_map(CUtensorMap *map, const void *base, int64_t pages, int hkv, int dim,
                    int box_tokens) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return fail(PDL_ERR_CUDA, "cudaGetDriverEntryPoint", "cuTensorMapEncodeTiled");
  const cuuint64_t dims[5] = {64u, 256u, (cuuint64_t)dim / 64, (cuuint64_t)hkv, (cuuint64_t)pages};
  const cuuint64_t strides[4] = {(cuuint64_t)hkv * dim * 2, 128u, (cuuint64_t)dim * 2,
                                 (cuuint64_t)256 * hkv * dim * 2};
  const cuuint32_t box[5] = {64u, (cuuint32_t)box_tokens, (cuuint32_t)dim / 64, 1u, 1u};
  const cuuint32_t elem[5] = {1u, 1u, 1u, 1u, 1u};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void *>(base), dims,
                        strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char detail[96];
    snprintf(detail, sizeof(detail), "CUresult %d", (int)r);
    return fail(PDL_ERR_CUDA, "cuTensorMapEncodeTiled", detail);
  }
  return PDL_OK;
}

// Encoded descriptors are cached per host thread: a decode loop reuses the
// same pools call after call, and encoding is pure host work.
struct PoolMapEntry {
  const void *base;
  int64_t pages;
  int hkv, dim, box;
  CUtensorMap map;
};
constexpr int kPoolMapCache = 8;
thread_local PoolMapEntry g_pool_maps[kPoolMapCache];
thread_local int g_pool_map_next = 0;

int cached_pool_map(CUtensorMap *map, const void *base, int64_t pages, int hkv, int dim,
                    int box_tokens) {
  for (int i = 0; i < kPoolMapCache; ++i) {
    const PoolMapEntry &e = g_pool_maps[i];
    if (e.base == base && base != nullptr && e.pages == pages && e.hkv == hkv && e.dim == dim &&
        e.box == box_tokens) {
      *map = e.map;
      return PDL_OK;
    }
  }
  const int st = encode_pool_map(map, base, pages, hkv, dim, box_tokens);
  if (st != PDL_OK) return st;
  PoolMapEntry &slot = g_pool_maps[g_pool_map_next];
  g_pool_map_next = (g_pool_map_next + 1) % kPoolMapCache;
  slot.base = base;
  slot.pages = pages;
  slot.hkv = hkv;
  slot.dim = dim;
  slot.box = box_tokens;
  slot.map = *map;
  return PDL_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool valid_dim(int d) { return d == 64 || d == 128 || d == 256; }

// Which partition kernel serves this launch.  Measured on B200 at ~1 GB of
// KV: the CUDA-core kernel is at or above the tensor-core one for 1 and 2
// query heads per KV head and becomes issue-bound from 4 (ncu: 54% issue
// active, 39% DRAM throughput at D=256), where the tensor-core kernel stays
// DRAM-bound; so AUTO switches at 3.
int choose_kernel(const PdlDecodeArgs &a) {
  const int group = a.num_heads / a.num_kv_heads;
  if (a.kernel == PDL_KERNEL_SIMT) return PDL_KERNEL_SIMT;
  if (a.kernel == PDL_KERNEL_MMA) return PDL_KERNEL_MMA;
  return group >= 3 ? PDL_KERNEL_MMA : PDL_KERNEL_SIMT;
}

// Checks shared by every launch entry point; mirrors the tensor contract of
// the reference's _validate (src/paged_decode/runtime.py:46-84) on raw
// pointers and sizes.
int validate_common(const PdlDecodeArgs *a) {
  if (a == nullptr) return PDL_ERR_NULL;
  if (!valid_dim(a->head_dim)) return PDL_ERR_GEOMETRY;
  if (a->num_heads <= 0 || a->num_kv_heads <= 0 || a->num_heads % a->num_kv_heads)
    return PDL_ERR_GEOMETRY;
  if (a->batch <= 0 || a->batch > 65535) return PDL_ERR_SHAPE;
  if (!std::isfinite(a->scale)) return PDL_ERR_SCALE;
  if (a->splits <= 0 || a->tokens_per_split < 0) return PDL_ERR_SPLITS;
  if (a->tokens_per_split == 0 && a->splits != 1) return PDL_ERR_SPLITS;
  if (a->protocol != PDL_PROTOCOL_LSE && a->protocol != PDL_PROTOCOL_MLA) return PDL_ERR_SHAPE;
  if (a->flags & ~(PDL_FLAG_SKIP_EMPTY | PDL_FLAG_DIRECT_SINGLE | PDL_FLAG_DYNAMIC |
                   PDL_FLAG_BALANCED))
    return fail(PDL_ERR_SHAPE, "flags", "unknown PdlFlags bit");
  if ((a->flags & PDL_FLAG_BALANCED) && a->tokens_per_split == 0)
    return fail(PDL_ERR_SPLITS, "flags", "balanced partitions need a granule (tokens_per_split)");
  return PDL_OK;
}

int validate_partition_inputs(const PdlDecodeArgs *a) {
  if (!a->q || !a->k_cache || !a->v_cache || !a->block_table || !a->lengths) return PDL_ERR_NULL;
  if (a->num_pages <= 0 || a->num_pages > INT32_MAX) return PDL_ERR_SHAPE;
  if (a->table_width <= 0 || a->table_stride < a->table_width) return PDL_ERR_SHAPE;
  if ((int64_t)a->table_width * PDL_PAGE_SIZE > INT32_MAX) return PDL_ERR_SHAPE;
  if (a->q_stride_head < a->head_dim || a->q_stride_batch < 1) return PDL_ERR_SHAPE;
  if (!aligned(a->k_cache, 16) || !aligned(a->v_cache, 16)) return PDL_ERR_ALIGNMENT;
  if (!aligned(a->q, 2)) return PDL_ERR_ALIGNMENT;
  if (a->tokens_per_split > 0 && !(a->flags & PDL_FLAG_BALANCED)) {
    // Every token the table can address must belong to some partition
    // (balanced partitions always cover the row).
    const int64_t covered = (int64_t)a->splits * a->tokens_per_split;
    if (covered < (int64_t)a->table_width * PDL_PAGE_SIZE) return PDL_ERR_SPLITS;
  }
  return PDL_OK;
}

int validate_workspace(const PdlDecodeArgs *a) {
  if (a->protocol == PDL_PROTOCOL_LSE) {
    if (!a->partial || !a->lse) return PDL_ERR_WORKSPACE;
    if (!aligned(a->partial, 16)) return PDL_ERR_ALIGNMENT;
  } else {
    if (!a->maxima || !a->denoms || !a->accums) return PDL_ERR_WORKSPACE;
    if (!aligned(a->accums, 16)) return PDL_ERR_ALIGNMENT;
  }
  return PDL_OK;
}

int validate_out(const PdlDecodeArgs *a) {
  if (!a->out) return PDL_ERR_NULL;
  if (!aligned(a->out, 16)) return PDL_ERR_ALIGNMENT;
  return PDL_OK;
}

int status_from_cuda(cudaError_t e, const char *where) {
  return e == cudaSuccess ? PDL_OK : cuda_fail(where, e);
}

// Launch the partition kernel in `mode` (MODE_LSE / MODE_MLA / MODE_DIRECT).
int run_partition(const PdlDecodeArgs *a, int mode, cudaStream_t stream) {
  DeviceState *dev = nullptr;
  int st = current_device_state(&dev);
  if (st != PDL_OK) return st;
  const int which = choose_kernel(*a);
  const int group = a->num_heads / a->num_kv_heads;
  int per_cta = 0, box = 0;
  if (which == PDL_KERNEL_SIMT) {
    per_cta = simt_heads_per_cta(group);
    box = simt_tile_tokens(a->head_dim);
  } else {
    per_cta = mma_heads_per_cta(group, a->head_dim);
    box = mma_tile_tokens(a->head_dim);
    if (per_cta <= 0) return PDL_ERR_KERNEL;
  }
  const int nsub = (group + per_cta - 1) / per_cta;
  const int64_t items = (int64_t)a->splits * a->num_kv_heads * nsub * a->batch;
  // Item indices (and the fill items added per row) stay in int32.
  if (items + a->batch > INT32_MAX) return PDL_ERR_SHAPE;

  CUtensorMap kmap, vmap;
  st = cached_pool_map(&kmap, a->k_cache, a->num_pages, a->num_kv_heads, a->head_dim, box);
  if (st != PDL_OK) return st;
  st = cached_pool_map(&vmap, a->v_cache, a->num_pages, a->num_kv_heads, a->head_dim, box);
  if (st != PDL_OK) return st;

  KernelLaunch L;
  std::memset(&L, 0, sizeof(L));
  L.k_map = &kmap;
  L.v_map = &vmap;
  L.head_dim = a->head_dim;
  L.group_per_cta = per_cta;
  L.sm_count = dev->sm_count;
  PartitionParams &p = L.params;
  p.q = static_cast<const __nv_bfloat16 *>(a->q);
  p.q_stride_batch = a->q_stride_batch;
  p.q_stride_head = a->q_stride_head;
  p.table = a->block_table;
  p.table_stride = a->table_stride;
  p.table_width = a->table_width;
  p.lengths = a->lengths;
  p.batch = a->batch;
  p.num_heads = a->num_heads;
  p.num_kv_heads = a->num_kv_heads;
  p.group = group;
  p.nsub = nsub;
  p.tokens_per_split = a->tokens_per_split > 0 ? a->tokens_per_split : (1 << 30);
  p.splits = a->splits;
  p.n_items = (int32_t)items;
  p.log2_scale = a->scale * 1.4426950408889634f;
  p.mode = mode;
  p.q_vec16 = aligned(a->q, 16) && (a->q_stride_batch % 8 == 0) && (a->q_stride_head % 8 == 0);
  p.write_empty = (a->flags & PDL_FLAG_SKIP_EMPTY) ? 0 : 1;
  // A fill item stores whole empty partitions of all heads of a row, about
  // 128 KB: a launch's fills then take a few items per row, not one per
  // partition (each item costs the producer a schedule decode, microseconds
  // that fills of a few KB cannot hide).
  p.fill_splits =
      (int)std::max<int64_t>(1, 131072 / ((int64_t)a->num_heads * (a->head_dim + 1) * 4));
  p.out = static_cast<__nv_bfloat16 *>(a->out);
  p.partial = a->partial;
  p.lse = a->lse;
  p.maxima = a->maxima;
  p.denoms = a->denoms;
  p.accums = a->accums;
  p.fault = dev->fault;
  // Dynamic scheduling: counters[0] counts claimed items, counters[1]
  // finished CTAs.  The kernel uses them only when a launch has more live
  // items than CTAs (each CTA's first item is blockIdx.x, no atomic).
  p.sched = (a->flags & PDL_FLAG_DYNAMIC) ? a->counters : nullptr;
  p.balanced = (a->flags & PDL_FLAG_BALANCED) ? 1 : 0;
  const cudaError_t e = which == PDL_KERNEL_SIMT ? launch_partition_simt(L, stream)
                                                 : launch_partition_mma(L, stream);
  return status_from_cuda(e, which == PDL_KERNEL_SIMT ? "partition (simt)" : "partition (mma)");
}

// `after_partition`: the launch directly follows this library's partition
// kernel on the stream (pdl_paged_decode), so the merge may read the lengths
// before its dependency wait.
int run_merge(const PdlDecodeArgs *a, cudaStream_t stream, bool after_partition) {
  MergeParams m;
  std::memset(&m, 0, sizeof(m));
  m.partial = a->partial;
  m.lse = a->lse;
  m.maxima = a->maxima;
  m.denoms = a->denoms;
  m.accums = a->accums;
  m.out = static_cast<__nv_bfloat16 *>(a->out);
  // Partitions past ceil(len / tokens_per_split) are empty and weigh exactly
  // 0, so the merge reads only the live ones whenever lengths are known.
  m.lengths = a->lengths;
  m.early_lengths = after_partition ? 1 : 0;
  m.balanced = (a->flags & PDL_FLAG_BALANCED) ? 1 : 0;
  m.cap_tokens = a->table_width * PDL_PAGE_SIZE;
  m.num_heads = a->num_heads;
  m.tokens_per_split = a->tokens_per_split > 0 ? a->tokens_per_split : (1 << 30);
  m.rows = a->batch * a->num_heads;
  m.splits = a->splits;
  m.protocol = a->protocol == PDL_PROTOCOL_LSE ? MODE_LSE : MODE_MLA;
  m.row_stride = (int64_t)a->splits * a->head_dim;
  m.part_stride = a->head_dim;
  m.w_row_stride = a->splits;
  m.w_part_stride = 1;
  return status_from_cuda(launch_merge(m, a->head_dim, stream), "merge");
}

float to_f32(double x) { return static_cast<float>(x); }

}  // namespace
}  // namespace pdl

using namespace pdl;

extern "C" int pdl_abi_version(void) { return PDL_ABI_VERSION; }

extern "C" const char *pdl_last_error(void) { return g_last_error; }

extern "C" const char *pdl_status_string(int status) {
  switch (status) {
    case PDL_OK: return "ok";
    case PDL_ERR_NULL: return "null pointer";
    case PDL_ERR_GEOMETRY: return "unsupported geometry";
    case PDL_ERR_SHAPE: return "invalid shape or stride";
    case PDL_ERR_WORKSPACE: return "invalid or missing preallocated split-K workspace";
    case PDL_ERR_SCALE: return "invalid scale";
    case PDL_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case PDL_ERR_SPLITS: return "invalid split configuration";
    case PDL_ERR_CUDA: return "CUDA call failed";
    case PDL_ERR_DEVICE: return "no usable sm_100 device";
    case PDL_ERR_KERNEL: return "kernel variant unavailable for this shape";
    case PDL_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" int pdl_spec_geometry(const PdlSpec *spec, int32_t *partitions, int32_t *table_width,
                                 int64_t *split_workspace_bytes) {
  if (!spec) return PDL_ERR_NULL;
  if (spec->max_batch <= 0 || spec->num_heads <= 0 || spec->num_kv_heads <= 0 ||
      spec->max_context_len <= 0)
    return PDL_ERR_SHAPE;
  if (!valid_dim(spec->head_dim) || spec->page_size != PDL_PAGE_SIZE ||
      spec->num_heads % spec->num_kv_heads)
    return PDL_ERR_GEOMETRY;
  const int64_t parts = ((int64_t)spec->max_context_len + 1023) / 1024;
  const int64_t width = ((int64_t)spec->max_context_len + PDL_PAGE_SIZE - 1) / PDL_PAGE_SIZE;
  if (partitions) *partitions = (int32_t)parts;
  if (table_width) *table_width = (int32_t)width;
  if (split_workspace_bytes)
    *split_workspace_bytes =
        (int64_t)spec->max_batch * spec->num_heads * parts * (spec->head_dim + 2) * 4;
  return PDL_OK;
}

// Static plan: same integer and float32 steps as the reference heuristic
// (src/paged_decode/splitkv_plan.py:26-56).  Python floats are doubles there;
// every _f32() rounding is a cast to float here.
extern "C" int pdl_splitkv_plan(const PdlSpec *spec, int32_t sm_count, int32_t num_splits,
                                PdlPlan *plan) {
  if (!spec || !plan) return PDL_ERR_NULL;
  int st = pdl_spec_geometry(spec, nullptr, nullptr, nullptr);
  if (st != PDL_OK) return st;
  if (sm_count < 1) return PDL_ERR_SHAPE;
  if (num_splits < 0 || num_splits > 128) return PDL_ERR_SPLITS;
  if (spec->num_heads / spec->num_kv_heads > 16) return PDL_ERR_GEOMETRY;
  const int tile = spec->head_dim == 64 ? 256 : (spec->head_dim == 128 ? 128 : 64);
  const int64_t capacity = ((int64_t)spec->max_context_len + 255) / 256 * 256;
  const int64_t blocks = (capacity + tile - 1) / tile;
  int64_t splits = num_splits;
  if (splits == 0) {
    const int64_t work = (int64_t)spec->max_batch * spec->num_kv_heads;
    const int64_t virt = (int64_t)sm_count * 2;
    const float threshold = to_f32((double)to_f32(0.8) * (double)virt);
    if ((double)work >= (double)threshold) {
      splits = 1;
    } else {
      const int64_t maximum = std::min<int64_t>(std::min<int64_t>(128, virt), blocks);
      float eff[129];
      bool ok[129];
      float best = 0.f;
      for (int64_t n = 1; n <= maximum; ++n) {
        ok[n] = n == 1 || (blocks + n - 1) / n != (blocks + n - 2) / (n - 1);
        if (!ok[n]) continue;
        const float waves = to_f32((double)to_f32((double)(work * n)) / (double)virt);
        eff[n] = to_f32((double)waves / std::ceil((double)waves));
        best = std::max(best, eff[n]);
      }
      splits = 1;
      for (int64_t n = 1; n <= maximum; ++n) {
        if (ok[n] && (double)eff[n] >= 0.85 * (double)best) {
          splits = n;
          break;
        }
      }
    }
  }
  int64_t padded = 1;
  while (padded < splits) padded <<= 1;
  const int64_t merge_rows = spec->head_dim % 128 == 0 ? 4 : 8;
  plan->splits = (int32_t)splits;
  plan->tile_tokens = tile;
  plan->tokens_per_split = (int32_t)((blocks + splits - 1) / splits * tile);
  plan->table_capacity_tokens = (int32_t)capacity;
  plan->lse_lanes = (int32_t)std::min<int64_t>(padded, 128 / merge_rows);
  plan->sm_count = sm_count;
  plan->explicit_splits = num_splits ? 1 : 0;
  plan->balanced = 0;
  return PDL_OK;
}

// Split plan for this library's persistent, dynamically scheduled kernels:
// about one work item per CTA slot (two CTAs per SM; measured best for
// uniform batches), items of at most 4096 tokens so variable-length batches
// balance, and never smaller than one tile (the partition sizes stay
// multiples of the reference plan's tile, so the merge and workspace layouts
// are unchanged).
extern "C" int pdl_b200_plan(const PdlSpec *spec, int32_t sm_count, PdlPlan *plan) {
  if (!spec || !plan) return PDL_ERR_NULL;
  int st = pdl_spec_geometry(spec, nullptr, nullptr, nullptr);
  if (st != PDL_OK) return st;
  if (sm_count < 1) return PDL_ERR_SHAPE;
  const int tile = spec->head_dim == 64 ? 256 : (spec->head_dim == 128 ? 128 : 64);
  const int64_t capacity = ((int64_t)spec->max_context_len + 255) / 256 * 256;
  const int64_t blocks = (capacity + tile - 1) / tile;
  const int64_t groups = (int64_t)spec->max_batch * spec->num_kv_heads;
  const int64_t slots = 2LL * sm_count;
  // One wave of items at most (rounding up would leave a few items for a
  // second wave that a handful of CTAs stream alone), and items of at most
  // 4096 tokens so variable lengths balance under dynamic scheduling.
  int64_t splits = std::max<int64_t>(std::max<int64_t>(slots / groups, 1), (capacity + 4095) / 4096);
  // Up to D = 128 an item's fixed cost is small, so a partial wave of long
  // items becomes two full waves of shorter ones (measured, B=2 x 8 KV heads
  // x 64k tokens: 304 items of 3456 tokens 0.76 of copy bandwidth, 576 of
  // 1920 tokens 1.01).  At D = 256 the per-item cost dominates (B=32: 256
  // items 0.81, 384 items 0.78) and one wave stays.
  if (spec->head_dim <= 128 && groups * splits < 2 * slots && capacity / splits > 1024)
    splits = (2 * slots + groups - 1) / groups;
  // At D = 256, between one and two waves of whole-row items the second wave
  // leaves most CTAs idle; two balanced partitions per row (3.5 waves) keep
  // them busy (config 3 B=128 per step: 173.6 -> 171.8 us at ctx 2064, the
  // partition kernel 0.963 -> 0.992 of copy bandwidth; 54.7 -> 53.3 us at
  // ctx 528.  B=64, one wave of rows, stays at 1: 86.5 vs 90.5 us).
  const bool d256_rows_wave = spec->head_dim == 256 && splits == 1 && groups > slots &&
                              groups < 2 * slots;
  if (d256_rows_wave) splits = 2;
  splits = std::min<int64_t>(std::max<int64_t>(splits, 1), blocks);
  const int64_t tps = (blocks + splits - 1) / splits * tile;
  splits = (capacity + tps - 1) / tps;  // drop partitions that would always be empty
  // One wave of long D = 256 items: the plan is made from the table capacity,
  // but rows are often shorter (config 3: 2064 of 2560 tokens splits into
  // 1280 + 784 with fixed bounds), so the plan recommends partitions that
  // follow each row's length (PDL_FLAG_BALANCED, granule tile_tokens).
  const bool balanced = spec->head_dim == 256 && splits > 1 && tps > 4 * tile &&
                        (groups * splits <= slots || d256_rows_wave);
  int64_t padded = 1;
  while (padded < splits) padded <<= 1;
  plan->splits = (int32_t)splits;
  plan->tile_tokens = tile;
  plan->tokens_per_split = (int32_t)tps;
  plan->table_capacity_tokens = (int32_t)capacity;
  plan->lse_lanes = (int32_t)std::min<int64_t>(padded, 32);
  plan->sm_count = sm_count;
  plan->explicit_splits = 1;
  plan->balanced = balanced ? 1 : 0;
  return PDL_OK;
}

extern "C" int pdl_partition(const PdlDecodeArgs *args, pdl_stream_t stream) {
  int st = validate_common(args);
  if (st == PDL_OK) st = validate_partition_inputs(args);
  if (st != PDL_OK) return st;
  if ((args->flags & PDL_FLAG_DYNAMIC) && !args->counters)
    return fail(PDL_ERR_WORKSPACE, "pdl_partition", "dynamic scheduling needs counters");
  const bool direct = args->tokens_per_split == 0;
  st = direct ? validate_out(args) : validate_workspace(args);
  if (st != PDL_OK) return st;
  const int mode = direct ? MODE_DIRECT
                          : (args->protocol == PDL_PROTOCOL_LSE ? MODE_LSE : MODE_MLA);
  return run_partition(args, mode, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int pdl_merge(const PdlDecodeArgs *args, pdl_stream_t stream) {
  int st = validate_common(args);
  if (st != PDL_OK) return st;
  if ((args->flags & PDL_FLAG_SKIP_EMPTY) && !args->lengths) return PDL_ERR_NULL;
  st = validate_workspace(args);
  if (st == PDL_OK) st = validate_out(args);
  if (st != PDL_OK) return st;
  return run_merge(args, reinterpret_cast<cudaStream_t>(stream), false);
}

extern "C" int pdl_lse_merge(const PdlMergeArgs *args, pdl_stream_t stream) {
  if (args == nullptr || args->partial == nullptr || args->lse == nullptr) return PDL_ERR_NULL;
  if (!valid_dim(args->head_dim)) return PDL_ERR_GEOMETRY;
  if (args->rows <= 0 || args->parts <= 0) return PDL_ERR_SHAPE;
  if (!args->out && !args->out_partial && !args->out_lse) return PDL_ERR_NULL;
  // Every partition row must start on a 16-byte boundary for vector loads.
  if (!aligned(args->partial, 16) || args->row_stride % 4 || args->part_stride % 4)
    return PDL_ERR_ALIGNMENT;
  if ((args->out && !aligned(args->out, 16)) ||
      (args->out_partial && !aligned(args->out_partial, 16)))
    return PDL_ERR_ALIGNMENT;
  MergeParams m;
  std::memset(&m, 0, sizeof(m));
  m.partial = args->partial;
  m.lse = args->lse;
  m.row_stride = args->row_stride;
  m.part_stride = args->part_stride;
  m.w_row_stride = args->lse_row_stride;
  m.w_part_stride = args->lse_part_stride;
  m.out = static_cast<__nv_bfloat16 *>(args->out);
  m.out_partial = args->out_partial;
  m.out_lse = args->out_lse;
  m.num_heads = 1;
  m.tokens_per_split = 1 << 30;
  m.rows = args->rows;
  m.splits = args->parts;
  m.protocol = MODE_LSE;
  return status_from_cuda(launch_merge(m, args->head_dim, reinterpret_cast<cudaStream_t>(stream)),
                          "lse merge");
}

// ---------------------------------------------------------------------------
// Peer exchange (context-parallel combine).

extern "C" int pdl_exchange_plan(int32_t rows, int32_t head_dim, int32_t world, int32_t sm_count,
                                 int32_t emulate_ranks, PdlExchangePlan *plan) {
  using namespace pdl;
  if (plan == nullptr) return PDL_ERR_NULL;
  if (!valid_dim(head_dim)) return fail(PDL_ERR_GEOMETRY, "exchange plan", "head_dim must be 64, 128 or 256");
  if (rows <= 0 || sm_count <= 0) return fail(PDL_ERR_SHAPE, "exchange plan", "rows and sm_count must be positive");
  if (world < 1 || world > PDL_MAX_PEERS) return fail(PDL_ERR_SHAPE, "exchange plan", "world must be 1..8");
  static_assert(PDL_MAX_PEERS == kMaxPeers, "peer limit mismatch");
  std::memset(plan, 0, sizeof(*plan));
  plan->ctas = exchange_ctas(rows, head_dim, world, sm_count, emulate_ranks != 0);
  plan->block_words = (int64_t)rows * head_dim + 2 * (((int64_t)rows + 1) / 2);
  plan->data_offset = kExchangeHeaderBytes;
  plan->buffer_bytes = kExchangeHeaderBytes + 2 * (int64_t)world * plan->block_words * 8;
  return PDL_OK;
}

extern "C" int pdl_peer_buffer_create(int64_t bytes, void **dev_ptr, PdlIpcHandle *handle) {
  using namespace pdl;
  if (dev_ptr == nullptr) return PDL_ERR_NULL;
  if (bytes <= 0) return fail(PDL_ERR_SHAPE, "peer buffer", "size must be positive");
  *dev_ptr = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return cuda_fail("cudaMalloc(peer buffer)", e);
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess && handle != nullptr) {
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(PdlIpcHandle), "IPC handle size");
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) std::memcpy(handle->bytes, &h, sizeof(h));
  }
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail("peer buffer set-up", e);
  }
  *dev_ptr = p;
  return PDL_OK;
}

extern "C" int pdl_peer_buffer_open(const PdlIpcHandle *handle, void **dev_ptr) {
  using namespace pdl;
  if (handle == nullptr || dev_ptr == nullptr) return PDL_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  void *p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail("cudaIpcOpenMemHandle", e);
  *dev_ptr = p;
  return PDL_OK;
}

extern "C" int pdl_peer_buffer_close(void *dev_ptr) {
  using namespace pdl;
  if (dev_ptr == nullptr) return PDL_ERR_NULL;
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? PDL_OK : cuda_fail("cudaIpcCloseMemHandle", e);
}

extern "C" int pdl_peer_buffer_free(void *dev_ptr) {
  using namespace pdl;
  if (dev_ptr == nullptr) return PDL_ERR_NULL;
  const cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? PDL_OK : cuda_fail("cudaFree(peer buffer)", e);
}

extern "C" int pdl_exchange_merge(const PdlExchangeArgs *args, pdl_stream_t stream) {
  using namespace pdl;
  if (args == nullptr || args->partial == nullptr || args->lse == nullptr || args->out == nullptr)
    return PDL_ERR_NULL;
  const PdlExchangeArgs &a = *args;
  if (!valid_dim(a.head_dim)) return fail(PDL_ERR_GEOMETRY, "exchange", "head_dim must be 64, 128 or 256");
  if (a.rows <= 0 || a.parts <= 0) return fail(PDL_ERR_SHAPE, "exchange", "rows and parts must be positive");
  if (a.world < 1 || a.world > PDL_MAX_PEERS) return fail(PDL_ERR_SHAPE, "exchange", "world must be 1..8");
  if (!a.emulate_ranks && (a.rank < 0 || a.rank >= a.world))
    return fail(PDL_ERR_SHAPE, "exchange", "rank outside [0, world)");
  for (int q = 0; q < a.world; ++q) {
    if (a.buffers[q] == nullptr) return fail(PDL_ERR_NULL, "exchange", "missing peer buffer");
    if (!aligned(a.buffers[q], 256)) return fail(PDL_ERR_ALIGNMENT, "exchange", "peer buffer not 256-byte aligned");
  }
  if (a.lengths != nullptr &&
      (a.num_heads <= 0 || a.rows % a.num_heads != 0 || a.tokens_per_split <= 0))
    return fail(PDL_ERR_SHAPE, "exchange", "lengths need num_heads dividing rows and tokens_per_split > 0");
  if (!aligned(a.partial, 16) || !aligned(a.out, 16))
    return fail(PDL_ERR_ALIGNMENT, "exchange", "partial and out must be 16-byte aligned");
  if (a.timeout_us > 10u * 1000u * 1000u) return fail(PDL_ERR_SHAPE, "exchange", "timeout above 10 s");
  DeviceState *dev = nullptr;
  int st = current_device_state(&dev);
  if (st != PDL_OK) return st;
  PdlExchangePlan plan;
  st = pdl_exchange_plan(a.rows, a.head_dim, a.world, dev->sm_count, a.emulate_ranks, &plan);
  if (st != PDL_OK) return st;
  ExchangeParams p;
  std::memset(&p, 0, sizeof(p));
  p.partial = a.partial;
  p.lse = a.lse;
  p.lengths = a.lengths;
  p.num_heads = a.lengths != nullptr ? a.num_heads : 1;
  p.tokens_per_split = a.lengths != nullptr ? a.tokens_per_split : 1;
  p.rows = a.rows;
  p.splits = a.parts;
  p.rank = a.emulate_ranks ? 0 : a.rank;
  p.world = a.world;
  p.emulate = a.emulate_ranks ? 1 : 0;
  p.ctas = plan.ctas;
  p.block = plan.block_words;
  for (int q = 0; q < a.world; ++q) p.buffers[q] = static_cast<unsigned char *>(a.buffers[q]);
  p.out = static_cast<__nv_bfloat16 *>(a.out);
  p.timeout_ns = (uint64_t)(a.timeout_us ? a.timeout_us : 1000u * 1000u) * 1000ull;
  p.fault = dev->fault;
  return status_from_cuda(launch_exchange(p, a.head_dim, reinterpret_cast<cudaStream_t>(stream)),
                          "exchange merge");
}

extern "C" int pdl_paged_decode(const PdlDecodeArgs *args, pdl_stream_t stream) {
  int st = validate_common(args);
  if (st == PDL_OK) st = validate_partition_inputs(args);
  if (st == PDL_OK) st = validate_out(args);
  if (st != PDL_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((args->flags & PDL_FLAG_DYNAMIC) && !args->counters)
    return fail(PDL_ERR_WORKSPACE, "pdl_paged_decode", "dynamic scheduling needs counters");
  const bool direct = args->tokens_per_split == 0 ||
                      (args->splits == 1 && (args->flags & PDL_FLAG_DIRECT_SINGLE));
  if (direct) return run_partition(args, MODE_DIRECT, s);
  st = validate_workspace(args);
  if (st != PDL_OK) return st;
  const int mode = args->protocol == PDL_PROTOCOL_LSE ? MODE_LSE : MODE_MLA;
  st = run_partition(args, mode, s);
  if (st != PDL_OK) return st;
  return run_merge(args, s, true);
}

extern "C" int pdl_append_kv(const PdlAppendArgs *args, pdl_stream_t stream) {
  if (args == nullptr || !args->key || !args->value || !args->k_cache || !args->v_cache)
    return PDL_ERR_NULL;
  if (!valid_dim(args->head_dim) || args->num_kv_heads <= 0) return PDL_ERR_GEOMETRY;
  if (args->n_tokens < 0 || args->num_pages <= 0) return PDL_ERR_SHAPE;
  if (args->key_stride_head < args->head_dim || args->value_stride_head < args->head_dim)
    return PDL_ERR_SHAPE;
  if (!args->slot_mapping) {
    if (!args->block_table || !args->lengths) return PDL_ERR_NULL;
    if (args->table_width <= 0 || args->table_stride < args->table_width) return PDL_ERR_SHAPE;
  }
  if (!aligned(args->k_cache, 16) || !aligned(args->v_cache, 16)) return PDL_ERR_ALIGNMENT;
  if (!aligned(args->key, 2) || !aligned(args->value, 2)) return PDL_ERR_ALIGNMENT;
  AppendParams p;
  std::memset(&p, 0, sizeof(p));
  p.key = static_cast<const __nv_bfloat16 *>(args->key);
  p.value = static_cast<const __nv_bfloat16 *>(args->value);
  p.key_stride_token = args->key_stride_token;
  p.key_stride_head = args->key_stride_head;
  p.value_stride_token = args->value_stride_token;
  p.value_stride_head = args->value_stride_head;
  p.k_cache = static_cast<__nv_bfloat16 *>(args->k_cache);
  p.v_cache = static_cast<__nv_bfloat16 *>(args->v_cache);
  p.num_pages = args->num_pages;
  p.n_tokens = args->n_tokens;
  p.num_kv_heads = args->num_kv_heads;
  p.head_dim = args->head_dim;
  p.slot_mapping = args->slot_mapping;
  p.table = args->block_table;
  p.table_stride = args->table_stride;
  p.table_width = args->table_width;
  p.lengths = args->lengths;
  p.increment = args->increment_lengths ? 1 : 0;
  p.key_vec16 = aligned(args->key, 16) && args->key_stride_token % 8 == 0 &&
                args->key_stride_head % 8 == 0;
  p.value_vec16 = aligned(args->value, 16) && args->value_stride_token % 8 == 0 &&
                  args->value_stride_head % 8 == 0;
  return status_from_cuda(launch_append(p, reinterpret_cast<cudaStream_t>(stream)), "append");
}

extern "C" int pdl_read_fault(uint32_t *fault, int clear) {
  if (!fault) return PDL_ERR_NULL;
  DeviceState *dev = nullptr;
  int st = current_device_state(&dev);
  if (st != PDL_OK) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return PDL_ERR_CUDA;
  if (cudaMemcpy(fault, dev->fault, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
    return PDL_ERR_CUDA;
  if (clear && cudaMemset(dev->fault, 0, sizeof(uint32_t)) != cudaSuccess) return PDL_ERR_CUDA;
  return PDL_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free decode: pdl_paged_decode_static_scratch.
//
// Some callers cannot allocate device memory for the split workspace: an
// engine that reserved (nearly) all free HBM for its KV page pool at start-up
// and leaves no room for extra buffers, a host that reaches this library
// through an FFI and only holds device pointers handed to it by an engine
// that owns every allocation, or a code path that must not call cudaMalloc /
// cudaFree because those calls can synchronise the whole device.  For them
// the partial + LSE workspace lives in the file-scope device array below,
// which every GPU that loads this library keeps until the process exits.
//
// The caller still passes q, K/V, table, lengths and the output; the
// workspace pointers in PdlDecodeArgs are ignored.  The array is shared by
// all calls on a device and keeps the last call's contents; nothing in it
// has to start at zero, because the partition kernel stores every partition
// the merge reads.  Two calls whose work overlaps on the GPU (different
// streams, or graphs replayed concurrently) race on the array.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_pdl_static_scratch[PDL_STATIC_SCRATCH_BYTES / sizeof(float)];

namespace pdl {
namespace {

float *g_static_scratch[kMaxDevices];  // device address of the array, per device
std::mutex g_static_scratch_mutex;

// Set up once per device, with that device current: the host-side name of a
// __device__ array is only a stand-in, so its device address is fetched with
// cudaGetSymbolAddress and passed to the kernels.
int static_scratch_for_current_device(float **out) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return PDL_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch[dev] == nullptr) {
    void *addr = nullptr;
    const cudaError_t r = cudaGetSymbolAddress(&addr, g_pdl_static_scratch);
    if (r != cudaSuccess) return cuda_fail("cudaGetSymbolAddress(static scratch)", r);
    g_static_scratch[dev] = static_cast<float *>(addr);
  }
  *out = g_static_scratch[dev];
  return PDL_OK;
}

}  // namespace
}  // namespace pdl

extern "C" int pdl_paged_decode_static_scratch(const PdlDecodeArgs *args, pdl_stream_t stream) {
  int st = validate_common(args);
  if (st == PDL_OK) st = validate_partition_inputs(args);
  if (st == PDL_OK) st = validate_out(args);
  if (st != PDL_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((args->flags & PDL_FLAG_DYNAMIC) && !args->counters)
    return fail(PDL_ERR_WORKSPACE, "pdl_paged_decode_static_scratch",
                "dynamic scheduling needs counters");
  if (args->tokens_per_split == 0) return run_partition(args, MODE_DIRECT, s);  // no workspace
  const int64_t rows = (int64_t)args->batch * args->num_heads * args->splits;
  const int64_t bytes = rows * (args->head_dim + 1) * (int64_t)sizeof(float);
  if (bytes > (int64_t)PDL_STATIC_SCRATCH_BYTES) {
    char detail[160];
    snprintf(detail, sizeof(detail),
             "needs %lld bytes of scratch (batch*num_heads*splits*(head_dim+1)*4); "
             "the static scratch holds %lld",
             (long long)bytes, (long long)PDL_STATIC_SCRATCH_BYTES);
    return fail(PDL_ERR_WORKSPACE, "pdl_paged_decode_static_scratch", detail);
  }
  float *scratch = nullptr;
  st = static_scratch_for_current_device(&scratch);
  if (st != PDL_OK) return st;
  PdlDecodeArgs a = *args;
  a.protocol = PDL_PROTOCOL_LSE;
  a.partial = scratch;
  a.lse = scratch + rows * args->head_dim;  // 256-byte aligned: head_dim is a multiple of 64
  a.maxima = a.denoms = a.accums = nullptr;
  if (a.splits == 1 && (a.flags & PDL_FLAG_DIRECT_SINGLE)) return run_partition(&a, MODE_DIRECT, s);
  st = run_partition(&a, MODE_LSE, s);
  if (st != PDL_OK) return st;
  return run_merge(&a, s, true);
}
