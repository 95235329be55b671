// pdl_append.cu -- write new K/V rows into the paged cache (the step before decode).
//
// One CTA per new token; its threads copy the token's num_kv_heads * head_dim
// BF16 values of K and of V in 16-byte chunks (2-byte chunks when a source
// is not 16-byte aligned).  The destination slot comes from either
//   * a slot mapping (nano-vLLM store_kvcache, reference overlay
//     nanovllm/layers/attention.py:10-40): slot = page * 256 + offset,
//     -1 = skip the token; or
//   * the block table at each row's current length (the Qwen3.5 runner's
//     paged update, reference src/paged_decode/hybrid.py:63-72, for one
//     decode position): row b writes position lengths[b], i.e. page
//     table[b][len / 256], slot len % 256; with `increment` the row's length
//     becomes len + 1 (read and written by the one thread that resolves the
//     slot).
// Slots outside the pool and rows whose table is full are skipped, so a bad
// mapping can never write outside the cache.
#include "pdl_device.cuh"

namespace pdl {
namespace {

constexpr int APPEND_THREADS = 128;

__device__ __forceinline__ void copy_row(const __nv_bfloat16 *src, int64_t head_stride,
                                         __nv_bfloat16 *dst, int hkv, int dim, bool vec) {
  const int chunks = hkv * dim / 8;
  if (vec) {
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      const int h = c / (dim / 8), o = (c % (dim / 8)) * 8;
      const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src + h * head_stride + o));
      *reinterpret_cast<uint4 *>(dst + h * dim + o) = v;
    }
  } else {
    for (int e = threadIdx.x; e < hkv * dim; e += blockDim.x) {
      const int h = e / dim, o = e % dim;
      dst[h * dim + o] = src[h * head_stride + o];
    }
  }
}

__global__ void __launch_bounds__(APPEND_THREADS) append_kernel(const AppendParams p) {
  const int t = blockIdx.x;
  __shared__ long long s_slot;
  if (threadIdx.x == 0) {
    int64_t slot = -1;
    if (p.slot_mapping != nullptr) {
      slot = __ldg(p.slot_mapping + t);
    } else {
      const int len = p.lengths[t];
      if (len >= 0 && len < p.table_width * 256) {
        const int page = __ldg(p.table + (int64_t)t * p.table_stride + len / 256);
        if (page >= 0 && page < p.num_pages) slot = (int64_t)page * 256 + len % 256;
      }
      // Only this thread reads the row's length, so the increment cannot race.
      if (slot >= 0 && p.increment) p.lengths[t] = len + 1;
    }
    s_slot = slot < 0 || slot >= p.num_pages * 256 ? -1 : slot;
  }
  __syncthreads();
  const int64_t slot = s_slot;
  if (slot < 0) return;
  const int64_t row_elems = (int64_t)p.num_kv_heads * p.head_dim;
  copy_row(p.key + t * p.key_stride_token, p.key_stride_head, p.k_cache + slot * row_elems,
           p.num_kv_heads, p.head_dim, p.key_vec16);
  copy_row(p.value + t * p.value_stride_token, p.value_stride_head, p.v_cache + slot * row_elems,
           p.num_kv_heads, p.head_dim, p.value_vec16);
}

}  // namespace

cudaError_t launch_append(const AppendParams &params, cudaStream_t stream) {
  if (params.n_tokens <= 0) return cudaSuccess;
  append_kernel<<<params.n_tokens, APPEND_THREADS, 0, stream>>>(params);
  return cudaGetLastError();
}

}  // namespace pdl
