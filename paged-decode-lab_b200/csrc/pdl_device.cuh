// pdl_device.cuh -- device helpers shared by the sm_100a decode kernels:
// mbarrier pipeline primitives with bounded waits, 5-D TMA tile loads,
// BF16 unpacking and the fault word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "pdl_internal.h"

namespace pdl {

constexpr unsigned FULL_MASK = 0xffffffffu;

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t WAIT_LIMIT_NS = 1000ull * 1000ull * 1000ull;  // 1 s

// Fault codes recorded (OR-ed) into the per-device fault word.
enum FaultBits : uint32_t {
  FAULT_PRODUCER_EMPTY_WAIT = 1u << 0,  // producer gave up waiting for a free stage
  FAULT_CONSUMER_FULL_WAIT = 1u << 1,   // consumer gave up waiting for a TMA tile
  FAULT_DRAIN_WAIT = 1u << 2,           // in-flight copies did not land at exit
  FAULT_SMEM_ALIGN = 1u << 3,           // dynamic shared memory not 1024-byte aligned
  FAULT_EXCHANGE_WAIT = 1u << 4,        // a peer's exchange flag did not arrive in time
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking check whether the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bring the 128-byte line holding `addr` into L1 ahead of its load.
__device__ __forceinline__ void prefetch_l1(const void *addr) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(addr));
}

// Wait for the phase with the given parity.  Gives up after WAIT_LIMIT_NS,
// records `code` in the fault word and returns false; the caller then stops
// issuing work and exits.  A healthy pipeline never reaches the slow path.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint32_t *fault, uint32_t code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > WAIT_LIMIT_NS) {
      if (fault) atomicOr(fault, code);
      return false;
    }
  }
}

// Pipeline wait shared by producer and consumers.  Once any warp of the CTA
// has given up (abort flag set), later waits return false at once so every
// warp still walks the same control flow (and reaches the same named
// barriers) without blocking again.
__device__ __forceinline__ bool pipeline_wait(uint64_t *bar, uint32_t parity, uint32_t *fault,
                                              uint32_t code, volatile int *abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait_bounded(bar, parity, fault, code)) return true;
  *abort_flag = 1;
  return false;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// KV pages are streamed once per launch: mark them evict-first in L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Tokens per partition of a row of (clamped) length len split into `splits`
// balanced partitions of whole granules: granule * ceil(ceil(len / splits) /
// granule); 0 for an empty row.  Partition p covers [p * span, (p + 1) *
// span) of the row; the partition and merge kernels both use this.
__host__ __device__ __forceinline__ int64_t balanced_span(int len, int splits, int granule) {
  const int64_t per = ((int64_t)len + splits - 1) / splits;
  return (per + granule - 1) / granule * granule;
}

// 5-D tiled TMA load (no multicast) into CTA shared memory; completion is
// signalled on `bar` as transaction bytes.  Coordinates are innermost first.
__device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, int c4, uint64_t *bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a sub-tile
// written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (rows of 128 bytes, chunk
// index XOR-ed with row % 8; the sub-tile base is 1024-byte aligned).
__device__ __forceinline__ uint32_t swizzle128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ---------------------------------------------------------------- numerics
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t x) {
  // BF16 is the upper half of an FP32 bit pattern.
  return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
}

// Hardware base-2 exponential (PTX ex2.approx); exp2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Named barrier over `count` threads (consumer warps only).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Programmatic dependent launch: a kernel launched after this one with
// programmatic stream serialization may start once every CTA here has
// executed launch_dependents (or exited); it must call grid_dependency_wait
// before touching this kernel's outputs, which returns once this kernel has
// completed and its memory operations are visible.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Host: launch `kernel` with programmatic stream serialization, so it may be
// scheduled while the previous kernel in the stream still runs (once that
// kernel has executed allow_dependent_launch in every CTA); the kernel must
// call grid_dependency_wait before touching anything the previous kernels
// write or read.  Without such a trigger it behaves like a plain launch.
template <typename... KArgs, typename... Args>
cudaError_t launch_programmatic(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

constexpr float LN2 = 0.6931471805599453f;

}  // namespace pdl
