// common.cuh -- device helpers shared by the SlipStream CUDA kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SS_DEVINL __device__ __forceinline__

namespace ss {

constexpr int kWarp = 32;
constexpr int kMaxGroupRows = 8;

// GGML tensor type ids (SlipStream/src/core/gguf_loader.h:41-55).
enum : int { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12 };

// ---- programmatic dependent launch (PTX griddepcontrol, sm_90+) ----------
// wait: block until the preceding kernel in the stream has completed and its
// writes are visible.  launch_dependents: let the next kernel start launching.
SS_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SS_DEVINL void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Bulk prefetch of [ptr, ptr+bytes) into L2 (no shared memory, no completion
// tracking).  ptr must be 16-byte aligned and bytes a multiple of 16.
SS_DEVINL void prefetch_l2_bulk(const void* ptr, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

// Streaming 128-bit load that bypasses L1 allocation (weights are read once).
// Not volatile: these read immutable weights, so the compiler may hoist and
// batch them (that is what keeps many rows in flight per warp).
SS_DEVINL uint4 ldg_stream(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
SS_DEVINL uint16_t ldg_u16(const void* p) {
  uint16_t v;
  asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// ---- mbarrier + bulk async copy (TMA engine, non-tensor form) -------------
SS_DEVINL uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
SS_DEVINL void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
SS_DEVINL void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
SS_DEVINL void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
SS_DEVINL bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `budget` SM clock cycles (then the caller
// reports an error instead of hanging the GPU).
SS_DEVINL bool mbar_wait_bounded(uint32_t bar, uint32_t parity, long long budget) {
  if (mbar_try_wait(bar, parity)) return true;  // common case: no clock read
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > budget) return false;
  }
  return true;
}
// Global -> shared bulk copy completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16).
SS_DEVINL void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
SS_DEVINL uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
SS_DEVINL uint16_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

constexpr long long kWaitBudget = 1LL << 31;  // ~1 s of SM clocks
// the budget of one failure-path test step (ss_cuda_test_fail_next_step)
constexpr long long kTestWaitBudget = 1LL << 22;  // ~2 ms

SS_DEVINL float half_bits_to_float(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

SS_DEVINL float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
SS_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Order-preserving encoding of a non-negative float for atomicMax.
SS_DEVINL unsigned int float_as_ordered(float f) { return __float_as_uint(f); }

// Block-wide sum for blockDim.x <= 1024; `scratch` needs 32 floats.  All
// threads receive the result.
SS_DEVINL float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.0f;
  if (warp == 0) {
    t = lane < nw ? scratch[lane] : 0.0f;
    t = warp_sum(t);
    if (lane == 0) scratch[0] = t;
  }
  __syncthreads();
  return scratch[0];
}

}  // namespace ss
