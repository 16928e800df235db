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
enum : int { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ8_0 = 8 };

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
SS_DEVINL uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
SS_DEVINL uint16_t ldg_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

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
