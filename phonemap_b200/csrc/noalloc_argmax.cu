// noalloc_argmax.cu -- greedy argmax over device logits without allocating.
//
// Some callers cannot allocate device memory at the point where they need a
// greedy token: code running while a stream is being captured into a CUDA
// graph (cudaMalloc is not capturable), or hosts that hand this library only
// pre-sized buffers from their own memory pool.  ss_cuda_argmax_noalloc serves
// them: it is the same two-level reduction as the lm_head epilogue
// (gemv.cuh -- per-CTA maxima to scratch, the last CTA to finish reduces them),
// but its scratch lives in the file-scope array below instead of memory
// allocated by a context.
//
// The array is part of this library's device image: every GPU that loads the
// library holds it (about 8 KiB) until the process exits.  All calls share it,
// so calls whose kernels overlap on the GPU (different streams, or different
// host threads, without ordering between them) race on it and must not be
// issued; calls on one stream are ordered and safe.
#include <cuda_runtime.h>

#include <mutex>

#include "gemv.cuh"
#include "slipstream_cuda.h"

#define SS_API extern "C" __attribute__((visibility("default")))

namespace ss {
namespace {

constexpr int kNoAllocThreads = 256;
constexpr int kNoAllocItems = 16;                   // values per thread
constexpr int kNoAllocMaxBlocks = 1024;
constexpr long long kNoAllocMaxN =
    (long long)kNoAllocMaxBlocks * kNoAllocThreads * kNoAllocItems;  // 4,194,304

struct NoAllocScratch {
  unsigned long long partial[kNoAllocMaxBlocks];  // packed (value, index) per CTA
  unsigned int count;                              // CTAs finished; reset to 0 by the last one
};

static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

__global__ void __launch_bounds__(kNoAllocThreads)
argmax_noalloc_kernel(const float* __restrict__ v, int n, int* __restrict__ out,
                      NoAllocScratch* scratch) {
  __shared__ unsigned long long wbest[kNoAllocThreads / 32];
  __shared__ bool is_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned long long best = 0;
  for (int i = blockIdx.x * kNoAllocThreads + tid; i < n; i += gridDim.x * kNoAllocThreads) {
    const unsigned long long pk = pack_argmax(v[i], i);
    best = pk > best ? pk : best;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (lane == 0) wbest[warp] = best;
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kNoAllocThreads / 32; w++) b = wbest[w] > b ? wbest[w] : b;
    scratch->partial[blockIdx.x] = b;
    __threadfence();
    is_last = atomicAdd(&scratch->count, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  unsigned long long b = 0;
  for (int i = tid; i < (int)gridDim.x; i += kNoAllocThreads) {
    const unsigned long long p = *((volatile unsigned long long*)scratch->partial + i);
    b = p > b ? p : b;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
    b = other > b ? other : b;
  }
  if (lane == 0) wbest[warp] = b;
  __syncthreads();
  if (tid == 0) {
    unsigned long long bb = 0;
    for (int w = 0; w < kNoAllocThreads / 32; w++) bb = wbest[w] > bb ? wbest[w] : bb;
    // every element packs above 0 (index 0 always exists), so bb == 0 cannot
    // happen for n >= 1; index 0 is the answer of an empty scan all the same
    *out = bb == 0 ? 0 : unpack_argmax_index(bb);
    scratch->count = 0;
  }
}

// Device address of g_noalloc_scratch, looked up once per device.  In host
// code the symbol's name is only a host-side stand-in, never a device address.
std::mutex g_noalloc_mu;
NoAllocScratch* g_noalloc_ptr[64] = {};

}  // namespace
}  // namespace ss

using namespace ss;

SS_API int ss_cuda_argmax_noalloc(const float* d_values, int32_t n, int32_t* d_index, void* stream) {
  if (!d_values || !d_index || n <= 0) return SS_CUDA_ERROR_INVALID_PARAMS;
  if ((long long)n > kNoAllocMaxN) return SS_CUDA_ERROR_INVALID_PARAMS;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SS_CUDA_ERROR_BACKEND;
  NoAllocScratch* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return SS_CUDA_ERROR_BACKEND;
      }
      g_noalloc_ptr[dev] = static_cast<NoAllocScratch*>(p);
    }
    scratch = g_noalloc_ptr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the completion counter must start at zero (the last CTA also resets it)
  if (cudaMemsetAsync(&scratch->count, 0, sizeof(unsigned int), s) != cudaSuccess)
    return SS_CUDA_ERROR_BACKEND;
  const long long per_block = (long long)kNoAllocThreads * kNoAllocItems;
  const int blocks = (int)((n + per_block - 1) / per_block);
  argmax_noalloc_kernel<<<blocks, kNoAllocThreads, 0, s>>>(d_values, n, d_index, scratch);
  return cudaGetLastError() == cudaSuccess ? SS_CUDA_OK : SS_CUDA_ERROR_BACKEND;
}
