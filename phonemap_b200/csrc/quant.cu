// quant.cu -- every GGUF block type of SlipStream's ss_dequantize
// (SlipStream/src/core/quantize.c:58-442) on the device, and the Q4_K matvec
// of its Metal backend (metal_backend.m:111-154, ss_metal_matvec_q4_K).
//
// Each value is computed the way the reference computes it: float16 fields
// converted exactly, then each product, sum and difference of the formula
// rounded on its own in the reference's order (explicit __fmul_rn / __fadd_rn /
// __fsub_rn, so nothing is contracted into an FMA) -- bit-identical to the
// reference's CPU build, which has no FMA.  The matvec dequantizes the same
// way and accumulates in fp32 in its own order (one warp per row).
#include "quant.h"

#include <cuda_fp16.h>

#include <algorithm>

namespace ss {
namespace {

__device__ __forceinline__ float qt_half(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}
__device__ __forceinline__ uint32_t qt_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Scale and min of sub-block j (0..7) of a Q4_K / Q5_K super-block: 6 bits
// each, sub-blocks 0-3 in the low bits of bytes j and j + 4, sub-blocks 4-7
// split between the nibbles of byte j + 4 and the top bits of bytes j - 4 and
// j (quantize.c:268-276).
__device__ __forceinline__ void qt_k4_scale(int j, const uint8_t* sc, float& s, float& m) {
  int a, b;
  if (j < 4) {
    a = sc[j] & 63;
    b = sc[j + 4] & 63;
  } else {
    a = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
    b = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
  s = (float)a;
  m = (float)b;
}

// Value e of the block at blk.
__device__ float qt_value(int type, const uint8_t* blk, int e) {
  switch (type) {
    case 2: {  // Q4_0 (quantize.c:60-72)
      const uint8_t q = blk[2 + (e & 15)];
      return __fmul_rn(qt_half(blk), (float)((e < 16 ? (q & 0xF) : (q >> 4)) - 8));
    }
    case 3: {  // Q4_1 (:76-89)
      const uint8_t q = blk[4 + (e & 15)];
      return __fadd_rn(__fmul_rn(qt_half(blk), (float)(e < 16 ? (q & 0xF) : (q >> 4))), qt_half(blk + 2));
    }
    case 6: {  // Q5_0 (:93-112)
      const uint8_t q = blk[6 + (e & 15)];
      const int v = (e < 16 ? (q & 0xF) : (q >> 4)) | (int)(((qt_u32(blk + 2) >> e) & 1u) << 4);
      return __fmul_rn((float)(v - 16), qt_half(blk));
    }
    case 7: {  // Q5_1 (:116-135)
      const uint8_t q = blk[8 + (e & 15)];
      const int v = (e < 16 ? (q & 0xF) : (q >> 4)) | (int)(((qt_u32(blk + 4) >> e) & 1u) << 4);
      return __fadd_rn(__fmul_rn((float)v, qt_half(blk)), qt_half(blk + 2));
    }
    case 8:  // Q8_0 (:139-149)
      return __fmul_rn(qt_half(blk), (float)(int8_t)blk[2 + e]);
    case 9:  // Q8_1 (:153-163): fp32 scale
      return __fmul_rn(__uint_as_float(qt_u32(blk)), (float)(int8_t)blk[8 + e]);
    case 10: {  // Q2_K (:180-215)
      const int h = e >> 7, r = e & 31, j = (e & 127) >> 5;
      const uint8_t s8 = blk[8 * h + 2 * j + (r >> 4)];
      const float dl = __fmul_rn(qt_half(blk + 80), (float)(s8 & 0xF));
      const float ml = __fmul_rn(qt_half(blk + 82), (float)(s8 >> 4));
      const int q = (blk[16 + 32 * h + r] >> (2 * j)) & 3;
      return __fsub_rn(__fmul_rn(dl, (float)q), ml);
    }
    case 11: {  // Q3_K (:219-263)
      const int h = e >> 7, r = e & 31, j = (e & 127) >> 5, i = 8 * h + 2 * j + (r >> 4);
      const int low = i < 8 ? (blk[96 + i] & 0xF) : (blk[96 + i - 8] >> 4);
      const int top = (blk[104 + (i & 3)] >> (2 * (i >> 2))) & 3;
      const float dl = __fmul_rn(qt_half(blk + 108), (float)((low | (top << 4)) - 32));
      const int q = ((blk[32 + 32 * h + r] >> (2 * j)) & 3) - ((blk[r] & (1 << (4 * h + j))) ? 0 : 4);
      return __fmul_rn(dl, (float)q);
    }
    case 12:    // Q4_K (:278-308)
    case 13: {  // Q5_K (:312-348)
      const int c = e >> 6, hi = (e >> 5) & 1, l = e & 31;
      float s, m;
      qt_k4_scale(2 * c + hi, blk + 4, s, m);
      const float d1 = __fmul_rn(qt_half(blk), s), m1 = __fmul_rn(qt_half(blk + 2), m);
      int q;
      if (type == 12) {
        const uint8_t b = blk[16 + 32 * c + l];
        q = hi ? (b >> 4) : (b & 0xF);
      } else {
        const uint8_t b = blk[48 + 32 * c + l];
        q = (hi ? (b >> 4) : (b & 0xF)) + (((blk[16 + l] >> (2 * c + hi)) & 1) ? 16 : 0);
      }
      return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case 14: {  // Q6_K (:352-383): (d * scale) * q
      const int h = e >> 7, g = (e & 127) >> 5, l = e & 31;
      const uint8_t lo = blk[64 * h + ((g & 1) ? l + 32 : l)];
      const int nib = (g & 2) ? (lo >> 4) : (lo & 0xF);
      const int q = (int)(int8_t)(nib | (((blk[128 + 32 * h + l] >> (2 * g)) & 3) << 4)) - 32;
      const int8_t sc = (int8_t)blk[192 + 8 * h + (l >> 4) + 2 * g];
      return __fmul_rn(__fmul_rn(qt_half(blk + 208), (float)sc), (float)q);
    }
    default:
      return 0.0f;
  }
}

__global__ void dequant_any_kernel(const uint8_t* __restrict__ src, long long n, int type, int bs, int ts,
                                   float* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    if (type == 0) {
      out[i] = __uint_as_float(qt_u32(src + 4 * i));
    } else if (type == 1) {
      out[i] = qt_half(src + 2 * i);
    } else {
      const long long b = i / bs;
      out[i] = qt_value(type, src + b * ts, (int)(i - b * bs));
    }
  }
}

// One warp per row; lane l takes values 8 l .. 8 l + 7 of every super-block
// (one sub-block's scale and min, 8 bytes of quants, 8 inputs).
constexpr int kQ4kWarps = 8;
__global__ void __launch_bounds__(32 * kQ4kWarps) matvec_q4k_kernel(const uint8_t* __restrict__ w,
                                                                    const float* __restrict__ x,
                                                                    float* __restrict__ out, int rows, int cols) {
  const int row = blockIdx.x * kQ4kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nb = cols >> 8;
  const int e0 = lane * 8, c = e0 >> 6, hi = (e0 >> 5) & 1, off = e0 & 31;
  const uint8_t* rp = w + (size_t)row * nb * 144;
  float acc = 0.0f;
  for (int b = 0; b < nb; b++) {
    const uint8_t* blk = rp + (size_t)b * 144;
    float s, m;
    qt_k4_scale(2 * c + hi, blk + 4, s, m);
    const float d1 = __fmul_rn(qt_half(blk), s), m1 = __fmul_rn(qt_half(blk + 2), m);
    const uint2 qv = *reinterpret_cast<const uint2*>(blk + 16 + 32 * c + off);
    const float4 x0 = __ldg(reinterpret_cast<const float4*>(x + 256 * b + e0));
    const float4 x1 = __ldg(reinterpret_cast<const float4*>(x + 256 * b + e0 + 4));
    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const uint32_t word = k < 4 ? qv.x : qv.y;
      const int byte = (word >> (8 * (k & 3))) & 0xFF;
      const int q = hi ? (byte >> 4) : (byte & 0xF);
      acc = fmaf(__fsub_rn(__fmul_rn(d1, (float)q), m1), xv[k], acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[row] = acc;
}

}  // namespace

size_t quant_type_size(int type) {
  switch (type) {
    case 0: return 4;
    case 1: return 2;
    case 2: return 18;
    case 3: return 20;
    case 6: return 22;
    case 7: return 24;
    case 8: return 34;
    case 9: return 40;
    case 10: return 84;
    case 11: return 110;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    default: return 0;
  }
}

int quant_block_size(int type) {
  if (type == 0 || type == 1) return 1;
  return type >= 10 && type <= 14 ? 256 : 32;
}

cudaError_t dequant_launch(const uint8_t* src, long long n, int type, float* out, cudaStream_t s) {
  const size_t ts = quant_type_size(type);
  const int bs = quant_block_size(type);
  if (!ts || n <= 0 || n % bs) return cudaErrorInvalidValue;
  const long long grid = std::min<long long>((n + 255) / 256, 4096);
  dequant_any_kernel<<<(unsigned)grid, 256, 0, s>>>(src, n, type, bs, (int)ts, out);
  return cudaGetLastError();
}

cudaError_t matvec_q4k_launch(const uint8_t* w, const float* x, float* out, int rows, int cols, cudaStream_t s) {
  if (rows <= 0 || cols <= 0 || cols % 256 || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(x) & 15))
    return cudaErrorInvalidValue;
  matvec_q4k_kernel<<<(rows + kQ4kWarps - 1) / kQ4kWarps, 32 * kQ4kWarps, 0, s>>>(w, x, out, rows, cols);
  return cudaGetLastError();
}

}  // namespace ss
