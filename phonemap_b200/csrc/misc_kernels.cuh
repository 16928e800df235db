// misc_kernels.cuh -- embedding gather, weight repack, dequantisation, fp32 GEMV.
#pragma once
#include "common.cuh"

namespace ss {

// Step entry: h = token_embd[token at pos] (SlipStream/src/core/layer_scheduler.c:
// 584-587, F32 embeddings) and clear the |k| / |v| maxima slots of every layer
// before the QKV GEMVs accumulate into them.
struct EmbedParams {
  const float* embd;    // [vocab][d] fp32
  int d, vocab, n_layers, ctx;
  const int* seq_tokens;
  const int* d_pos;
  float* h;
  unsigned int* amax;    // [L][2]: |k|, |v| maxima of the current position
  int* err;
};

__global__ void embed_kernel(const EmbedParams p) {
  pdl_wait();
  const int pos = *p.d_pos;
  if (pos < 0 || pos >= p.ctx) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, 1);
    return;
  }
  int tok = p.seq_tokens[pos];
  if (tok < 0 || tok >= p.vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, 2);
    tok = 0;
  }
  const float* row = p.embd + (size_t)tok * p.d;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.d; i += gridDim.x * blockDim.x)
    p.h[i] = row[i];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < 2 * p.n_layers; i += blockDim.x) p.amax[i] = 0u;
  pdl_trigger();
}

// Tensor parallelism: the argmax all-reduce left the global best (value, index)
// in *best; write the token of pos + 1 and advance the position, as the
// argmax epilogue does without tensor parallelism.
__global__ void tp_finish_kernel(const unsigned long long* best, int* d_pos, const int* fixed_until,
                                 int* seq_tokens, int ctx) {
  const int tok = 0x7fffffff - (int)(unsigned)(*best & 0xffffffffu);
  const int pos = *d_pos;
  if (pos + 1 < ctx && pos + 1 >= *fixed_until) seq_tokens[pos + 1] = tok;
  seq_tokens[ctx] = tok;
  *d_pos = pos + 1;
}

// GGUF blocks (AoS, 18 B Q4_0 / 34 B Q8_0 per 32 weights) -> row-interleaved
// layout (see gemv.cuh).  Source row r goes to destination row
// r * dst_row_mul + dst_row_add, so gate/up rows can be interleaved and
// Q/K/V stacked; of each source row (src_nb blocks) blocks src_b0 .. src_b0 +
// cols/32 are taken (a column slice, for tensor parallelism).  One thread per
// block.
__global__ void repack_kernel(const uint8_t* __restrict__ src, int rows, int cols, int type,
                              uint8_t* __restrict__ dst, int row_stride, int scale_off,
                              int dst_row_mul, int dst_row_add, int src_nb, int src_b0) {
  const int nb = cols / 32;
  const int bsz = type == kQ4_0 ? 18 : 34;
  const int qsz = bsz - 2;
  const long long total = (long long)rows * nb;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
    const uint8_t* s = src + ((long long)r * src_nb + src_b0 + b) * bsz;
    uint8_t* drow = dst + (size_t)(r * dst_row_mul + dst_row_add) * row_stride;
    drow[scale_off + 2 * b] = s[0];
    drow[scale_off + 2 * b + 1] = s[1];
    for (int j = 0; j < qsz; j++) drow[b * qsz + j] = s[2 + j];
  }
}

// GGUF blocks -> tiled layout (step_kernel.cuh): tiles of 4 rows, the rows'
// quant bytes row-major, then the nb x 4 fp16 scales block-major.  Source row r
// goes to destination row r * dst_row_mul + dst_row_add.
__global__ void repack_tiled_kernel(const uint8_t* __restrict__ src, int rows, int cols, int type,
                                    uint8_t* __restrict__ dst, int tile_bytes, int dst_row_mul,
                                    int dst_row_add, int src_nb, int src_b0) {
  const int nb = cols / 32;
  const int bsz = type == kQ4_0 ? 18 : 34;
  const int qsz = bsz - 2;
  const long long total = (long long)rows * nb;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
    const uint8_t* s = src + ((long long)r * src_nb + src_b0 + b) * bsz;
    const int R = r * dst_row_mul + dst_row_add;
    uint8_t* tile = dst + (size_t)(R >> 2) * tile_bytes;
    const int ri = R & 3;
    tile[4 * nb * qsz + b * 8 + ri * 2] = s[0];
    tile[4 * nb * qsz + b * 8 + ri * 2 + 1] = s[1];
    uint8_t* q = tile + (size_t)ri * nb * qsz + b * qsz;
    for (int j = 0; j < qsz; j++) q[j] = s[2 + j];
  }
}

// Dequantise rows of a tiled matrix (rows src_row_mul * r + src_row_add).
__global__ void dequant_tiled_kernel(const uint8_t* __restrict__ w, int rows, int cols, int type,
                                     int tile_bytes, int src_row_mul, int src_row_add,
                                     float* __restrict__ out) {
  const int nb = cols / 32;
  const int qsz = type == kQ4_0 ? 16 : 32;
  const long long total = (long long)rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i - (long long)r * cols);
    const int b = c >> 5, j = c & 31;
    const int R = r * src_row_mul + src_row_add;
    const uint8_t* tile = w + (size_t)(R >> 2) * tile_bytes;
    const int ri = R & 3;
    const uint8_t* sp = tile + 4 * nb * qsz + b * 8 + ri * 2;
    const float d = half_bits_to_float((uint16_t)sp[0] | ((uint16_t)sp[1] << 8));
    const uint8_t* q = tile + (size_t)ri * nb * qsz + b * qsz;
    float v;
    if (type == kQ4_0) {
      const uint8_t byte = q[j & 15];
      const int qq = j < 16 ? (byte & 0xF) : (byte >> 4);
      v = __fmul_rn(d, (float)(qq - 8));
    } else {
      v = __fmul_rn(d, (float)(int8_t)q[j]);
    }
    out[i] = v;
  }
}

// Dequantise a row-interleaved matrix back to fp32 rows (for bit-exactness
// checks against the reference dequantiser, quantize.c:60-72 / :139-149):
// value = fp32(d) * (q - 8) (Q4_0) or fp32(d) * q (Q8_0), one rounding.
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ w, int rows, int cols, int type,
                                    int row_stride, int scale_off, int src_row_mul,
                                    int src_row_add, float* __restrict__ out) {
  const long long total = (long long)rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i - (long long)r * cols);
    const int b = c >> 5, j = c & 31;
    const uint8_t* row = w + (size_t)(r * src_row_mul + src_row_add) * row_stride;
    const uint16_t dh = (uint16_t)row[scale_off + 2 * b] | ((uint16_t)row[scale_off + 2 * b + 1] << 8);
    const float d = half_bits_to_float(dh);
    float v;
    if (type == kQ4_0) {
      const uint8_t byte = row[b * 16 + (j & 15)];
      const int q = j < 16 ? (byte & 0xF) : (byte >> 4);
      v = __fmul_rn(d, (float)(q - 8));
    } else {
      v = __fmul_rn(d, (float)(int8_t)row[b * 32 + j]);
    }
    out[i] = v;
  }
}

// fp32 GEMV (twin of the Metal `matvec` kernel, metal_backend.m:23-46): warp per
// row, float4 loads.
__global__ void matvec_f32_kernel(const float* __restrict__ w, const float* __restrict__ x,
                                  float* __restrict__ out, int rows, int cols) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* row = w + (size_t)warp * cols;
  float s = 0.0f;
  if ((cols & 3) == 0) {
    for (int i = lane * 4; i < cols; i += 128) {
      const float4 a = *reinterpret_cast<const float4*>(row + i);
      const float4 b = *reinterpret_cast<const float4*>(x + i);
      s = fmaf(a.x, b.x, s); s = fmaf(a.y, b.y, s); s = fmaf(a.z, b.z, s); s = fmaf(a.w, b.w, s);
    }
  } else {
    for (int i = lane; i < cols; i += 32) s = fmaf(row[i], x[i], s);
  }
  s = warp_sum(s);
  if (lane == 0) out[warp] = s;
}

}  // namespace ss
