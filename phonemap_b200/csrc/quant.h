// quant.h -- the GGUF block types SlipStream dequantizes, on the device
// (quant.cu): dequantization of every type of SlipStream/src/core/quantize.c:
// 389-442 and the Q4_K matvec twin of ss_metal_matvec_q4_K.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace ss {

// Bytes per block of a ggml type (0: not a type the reference dequantizes)
// and values per block (SlipStream/src/core/gguf_loader.c:22-60).
size_t quant_type_size(int type);
int quant_block_size(int type);
// out[0, n) = the values of the blocks at src (n a multiple of the block size).
cudaError_t dequant_launch(const uint8_t* src, long long n, int type, float* out, cudaStream_t s);
// out[r] = sum_c W[r][c] x[c] for a Q4_K matrix in GGUF row order (cols a
// multiple of 256; w 16-byte aligned).
cudaError_t matvec_q4k_launch(const uint8_t* w, const float* x, float* out, int rows, int cols, cudaStream_t s);

}  // namespace ss
