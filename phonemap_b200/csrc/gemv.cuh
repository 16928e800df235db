// gemv.cuh -- batch-1 dequantize-and-matvec for Q4_0 / Q8_0 weights on sm_100a.
//
// Replaces SlipStream's per-row "dequantize into a temp, then dot" CPU loop
// (SlipStream/src/core/quantize.c:446-494) and the one-thread-per-row Metal
// kernel (SlipStream/src/backends/metal_backend.m:55-91).  Same math -- every
// weight is d * (q - 8) (Q4_0) or d * q (Q8_0) with d the block's fp16 scale
// widened exactly to fp32, products and sums in fp32 -- in a different
// summation order.
//
// Layout ("row-interleaved"): the uploader repacks each GGUF matrix so that row
// r occupies `row_stride` bytes at `data + r * row_stride`:
//     [nb blocks of quants, 16 B (Q4_0) or 32 B (Q8_0) each]
//     [nb fp16 scales][zero pad to 16 B]
// The quant bytes of a block are the GGUF block's bytes unchanged (Q4_0 byte j
// holds q[j] in its low nibble and q[j+16] in its high nibble), so every weight
// decodes to the same value as the reference's dequantizer.  Bytes per weight
// are the GGUF ones (18/32, 34/32) plus < 16 B of padding per row.
//
// Work split ("x-stationary"): a CTA has one thread per 32-column block
// (blockDim = nb rounded up to a warp).  Each thread keeps its block's 32
// activations in registers for every row the CTA owns, streams that block of
// each row with one 128-bit load (two for Q8_0), and the CTA reduces each row
// once at the end.  A CTA owns a contiguous range of rows, so one bulk L2
// prefetch covers its whole share of the matrix; it is issued before the
// programmatic-dependent-launch wait so the weight stream overlaps the tail of
// the previous kernel.
//
// Inner product in exact integer arithmetic: each thread converts its 32
// activations once per CTA to block fixed point -- m_j = round(x_j * 2^(22-e))
// with 2^e > max |x_j| of the block, so x_j = m_j * 2^(e-22) to 23 bits -- and
// splits m_j into three signed base-256 digits (byte planes).  A row's block
// then costs dp4a instructions only: sum_j (q_j - zp) * m_j =
// sum_p 256^p * sum_j q_j * s_pj  -  zp * sum_j m_j, exact in int32, with the
// zero-point term folded into the accumulators' initial values.  Three int->float
// conversions and two fused multiply-adds combine the planes; the fp16 scale d
// and 2^(e-22) scale the result.  Q4_0: 8 weights per SHF + 2 LOP3 + 6 dp4a;
// Q8_0: 4 weights per 3 dp4a.
#pragma once
#include "common.cuh"

namespace ss {

struct QMatrix {
  const uint8_t* data;
  int rows, cols;
  int row_stride;  // bytes per row
  int scale_off;   // byte offset of the fp16 scales within a row
  int type;        // kQ4_0 or kQ8_0
};

enum class XSrc : int { Plain = 0, RmsNorm = 1 };
enum class Epi : int { Store = 0, Residual = 1, QKV = 2, SwiGLU = 3, Argmax = 4 };

struct GemvParams {
  QMatrix w;
  const float* x;        // Plain: the input vector; RmsNorm: the residual stream h
  const float* norm_w;   // RmsNorm weight (fp32, cols)
  float eps;
  float* out;            // Store/Residual/QKV: [rows]; SwiGLU: [rows/2]; Argmax: logits (nullable)
  const float* residual; // Residual: out[r] = acc + residual[r]
  // QKV epilogue: RoPE on the q and k rows, |k| and |v| maxima for the int8 cache
  int q_rows, kv_rows, head_dim, rope_dim;
  const float2* rope_tab;    // [ctx][rope_dim/2] (cos, sin)
  const int* d_pos;
  unsigned int* amax_k;      // slot for (layer, pos) = amax_k[pos] (already offset by layer)
  unsigned int* amax_v;
  // Argmax epilogue
  unsigned long long* am_part;  // one packed (value, index) per CTA
  unsigned int* am_count;
  int* seq_tokens;              // token of every position
  const int* fixed_until;       // positions below this hold prompt tokens
  int* d_pos_rw;                // advanced by one after the step
  int ctx;
  int* err;
  int rows_per_cta;
  int prefetch;
  // bulk-copy pipeline: `nstage` shared-memory slots of `stage_rows` rows
  int nstage, stage_rows;
};

// ---- per-block dot products --------------------------------------------
// One thread's 32 activations as block fixed point in three signed byte planes
// (natural order: word w of plane p holds digits p of weights 4w .. 4w+3).
struct XPlanes {
  int pl[3][8];
  int init[3];  // accumulator start: -zero_point * sum_j s_pj
  float fb;     // 2^(e-22), the value of one unit of m
};

SS_DEVINL float pow2i(int k) { return __int_as_float((k + 127) << 23); }  // 2^k, -126 <= k <= 127

template <int ZP>
SS_DEVINL XPlanes make_planes(const float (&xv)[32]) {
  XPlanes xp;
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(xv[j]));
  int e = 0;
  if (amax >= 1e-30f) frexpf(amax, &e);  // amax < 2^e
  const bool live = amax >= 1e-30f;      // smaller blocks contribute nothing measurable
  const float sc = live ? pow2i(22 - e) : 0.0f;
  xp.fb = live ? pow2i(e - 22) : 0.0f;
  int sum[3] = {0, 0, 0};
#pragma unroll
  for (int w = 0; w < 8; w++) {
    unsigned b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int m = __float2int_rn(xv[4 * w + i] * sc);  // |m| <= 2^22
      const int s0 = ((m + 128) & 255) - 128;
      const int m1 = (m - s0) >> 8;
      const int s1 = ((m1 + 128) & 255) - 128;
      const int s2 = (m1 - s1) >> 8;                   // |s2| <= 64
      b0 |= (unsigned)(s0 & 255) << (8 * i);
      b1 |= (unsigned)(s1 & 255) << (8 * i);
      b2 |= (unsigned)(s2 & 255) << (8 * i);
      sum[0] += s0; sum[1] += s1; sum[2] += s2;
    }
    xp.pl[0][w] = (int)b0;
    xp.pl[1][w] = (int)b1;
    xp.pl[2][w] = (int)b2;
  }
#pragma unroll
  for (int p = 0; p < 3; p++) xp.init[p] = -ZP * sum[p];
  return xp;
}

SS_DEVINL int dp4a_us(unsigned a, int b, int c) {  // unsigned bytes . signed bytes
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
SS_DEVINL int dp4a_ss(int a, int b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
SS_DEVINL float combine_planes(int a0, int a1, int a2) {  // |a_p| < 2^24: exact conversions
  return fmaf((float)a2, 65536.0f, fmaf((float)a1, 256.0f, (float)a0));
}

// Q4_0 block: sum_j (q_j - 8) * m_j, in units of 2^(e-22).
SS_DEVINL float dot_q4_block(const uint4 q, const XPlanes& xp) {
  int a0 = xp.init[0], a1 = xp.init[1], a2 = xp.init[2];
  const unsigned wq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const unsigned lo = wq[t] & 0x0F0F0F0Fu;          // q[4t .. 4t+3]
    const unsigned hi = (wq[t] >> 4) & 0x0F0F0F0Fu;   // q[16+4t .. 16+4t+3]
    a0 = dp4a_us(lo, xp.pl[0][t], a0);
    a1 = dp4a_us(lo, xp.pl[1][t], a1);
    a2 = dp4a_us(lo, xp.pl[2][t], a2);
    a0 = dp4a_us(hi, xp.pl[0][4 + t], a0);
    a1 = dp4a_us(hi, xp.pl[1][4 + t], a1);
    a2 = dp4a_us(hi, xp.pl[2][4 + t], a2);
  }
  return combine_planes(a0, a1, a2);
}

// Q8_0 block: sum_j q_j * m_j, in units of 2^(e-22).
SS_DEVINL float dot_q8_block(const uint4 qa, const uint4 qb, const XPlanes& xp) {
  int a0 = 0, a1 = 0, a2 = 0;
  const unsigned wq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int t = 0; t < 8; t++) {
    a0 = dp4a_ss((int)wq[t], xp.pl[0][t], a0);
    a1 = dp4a_ss((int)wq[t], xp.pl[1][t], a1);
    a2 = dp4a_ss((int)wq[t], xp.pl[2][t], a2);
  }
  return combine_planes(a0, a1, a2);
}

// ---- warp "transpose" reductions -----------------------------------------
// Reduce G per-lane values over the 32 lanes in G + 5 - log2(G)... shuffles:
// after the call, lanes with (lane & (32/G - 1)) == 0 hold the sum of value
// index row_of_lane(lane).
template <int G>
SS_DEVINL float warp_reduce_rows(float (&a)[G], int lane);

template <>
SS_DEVINL float warp_reduce_rows<1>(float (&a)[1], int lane) {
  return warp_sum(a[0]);
}
template <>
SS_DEVINL float warp_reduce_rows<2>(float (&a)[2], int lane) {
  const bool hi = lane & 16;
  float v = (hi ? a[1] : a[0]) + __shfl_xor_sync(0xffffffffu, hi ? a[0] : a[1], 16);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <>
SS_DEVINL float warp_reduce_rows<4>(float (&a)[4], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8;
  float b0 = (b4 ? a[2] : a[0]) + __shfl_xor_sync(0xffffffffu, b4 ? a[0] : a[2], 16);
  float b1 = (b4 ? a[3] : a[1]) + __shfl_xor_sync(0xffffffffu, b4 ? a[1] : a[3], 16);
  float v = (b3 ? b1 : b0) + __shfl_xor_sync(0xffffffffu, b3 ? b0 : b1, 8);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <>
SS_DEVINL float warp_reduce_rows<8>(float (&a)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float b[4], c[2];
#pragma unroll
  for (int i = 0; i < 4; i++)
    b[i] = (b4 ? a[i + 4] : a[i]) + __shfl_xor_sync(0xffffffffu, b4 ? a[i] : a[i + 4], 16);
#pragma unroll
  for (int i = 0; i < 2; i++)
    c[i] = (b3 ? b[i + 2] : b[i]) + __shfl_xor_sync(0xffffffffu, b3 ? b[i] : b[i + 2], 8);
  float v = (b2 ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, b2 ? c[0] : c[1], 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}
template <int G>
SS_DEVINL int row_of_lane(int lane) {
  if (G == 1) return 0;
  if (G == 2) return (lane >> 4) & 1;
  if (G == 4) return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
  return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}

// Packs (value, index) so that unsigned max picks the larger value and, among
// equal values, the lower index (ss_argmax, SlipStream/src/core/tensor.c:318-328).
SS_DEVINL unsigned long long pack_argmax(float v, int idx) {
  unsigned b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  if (v != v) b = 0;  // NaN never wins
  return ((unsigned long long)b << 32) | (unsigned)(0x7fffffff - idx);
}
SS_DEVINL int unpack_argmax_index(unsigned long long p) {
  return 0x7fffffff - (int)(unsigned)(p & 0xffffffffu);
}

// ---- the kernel ------------------------------------------------------------
// Threads: RG row-groups of NBT = blockDim.x / RG threads; thread (rg, blk)
// owns column block blk and, within every pipeline stage, rows
// rg*2 .. rg*2+1 of the stage (stage_rows = 2 * RG).
//
// Pipeline: thread 0 streams the CTA's contiguous row range global -> shared
// in stages of stage_rows rows with cp.async.bulk (one copy per stage, tracked
// by an mbarrier), keeping `nstage` stages in flight; the remaining range is
// bulk-prefetched into L2.  All of this is issued before the programmatic-
// dependent-launch wait, since weights never depend on the previous kernel.
template <int TYPE, XSrc XS, Epi EPI, int RG>
__global__ void __launch_bounds__(512) gemv_kernel(const GemvParams p) {
  constexpr int G = 2;  // rows per warp per stage
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = blockDim.x >> 5;
  const int nbt = blockDim.x / RG;          // threads per row-group
  const int nwb = nbt >> 5;                 // warps per row-group
  const int rg = tid / nbt;
  const int blk = tid - rg * nbt;
  const int wl = blk >> 5;                  // warp index inside the row-group
  const int nb = p.w.cols >> 5;
  const bool active = blk < nb;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(r0 + p.rows_per_cta, p.w.rows);
  const int nrows = max(r1 - r0, 0);
  const int SR = p.stage_rows;
  const int nst = (nrows + SR - 1) / SR;
  const uint32_t stage_bytes = (uint32_t)(SR * p.w.row_stride);
  uint8_t* ring = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + (size_t)p.nstage * stage_bytes);
  float* red = reinterpret_cast<float*>(bars + p.nstage);   // [nwb][rows_per_cta]
  float* scratch = red + nwb * p.rows_per_cta;             // 64 floats
  __shared__ int s_abort;
  const uint8_t* base = p.w.data + (size_t)r0 * p.w.row_stride;

  auto issue = [&](int i) {
    const int rows_i = min(SR, nrows - i * SR);
    const uint32_t bytes = (uint32_t)(rows_i * p.w.row_stride);
    const uint32_t bar = smem_addr(bars + (i % p.nstage));
    mbar_expect_tx(bar, bytes);
    bulk_g2s(smem_addr(ring + (size_t)(i % p.nstage) * stage_bytes),
             base + (size_t)i * SR * p.w.row_stride, bytes, bar);
  };
  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < p.nstage; i++) mbar_init(smem_addr(bars + i), 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0) {
    const int first = min(p.nstage, nst);
    for (int i = 0; i < first; i++) issue(i);
    if (p.prefetch && nst > first) {
      const size_t off = (size_t)first * SR * p.w.row_stride;
      prefetch_l2_bulk(base + off, (uint32_t)((size_t)nrows * p.w.row_stride - off));
    }
  }
  pdl_wait();

  // ---- prologue: this thread's 32 activations as block fixed-point byte planes
  XPlanes xp;
  {
    float xv[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (active) v = *reinterpret_cast<const float4*>(p.x + blk * 32 + i);
      xv[i] = v.x; xv[i + 1] = v.y; xv[i + 2] = v.z; xv[i + 3] = v.w;
    }
    if constexpr (XS == XSrc::RmsNorm) {
      // SlipStream/src/backends/cpu_neon.c:109-115: ss = sum x^2,
      // scale = 1 / sqrtf(ss / n + eps), out = x * scale * w.  Each row-group
      // of threads holds all n values, so ss is a block reduction (counted once).
      float4 wv4[8];
#pragma unroll
      for (int i = 0; i < 8; i++)
        wv4[i] = active ? *reinterpret_cast<const float4*>(p.norm_w + blk * 32 + 4 * i)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
      float ss = 0.0f;
      if (rg == 0) {
#pragma unroll
        for (int i = 0; i < 32; i++) ss = fmaf(xv[i], xv[i], ss);
      }
      ss = block_sum(ss, scratch);
      const float scale = 1.0f / sqrtf(ss / (float)p.w.cols + p.eps);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        xv[4 * i] = __fmul_rn(__fmul_rn(xv[4 * i], scale), wv4[i].x);
        xv[4 * i + 1] = __fmul_rn(__fmul_rn(xv[4 * i + 1], scale), wv4[i].y);
        xv[4 * i + 2] = __fmul_rn(__fmul_rn(xv[4 * i + 2], scale), wv4[i].z);
        xv[4 * i + 3] = __fmul_rn(__fmul_rn(xv[4 * i + 3], scale), wv4[i].w);
      }
    }
    xp = make_planes<TYPE == kQ4_0 ? 8 : 0>(xv);
  }
  pdl_trigger();

  // ---- main loop over pipeline stages
  int i = 0;
  for (; i < nst; i++) {
    const int slot = i % p.nstage;
    if (!mbar_wait_bounded(smem_addr(bars + slot), (uint32_t)((i / p.nstage) & 1), kWaitBudget)) {
      atomicOr(p.err, 4);
      s_abort = 1;
    }
    const int rows_i = min(SR, nrows - i * SR);
    const uint8_t* st = ring + (size_t)slot * stage_bytes;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
      const int k = rg * G + g;
      acc[g] = 0.0f;
      if (active && k < rows_i) {
        const uint8_t* rowp = st + (size_t)k * p.w.row_stride;
        const float d = half_bits_to_float(lds16(rowp + p.w.scale_off + blk * 2));
        float sdot;
        if constexpr (TYPE == kQ4_0) sdot = dot_q4_block(lds128(rowp + blk * 16), xp);
        else sdot = dot_q8_block(lds128(rowp + blk * 32), lds128(rowp + blk * 32 + 16), xp);
        acc[g] = sdot * (d * xp.fb);
      }
    }
    const float v = warp_reduce_rows<G>(acc, lane);
    const int rr = rg * G + row_of_lane<G>(lane);
    if ((lane & (32 / G - 1)) == 0 && rr < rows_i) red[wl * p.rows_per_cta + i * SR + rr] = v;
    __syncthreads();  // every thread is done with this slot
    if (s_abort) break;
    if (tid == 0 && i + p.nstage < nst) issue(i + p.nstage);
  }
  if (s_abort) {
    // drain the copies still in flight (bounded), then leave without output
    if (tid == 0) {
      const int issued = min(nst, i + p.nstage);
      for (int j = max(0, issued - p.nstage); j < issued; j++)
        mbar_wait_bounded(smem_addr(bars + j % p.nstage), (uint32_t)((j / p.nstage) & 1), kWaitBudget);
    }
    return;
  }

  // ---- epilogue
  auto row_sum = [&](int lr_) {
    float s = 0.0f;
    for (int w = 0; w < nwb; w++) s += red[w * p.rows_per_cta + lr_];
    return s;
  };

  if constexpr (EPI == Epi::Store || EPI == Epi::Residual) {
    for (int lr = tid; lr < nrows; lr += blockDim.x) {
      const int r = r0 + lr;
      float v = row_sum(lr);
      if constexpr (EPI == Epi::Residual) v = __fadd_rn(v, p.residual[r]);
      p.out[r] = v;
    }
  } else if constexpr (EPI == Epi::SwiGLU) {
    // rows 2i (gate) and 2i+1 (up); SlipStream/src/core/layer_scheduler.c:533-549:
    // up *= g / (1 + expf(-g)).
    for (int lp = tid; lp * 2 < nrows; lp += blockDim.x) {
      const float g = row_sum(2 * lp), u = row_sum(2 * lp + 1);
      p.out[(r0 >> 1) + lp] = __fmul_rn(u, __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
    }
  } else if constexpr (EPI == Epi::QKV) {
    // RoPE (non-NeoX, SlipStream/src/core/tensor.c:249-274) on q and k rows,
    // then the |k| / |v| maxima feeding the int8 cache scale
    // (layer_scheduler.c:101-111).
    const int pos = *p.d_pos;
    if (pos < 0 || pos >= p.ctx) return;  // host bounds positions; never index past the table
    float mk = 0.0f, mv = 0.0f;
    for (int lp = tid; lp * 2 < nrows; lp += blockDim.x) {
      const int r = r0 + 2 * lp;
      float a = row_sum(2 * lp), b = row_sum(2 * lp + 1);
      if (r < p.q_rows + p.kv_rows) {
        const int i = r % p.head_dim;
        if (i < p.rope_dim) {
          const float2 cs = p.rope_tab[(size_t)pos * (p.rope_dim >> 1) + (i >> 1)];
          const float na = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
          const float nb2 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
          a = na; b = nb2;
        }
        if (r >= p.q_rows) mk = fmaxf(mk, fmaxf(fabsf(a), fabsf(b)));
      } else {
        mv = fmaxf(mv, fmaxf(fabsf(a), fabsf(b)));
      }
      p.out[r] = a;
      p.out[r + 1] = b;
    }
    mk = warp_max(mk);
    mv = warp_max(mv);
    __syncthreads();
    if (lane == 0) { scratch[warp] = mk; scratch[32 + warp] = mv; }
    __syncthreads();
    if (tid == 0) {
      float a = 0.0f, b = 0.0f;
      for (int w = 0; w < nw; w++) { a = fmaxf(a, scratch[w]); b = fmaxf(b, scratch[32 + w]); }
      if (a > 0.0f) atomicMax(p.amax_k + pos, float_as_ordered(a));
      if (b > 0.0f) atomicMax(p.amax_v + pos, float_as_ordered(b));
    }
  } else if constexpr (EPI == Epi::Argmax) {
    unsigned long long best = 0;
    for (int lr = tid; lr < nrows; lr += blockDim.x) {
      const int r = r0 + lr;
      const float v = row_sum(lr);
      if (p.out) p.out[r] = v;
      const unsigned long long pk = pack_argmax(v, r);
      best = pk > best ? pk : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    __shared__ unsigned long long wbest[32];
    __shared__ bool is_last;
    if (lane == 0) wbest[warp] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = 0;
      for (int w = 0; w < nw; w++) b = wbest[w] > b ? wbest[w] : b;
      p.am_part[blockIdx.x] = b;
      __threadfence();
      is_last = atomicAdd(p.am_count, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      unsigned long long b = 0;
      for (int i = tid; i < (int)gridDim.x; i += blockDim.x) {
        const unsigned long long v = *((volatile unsigned long long*)p.am_part + i);
        b = v > b ? v : b;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
        b = other > b ? other : b;
      }
      if (lane == 0) wbest[warp] = b;
      __syncthreads();
      if (tid == 0) {
        unsigned long long bb = 0;
        for (int w = 0; w < nw; w++) bb = wbest[w] > bb ? wbest[w] : bb;
        const int tok = unpack_argmax_index(bb);
        const int pos = *p.d_pos_rw;
        if (pos + 1 < p.ctx && pos + 1 >= *p.fixed_until) p.seq_tokens[pos + 1] = tok;
        p.seq_tokens[p.ctx] = tok;  // last argmax, whatever the position
        *p.d_pos_rw = pos + 1;
        *p.am_count = 0;
      }
    }
  }
}

}  // namespace ss
