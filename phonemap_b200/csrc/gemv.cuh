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
  unsigned int* amax_k;      // this layer's slot for the current position's maximum
  unsigned int* amax_v;
  // Argmax epilogue
  int index_base;               // global index of row 0 (tensor parallelism: vocab slice start)
  unsigned long long* tp_best;  // non-null: the last CTA leaves the packed best here (an
                                // all-reduce and tp_finish_kernel complete the step)
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
  float c[3];   // (1, 256, 65536) * 2^(e-22): value of one unit of each plane
};

SS_DEVINL float pow2i(int k) { return __int_as_float((k + 127) << 23); }  // 2^k, -126 <= k <= 127

SS_DEVINL int sext8(int v) {  // sign-extend the low byte (prmt sign-replicate mode)
  int r;
  asm("prmt.b32 %0, %1, 0, 0x8880;" : "=r"(r) : "r"(v));
  return r;
}
SS_DEVINL unsigned pack_low_bytes(int a, int b, int c, int d) {  // a.b0 | b.b0<<8 | c.b0<<16 | d.b0<<24
  unsigned ab, cd, r;
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(ab) : "r"(a), "r"(b));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(cd) : "r"(c), "r"(d));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(r) : "r"(ab), "r"(cd));
  return r;
}

template <int ZP>
SS_DEVINL XPlanes make_planes(const float (&xv)[32]) {
  XPlanes xp;
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(xv[j]));
  // 2^e > amax: e = unbiased exponent of amax + 1 (blocks below 1e-30
  // contribute nothing measurable and become zero)
  const bool live = amax >= 1e-30f;
  const int e = (int)((__float_as_uint(amax) >> 23) & 255u) - 126;
  const float sc = live ? pow2i(22 - e) : 0.0f;
  xp.c[0] = live ? pow2i(e - 22) : 0.0f;
  xp.c[1] = live ? pow2i(e - 14) : 0.0f;
  xp.c[2] = live ? pow2i(e - 6) : 0.0f;
  int sum[3] = {0, 0, 0};
#pragma unroll
  for (int w = 0; w < 8; w++) {
    int d0[4], d1[4], d2[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      // balanced base-256 digits of m = round(x * 2^(22-e)), |m| <= 2^22
      const int m = __float2int_rn(xv[4 * w + i] * sc);
      d0[i] = sext8(m);
      const int m1 = (m - d0[i]) >> 8;
      d1[i] = sext8(m1);
      d2[i] = (m1 - d1[i]) >> 8;  // |d2| <= 64
    }
    xp.pl[0][w] = (int)pack_low_bytes(d0[0], d0[1], d0[2], d0[3]);
    xp.pl[1][w] = (int)pack_low_bytes(d1[0], d1[1], d1[2], d1[3]);
    xp.pl[2][w] = (int)pack_low_bytes(d2[0], d2[1], d2[2], d2[3]);
    if (ZP != 0) {
#pragma unroll
      for (int p = 0; p < 3; p++) {
        int acc;
        asm("dp4a.s32.s32 %0, %1, 0x01010101, %2;" : "=r"(acc) : "r"(xp.pl[p][w]), "r"(sum[p]));
        sum[p] = acc;
      }
    }
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
// fb * (a0 + 256 a1 + 65536 a2); |a_p| < 2^24, so the conversions are exact,
// and c = (fb, 256 fb, 65536 fb) are exact powers-of-two multiples.
SS_DEVINL float combine_planes(int a0, int a1, int a2, const float (&c)[3]) {
  return fmaf((float)a2, c[2], fmaf((float)a1, c[1], (float)a0 * c[0]));
}

// Q4_0 block: sum_j (q_j - 8) * x_j (x in block fixed point).
SS_DEVINL float dot_q4_block(const uint4 q, const XPlanes& xp) {
  // two accumulators per plane (low / high nibbles): 6 independent chains
  int a0 = xp.init[0], a1 = xp.init[1], a2 = xp.init[2], b0 = 0, b1 = 0, b2 = 0;
  const unsigned wq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const unsigned lo = wq[t] & 0x0F0F0F0Fu;          // q[4t .. 4t+3]
    const unsigned hi = (wq[t] >> 4) & 0x0F0F0F0Fu;   // q[16+4t .. 16+4t+3]
    a0 = dp4a_us(lo, xp.pl[0][t], a0);
    a1 = dp4a_us(lo, xp.pl[1][t], a1);
    a2 = dp4a_us(lo, xp.pl[2][t], a2);
    b0 = dp4a_us(hi, xp.pl[0][4 + t], b0);
    b1 = dp4a_us(hi, xp.pl[1][4 + t], b1);
    b2 = dp4a_us(hi, xp.pl[2][4 + t], b2);
  }
  return combine_planes(a0 + b0, a1 + b1, a2 + b2, xp.c);
}

// Q8_0 block: sum_j q_j * x_j (x in block fixed point).
SS_DEVINL float dot_q8_block(const uint4 qa, const uint4 qb, const XPlanes& xp) {
  int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
  const unsigned wa[4] = {qa.x, qa.y, qa.z, qa.w};
  const unsigned wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    a0 = dp4a_ss((int)wa[t], xp.pl[0][t], a0);
    a1 = dp4a_ss((int)wa[t], xp.pl[1][t], a1);
    a2 = dp4a_ss((int)wa[t], xp.pl[2][t], a2);
    b0 = dp4a_ss((int)wb[t], xp.pl[0][4 + t], b0);
    b1 = dp4a_ss((int)wb[t], xp.pl[1][4 + t], b1);
    b2 = dp4a_ss((int)wb[t], xp.pl[2][4 + t], b2);
  }
  return combine_planes(a0 + b0, a1 + b1, a2 + b2, xp.c);
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

// Packs (value, index) so that the unsigned maximum over all elements is the
// index ss_argmax returns (SlipStream/src/core/tensor.c:318-328: start from
// x[0], move only on a strict `>`):
//   * a larger value wins; among equal values the lower index (the first);
//   * -0.0 and +0.0 compare equal there, so both map to the key of +0.0;
//   * a NaN at index > 0 never compares greater, so it gets the lowest key;
//   * a NaN at index 0 is never replaced (nothing compares greater than it),
//     so it gets the highest key and index 0 wins outright.
// A NaN anywhere else with every other value NaN leaves index 0 (lowest key,
// lowest index), as the reference does.
SS_DEVINL unsigned long long pack_argmax(float v, int idx) {
  unsigned b;
  if (v != v) {
    b = idx == 0 ? 0xffffffffu : 0u;
  } else {
    b = v == 0.0f ? 0u : __float_as_uint(v);  // -0.0 -> +0.0
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  }
  return ((unsigned long long)b << 32) | (unsigned)(0x7fffffff - idx);
}
SS_DEVINL int unpack_argmax_index(unsigned long long p) {
  return 0x7fffffff - (int)(unsigned)(p & 0xffffffffu);
}

// ---- the kernel ------------------------------------------------------------
// Warp roles: warp 0 is the producer, warps 1.. the consumers.  Consumers form
// RG row-groups of NBT = nb rounded up to 32 threads; consumer thread
// (rg, blk) owns column block blk and, in every pipeline stage, rows
// rg*G .. rg*G+G-1 of the stage (stage_rows = G * RG).
//
// Pipeline: the producer's lane 0 streams the CTA's contiguous row range
// global -> shared in stages of stage_rows rows, one cp.async.bulk per stage,
// through a ring of `nstage` slots.  Each slot has a "full" mbarrier (completed
// by the copy's byte count) and an "empty" mbarrier (one arrival per consumer
// warp), so consumer warps run independently of each other and the producer
// refills a slot as soon as every warp is done with it.  The first `nstage`
// copies and a bulk L2 prefetch of the rest of the range are issued before the
// programmatic-dependent-launch wait: weights never depend on the previous
// kernel.  Every mbarrier wait is bounded; on expiry the kernel records an
// error bit, drains its copies and returns without writing outputs.
// Named barrier over `count` threads.  The non-aligned form: it waits for all
// non-exited threads of each arriving warp itself, so it stays correct when a
// warp reaches it diverged -- single-thread work (`if (tid == 0) ...`) often
// directly precedes it, and nothing forces the compiler to reconverge before an
// opaque asm statement (bar.sync, the aligned form, requires that).
SS_DEVINL void named_bar_sync(int id, int count) {
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
SS_DEVINL void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

constexpr int kGemvG = 4;  // rows per consumer warp per stage
constexpr int kGemvMaxNb = 512;  // column blocks of one GEMV: one per consumer thread of a row-group

template <int TYPE, XSrc XS, Epi EPI, int RG>
__global__ void __launch_bounds__(544) gemv_kernel(const GemvParams p) {
  constexpr int G = kGemvG;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = blockDim.x >> 5;
  const int ncw = nw - 1;                   // consumer warps
  const int nwb = ncw / RG;                 // consumer warps per row-group
  const int cw = warp - 1;                  // consumer warp index (-1: producer)
  const int rg = cw >= 0 ? cw / nwb : 0;
  const int wl = cw >= 0 ? cw - rg * nwb : 0;
  const int blk = wl * 32 + lane;
  const int nb = p.w.cols >> 5;
  const bool active = cw >= 0 && blk < nb;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(r0 + p.rows_per_cta, p.w.rows);
  const int nrows = max(r1 - r0, 0);
  const int SR = p.stage_rows;
  const int nst = (nrows + SR - 1) / SR;
  const uint32_t stage_bytes = (uint32_t)(SR * p.w.row_stride);
  uint8_t* ring = smem_raw;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + (size_t)p.nstage * stage_bytes);
  uint64_t* empty = full + p.nstage;
  float* red = reinterpret_cast<float*>(empty + p.nstage);  // [nwb][rows_per_cta]
  float* scratch = red + nwb * p.rows_per_cta;             // 64 floats
  __shared__ int s_abort;
  const uint8_t* base = p.w.data + (size_t)r0 * p.w.row_stride;

  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < p.nstage; i++) {
      mbar_init(smem_addr(full + i), 1);
      mbar_init(smem_addr(empty + i), (uint32_t)ncw);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (cw < 0) {
    // ---------------- producer warp
    if (lane == 0) {
      auto issue = [&](int i) {
        const int rows_i = min(SR, nrows - i * SR);
        const uint32_t bytes = (uint32_t)(rows_i * p.w.row_stride);
        const uint32_t bar = smem_addr(full + (i % p.nstage));
        mbar_expect_tx(bar, bytes);
        bulk_g2s(smem_addr(ring + (size_t)(i % p.nstage) * stage_bytes),
                 base + (size_t)i * SR * p.w.row_stride, bytes, bar);
      };
      const int first = min(p.nstage, nst);
      for (int i = 0; i < first; i++) issue(i);
      if (p.prefetch && nst > first) {
        const size_t off = (size_t)first * SR * p.w.row_stride;
        prefetch_l2_bulk(base + off, (uint32_t)((size_t)nrows * p.w.row_stride - off));
      }
      int i = first;
      for (; i < nst; i++) {
        const int slot = i % p.nstage;
        if (!mbar_wait_bounded(smem_addr(empty + slot), (uint32_t)((i / p.nstage - 1) & 1),
                               kWaitBudget)) {
          atomicOr(p.err, 4);
          s_abort = 1;
          break;
        }
        issue(i);
      }
      if (s_abort) {  // drain what is in flight before the CTA can exit
        for (int j = max(0, i - p.nstage); j < i; j++)
          mbar_wait_bounded(smem_addr(full + j % p.nstage), (uint32_t)((j / p.nstage) & 1),
                            kWaitBudget);
      }
    }
  } else {
    // ---------------- consumer warps
    pdl_wait();
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
        // scale = 1 / sqrtf(ss / n + eps), out = x * scale * w.  Row-group 0
        // holds all n values, so ss is a sum over its threads.
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
        ss = warp_sum(ss);
        if (lane == 0) scratch[cw] = ss;
        named_bar_sync(1, ncw * 32);
        ss = 0.0f;
        for (int w = 0; w < ncw; w++) ss += scratch[w];
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

    // Per-thread byte offsets inside a slot, fixed for the whole loop.  Rows
    // past the end of a partial last stage are computed from stale slot bytes
    // and never stored; lanes past the last block read block 0 and carry zero
    // activations (xp is zero for them), so neither needs a per-row test.
    const int bsafe = active ? blk : 0;
    const uint32_t ring_base = smem_addr(ring);
    const uint32_t q_off = (uint32_t)((rg * G) * p.w.row_stride + bsafe * (TYPE == kQ4_0 ? 16 : 32));
    const uint32_t s_off = (uint32_t)((rg * G) * p.w.row_stride + p.w.scale_off + bsafe * 2);
    const uint32_t rs = (uint32_t)p.w.row_stride;
    float* red_w = red + wl * p.rows_per_cta + rg * G + row_of_lane<G>(lane);
    const bool writer = (lane & (32 / G - 1)) == 0;
    int slot = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nst; i++) {
      if (!mbar_wait_bounded(smem_addr(full + slot), phase, kWaitBudget)) {
        atomicOr(p.err, 4);
        s_abort = 1;
        break;
      }
      const uint32_t st = ring_base + (uint32_t)slot * stage_bytes;
      uint4 qa[G], qb[G];
      uint16_t sc[G];
#pragma unroll
      for (int g = 0; g < G; g++) {
        const uint32_t rq = st + q_off + (uint32_t)g * rs;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sc[g]) : "r"(st + s_off + (uint32_t)g * rs));
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(qa[g].x), "=r"(qa[g].y), "=r"(qa[g].z), "=r"(qa[g].w) : "r"(rq));
        if constexpr (TYPE == kQ8_0)
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(qb[g].x), "=r"(qb[g].y), "=r"(qb[g].z), "=r"(qb[g].w) : "r"(rq + 16));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(empty + slot));  // slot free for the producer
      float acc[G];
#pragma unroll
      for (int g = 0; g < G; g++) {
        float sdot;
        if constexpr (TYPE == kQ4_0) sdot = dot_q4_block(qa[g], xp);
        else sdot = dot_q8_block(qa[g], qb[g], xp);
        acc[g] = sdot * half_bits_to_float(sc[g]);
      }
      const float v = warp_reduce_rows<G>(acc, lane);
      const int rr = rg * G + row_of_lane<G>(lane);
      if (writer && rr < nrows - i * SR) red_w[i * SR] = v;
      if (++slot == p.nstage) { slot = 0; phase ^= 1u; }
    }
  }
  __syncthreads();
  if (s_abort) return;

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
      // (tensor parallelism: only rank 0 adds the residual before the all-reduce)
      if constexpr (EPI == Epi::Residual)
        if (p.residual) v = __fadd_rn(v, p.residual[r]);
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
      if (a > 0.0f) atomicMax(p.amax_k, float_as_ordered(a));
      if (b > 0.0f) atomicMax(p.amax_v, float_as_ordered(b));
    }
  } else if constexpr (EPI == Epi::Argmax) {
    unsigned long long best = 0;
    for (int lr = tid; lr < nrows; lr += blockDim.x) {
      const int r = r0 + lr;
      const float v = row_sum(lr);
      if (p.out) p.out[r] = v;
      const unsigned long long pk = pack_argmax(v, p.index_base + r);
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
      if (tid == 0 && p.tp_best) {
        unsigned long long bb = 0;
        for (int w = 0; w < nw; w++) bb = wbest[w] > bb ? wbest[w] : bb;
        *p.tp_best = bb;
        *p.am_count = 0;
      } else if (tid == 0) {
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
