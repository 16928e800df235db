// batch_kernels.cuh -- the many-token decoder step around the tensor-core
// product (qgemm.cuh): T tokens, each with its own sequence and position,
// through every layer at once.  Serves the prompt (ss_scheduler_prefill,
// SlipStream/src/core/layer_scheduler.c:681-803: the reference runs the prompt
// token by token, layer-major; each token's layer l depends only on the cache
// rows of earlier positions at layer l, so writing the batch's K/V rows first
// and then attending causally gives the same result) and several sequences
// decoded together.
//
// Per layer (process_layer, layer_scheduler.c:291-567): RMSNorm -> QKV
// product -> RoPE + int8 K/V append (bt_qkv_kernel) -> attention over each
// token's own cache rows (bt_attn_kernel) -> O product + residual -> RMSNorm
// -> gate/up product -> SwiGLU -> down product + residual.  The products
// leave per-split partial sums; each consumer below adds them in split order.
// The elementwise steps between products (residual add, SwiGLU, the merge of
// the attention slots) run inside the next product's activation prep
// (bt_prep_kernel), so a layer is 9 kernels.  Every kernel here waits for its
// predecessor with griddepcontrol (programmatic dependent launch) before it
// touches global memory, and lets its successor launch at once.
#pragma once
#include <cooperative_groups.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "qgemm.cuh"

namespace ss {

// Where token t of the batch goes: its sequence, position, and token id.
struct BatchTokens {
  const int* tok;   // [T]
  const int* pos;   // [T]
  const int* seq;   // [T]
};

// KV cache of every sequence: sequence s, layer l at kc + s * seq_stride +
// l * ctx * kvd, head-major [nkv][ctx][hd] inside a layer; scales at
// ks + s * sc_stride + l * ctx.
struct BatchKv {
  int8_t* kc;
  int8_t* vc;
  float* ks;
  float* vs;
  size_t seq_stride, sc_stride;
  int ctx;
};

SS_DEVINL float split_sum(const float* part, int nsplit, size_t n, size_t i) {
  float v = part[i];
  for (int s = 1; s < nsplit; s++) v += part[(size_t)s * n + i];
  return v;
}

// h[t] = token_embd[tok[t]] (layer_scheduler.c:584-587); tokens outside the
// vocabulary set error bit 2 and read row 0.
__global__ void bt_embed_kernel(const float* __restrict__ embd, int d, int vocab, BatchTokens bt, int T,
                                float* __restrict__ h, int* err, unsigned* __restrict__ zero, int nzero) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  // the pass's K/V maxima and greedy-choice words start at zero
  if (t == 0 && blockIdx.x == 0)
    for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0u;
  int tok = bt.tok[t];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, 2);
    tok = 0;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x)
    h[(size_t)t * d + i] = embd[(size_t)tok * d + i];
}

// q|k|v of every token = the product's split sums, with RoPE on q and k
// (non-NeoX, tensor.c:249-274, the table built on the host with the
// reference's expressions): q to qout[t], k | v (fp32) to kvtmp[t], and the
// largest |k| and |v| of each token into amax[t] (float bits as unsigned:
// non-negative floats order like their bits, so the maximum is exact and
// independent of the order).  One thread per (q, k) or (k, k+1) pair.
__global__ void bt_qkv_kernel(const float* __restrict__ part, int nsplit, int T, int rows, int qd, int kvd,
                              int hd, int rope_dim, const float2* __restrict__ rope_tab, BatchTokens bt,
                              float* __restrict__ qout, float* __restrict__ kvtmp, unsigned* __restrict__ amax) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const int pr = blockIdx.x * blockDim.x + threadIdx.x;
  const int r = 2 * pr;
  float mk = 0.0f, mv = 0.0f;
  if (r < rows) {
    const size_t n = (size_t)T * rows;
    float a = split_sum(part, nsplit, n, (size_t)t * rows + r);
    float b = split_sum(part, nsplit, n, (size_t)t * rows + r + 1);
    if (r < qd + kvd) {
      const int i = r % hd;
      if (i < rope_dim) {
        const float2 cs = rope_tab[(size_t)bt.pos[t] * (rope_dim >> 1) + (i >> 1)];
        const float na = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        const float nb = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
        a = na;
        b = nb;
      }
    }
    if (r < qd) {
      qout[(size_t)t * qd + r] = a;
      qout[(size_t)t * qd + r + 1] = b;
    } else {
      kvtmp[(size_t)t * 2 * kvd + (r - qd)] = a;
      kvtmp[(size_t)t * 2 * kvd + (r - qd) + 1] = b;
      if (r < qd + kvd) mk = fmaxf(fabsf(a), fabsf(b));
      else mv = fmaxf(fabsf(a), fabsf(b));
    }
  }
  mk = warp_max(mk);
  mv = warp_max(mv);
  if ((threadIdx.x & 31) == 0) {
    if (mk > 0.0f) atomicMax(amax + 2 * t, __float_as_uint(mk));
    if (mv > 0.0f) atomicMax(amax + 2 * t + 1, __float_as_uint(mv));
  }
}

// The int8 K/V row of each token at (sequence, layer, position) with one
// scale per row over the whole kv_dim (kv_turboquant_encode,
// layer_scheduler.c:101-118: scale = max / 127, q = roundf(v / scale)).
__global__ void bt_kv_encode_kernel(const float* __restrict__ kvtmp, const unsigned* __restrict__ amax, int kvd,
                                    int hd, BatchTokens bt, BatchKv kv, int layer) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int pos = bt.pos[t], seq = bt.seq[t];
  const float k_scale = __uint_as_float(amax[2 * t]) / 127.0f;   // layer_scheduler.c:109-110
  const float v_scale = __uint_as_float(amax[2 * t + 1]) / 127.0f;
  if (i < kvd) {
    const float kinv = k_scale > 0.0f ? 1.0f / k_scale : 0.0f;
    const float vinv = v_scale > 0.0f ? 1.0f / v_scale : 0.0f;
    const int kvh = i / hd, j = i - kvh * hd;
    const size_t o = seq * kv.seq_stride + (size_t)layer * kv.ctx * kvd + ((size_t)kvh * kv.ctx + pos) * hd + j;
    kv.kc[o] = kv_encode(kvtmp[(size_t)t * 2 * kvd + i], kinv);
    kv.vc[o] = kv_encode(kvtmp[(size_t)t * 2 * kvd + kvd + i], vinv);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    kv.ks[seq * kv.sc_stride + (size_t)layer * kv.ctx + pos] = k_scale;
    kv.vs[seq * kv.sc_stride + (size_t)layer * kv.ctx + pos] = v_scale;
  }
}

// Attention (layer_scheduler.c:415-468; softmax tensor.c:154-173) of every
// token over positions 0..pos of its sequence, split over the positions as
// flash-decoding does: CTA (kv head, token, slot s) takes the chunks of
// kBtAttnChunk cached positions s, s + kBtAttnSlots, ... up to pos, for the G
// query heads that share the kv head.  Per chunk: the int8 K and V rows and
// their scales are staged in shared memory (coalesced 16-byte loads), scores
// s_j = (q . k_j) * k_scale_j * (1/sqrt(hd)) (two threads per position, each
// K value converted once for all G heads), then a running softmax (max m, sum
// l, output o rescaled when m grows) and o += p_j v_scale_j v_j (each thread
// four elements of a group of positions).  The slot's (m, l, o) go to `part`;
// the O product's prep merges the slots.  The result equals the reference's
// softmax-weighted sum of dec(V_j) up to fp32 rounding order.
constexpr int kBtAttnChunk = 128;   // positions per chunk
constexpr int kBtAttnSlots = 16;    // position slots (CTAs) per (kv head, token)
constexpr int kBtAttnMaxG = 8;      // query heads per kv head
constexpr int kBtAttnThreads = 256;

__host__ __device__ constexpr size_t bt_attn_smem(int hd, int G) {
  // q[G][hd] | scores[G][chunk] | k scale, v scale [chunk] | m, l, corr [G]
  // | K chunk, V chunk [chunk][hd] int8 (after the last chunk: the position
  // groups' partial outputs [threads / (hd / 4)][G][hd] fp32)
  return (size_t)(G * hd + G * kBtAttnChunk + 2 * kBtAttnChunk + 4 * kBtAttnMaxG) * sizeof(float) +
         ((size_t)2 * kBtAttnChunk * hd > (size_t)4096 * G ? (size_t)2 * kBtAttnChunk * hd : (size_t)4096 * G);
}

// Four signed bytes as floats, exactly: byte ^ 0x80 (in [0, 255]) in the low
// mantissa bits of 2^23, minus 2^23 + 128.
SS_DEVINL void s8x4_to_f32(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
}

// part layout: [T][nh][slots][hd + 2]: m, l, then o[hd].
__global__ void __launch_bounds__(kBtAttnThreads) bt_attn_kernel(const float* __restrict__ q, BatchTokens bt,
                                                                 BatchKv kv, int layer, int nh, int nkv, int hd,
                                                                 float scale, float* __restrict__ part) {
  extern __shared__ float sm[];
  pdl_wait();
  pdl_trigger();
  const int kvh = blockIdx.x, t = blockIdx.y, slot = blockIdx.z;
  const int pos = bt.pos[t], seq = bt.seq[t];
  if (slot * kBtAttnChunk > pos) return;  // no chunk for this slot (the merge skips it)
  const int G = nh / nkv, kvd = nkv * hd, qd = nh * hd;
  float* qs = sm;                               // [G][hd]
  float* sc = qs + G * hd;                      // [G][chunk]
  float* sks = sc + G * kBtAttnChunk;           // [chunk]
  float* svs = sks + kBtAttnChunk;              // [chunk]
  float* sml = svs + kBtAttnChunk;              // m[G] | l[G] | corr[G] | pad
  int8_t* sk = reinterpret_cast<int8_t*>(sml + 4 * kBtAttnMaxG);
  int8_t* sv = sk + kBtAttnChunk * hd;
  float* red = reinterpret_cast<float*>(sk);    // after the last chunk
  const int tid = threadIdx.x, nt = kBtAttnThreads;
  for (int i = tid; i < G * hd; i += nt) qs[i] = q[(size_t)t * qd + (size_t)kvh * G * hd + i];
  if (tid < G) {
    sml[tid] = -INFINITY;
    sml[kBtAttnMaxG + tid] = 0.0f;
  }
  const size_t lbase = seq * kv.seq_stride + (size_t)layer * kv.ctx * kvd + (size_t)kvh * kv.ctx * hd;
  const int8_t* kc = kv.kc + lbase;
  const int8_t* vc = kv.vc + lbase;
  const float* ks = kv.ks + seq * kv.sc_stride + (size_t)layer * kv.ctx;
  const float* vs = kv.vs + seq * kv.sc_stride + (size_t)layer * kv.ctx;
  // PV mapping: element quad eq, position group pg
  const int nq = hd >> 2, eq = tid % nq, pg = tid / nq, npg = nt / nq;
  float o[kBtAttnMaxG][4];
#pragma unroll
  for (int h = 0; h < kBtAttnMaxG; h++)
#pragma unroll
    for (int k = 0; k < 4; k++) o[h][k] = 0.0f;
  const int vec = hd / 16;
  const int half = hd >> 1;
  for (int ch = slot; ch * kBtAttnChunk <= pos; ch += kBtAttnSlots) {
    const int c0 = ch * kBtAttnChunk, cn = min(kBtAttnChunk, pos + 1 - c0);
    __syncthreads();  // the previous chunk is consumed (and q, m, l are set)
    for (int k = tid; k < cn * vec; k += nt) {
      reinterpret_cast<int4*>(sk)[k] = __ldcg(reinterpret_cast<const int4*>(kc + (size_t)c0 * hd) + k);
      reinterpret_cast<int4*>(sv)[k] = __ldcg(reinterpret_cast<const int4*>(vc + (size_t)c0 * hd) + k);
    }
    for (int k = tid; k < cn; k += nt) {
      sks[k] = ks[c0 + k];
      svs[k] = vs[c0 + k];
    }
    __syncthreads();
    // scores: thread pair (2j, 2j+1) takes position j, one half of hd each
    for (int j0 = 0; j0 < cn; j0 += nt / 2) {
      const int j = j0 + (tid >> 1), hf = tid & 1;
      const int jr = min(j, cn - 1);  // past the chunk: a duplicate, not stored
      float dot[kBtAttnMaxG];
#pragma unroll
      for (int h = 0; h < kBtAttnMaxG; h++) dot[h] = 0.0f;
      const int8_t* kr = sk + jr * hd + hf * half;
      for (int i = 0; i < half; i += 16) {
        const uint4 kw = *reinterpret_cast<const uint4*>(kr + i);
        float kf[16];
        s8x4_to_f32(kw.x, kf);
        s8x4_to_f32(kw.y, kf + 4);
        s8x4_to_f32(kw.z, kf + 8);
        s8x4_to_f32(kw.w, kf + 12);
#pragma unroll
        for (int h = 0; h < kBtAttnMaxG; h++) {
          if (h < G) {
            const float4* qv = reinterpret_cast<const float4*>(qs + h * hd + hf * half + i);
#pragma unroll
            for (int u = 0; u < 4; u++) {
              const float4 qq = qv[u];
              dot[h] = fmaf(qq.x, kf[4 * u], dot[h]);
              dot[h] = fmaf(qq.y, kf[4 * u + 1], dot[h]);
              dot[h] = fmaf(qq.z, kf[4 * u + 2], dot[h]);
              dot[h] = fmaf(qq.w, kf[4 * u + 3], dot[h]);
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < kBtAttnMaxG; h++) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], 1);
      if (hf == 0 && j < cn)
#pragma unroll
        for (int h = 0; h < kBtAttnMaxG; h++)
          if (h < G) sc[h * kBtAttnChunk + j] = dot[h] * sks[j] * scale;
    }
    __syncthreads();
    // running softmax per head: warp h (G <= 8 warps)
    {
      const int w = tid >> 5, lane = tid & 31;
      if (w < G) {
        float mx = -INFINITY;
        for (int j = lane; j < cn; j += 32) mx = fmaxf(mx, sc[w * kBtAttnChunk + j]);
        mx = warp_max(mx);
        const float mo = sml[w], mn = fmaxf(mo, mx);
        float sum = 0.0f;
        for (int j = lane; j < cn; j += 32) {
          const float pj = expf(sc[w * kBtAttnChunk + j] - mn);
          sc[w * kBtAttnChunk + j] = pj * svs[j];  // the V scale joins the weight
          sum += pj;
        }
        sum = warp_sum(sum);
        if (lane == 0) {
          const float corr = mo == -INFINITY ? 0.0f : expf(mo - mn);
          sml[w] = mn;
          sml[kBtAttnMaxG + w] = sml[kBtAttnMaxG + w] * corr + sum;
          sml[2 * kBtAttnMaxG + w] = corr;
        }
      }
    }
    __syncthreads();
    // o = o * corr + sum_j w_j v_j over this thread's positions
#pragma unroll
    for (int h = 0; h < kBtAttnMaxG; h++) {
      if (h < G) {
        const float cr = sml[2 * kBtAttnMaxG + h];
#pragma unroll
        for (int k = 0; k < 4; k++) o[h][k] *= cr;
      }
    }
    for (int j = pg; j < cn; j += npg) {
      float vf[4];
      s8x4_to_f32(*reinterpret_cast<const uint32_t*>(sv + j * hd + 4 * eq), vf);
#pragma unroll
      for (int h = 0; h < kBtAttnMaxG; h++) {
        if (h < G) {
          const float wj = sc[h * kBtAttnChunk + j];
#pragma unroll
          for (int k = 0; k < 4; k++) o[h][k] = fmaf(wj, vf[k], o[h][k]);
        }
      }
    }
  }
  __syncthreads();  // the staging area becomes the position groups' partials
#pragma unroll
  for (int h = 0; h < kBtAttnMaxG; h++)
    if (h < G)
      *reinterpret_cast<float4*>(red + ((size_t)pg * G + h) * hd + 4 * eq) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
  __syncthreads();
  for (int idx = tid; idx < G * hd; idx += nt) {
    const int h = idx / hd, e = idx - h * hd;
    float acc = 0.0f;
    for (int g2 = 0; g2 < npg; g2++) acc += red[((size_t)g2 * G + h) * hd + e];
    float* pp = part + (((size_t)t * nh + (size_t)kvh * G + h) * kBtAttnSlots + slot) * (hd + 2);
    if (e == 0) {
      pp[0] = sml[h];
      pp[1] = sml[kBtAttnMaxG + h];
    }
    pp[2 + e] = acc;
  }
}

// ---- activation prep of a product, fused with the elementwise step before it

enum PrepMode : int {
  kPrepPlain = 0,   // x = the input row
  kPrepResid = 1,   // x = h + the previous product (residual add, layer_scheduler.c:484, :566);
                    //     the new h is also written out
  kPrepSwiGLU = 2,  // x = up * (g / (1 + expf(-g))) of the gate/up product (layer_scheduler.c:533-549)
  kPrepMerge = 3,   // x = the attention output, merged from the position slots
};

constexpr int kPrepMaxHeads = 128;  // query heads of one token (merge factors in shared memory)

struct PrepParams {
  const float* x;       // Plain, Resid: token t's row at x + (t + toff) * ld
  int ld;
  int n;                // elements per token (the product's columns)
  const float* norm_w;  // RMSNorm weight (nullptr: none)
  float eps;
  int T, TP, toff;      // tokens; B rows per piece; first source row
  float* post;          // [T]: the power of two each token's result is multiplied by
  __half* xq;           // the pieces, [nb][2][TP][32] canonical per block
  const float* part;    // Resid, SwiGLU: the previous product's partials [nsplit][ptok][prow]
  int nsplit, ptok, prow;
  float* h_out;         // Resid: the new residual stream (same row layout as x)
  const float* apart;   // Merge: attention slots [ptok][nh][slots][hd + 2]
  BatchTokens bt;
  int nh, hd;
};

template <int MODE>
SS_DEVINL float prep_elem(const PrepParams& p, int tr, int i, const float* mf, const float* minv) {
  if constexpr (MODE == kPrepPlain) {
    return p.x[(size_t)tr * p.ld + i];
  } else if constexpr (MODE == kPrepResid) {
    const size_t n = (size_t)p.ptok * p.prow;
    return __fadd_rn(split_sum(p.part, p.nsplit, n, (size_t)tr * p.prow + i), p.x[(size_t)tr * p.ld + i]);
  } else if constexpr (MODE == kPrepSwiGLU) {
    const size_t n = (size_t)p.ptok * p.prow;
    const float g = split_sum(p.part, p.nsplit, n, (size_t)tr * p.prow + 2 * i);
    const float u = split_sum(p.part, p.nsplit, n, (size_t)tr * p.prow + 2 * i + 1);
    return __fmul_rn(u, __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
  } else {
    const int h = i / p.hd, e = i - h * p.hd;
    const int ns = min(kBtAttnSlots, p.bt.pos[tr] / kBtAttnChunk + 1);
    const float* pp = p.apart + ((size_t)tr * p.nh + h) * kBtAttnSlots * (p.hd + 2) + 2 + e;
    // every slot's load issued before the chain of fmas that uses them
    float o[kBtAttnSlots];
#pragma unroll
    for (int s2 = 0; s2 < kBtAttnSlots; s2++) o[s2] = s2 < ns ? pp[(size_t)s2 * (p.hd + 2)] : 0.0f;
    float acc = 0.0f;
#pragma unroll
    for (int s2 = 0; s2 < kBtAttnSlots; s2++)
      if (s2 < ns) acc = fmaf(o[s2], mf[h * kBtAttnSlots + s2], acc);
    return acc * minv[h];
  }
}

// The activation pieces of a product (numerics in qgemm.cuh): a cluster of
// kPrepSlices CTAs per token row t < TP, CTA k computing the mode's values of
// slice k of the row (contiguous blocks) once, into shared memory, with its
// partial sum of squares and largest |x * w|; the partials meet through
// distributed shared memory (added in rank order, so every CTA of the token
// gets the same RMSNorm scale and power of two); then each CTA writes its
// slice's pieces (Resid: and the new h).  Rows t >= T write zero pieces.
constexpr int kPrepSlices = 8;         // CTAs per token (the cluster)
constexpr int kPrepMaxSlice = 4096;    // elements per slice (rows up to 32768)

template <int MODE>
__global__ void __launch_bounds__(512) bt_prep_kernel(const PrepParams p) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float vals[kPrepMaxSlice];
  __shared__ float red[64];
  __shared__ float s_part[2];  // this CTA's sum of squares, max |x * w|
  __shared__ float mf[MODE == kPrepMerge ? kPrepMaxHeads * kBtAttnSlots : 1];
  __shared__ float minv[MODE == kPrepMerge ? kPrepMaxHeads : 1];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, tr = t + p.toff;
  const int slice = (int)cluster.block_rank();
  const int nb = p.n >> 5;
  const int b0 = (int)((long long)nb * slice / kPrepSlices), b1 = (int)((long long)nb * (slice + 1) / kPrepSlices);
  const int i0 = b0 * 32, i1 = b1 * 32;
  const bool live = t < p.T;
  if (live) {
    if constexpr (MODE == kPrepMerge) {
      // per head of the slice: M = max m_s, f_s = e^(m_s - M), 1 / sum_s f_s l_s
      const int ns = min(kBtAttnSlots, p.bt.pos[tr] / kBtAttnChunk + 1);
      const int h0 = i0 / p.hd, h1 = (i1 + p.hd - 1) / p.hd;
      for (int h = h0 + (int)threadIdx.x; h < h1; h += blockDim.x) {
        const float* pp = p.apart + ((size_t)tr * p.nh + h) * kBtAttnSlots * (p.hd + 2);
        float M = -INFINITY;
        for (int s2 = 0; s2 < ns; s2++) M = fmaxf(M, pp[(size_t)s2 * (p.hd + 2)]);
        float L = 0.0f;
        for (int s2 = 0; s2 < ns; s2++) {
          const float f = expf(pp[(size_t)s2 * (p.hd + 2)] - M);
          mf[h * kBtAttnSlots + s2] = f;
          L = fmaf(pp[(size_t)s2 * (p.hd + 2) + 1], f, L);
        }
        minv[h] = 1.0f / L;
      }
      __syncthreads();
    }
    float ss = 0.0f, amax = 0.0f;
#pragma unroll 2
    for (int i = i0 + (int)threadIdx.x; i < i1; i += blockDim.x) {
      const float v = prep_elem<MODE>(p, tr, i, mf, minv);
      vals[i - i0] = v;
      ss = fmaf(v, v, ss);
      amax = fmaxf(amax, fabsf(p.norm_w ? v * p.norm_w[i] : v));
    }
    ss = warp_sum(ss);
    amax = warp_max(amax);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) {
      red[w] = ss;
      red[32 + w] = amax;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.0f, m = 0.0f;
      for (int i = 0; i < nw; i++) {
        tot += red[i];
        m = fmaxf(m, red[32 + i]);
      }
      s_part[0] = tot;
      s_part[1] = m;
    }
  }
  cluster.sync();  // every slice's partials are in place
  float sc = 0.0f, pre = 0.0f;
  if (live) {
    float tot = 0.0f, m = 0.0f;
    for (int r = 0; r < kPrepSlices; r++) {
      const float* rp = cluster.map_shared_rank(s_part, r);
      tot += rp[0];
      m = fmaxf(m, rp[1]);
    }
    sc = p.norm_w ? 1.0f / sqrtf(tot / (float)p.n + p.eps) : 1.0f;
    m *= sc;
    int e = m >= 1.17549435e-38f ? (int)((__float_as_uint(m) >> 23) & 255u) - 127 : 0;
    e = max(-126, min(126, e));
    pre = pow2i(-e);
    if (slice == 0 && threadIdx.x == 0) p.post[t] = pow2i(e);
  }
  cluster.sync();  // no CTA leaves while another still reads its partials
  for (int i = i0 + (int)threadIdx.x; i < i1; i += blockDim.x) {
    const int b = i >> 5, k = i & 31;
    float v = 0.0f;
    if (live) {
      v = vals[i - i0];
      if constexpr (MODE == kPrepResid) p.h_out[(size_t)tr * p.ld + i] = v;
      if (p.norm_w) v = __fmul_rn(__fmul_rn(v, sc), p.norm_w[i]);
      v = __fmul_rn(v, pre);
    }
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    uint8_t* blk = reinterpret_cast<uint8_t*>(p.xq) + (size_t)b * 2 * p.TP * 64;
    *reinterpret_cast<__half*>(blk + qg_canon16(t, k)) = hi;
    *reinterpret_cast<__half*>(blk + p.TP * 64 + qg_canon16(t, k)) = lo;
  }
}

// h[t][r] = the product + h (the last residual add of a pass whose final
// hidden states are needed without the lm_head: the embedding).
__global__ void bt_residual_kernel(const float* __restrict__ part, int nsplit, int T, int rows,
                                   const float* __restrict__ h, float* __restrict__ h_out) {
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)T * rows;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    h_out[i] = __fadd_rn(split_sum(part, nsplit, n, i), h[i]);
}

// Logits of token t (the product's split sums) and the packed (value,
// index) maximum (pack_argmax: ss_argmax's rule, tensor.c:318-328) into
// best[t] by atomicMax -- order-independent, so deterministic.
__global__ void bt_head_kernel(const float* __restrict__ part, int nsplit, int T, int vocab,
                               float* __restrict__ logits, unsigned long long* __restrict__ best) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const size_t n = (size_t)T * vocab;
  unsigned long long b = 0;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < vocab; r += gridDim.x * blockDim.x) {
    const float v = split_sum(part, nsplit, n, (size_t)t * vocab + r);
    logits[(size_t)t * vocab + r] = v;
    const unsigned long long pk = pack_argmax(v, r);
    b = pk > b ? pk : b;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
    b = other > b ? other : b;
  }
  if ((threadIdx.x & 31) == 0 && b) atomicMax(best + t, b);
}

// next[t] = the index in best[t] (index 0 when nothing was packed).
__global__ void bt_token_kernel(const unsigned long long* __restrict__ best, int T, int* __restrict__ next) {
  pdl_wait();
  pdl_trigger();
  const int t = threadIdx.x;
  if (t < T) next[t] = best[t] == 0 ? 0 : unpack_argmax_index(best[t]);
}

// Single-sequence step through the many-token kernels with its token and
// position on the device, as the decode step reads them (contexts without the
// persistent step): token seq_tokens[pos] of sequence 0 at pos = ctrl->pos.
// A position outside the context sets error bit 1, a token outside the
// vocabulary bit 2; either then reads row 0 / position 0 so every later
// access stays in bounds.
__global__ void bt_from_ctrl_kernel(const int* __restrict__ ctrl_pos, const int* __restrict__ seq_tokens, int ctx,
                                    int vocab, int* __restrict__ meta, int meta_stride, int* err) {
  if (threadIdx.x != 0) return;
  int pos = *ctrl_pos;
  if (pos < 0 || pos >= ctx) {
    atomicOr(err, 1);
    pos = 0;
  }
  int tok = seq_tokens[pos];
  if (tok < 0 || tok >= vocab) {
    atomicOr(err, 2);
    tok = 0;
  }
  meta[0] = tok;
  meta[meta_stride] = pos;
  meta[2 * meta_stride] = 0;
}

// After that step: its logits become the context's, its greedy token goes to
// seq_tokens[ctx] and, past the caller's tokens, to the next position; the
// position advances (the decode step's epilogue, gemv.cuh's argmax).
__global__ void bt_to_ctrl_kernel(int* __restrict__ ctrl_pos, const int* __restrict__ fixed_until,
                                  int* __restrict__ seq_tokens, int ctx, const int* __restrict__ next,
                                  const float* __restrict__ row, float* __restrict__ logits, int vocab) {
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) logits[i] = row[i];
  if (threadIdx.x == 0) {
    const int tok = next[0];
    const int pos = *ctrl_pos;
    if (pos >= 0 && pos + 1 < ctx && pos + 1 >= *fixed_until) seq_tokens[pos + 1] = tok;
    seq_tokens[ctx] = tok;
    *ctrl_pos = pos + 1;
  }
}

// ---- sentence embedding (ss_scheduler_embed, layer_scheduler.c:805-915):
// every prompt token's final hidden state through the final RMSNorm, summed
// over the tokens in order, times 1/n, then L2-normalised.

// Final RMSNorm scale of each of T tokens, 1 / sqrtf(ss / d + eps) with ss
// summed sequentially in element order, products and sums rounded apart
// (ss_rmsnorm -> cpu_neon.c:109-115, as the reference's C compiles).  One
// thread per token: the sum is one dependent chain either way.
__global__ void bt_norm_scale_kernel(const float* __restrict__ h, int T, int d, float eps,
                                     float* __restrict__ scale) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float* x = h + (size_t)t * d;
  float ss = 0.0f;
  for (int i = 0; i < d; i++) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  scale[t] = 1.0f / sqrtf(__fdiv_rn(ss, (float)d) + eps);
}

// sum[j] += (h[t][j] * scale[t]) * w[j] for t = 0..T-1 in order (the
// embedding's running sum, layer_scheduler.c:888-894; w: output_norm).
__global__ void bt_pool_kernel(const float* __restrict__ h, const float* __restrict__ scale, int T, int d,
                               const float* __restrict__ w, float* __restrict__ sum) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d) return;
  float acc = sum[j];
  for (int t = 0; t < T; t++) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(h[(size_t)t * d + j], scale[t]), w[j]));
  sum[j] = acc;
}

// out = sum * (1 / n), then times 1 / (sqrtf(sum_j out_j^2) + 1e-12f), the
// squares summed sequentially in element order (layer_scheduler.c:896-910).
// One block; the scaled vector is staged in shared memory (d floats).
__global__ void bt_embed_finish_kernel(const float* __restrict__ sum, int d, int n, float* __restrict__ out) {
  extern __shared__ float e[];
  __shared__ float s_scale;
  const float inv = 1.0f / (float)n;
  for (int j = threadIdx.x; j < d; j += blockDim.x) e[j] = __fmul_rn(sum[j], inv);
  __syncthreads();
  if (threadIdx.x == 0) {
    float l2 = 0.0f;
    for (int j = 0; j < d; j++) l2 = __fadd_rn(l2, __fmul_rn(e[j], e[j]));
    s_scale = 1.0f / __fadd_rn(sqrtf(l2), 1e-12f);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += blockDim.x) out[j] = __fmul_rn(e[j], s_scale);
}

// Greedy feedback of a batched decode step, on the device: each sequence's
// greedy token becomes its next input at the next position, and is recorded
// at ids[(pos + 1) * stride + t] (positions up to ctx).
__global__ void bt_feed_kernel(int* __restrict__ meta, int meta_stride, int T, int* __restrict__ ids,
                               int stride, int ctx) {
  const int t = threadIdx.x;
  if (t >= T) return;
  const int next = meta[3 * meta_stride + t];
  const int pos = meta[meta_stride + t] + 1;
  if (pos <= ctx) ids[(size_t)pos * stride + t] = next;
  meta[t] = next;
  meta[meta_stride + t] = pos < ctx ? pos : ctx - 1;
}

}  // namespace ss
