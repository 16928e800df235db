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
#pragma once
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"

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
                                float* __restrict__ h, int* err) {
  const int t = blockIdx.y;
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
// s_j = (q . k_j) * k_scale_j * (1/sqrt(hd)), then a running softmax (max m,
// sum l, output o rescaled when m grows).  The slot's (m, l, o) go to `part`;
// bt_attn_merge_kernel combines the slots.  The result equals the
// reference's softmax-weighted sum of dec(V_j) up to fp32 rounding order.
constexpr int kBtAttnChunk = 128;   // positions per chunk
constexpr int kBtAttnSlots = 16;    // position slots (CTAs) per (kv head, token)
constexpr int kBtAttnMaxG = 8;      // query heads per kv head

__host__ __device__ constexpr size_t bt_attn_smem(int hd, int G) {
  // q[G][hd] | scores[G][chunk] | k scale, v scale [chunk] | m, l, corr [G]
  // | K chunk, V chunk [chunk][hd] int8
  return (size_t)(G * hd + G * kBtAttnChunk + 2 * kBtAttnChunk + 4 * kBtAttnMaxG) * sizeof(float) +
         (size_t)2 * kBtAttnChunk * hd;
}

// part layout: [T][nh][slots][hd + 2]: m, l, then o[hd].
__global__ void __launch_bounds__(256) bt_attn_kernel(const float* __restrict__ q, BatchTokens bt, BatchKv kv,
                                                      int layer, int nh, int nkv, int hd, float scale,
                                                      float* __restrict__ part) {
  extern __shared__ float sm[];
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
  const int tid = threadIdx.x, nt = blockDim.x;
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
  // output elements of this thread: element e of heads hb, hb + hs, ...
  const int e = tid % hd, hb = tid / hd, hs = nt / hd;  // hd divides 256 (hd <= 256, power of two)
  float o[kBtAttnMaxG];
#pragma unroll
  for (int i = 0; i < kBtAttnMaxG; i++) o[i] = 0.0f;
  const int vec = hd / 16;
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
    // scores of (head, position) pairs
    for (int idx = tid; idx < G * cn; idx += nt) {
      const int h = idx / cn, j = idx - h * cn;
      const float* qh = qs + h * hd;
      const int8_t* kr = sk + j * hd;
      float dot = 0.0f;
      for (int i = 0; i < hd; i += 16) {
        const int4 kw = *reinterpret_cast<const int4*>(kr + i);
        const int8_t* kb = reinterpret_cast<const int8_t*>(&kw);
#pragma unroll
        for (int u = 0; u < 16; u++) dot = fmaf(qh[i + u], (float)kb[u], dot);
      }
      sc[h * kBtAttnChunk + j] = dot * sks[j] * scale;
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
    // o = o * corr + sum_j w_j v_j
#pragma unroll
    for (int i = 0; i < kBtAttnMaxG; i++) {
      const int h = hb + i * hs;
      if (h < G) o[i] *= sml[2 * kBtAttnMaxG + h];
    }
    for (int j = 0; j < cn; j++) {
      const float v = (float)sv[j * hd + e];
#pragma unroll
      for (int i = 0; i < kBtAttnMaxG; i++) {
        const int h = hb + i * hs;
        if (h < G) o[i] = fmaf(sc[h * kBtAttnChunk + j], v, o[i]);
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kBtAttnMaxG; i++) {
    const int h = hb + i * hs;
    if (h < G) {
      float* pp = part + (((size_t)t * nh + (size_t)kvh * G + h) * kBtAttnSlots + slot) * (hd + 2);
      if (e == 0) {
        pp[0] = sml[h];
        pp[1] = sml[kBtAttnMaxG + h];
      }
      pp[2 + e] = o[i];
    }
  }
}

// out[t][h][:] = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s over the
// slots that held positions (M = max m_s).
__global__ void bt_attn_merge_kernel(const float* __restrict__ part, BatchTokens bt, int nh, int hd,
                                     float* __restrict__ out) {
  const int h = blockIdx.x, t = blockIdx.y, e = threadIdx.x;
  const int pos = bt.pos[t];
  const int ns = min(kBtAttnSlots, pos / kBtAttnChunk + 1);
  const float* pp = part + ((size_t)t * nh + h) * kBtAttnSlots * (hd + 2);
  float M = -INFINITY;
  for (int s = 0; s < ns; s++) M = fmaxf(M, pp[(size_t)s * (hd + 2)]);
  float L = 0.0f, acc = 0.0f;
  for (int s = 0; s < ns; s++) {
    const float* ps = pp + (size_t)s * (hd + 2);
    const float f = expf(ps[0] - M);
    L = fmaf(ps[1], f, L);
    if (e < hd) acc = fmaf(ps[2 + e], f, acc);
  }
  if (e < hd) out[(size_t)t * nh * hd + (size_t)h * hd + e] = acc / L;
}

// h[t][r] += the product (layer_scheduler.c:484, :566).
__global__ void bt_residual_kernel(const float* __restrict__ part, int nsplit, int T, int rows,
                                   float* __restrict__ h) {
  const size_t n = (size_t)T * rows;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    h[i] = __fadd_rn(split_sum(part, nsplit, n, i), h[i]);
}

// act[t][j] = up * (g / (1 + expf(-g))) (layer_scheduler.c:533-549); the
// gate/up matrix interleaves gate (even rows) and up (odd rows).
__global__ void bt_swiglu_kernel(const float* __restrict__ part, int nsplit, int T, int ff,
                                 float* __restrict__ act) {
  const size_t n = (size_t)T * 2 * ff, m = (size_t)T * ff;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < m; i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / ff, j = i - t * ff;
    const float g = split_sum(part, nsplit, n, t * 2 * ff + 2 * j);
    const float u = split_sum(part, nsplit, n, t * 2 * ff + 2 * j + 1);
    act[i] = __fmul_rn(u, __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
  }
}

// Logits of token t (the product's split sums) and the packed (value,
// index) maximum (pack_argmax: ss_argmax's rule, tensor.c:318-328) into
// best[t] by atomicMax -- order-independent, so deterministic.
__global__ void bt_head_kernel(const float* __restrict__ part, int nsplit, int T, int vocab,
                               float* __restrict__ logits, unsigned long long* __restrict__ best) {
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
