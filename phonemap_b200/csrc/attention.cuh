// attention.cuh -- GQA decode attention over the int8 ("TurboQuant") KV cache.
//
// Replaces SlipStream/src/core/layer_scheduler.c:408-468: encode this token's
// K and V rows to int8 with one symmetric scale over the whole kv_dim
// (kv_turboquant_encode, :101-118), then for every query head h (kv head
// h / (nh / nkv)):  s_t = (q . dec(K_t)) * (1/sqrt(hd)) for t <= pos, softmax
// (tensor.c:154-173), out_h = sum_t p_t * dec(V_t), with dec(x) = x * scale_t.
//
// Grid (nsplit, nkv): a CTA handles one kv head and a contiguous slice of the
// positions 0..pos (pos is read on the device, so one CUDA graph serves every
// position) for all query heads of its GQA group.  It writes an unnormalised
// partial (running max m, sum l, o = sum exp(s - m) * v); the last CTA of the
// kv head to finish merges the partials (the standard split-softmax merge) and
// writes the heads' outputs.  The CTA whose slice contains `pos` also encodes
// and appends this token's K/V slice of its kv head -- the scale comes from the
// |k| / |v| maxima the QKV GEMV accumulated, so every CTA derives the same
// scale without another pass.
#pragma once
#include "common.cuh"

namespace ss {

struct AttnParams {
  const float* qkv;          // q [nh*hd] (roped) | k [kvd] (roped) | v [kvd]
  int8_t* kc;                // this layer's cache rows [ctx][kvd]
  int8_t* vc;
  float* ks;                 // this layer's scales [ctx]
  float* vs;
  const unsigned int* amax_k;  // this layer's |k| maxima [ctx]
  const unsigned int* amax_v;
  const int* d_pos;
  float* part_o;             // [nkv][nsplit][g][hd]
  float* part_ml;            // [nkv][nsplit][g][2]
  unsigned int* counters;    // [nkv]
  float* out;                // [nh*hd]
  int nh, nkv, hd, ctx, nsplit, chunk_max;
  float scale;               // 1 / sqrtf(hd), computed on the host as the reference does
};

// Encode one value as kv_turboquant_encode does: (int8_t)roundf(v * inv).
SS_DEVINL int8_t kv_encode(float v, float inv) { return (int8_t)(int)roundf(__fmul_rn(v, inv)); }

template <int DPL>  // dims per lane = hd / 32
__global__ void __launch_bounds__(128) attention_kernel(const AttnParams p) {
  extern __shared__ float sm[];
  const int split = blockIdx.x, kh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;
  const int g = p.nh / p.nkv, hd = p.hd, kvd = p.nkv * hd;
  float* s_sc = sm;                          // [g][chunk_max] scores -> probabilities
  float* s_red = sm + g * p.chunk_max;       // 64 floats
  __shared__ bool is_last;

  pdl_wait();
  const int pos = *p.d_pos;
  if (pos < 0 || pos >= p.ctx) return;  // host bounds positions; never index past the cache
  const int seq = pos + 1;
  const int chunk = (seq + p.nsplit - 1) / p.nsplit;
  const int t0 = min(split * chunk, seq), t1 = min(t0 + chunk, seq);
  const int n = t1 - t0;

  // scales of this token's rows (layer_scheduler.c:109-114)
  const float k_scale = __uint_as_float(p.amax_k[pos]) / 127.0f;
  const float v_scale = __uint_as_float(p.amax_v[pos]) / 127.0f;
  const float* qv = p.qkv;
  const float* kcur = p.qkv + p.nh * hd + kh * hd;
  const float* vcur = p.qkv + p.nh * hd + kvd + kh * hd;

  if (pos >= t0 && pos < t1) {
    const float kinv = k_scale > 0.0f ? 1.0f / k_scale : 0.0f;
    const float vinv = v_scale > 0.0f ? 1.0f / v_scale : 0.0f;
    for (int i = tid; i < hd; i += blockDim.x) {
      p.kc[(size_t)pos * kvd + kh * hd + i] = kv_encode(kcur[i], kinv);
      p.vc[(size_t)pos * kvd + kh * hd + i] = kv_encode(vcur[i], vinv);
    }
    if (kh == 0 && tid == 0) { p.ks[pos] = k_scale; p.vs[pos] = v_scale; }
    __syncthreads();
  }
  pdl_trigger();

  // ---- scores: warp per position, lane owns DPL dims
  float qr[8][DPL];
#pragma unroll
  for (int h = 0; h < 8; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++)
      qr[h][i] = h < g ? qv[(kh * g + h) * hd + lane * DPL + i] : 0.0f;

  for (int t = t0 + warp; t < t1; t += nwarp) {
    const int8_t* krow = p.kc + (size_t)t * kvd + kh * hd + lane * DPL;
    const float ksc = (t == pos) ? k_scale : p.ks[t];
    float kd[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) kd[i] = __fmul_rn((float)krow[i], ksc);
#pragma unroll
    for (int h = 0; h < 8; h++) {
      if (h < g) {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; i++) d = fmaf(qr[h][i], kd[i], d);
        d = warp_sum(d);
        if (lane == 0) s_sc[h * p.chunk_max + (t - t0)] = __fmul_rn(d, p.scale);
      }
    }
  }
  __syncthreads();

  // ---- per-head max / exp / sum over this slice (warp per head)
  for (int h = warp; h < g; h += nwarp) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, s_sc[h * p.chunk_max + i]);
    m = warp_max(m);
    float l = 0.0f;
    for (int i = lane; i < n; i += 32) {
      const float e = expf(s_sc[h * p.chunk_max + i] - m);
      s_sc[h * p.chunk_max + i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      float* ml = p.part_ml + (((size_t)kh * p.nsplit + split) * g + h) * 2;
      ml[0] = n > 0 ? m : -INFINITY;
      ml[1] = l;
    }
  }
  __syncthreads();

  // ---- o = sum_t e_t * dec(V_t): thread per (head, dim)
  for (int idx = tid; idx < g * hd; idx += blockDim.x) {
    const int h = idx / hd, i = idx - h * hd;
    float o = 0.0f;
    for (int t = t0; t < t1; t++) {
      const float vsc = (t == pos) ? v_scale : p.vs[t];
      const float vd = __fmul_rn((float)p.vc[(size_t)t * kvd + kh * hd + i], vsc);
      o = fmaf(s_sc[h * p.chunk_max + (t - t0)], vd, o);
    }
    p.part_o[(((size_t)kh * p.nsplit + split) * g + h) * hd + i] = o;
  }

  // ---- last CTA of this kv head merges the splits
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(p.counters + kh, 1u) == (unsigned)p.nsplit - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int idx = tid; idx < g * hd; idx += blockDim.x) {
    const int h = idx / hd, i = idx - h * hd;
    const volatile float* ml = p.part_ml + ((size_t)kh * p.nsplit * g + h) * 2;
    float M = -INFINITY;
    for (int s = 0; s < p.nsplit; s++) M = fmaxf(M, ml[(size_t)s * g * 2]);
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < p.nsplit; s++) {
      const float ms = ml[(size_t)s * g * 2];
      if (ms == -INFINITY) continue;
      const float f = expf(ms - M);
      L = fmaf(ml[(size_t)s * g * 2 + 1], f, L);
      O = fmaf(*((volatile float*)p.part_o + (((size_t)kh * p.nsplit + s) * g + h) * hd + i), f, O);
    }
    p.out[(kh * g + h) * hd + i] = O * (1.0f / L);
  }
  if (tid == 0) p.counters[kh] = 0;
  (void)s_red;
}

}  // namespace ss
