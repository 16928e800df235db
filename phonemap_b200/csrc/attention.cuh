// attention.cuh -- GQA decode attention over the int8 ("TurboQuant") KV cache.
//
// Replaces SlipStream/src/core/layer_scheduler.c:408-468: encode this token's
// K and V rows to int8 with one symmetric scale over the whole kv_dim
// (kv_turboquant_encode, :101-118), then for every query head h (kv head
// h / (nh / nkv)):  s_t = (q . dec(K_t)) * (1/sqrt(hd)) for t <= pos, softmax
// (tensor.c:154-173), out_h = sum_t p_t * dec(V_t), with dec(x) = x * scale_t.
//
// Grid (nsplit, nkv) in clusters of (nsplit, 1): the nsplit CTAs of one kv
// head split the positions 0..pos between them (pos is read on the device, so
// one CUDA graph serves every position) and serve all query heads of its GQA
// group.  Each CTA streams its positions through shared memory in tiles
// (cp.async, 16 B per thread-copy), keeps an online softmax (running max m,
// sum l, o = sum exp(s - m) * dec(V)), and the cluster merges the partials
// through distributed shared memory -- no global scratch, no atomics.
//
// The cached rows (t < pos) and the position itself do not depend on this
// step's QKV kernel, so the first tile is requested before the programmatic-
// dependent-launch wait.  The CTA whose slice contains `pos` encodes this
// token's K/V slice of its kv head (scale from the |k| / |v| maxima the QKV
// GEMV accumulated), appends it to the cache and uses it from registers.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"

namespace ss {

struct AttnParams {
  const float* qkv;          // q [nh*hd] (roped) | k [kvd] (roped) | v [kvd]
  int8_t* kc;                // this layer's cache rows, head-major [nkv][ctx][hd]
  int8_t* vc;
  float* ks;                 // this layer's scales [ctx]
  float* vs;
  const unsigned int* amax_k;  // this layer's |k| maximum of the current position (one slot)
  const unsigned int* amax_v;
  const int* d_pos;
  float* out;                // [nh*hd]
  int nh, nkv, hd, ctx, nsplit;
  float scale;               // 1 / sqrtf(hd), computed on the host as the reference does
};

constexpr int kAttnTile = 64;     // positions per shared-memory tile
constexpr int kAttnMaxG = 8;      // query heads per kv head
constexpr int kAttnThreads = 128;

// Encode one value as kv_turboquant_encode does: (int8_t)roundf(v * inv).
SS_DEVINL int8_t kv_encode(float v, float inv) { return (int8_t)(int)roundf(__fmul_rn(v, inv)); }

SS_DEVINL void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gsrc)
               : "memory");
}
SS_DEVINL void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem_dst)), "l"(gsrc)
               : "memory");
}
SS_DEVINL void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared-memory layout of one CTA.
template <int HD>
struct AttnSmem {
  int8_t k[kAttnTile][HD];
  int8_t v[kAttnTile][HD];
  float ksc[kAttnTile];
  float vsc[kAttnTile];
  float s[kAttnMaxG][kAttnTile];   // scores -> exp weights
  float q[kAttnMaxG][HD];
  float o[kAttnMaxG][HD];          // running numerator
  float m[kAttnMaxG];              // running max
  float l[kAttnMaxG];              // running sum
  float corr[kAttnMaxG];
};

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
  namespace cg = cooperative_groups;
  constexpr int DPL = HD / 32;  // dims per lane
  extern __shared__ __align__(16) uint8_t smraw[];
  AttnSmem<HD>& sm = *reinterpret_cast<AttnSmem<HD>*>(smraw);
  cg::cluster_group cluster = cg::this_cluster();
  const int split = blockIdx.x, kh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nwarp = kAttnThreads / 32;
  const int g = p.nh / p.nkv, kvd = p.nkv * HD;

  const int pos = *p.d_pos;  // stable for the whole step (advanced by the lm_head)
  const bool pos_ok = pos >= 0 && pos < p.ctx;
  const int seq = pos_ok ? pos + 1 : 0;
  const int chunk = (seq + p.nsplit - 1) / p.nsplit;
  const int t0 = min(split * chunk, seq), t1 = min(t0 + chunk, seq);

  // Request the cached rows t in [a, b) (t != pos) of the tile starting at `a`.
  auto load_tile = [&](int a, int b) {
    const int rows = b - a;
    constexpr int cpr = HD / 16;  // 16-byte chunks per row
    for (int c = tid; c < rows * cpr; c += kAttnThreads) {
      const int r = c / cpr, j = c - r * cpr;
      const int t = a + r;
      if (t == pos) continue;
      const size_t off = ((size_t)kh * p.ctx + t) * HD + j * 16;  // head-major rows
      cp_async16(&sm.k[r][j * 16], p.kc + off);
      cp_async16(&sm.v[r][j * 16], p.vc + off);
    }
    for (int r = tid; r < rows; r += kAttnThreads) {
      const int t = a + r;
      if (t == pos) continue;
      cp_async4(&sm.ksc[r], p.ks + t);
      cp_async4(&sm.vsc[r], p.vs + t);
    }
  };

  if (t1 > t0) load_tile(t0, min(t0 + kAttnTile, t1));
  pdl_wait();

  // this step's q (all heads of the group) and the scales of row `pos`
  float k_scale = 0.0f, v_scale = 0.0f;
  if (pos_ok) {
    k_scale = __uint_as_float(*p.amax_k) / 127.0f;  // layer_scheduler.c:109-110
    v_scale = __uint_as_float(*p.amax_v) / 127.0f;
  }
  for (int idx = tid; idx < g * HD; idx += kAttnThreads) {
    const int h = idx / HD, i = idx - h * HD;
    sm.q[h][i] = p.qkv[(kh * g + h) * HD + i];
    sm.o[h][i] = 0.0f;
  }
  if (tid < kAttnMaxG) { sm.m[tid] = -INFINITY; sm.l[tid] = 0.0f; }
  if (pos_ok && pos >= t0 && pos < t1) {
    // encode + append this token's K/V slice (layer_scheduler.c:409-413)
    const float kinv = k_scale > 0.0f ? 1.0f / k_scale : 0.0f;
    const float vinv = v_scale > 0.0f ? 1.0f / v_scale : 0.0f;
    const float* kcur = p.qkv + p.nh * HD + kh * HD;
    const float* vcur = kcur + kvd;
    for (int i = tid; i < HD; i += kAttnThreads) {
      const int8_t kq = kv_encode(kcur[i], kinv), vq = kv_encode(vcur[i], vinv);
      p.kc[((size_t)kh * p.ctx + pos) * HD + i] = kq;
      p.vc[((size_t)kh * p.ctx + pos) * HD + i] = vq;
      if ((pos - t0) < kAttnTile) {
        sm.k[pos - t0][i] = kq;
        sm.v[pos - t0][i] = vq;
      }
    }
    if (tid == 0) {
      if (kh == 0) { p.ks[pos] = k_scale; p.vs[pos] = v_scale; }
      if ((pos - t0) < kAttnTile) { sm.ksc[pos - t0] = k_scale; sm.vsc[pos - t0] = v_scale; }
    }
  }
  pdl_trigger();

  for (int a = t0; a < t1; a += kAttnTile) {
    const int b = min(a + kAttnTile, t1), n = b - a;
    if (a != t0) {
      __syncthreads();  // previous tile fully consumed
      load_tile(a, b);
      if (pos >= a && pos < b && tid < HD) {
        // row `pos` of a later tile: re-encode from registers (same values)
        const float kinv = k_scale > 0.0f ? 1.0f / k_scale : 0.0f;
        const float vinv = v_scale > 0.0f ? 1.0f / v_scale : 0.0f;
        const float* kcur = p.qkv + p.nh * HD + kh * HD;
        for (int i = tid; i < HD; i += kAttnThreads) {
          sm.k[pos - a][i] = kv_encode(kcur[i], kinv);
          sm.v[pos - a][i] = kv_encode(kcur[kvd + i], vinv);
        }
        if (tid == 0) { sm.ksc[pos - a] = k_scale; sm.vsc[pos - a] = v_scale; }
      }
    }
    cp_async_wait_all();
    __syncthreads();

    // scores: warp per position, lane owns DPL dims (layer_scheduler.c:434-444)
    for (int r = warp; r < n; r += nwarp) {
      const float ksc = sm.ksc[r];
      float kd[DPL];
#pragma unroll
      for (int i = 0; i < DPL; i++) kd[i] = __fmul_rn((float)sm.k[r][lane * DPL + i], ksc);
#pragma unroll
      for (int h = 0; h < kAttnMaxG; h++) {
        if (h < g) {
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < DPL; i++) d = fmaf(sm.q[h][lane * DPL + i], kd[i], d);
          d = warp_sum(d);
          if (lane == 0) sm.s[h][r] = __fmul_rn(d, p.scale);
        }
      }
    }
    __syncthreads();
    // online softmax update, warp per head
    for (int h = warp; h < g; h += nwarp) {
      float mt = -INFINITY;
      for (int r = lane; r < n; r += 32) mt = fmaxf(mt, sm.s[h][r]);
      mt = warp_max(mt);
      const float mold = sm.m[h];
      const float mnew = fmaxf(mold, mt);
      float lt = 0.0f;
      for (int r = lane; r < n; r += 32) {
        const float e = expf(sm.s[h][r] - mnew);
        sm.s[h][r] = e;
        lt += e;
      }
      lt = warp_sum(lt);
      if (lane == 0) {
        const float c = mold == -INFINITY ? 0.0f : expf(mold - mnew);
        sm.corr[h] = c;
        sm.l[h] = fmaf(sm.l[h], c, lt);
        sm.m[h] = mnew;
      }
    }
    __syncthreads();
    // o = o * corr + sum_t e_t * dec(V_t): thread per (head, dim)
    for (int idx = tid; idx < g * HD; idx += kAttnThreads) {
      const int h = idx / HD, i = idx - h * HD;
      float o = sm.o[h][i] * sm.corr[h];
      for (int r = 0; r < n; r++) o = fmaf(sm.s[h][r], __fmul_rn((float)sm.v[r][i], sm.vsc[r]), o);
      sm.o[h][i] = o;
    }
  }
  cp_async_wait_all();

  // ---- merge the nsplit partials of this kv head through DSMEM
  cluster.sync();
  // CTA `split` of the cluster merges output elements split*128 + tid, strided
  // by the cluster's thread count.
  const int nr = (int)cluster.num_blocks();
  for (int idx = split * kAttnThreads + tid; idx < g * HD; idx += p.nsplit * kAttnThreads) {
    const int h = idx / HD, i = idx - h * HD;
    float M = -INFINITY;
    for (int r = 0; r < nr; r++) {
      const AttnSmem<HD>* rs = cluster.map_shared_rank(&sm, r);
      M = fmaxf(M, rs->m[h]);
    }
    float L = 0.0f, O = 0.0f;
    for (int r = 0; r < nr; r++) {
      const AttnSmem<HD>* rs = cluster.map_shared_rank(&sm, r);
      const float mr = rs->m[h];
      if (mr == -INFINITY) continue;
      const float f = expf(mr - M);
      L = fmaf(rs->l[h], f, L);
      O = fmaf(rs->o[h][i], f, O);
    }
    if (pos_ok) p.out[(kh * g + h) * HD + i] = O * (1.0f / L);
  }
  cluster.sync();  // keep every CTA's shared memory alive until all reads are done
}

}  // namespace ss
