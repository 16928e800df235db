// qgemm.cuh -- many-token dequantize-and-multiply for Q4_0 / Q8_0 weights on
// the sm_100a tensor cores (tcgen05, TMEM accumulators, TMA weight tiles).
//
// Serves the paths where one pass over the weights is shared by several
// tokens: the prompt (ss_scheduler_prefill, SlipStream/src/core/
// layer_scheduler.c:681-803, which the reference runs token by token) and
// several sequences decoded together.  For T tokens x_t it computes, for every
// weight row r,
//     y[t][r] = sum_b d[r][b] * sum_{j < 32} w[r][32 b + j] * x_t[32 b + j]
// with w = q - 8 (Q4_0) or q (Q8_0) and d the block's fp16 scale widened to
// fp32 -- the reference's dequant-matvec (SlipStream/src/core/quantize.c:
// 446-494) for each token, in another summation order.
//
// Numerics (the same as the batch-1 kernels, gemv.cuh): each token's 32-value
// block is block fixed point -- m_j = round(x_j 2^(22-e)), 2^e > max |x| --
// split into three signed byte planes (qplanes_kernel).  A block's weights
// and planes meet in one integer tensor-core product per plane, exact in
// int32; the planes are combined in fp32 and scaled by d * 2^(e-22).
//
// Tensor-core mapping (one CTA tile = 128 weight rows):
//   A (M = 128 rows x K = 32): the block's weights as int8 -- Q4_0 nibbles
//       unpacked to 16 (q - 8) (exact; the 1/16 joins the scale), Q8_0 bytes
//       as they are -- written by the math warps into shared memory in the
//       UMMA canonical K-major layout (8-row x 16-byte core matrices);
//   B (N = 3 TP x K = 32): the block's activation planes, row p * TP + t for
//       plane p of token t (TP = T rounded up to 16; padding rows zero),
//       already in the canonical layout in global memory (qplanes_kernel);
//   D (128 lanes x N columns of TMEM, int32): one tcgen05.mma per block, two
//       TMEM buffers so block b's product runs while block b-1 is flushed.
// Weights arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle, no
// multicast) into a ring of stages of KC blocks x 128 rows, with the planes
// of those blocks (cp.async.bulk) and the fp16 scales.
//
// Work: units of (128-row tile, contiguous range of K chunks); a unit's
// partial sums go to out[split][t][r] and the consumer of the product adds
// the splits in order.  A persistent grid walks the units.
#pragma once
#include <cuda.h>  // CUtensorMap (the type only; maps are encoded on the host)

#include "common.cuh"
#include "gemv.cuh"

namespace ss {

constexpr int kQgRows = 128;        // weight rows per tile (UMMA M)
constexpr int kQgMaxT = 32;         // tokens per product (N = 3 * 32 = 96 at most)
constexpr int kQgStages = 4;        // ring stages
constexpr int kQgMathWarps = 8;     // two warpgroups: each covers all 128 TMEM lanes
constexpr int kQgThreads = 32 * (1 + kQgMathWarps);
constexpr int kQgTmemCols = 256;    // two D buffers of up to 96 columns (power of two >= 192)
constexpr int kQgABytes = kQgRows * 32;  // one block of A in the canonical layout

// Blocks per stage: the TMA box's inner extent is 128 bytes (the 128-byte
// swizzle span): 8 Q4_0 blocks of 16 quant bytes, 4 Q8_0 blocks of 32.
__host__ __device__ constexpr int qg_kc(int type) { return type == kQ4_0 ? 8 : 4; }

struct QGemmParams {
  int rows, nb, type;
  int tiled;            // 1: tiled weight layout (4-row tiles), 0: row-interleaved
  int T, TP;            // tokens; plane stride in the N dimension (T rounded up to 16)
  const int8_t* xq;     // [nb][3 TP][32] planes, canonical K-major per block
  const float* xc;      // [T][nb]: 2^(e-22), the value of one unit of plane 0
  float* out;           // [nsplit][T][rows] partial products
  int nsplit;           // K ranges per row tile
  int nchunks;          // nb / KC
  int ntile;            // row tiles
  int* err;
  long long wait_budget;
};

// Shared memory: [stages][quants 16 KB | scales 2 KB | planes KC*N*32]
// [A x 2][mbarriers][tmem address].
struct QgSmem {
  static constexpr int kQuant = 16384;   // 128 rows x 128 bytes
  static constexpr int kScale = 2048;    // 128 rows x KC (<= 8) fp16
  __host__ __device__ static int plane_bytes(int type, int TP) { return qg_kc(type) * 3 * TP * 32; }
  __host__ __device__ static int stage_bytes(int type, int TP) {
    return (kQuant + kScale + plane_bytes(type, TP) + 1023) / 1024 * 1024;
  }
  __host__ __device__ static int total(int type, int TP) {
    return 1024 /* alignment slack */ + kQgStages * stage_bytes(type, TP) + 2 * kQgABytes + 256;
  }
};

// ---- tcgen05 / TMA primitives (inline PTX) --------------------------------

SS_DEVINL void tma_load_3d(uint32_t dst, const void* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
SS_DEVINL void tma_load_2d(uint32_t dst, const void* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
SS_DEVINL void tmem_alloc(uint32_t dst_smem, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
SS_DEVINL void tmem_dealloc(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
SS_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SS_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy writes to shared memory (the unpacked A) made visible to the
// tensor core (async proxy).
SS_DEVINL void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8, one CTA.
SS_DEVINL void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// Arrives once on `bar` when every tcgen05 operation this thread issued before
// it has completed (the MMA's shared-memory reads included).
SS_DEVINL void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
// 16 consecutive 32-bit TMEM columns of this thread's lane.
SS_DEVINL void tmem_ld16(uint32_t taddr, int (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
        "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
SS_DEVINL void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand without swizzle:
// 8-row x 16-byte core matrices, the two 16-byte halves of K 128 bytes apart
// (leading byte offset), 8-row groups 256 bytes apart (stride byte offset);
// version 1 (sm_100).
SS_DEVINL uint64_t umma_desc_kmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         (1ull << 46);
}
// Instruction descriptor of kind::i8: D s32, A and B s8, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Exact int -> float for |v| < 2^22 (integer add + float add on the FMA
// pipes instead of the conversion unit).
SS_DEVINL float i2f_small(int v) {
  return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

// Wait on an mbarrier phase with a budget; false on expiry (error bit 4).
SS_DEVINL bool qg_wait(uint32_t bar, uint32_t parity, const QGemmParams& p) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > p.wait_budget) {
      atomicOr(p.err, 4);
      return false;
    }
  }
  return true;
}

// ---- activation planes -----------------------------------------------------

// Per-token RMSNorm scale (cpu_neon.c:109-115): 1 / sqrtf(sum x^2 / n + eps).
__global__ void __launch_bounds__(256) qg_rms_kernel(const float* __restrict__ x, int n, int ld, float eps,
                                                     float* __restrict__ scale) {
  __shared__ float red[32];
  const float* xt = x + (size_t)blockIdx.x * ld;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xt[i], xt[i], ss);
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) scale[blockIdx.x] = 1.0f / sqrtf(ss / (float)n + eps);
}

// Block fixed point of token t's block b into B's canonical layout: one warp
// per (token, block), lane j = element j.  With norm_w: x * scale[t] * w (the
// reference's rounding order).  Tokens in [T, TP) write zero planes.
__global__ void __launch_bounds__(256) qg_planes_kernel(const float* __restrict__ x, int ld, int nb,
                                                        const float* __restrict__ norm_w,
                                                        const float* __restrict__ scale, int T, int TP,
                                                        int8_t* __restrict__ xq, float* __restrict__ xc) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int t = blockIdx.y;
  if (b >= nb) return;
  float v = 0.0f;
  if (t < T) {
    v = x[(size_t)t * ld + b * 32 + lane];
    if (norm_w) v = __fmul_rn(__fmul_rn(v, scale[t]), norm_w[b * 32 + lane]);
  }
  const float amax = warp_max(fabsf(v));
  const bool live = amax >= 1e-30f;
  const int e = (int)((__float_as_uint(amax) >> 23) & 255u) - 126;
  const int m = live ? __float2int_rn(v * pow2i(22 - e)) : 0;
  const int d0 = sext8(m);
  const int m1 = (m - d0) >> 8;
  const int d1 = sext8(m1);
  const int d2 = (m1 - d1) >> 8;
  const int N = 3 * TP;
  int8_t* blk = xq + (size_t)b * N * 32;
  const int dig[3] = {d0, d1, d2};
#pragma unroll
  for (int pl = 0; pl < 3; pl++) {
    const int n = pl * TP + t;
    blk[(n >> 3) * 256 + (lane >> 4) * 128 + (n & 7) * 16 + (lane & 15)] = (int8_t)dig[pl];
  }
  if (lane == 0 && t < T) xc[(size_t)t * nb + b] = live ? pow2i(e - 22) : 0.0f;
}

// ---- the product -----------------------------------------------------------

// out[t][r] = sum over splits of part[s][t][r], in split order.
__global__ void qg_sum_kernel(const float* __restrict__ part, int nsplit, int T, int rows, float* __restrict__ out) {
  const int n = T * rows;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float v = part[i];
    for (int s2 = 1; s2 < nsplit; s2++) v += part[(size_t)s2 * n + i];
    out[i] = v;
  }
}

// The two tensor maps of one weight matrix (host-encoded).
struct QgMaps {
  CUtensorMap q, s;
};

// Unit u -> (row tile, chunk range).
SS_DEVINL void qg_unit(const QGemmParams& p, int u, int& tile, int& split, int& c0, int& c1) {
  tile = u / p.nsplit;
  split = u - tile * p.nsplit;
  c0 = (int)((long long)p.nchunks * split / p.nsplit);
  c1 = (int)((long long)p.nchunks * (split + 1) / p.nsplit);
}

SS_DEVINL bool qg_any(bool pred) {  // barrier over the 256 math threads that ORs a predicate
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n"
      " barrier.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(32 * kQgMathWarps)
      : "memory");
  return r != 0;
}

// Warp 0 (one lane) feeds the ring; warps 1..8 unpack A, issue the MMAs (one
// thread) and flush D: warp w owns TMEM lanes 32 (w % 4) .. +31 (weight rows),
// warpgroup g = (w - 1) / 4 the tokens 16 g .. 16 g + 15 of each row.
template <int TYPE>
__global__ void __launch_bounds__(kQgThreads, 1)
    qgemm_kernel(const QGemmParams p, const __grid_constant__ CUtensorMap qmap,
                 const __grid_constant__ CUtensorMap smap) {
  constexpr int KC = qg_kc(TYPE);
  extern __shared__ uint8_t qg_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qg_raw) + 1023) & ~(uintptr_t)1023);
  const int N = 3 * p.TP;
  const int SB = QgSmem::stage_bytes(TYPE, p.TP);
  const int PB = QgSmem::plane_bytes(TYPE, p.TP);
  uint8_t* abuf = smem + kQgStages * SB;                           // 2 x 4 KB, 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(abuf + 2 * kQgABytes);
  uint64_t* empty = full + kQgStages;
  uint64_t* dfull = empty + kQgStages;                             // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 2);
  __shared__ int s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nunits = p.ntile * p.nsplit;
  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < kQgStages; i++) {
      mbar_init(smem_addr(full + i), 1);
      mbar_init(smem_addr(empty + i), kQgMathWarps);
    }
    mbar_init(smem_addr(dfull), 1);
    mbar_init(smem_addr(dfull + 1), 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), kQgTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      const uint32_t tx = (uint32_t)(QgSmem::kQuant + KC * 8 * 32 + PB);
      int sc = 0;
      bool bad = false;
      for (int u = blockIdx.x; u < nunits && !bad; u += gridDim.x) {
        int tile, split, c0, c1;
        qg_unit(p, u, tile, split, c0, c1);
        for (int c = c0; c < c1; c++, sc++) {
          const int s = sc % kQgStages;
          if (sc >= kQgStages) {
            const uint32_t par = (uint32_t)(((sc / kQgStages) - 1) & 1);
            if (!mbar_try_wait(smem_addr(empty + s), par)) {
              const long long t0 = clock64();
              while (!mbar_try_wait(smem_addr(empty + s), par)) {
                if (*(volatile int*)&s_abort || clock64() - t0 > p.wait_budget) { bad = true; break; }
              }
              if (bad) break;
            }
          }
          uint8_t* st = smem + s * SB;
          const uint32_t fb = smem_addr(full + s);
          mbar_expect_tx(fb, tx);
          tma_load_3d(smem_addr(st), &qmap, c * KC * (TYPE == kQ4_0 ? 16 : 32), 0, 32 * tile, fb);
          tma_load_2d(smem_addr(st + QgSmem::kQuant), &smap, c * KC * 8, 32 * tile, fb);
          bulk_g2s(smem_addr(st + QgSmem::kQuant + QgSmem::kScale), p.xq + (size_t)c * KC * N * 32,
                   (uint32_t)PB, fb);
        }
      }
      // drain: the copies of the last stages may still be landing
      for (int g = max(0, sc - kQgStages); g < sc; g++)
        mbar_wait_bounded(smem_addr(full + g % kQgStages), (uint32_t)((g / kQgStages) & 1), p.wait_budget);
    }
    return;
  }

  // ---------------- math warps
  const int q = warp & 3;                 // TMEM lane quadrant of this warp
  const int r = 32 * q + lane;            // weight row within the tile
  const int g = (warp - 1) >> 2;          // warpgroup: token half
  const bool flusher = 16 * g < p.TP;
  const uint32_t idesc = umma_idesc_i8(kQgRows, N);
  const uint32_t t_lane = tmem + ((uint32_t)(32 * q) << 16);
  const bool issuer = tid == 32;
  float acc[16];
  int it = 0;        // blocks issued by this CTA so far (all units)
  int sc = 0;        // stages consumed
  bool bad = false;
  // pending block (issued, not yet flushed)
  int pend_it = -1, pend_stage = 0, pend_bl = 0, pend_b = 0;
  bool pend_last_of_stage = false;

  auto flush_pending = [&]() -> bool {
    // wait for the MMA of block pend_it; read its D; scale and accumulate
    const uint32_t db = (uint32_t)(pend_it & 1);
    if (!qg_wait(smem_addr(dfull + db), (uint32_t)((pend_it >> 1) & 1), p)) return false;
    tc_fence_after();
    if (flusher) {
      int v0[16], v1[16], v2[16];
      const uint32_t col = t_lane + db * 128 + 16 * g;
      tmem_ld16(col, v0);
      tmem_ld16(col + p.TP, v1);
      tmem_ld16(col + 2 * p.TP, v2);
      tmem_ld_wait();
      const uint8_t* sst = smem + pend_stage * SB + QgSmem::kQuant;
      const uint16_t dh = *reinterpret_cast<const uint16_t*>(sst + (((r >> 2) * KC + pend_bl) * 4 + (r & 3)) * 2);
      float d = half_bits_to_float(dh);
      if (TYPE == kQ4_0) d *= 0.0625f;  // A held 16 (q - 8)
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int t = 16 * g + i;
        if (t < p.T) {
          const float cx = __ldg(p.xc + (size_t)t * p.nb + pend_b);
          const float v = fmaf(i2f_small(v2[i]), 65536.0f, fmaf(i2f_small(v1[i]), 256.0f, i2f_small(v0[i])));
          acc[i] = fmaf(v, d * cx, acc[i]);
        }
      }
    }
    tc_fence_before();
    if (pend_last_of_stage) {
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(empty + pend_stage));
    }
    pend_it = -1;
    return true;
  };

  for (int u = blockIdx.x; u < nunits && !bad; u += gridDim.x) {
    int tile, split, c0, c1;
    qg_unit(p, u, tile, split, c0, c1);
#pragma unroll
    for (int i = 0; i < 16; i++) acc[i] = 0.0f;
    for (int c = c0; c < c1 && !bad; c++, sc++) {
      const int s = sc % kQgStages;
      bool ok = qg_wait(smem_addr(full + s), (uint32_t)((sc / kQgStages) & 1), p);
      uint8_t* st = smem + s * SB;
      const uint32_t qbase = smem_addr(st);
      for (int bl = 0; bl < KC; bl++, it++) {
        // unpack block bl of the stage into A[it & 1] (canonical K-major)
        const uint32_t a = smem_addr(abuf + (it & 1) * kQgABytes) + (uint32_t)((r >> 3) * 256 + (r & 7) * 16);
        if (ok) {
          if constexpr (TYPE == kQ4_0) {
            uint32_t w0, w1;
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];"
                         : "=r"(w0), "=r"(w1)
                         : "r"(qbase + r * 128 + ((bl ^ (r & 7)) << 4) + 8 * g));
            const uint32_t l0 = ((w0 << 4) & 0xF0F0F0F0u) ^ 0x80808080u, l1 = ((w1 << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
            const uint32_t h0 = (w0 & 0xF0F0F0F0u) ^ 0x80808080u, h1 = (w1 & 0xF0F0F0F0u) ^ 0x80808080u;
            asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(a + 8 * g), "r"(l0), "r"(l1) : "memory");
            asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(a + 128 + 8 * g), "r"(h0), "r"(h1) : "memory");
          } else {
            uint32_t w[4];
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                         : "r"(qbase + r * 128 + (((2 * bl + g) ^ (r & 7)) << 4)));
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a + 128 * g), "r"(w[0]), "r"(w[1]),
                         "r"(w[2]), "r"(w[3])
                         : "memory");
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        bad = qg_any(!ok);  // every math thread has written its part of A
        tc_fence_after();
        if (bad) break;
        if (issuer) {
          const uint64_t adesc = umma_desc_kmajor(smem_addr(abuf + (it & 1) * kQgABytes));
          const uint64_t bdesc =
              umma_desc_kmajor(smem_addr(st + QgSmem::kQuant + QgSmem::kScale + bl * N * 32));
          umma_i8(tmem + (uint32_t)((it & 1) * 128), adesc, bdesc, idesc, 0u);
          umma_commit(smem_addr(dfull + (it & 1)));
        }
        if (pend_it >= 0) ok = flush_pending();
        pend_it = it;
        pend_stage = s;
        pend_bl = bl;
        pend_b = c * KC + bl;
        pend_last_of_stage = bl == KC - 1;
      }
    }
    if (bad) break;
    // the unit's last block, then its partial sums
    const bool ok = flush_pending();
    bad = qg_any(!ok);
    if (bad) break;
    if (flusher) {
      const int row = tile * kQgRows + r;
      if (row < p.rows) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int t = 16 * g + i;
          if (t < p.T) p.out[((size_t)split * p.T + t) * p.rows + row] = acc[i];
        }
      }
    }
  }
  if (bad) {
    if (tid == 32) {
      s_abort = 1;
      // no MMA may still write TMEM when it is freed
      if (pend_it >= 0)
        mbar_wait_bounded(smem_addr(dfull + (pend_it & 1)), (uint32_t)((pend_it >> 1) & 1), p.wait_budget);
    }
  }
  tc_fence_before();
  named_bar_sync(1, 32 * kQgMathWarps);
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kQgTmemCols);
}

}  // namespace ss
