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
// Numerics.  The weights enter the tensor core exactly: Q4_0 values q - 8
// and Q8_0 values q are small integers, exact in fp16.  Each token's input
// vector (RMSNormed in the reference's rounding order where the layer has a
// norm) is scaled by a power of two so its largest element lies in [1, 2) and
// split into two fp16 pieces, hi = fp16(x) and lo = fp16(x - hi) -- 22 bits of
// the fp32 value.  One block's dot products are then tensor-core products
// with fp32 accumulation (both pieces into the same accumulator); each block's
// result is scaled by its fp16 scale d in fp32 and summed over the blocks, and
// the token's power of two is undone at the end.
//
// Tensor-core mapping (one CTA tile = 128 weight rows):
//   A (M = 128 rows x K = 32 per block): the block's weights as fp16, written
//       by the math warps into tensor memory with tcgen05.st (row r in lane r,
//       two consecutive K elements per 32-bit column: 16 columns per block),
//       so the unpacked weights never pass through shared memory;
//   B (N = 2 TP x K = 32): the block's activation pieces, rows 0..TP-1 the
//       hi pieces of tokens 0..TP-1 and rows TP..2TP-1 their lo pieces (TP =
//       T rounded up to 8, 16 or 32; padding rows zero), already in the
//       canonical layout in global memory (bt_prep_kernel);
//   D (128 lanes x 2 TP columns of TMEM per block, fp32): two tcgen05.mma
//       kind::f16 per block (the two K halves of 16); column t holds token
//       t's hi product, column TP + t its lo product, added at the flush.
// A group (qg_group(TP) blocks) is the unit of work of the math warps: they
// unpack its blocks into one of two TMEM A buffers, one elected lane issues
// its MMAs into one of two TMEM D regions, and while those run the warps flush
// the previous group's region and unpack the next group.
// Weights arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle, no
// multicast) into a ring of stages of KC blocks x 128 rows (one or two
// groups), with the pieces of those blocks (cp.async.bulk) and the fp16
// scales.
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
constexpr int kQgMaxT = 32;         // tokens per product (N = 2 * 32 = 64 at most)
constexpr int kQgStages = 4;        // ring stages
constexpr int kQgUnpackWarps = 16;  // four warpgroups: each covers all 128 TMEM lanes
constexpr int kQgFlushWarps = 8;    // two per TMEM lane quadrant (each half of the tokens)
constexpr int kQgThreads = 32 * (2 + kQgUnpackWarps + kQgFlushWarps);  // + producer, MMA issuer
constexpr int kQgACols = 16;        // TMEM columns of one block of A (128 rows x 32 fp16)
constexpr int kQgTmemCols = 512;    // D regions, then A buffers

// Token rows per piece: T rounded up to 8, 16 or 32.
__host__ __device__ constexpr int qg_tp(int T) { return T <= 8 ? 8 : T <= 16 ? 16 : 32; }
// Blocks per MMA group (one A buffer, one D region): two D regions of
// G x 2 TP columns and two A buffers of G x 16 columns fit the 512 TMEM columns.
__host__ __device__ constexpr int qg_group(int TP) { return TP == 32 ? 2 : 4; }

// Blocks per stage: the TMA box's inner extent is 128 bytes (the 128-byte
// swizzle span): 8 Q4_0 blocks of 16 quant bytes, 4 Q8_0 blocks of 32.
__host__ __device__ constexpr int qg_kc(int type) { return type == kQ4_0 ? 8 : 4; }

struct QGemmParams {
  int rows, nb, type;
  int tiled;            // 1: tiled weight layout (4-row tiles), 0: row-interleaved
  int T, TP;            // tokens; B rows per piece (qg_tp(T))
  const __half* xq;     // [nb][2 pieces][TP][32] activation pieces, canonical K-major per block
  const float* post;    // [T]: the power of two each token's result is multiplied by
  float* out;           // [nsplit][T][rows] partial products
  int nsplit;           // K ranges per row tile
  int nchunks;          // nb / KC
  int ntile;            // row tiles
  int* err;
  long long wait_budget;
};

// Shared memory: [stages][quants 16 KB | scales 2 KB | pieces KC*2*TP*64]
// [mbarriers][tmem address].  A lives in TMEM.
struct QgSmem {
  static constexpr int kQuant = 16384;   // 128 rows x 128 bytes
  static constexpr int kScale = 2048;    // 128 rows x KC (<= 8) fp16
  __host__ __device__ static int plane_bytes(int type, int TP) { return qg_kc(type) * 2 * TP * 64; }
  __host__ __device__ static int stage_bytes(int type, int TP) {
    return (kQuant + kScale + plane_bytes(type, TP) + 1023) / 1024 * 1024;
  }
  __host__ __device__ static int total(int type, int TP) {
    return 1024 /* alignment slack */ + kQgStages * stage_bytes(type, TP) + 256;
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

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 operands, fp32
// accumulator), one CTA; accum = 0 overwrites D.  Executed by a whole warp
// with warp-uniform operands; one elected lane issues the MMA.
SS_DEVINL void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// The same with A in tensor memory (a_tmem: the column of its K = 16 slice).
SS_DEVINL void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
// Four consecutive 32-bit TMEM columns of this thread's lane (whole warp).
SS_DEVINL void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}
SS_DEVINL void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Arrives once on `bar` when every tcgen05 operation the issuing lane issued
// before it has completed (the MMA's shared-memory reads included).  Executed
// by the whole issuing warp; the elected lane commits.
SS_DEVINL void umma_commit(uint32_t bar) {
  asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
               " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(bar)
               : "memory");
}
// 4 / 8 / 16 consecutive 32-bit TMEM columns of this thread's lane.
SS_DEVINL void tmem_ld2(uint32_t taddr, int* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];"
               : "=r"(v[0]), "=r"(v[1])
               : "r"(taddr)
               : "memory");
}
SS_DEVINL void tmem_ld4(uint32_t taddr, int* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr)
               : "memory");
}
SS_DEVINL void tmem_ld8p(uint32_t taddr, int* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                 "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
SS_DEVINL void tmem_ld8(uint32_t taddr, int (&v)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                 "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
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

// Shared-memory matrix descriptor of a K-major fp16 operand without swizzle:
// 8-row x 16-byte (8-element) core matrices, the K-adjacent core matrices 128
// bytes apart (leading byte offset), 8-row groups 512 bytes apart (four core
// matrices of K = 32: stride byte offset); version 1 (sm_100).  One MMA (K =
// 16) spans two core matrices along K.
SS_DEVINL uint64_t umma_desc_kmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) |
         (1ull << 46);
}
// Instruction descriptor of kind::f16: D f32, A and B fp16, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Byte offset of element (row, k) of a block (K = 32 fp16) in the canonical
// layout: [row / 8][k / 8][row % 8][k % 8].
__host__ __device__ constexpr int qg_canon16(int row, int k) {
  return (row >> 3) * 512 + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2;
}

// ---- activation planes -----------------------------------------------------

// The pieces are built by bt_prep_kernel (batch_kernels.cuh): per token, the
// RMSNorm scale 1 / sqrtf(sum x^2 / n + eps) (cpu_neon.c:109-115) where the
// product has a norm, and a power of two 2^-e that brings the largest input
// element (after the norm) near [1, 2); x' = (x * scale * w) * 2^-e, hi =
// fp16(x'), lo = fp16(x' - hi); post[t] = 2^e undoes the scaling at the end.

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

// Two words of Q4_0 quant bytes (bytes 8 j .. 8 j + 7 of a block) -> the
// fp16 values q - 8 of their low (hi = false) or high nibbles, in element
// order as four fp16 pairs.  fp16 1024 + q is the bit pattern 0x6400 | q.
SS_DEVINL void q4_to_f16x8(uint32_t w0, uint32_t w1, bool hi, uint32_t (&h)[4]) {
  const __half2 off = __floats2half2_rn(1032.0f, 1032.0f);
  const uint32_t w[2] = {hi ? w0 >> 4 : w0, hi ? w1 >> 4 : w1};
#pragma unroll
  for (int i = 0; i < 2; i++) {
    uint32_t p01, p23;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(p01) : "r"(w[i]), "r"(0u));  // bytes 0, 1 -> half lanes
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(p23) : "r"(w[i]), "r"(0u));  // bytes 2, 3
    uint32_t a = (p01 & 0x000F000Fu) | 0x64006400u, c = (p23 & 0x000F000Fu) | 0x64006400u;
    const __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), off);
    const __half2 hc = __hsub2(*reinterpret_cast<__half2*>(&c), off);
    h[2 * i] = *reinterpret_cast<const uint32_t*>(&ha);
    h[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&hc);
  }
}
// Two words of Q8_0 quants -> fp16 q (1024 + (q + 128) - 1152).
SS_DEVINL void q8_to_f16x8(uint32_t w0, uint32_t w1, uint32_t (&h)[4]) {
  const __half2 off = __floats2half2_rn(1152.0f, 1152.0f);
  const uint32_t w[2] = {w0 ^ 0x80808080u, w1 ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 2; i++) {
    uint32_t a, c;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(a) : "r"(w[i]), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(c) : "r"(w[i]), "r"(0x64646464u));
    const __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), off);
    const __half2 hc = __hsub2(*reinterpret_cast<__half2*>(&c), off);
    h[2 * i] = *reinterpret_cast<const uint32_t*>(&ha);
    h[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&hc);
  }
}

// Warp roles: warp 0 (one lane) feeds the ring; warp 1 issues the MMAs (one
// elected lane); warps 2..17 unpack A -- warp w writes TMEM lanes
// 32 (w % 4) .. +31 (weight rows), warpgroup g = (w - 2) / 4 elements
// 8 g .. 8 g + 7 of each block (one core matrix); warps 18..25 flush D -- the
// same lane quadrants, tokens (w - 18) / 4 * TP/2 .. + TP/2 - 1.  The roles
// meet only at mbarriers: a group's A written (a_ready, 16 warp arrivals),
// its MMAs done (dfull, a commit), its TMEM region flushed (d_free, 8
// arrivals), a stage's slot free (empty: its quants unpacked and its last
// group flushed, 24 arrivals).  Unpacking the next group, the MMAs of this
// one and the flush of the previous one run at the same time.
template <int TYPE, int TP>
__global__ void __maxnreg__(72)
    qgemm_kernel(const QGemmParams p, const __grid_constant__ CUtensorMap qmap,
                 const __grid_constant__ CUtensorMap smap) {
  constexpr int KC = qg_kc(TYPE);
  constexpr int G = qg_group(TP);
  constexpr int NG = KC / G;  // groups per stage
  constexpr uint32_t kACol0 = 2 * G * 2 * TP;  // TMEM: D regions, then the two A buffers
  static_assert(kACol0 + 2 * G * kQgACols <= kQgTmemCols, "TMEM columns");
  static_assert(KC % G == 0, "stage = whole groups");
  static_assert(TP == 8 || TP == 16 || TP == 32, "token rows per piece");
  extern __shared__ uint8_t qg_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qg_raw) + 1023) & ~(uintptr_t)1023);
  const int SB = QgSmem::stage_bytes(TYPE, TP);
  const int PB = QgSmem::plane_bytes(TYPE, TP);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kQgStages * SB);
  uint64_t* empty = full + kQgStages;
  uint64_t* dfull = empty + kQgStages;                             // [2]: MMAs of a group done
  uint64_t* a_ready = dfull + 2;                                   // [2]: A of a group written
  uint64_t* d_free = a_ready + 2;                                  // [2]: TMEM region flushed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_free + 2);
  __shared__ int s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nunits = p.ntile * p.nsplit;
  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < kQgStages; i++) {
      mbar_init(smem_addr(full + i), 1);
      mbar_init(smem_addr(empty + i), kQgUnpackWarps + kQgFlushWarps);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(smem_addr(dfull + i), 1);
      mbar_init(smem_addr(a_ready + i), kQgUnpackWarps);
      mbar_init(smem_addr(d_free + i), kQgFlushWarps);
    }
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), kQgTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // programmatic dependent launch: the weights do not depend on the previous
  // kernel; the pieces, post[] and the outputs' readers do (pdl_wait below)
  pdl_trigger();
  // bounded wait that also gives up when another role aborted
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(a, parity)) {
      if (*(volatile int*)&s_abort) return false;
      if (clock64() - t0 > p.wait_budget) {
        atomicOr(p.err, 4);
        *(volatile int*)&s_abort = 1;
        return false;
      }
    }
    return true;
  };
  constexpr int kEndWarps = 1 + kQgUnpackWarps + kQgFlushWarps;  // issuer + unpack + flush

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
          if (sc >= kQgStages && !wait(empty + s, (uint32_t)(((sc / kQgStages) - 1) & 1))) {
            bad = true;
            break;
          }
          uint8_t* st = smem + s * SB;
          const uint32_t fb = smem_addr(full + s);
          mbar_expect_tx(fb, tx);
          tma_load_3d(smem_addr(st), &qmap, c * KC * (TYPE == kQ4_0 ? 16 : 32), 0, 32 * tile, fb);
          tma_load_2d(smem_addr(st + QgSmem::kQuant), &smap, c * KC * 8, 32 * tile, fb);
          if (sc == 0) pdl_wait();  // the pieces were written by the previous kernel
          bulk_g2s(smem_addr(st + QgSmem::kQuant + QgSmem::kScale),
                   reinterpret_cast<const uint8_t*>(p.xq) + (size_t)c * PB, (uint32_t)PB, fb);
        }
      }
      // drain: the copies of the last stages may still be landing
      for (int g = max(0, sc - kQgStages); g < sc; g++)
        mbar_wait_bounded(smem_addr(full + g % kQgStages), (uint32_t)((g / kQgStages) & 1), p.wait_budget);
    }
    return;
  }

  const uint32_t idesc = umma_idesc_f16(kQgRows, 2 * TP);
  if (warp == 1) {
    // ---------------- MMA issuer (the whole warp runs the loop; one elected lane issues)
    int gc = 0, sc = 0;
    bool bad = false;
    for (int u = blockIdx.x; u < nunits && !bad; u += gridDim.x) {
      int tile, split, c0, c1;
      qg_unit(p, u, tile, split, c0, c1);
      for (int c = c0; c < c1 && !bad; c++, sc++) {
        const int s = sc % kQgStages;
        bad = !wait(full + s, (uint32_t)((sc / kQgStages) & 1));
        uint8_t* st = smem + s * SB;
        for (int h = 0; h < NG && !bad; h++, gc++) {
          if (!wait(a_ready + (gc & 1), (uint32_t)((gc >> 1) & 1)) ||
              (gc >= 2 && !wait(d_free + (gc & 1), (uint32_t)(((gc - 2) >> 1) & 1)))) {
            bad = true;
            break;
          }
          tc_fence_after();
          const uint32_t dt = tmem + (uint32_t)((gc & 1) * G * 2 * TP);
          const uint32_t at = tmem + kACol0 + (uint32_t)((gc & 1) * G * kQgACols);
          const uint64_t bdesc0 = umma_desc_kmajor(smem_addr(st + QgSmem::kQuant + QgSmem::kScale) +
                                                   (uint32_t)(h * G * 2 * TP * 64));
          // descriptor start addresses advance in 16-byte units; a K half of
          // A is 8 TMEM columns
#pragma unroll
          for (int bl = 0; bl < G; bl++)
#pragma unroll
            for (int kh = 0; kh < 2; kh++)  // K halves of 16
              umma_f16_ts(dt + (uint32_t)(bl * 2 * TP), at + (uint32_t)(bl * kQgACols + 8 * kh),
                          bdesc0 + (uint64_t)((bl * 2 * TP * 64 + 256 * kh) >> 4), idesc, kh ? 1u : 0u);
          umma_commit(smem_addr(dfull + (gc & 1)));
        }
      }
    }
    // no MMA may still write TMEM when it is freed: wait for the last commit
    if (gc > 0) {
      const int last = gc - 1;
      mbar_wait_bounded(smem_addr(dfull + (last & 1)), (uint32_t)((last >> 1) & 1), p.wait_budget);
    }
    tc_fence_before();
    named_bar_sync(1, 32 * kEndWarps);
    tc_fence_after();
    tmem_dealloc(tmem, kQgTmemCols);
    return;
  }

  const int q = warp & 3;                 // TMEM lane quadrant of this warp
  const int r = 32 * q + lane;            // weight row within the tile
  const uint32_t t_lane = tmem + ((uint32_t)(32 * q) << 16);
  if (warp < 2 + kQgUnpackWarps) {
    // ---------------- unpack warps (2..17)
    const int g = (warp - 2) >> 2;        // warpgroup 0..3
    // this thread's quant bytes of a block: Q4_0 bytes 8 (g & 1) .. +7 (low
    // nibbles for g < 2, high for g >= 2); Q8_0 bytes 8 g .. 8 g + 7
    const int qchunk_off = TYPE == kQ4_0 ? 0 : (g >> 1);
    const uint32_t qbyte = (uint32_t)(8 * (g & 1));
    int gc = 0, sc = 0;
    bool bad = false;
    for (int u = blockIdx.x; u < nunits && !bad; u += gridDim.x) {
      int tile, split, c0, c1;
      qg_unit(p, u, tile, split, c0, c1);
      for (int c = c0; c < c1 && !bad; c++, sc++) {
        const int s = sc % kQgStages;
        if (!wait(full + s, (uint32_t)((sc / kQgStages) & 1))) {
          bad = true;
          break;
        }
        const uint32_t qrow = smem_addr(smem + s * SB) + (uint32_t)(r * 128);
#pragma unroll 1
        for (int h = 0; h < NG; h++, gc++) {
          // A buffer (gc & 1) was last read by the MMAs of group gc - 2
          if (gc >= 2 && !wait(dfull + (gc & 1), (uint32_t)(((gc - 2) >> 1) & 1))) {
            bad = true;
            break;
          }
          tc_fence_after();
          // this warp writes its 32 lanes, columns 4 g .. 4 g + 3 of each block
          const uint32_t ab = t_lane + kACol0 + (uint32_t)((gc & 1) * G * kQgACols + 4 * g);
          uint32_t w[G][2];
#pragma unroll
          for (int bl = 0; bl < G; bl++) {
            const int blk = h * G + bl;  // block within the stage
            const int chunk = TYPE == kQ4_0 ? blk : 2 * blk + qchunk_off;
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];"
                         : "=r"(w[bl][0]), "=r"(w[bl][1])
                         : "r"(qrow + ((chunk ^ (r & 7)) << 4) + qbyte));
          }
#pragma unroll
          for (int bl = 0; bl < G; bl++) {
            uint32_t hh[4];
            if constexpr (TYPE == kQ4_0) q4_to_f16x8(w[bl][0], w[bl][1], g >= 2, hh);
            else q8_to_f16x8(w[bl][0], w[bl][1], hh);
            tmem_st4(ab + (uint32_t)(bl * kQgACols), hh);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(a_ready + (gc & 1)));
        }
        if (bad) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(empty + s));  // this stage's quants are read
      }
    }
    tc_fence_before();
    named_bar_sync(1, 32 * kEndWarps);
    return;
  }

  // ---------------- flush warps (18..25)
  pdl_wait();  // post[] and the outputs' previous readers
  constexpr int th = TP >> 1;             // tokens flushed per warp (4, 8 or 16)
  const int t0 = ((warp - 2 - kQgUnpackWarps) >> 2) * th;
  float acc[th];
  int gc = 0, sc = 0;
  bool bad = false;
  for (int u = blockIdx.x; u < nunits && !bad; u += gridDim.x) {
    int tile, split, c0, c1;
    qg_unit(p, u, tile, split, c0, c1);
#pragma unroll
    for (int i = 0; i < th; i++) acc[i] = 0.0f;
    for (int c = c0; c < c1 && !bad; c++, sc++) {
      const int s = sc % kQgStages;
      if (!wait(full + s, (uint32_t)((sc / kQgStages) & 1))) {  // the stage's scales
        bad = true;
        break;
      }
      const uint8_t* sst = smem + s * SB + QgSmem::kQuant;
#pragma unroll 1
      for (int h = 0; h < NG; h++, gc++) {
        if (!wait(dfull + (gc & 1), (uint32_t)((gc >> 1) & 1))) {
          bad = true;
          break;
        }
        tc_fence_after();
        const uint32_t region = (uint32_t)((gc & 1) * G * 2 * TP);
#pragma unroll
        for (int bl = 0; bl < G; bl++) {
          int hv[th], lv[th];
          const uint32_t col = t_lane + region + (uint32_t)(bl * 2 * TP + t0);
          if constexpr (th == 16) {
            tmem_ld16(col, hv);
            tmem_ld16(col + (uint32_t)TP, lv);
          } else if constexpr (th == 8) {
            tmem_ld8p(col, hv);
            tmem_ld8p(col + (uint32_t)TP, lv);
          } else {
            tmem_ld4(col, hv);
            tmem_ld4(col + (uint32_t)TP, lv);
          }
          const int blk = h * G + bl;
          const float d = half_bits_to_float(
              *reinterpret_cast<const uint16_t*>(sst + (((r >> 2) * KC + blk) * 4 + (r & 3)) * 2));
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < th; i++) acc[i] = fmaf(__int_as_float(hv[i]) + __int_as_float(lv[i]), d, acc[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_addr(d_free + (gc & 1)));
          if (h == NG - 1) mbar_arrive(smem_addr(empty + s));  // the stage's last group is flushed
        }
      }
    }
    if (bad) break;
    const int row = tile * kQgRows + r;
    if (row < p.rows) {
#pragma unroll
      for (int i = 0; i < th; i++) {
        const int t = t0 + i;
        if (t < p.T) p.out[((size_t)split * p.T + t) * p.rows + row] = acc[i] * p.post[t];
      }
    }
  }
  tc_fence_before();
  named_bar_sync(1, 32 * kEndWarps);
}

}  // namespace ss
