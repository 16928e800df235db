// step_kernel.cuh -- one decode step of SlipStream's llama path as a single
// persistent kernel on sm_100a.
//
// Same computation as ss_scheduler_forward (SlipStream/src/core/
// layer_scheduler.c:571-679): embedding, L x (RMSNorm, Q/K/V matvec + RoPE,
// int8 KV append + attention, O matvec + residual, RMSNorm, gate/up matvec +
// SwiGLU, down matvec + residual), final RMSNorm, lm_head, greedy argmax.
//
// Execution model.  One CTA per SM (grid = SM count, cooperative launch so all
// are co-resident), 20 warps: warp 0 is a *producer* that streams every weight
// tile this CTA will ever touch during the step -- all phases, back to back --
// from HBM into a shared-memory ring with cp.async.bulk, gated only by ring
// slots being free, plus a bulk L2 prefetch of the next phase's range.  It
// never waits for activations, so HBM keeps streaming across phase
// boundaries.  Warps 4..19 are *consumers*: for each phase they wait at a
// grid-wide barrier for the phase's input, then consume their share of the
// ring and write the phase's outputs.  The phases are
//     EMBED | per layer: QKV, ATT, O, GU, DOWN | HEAD
// separated by grid barriers (monotonic counter, bounded spin).
//
// Weight layout ("tiled"): a matrix is stored as tiles of 4 rows; a tile holds
// the 4 rows' quant bytes row-major (block b of row i at i*nb*QB + b*QB, the
// GGUF block bytes unchanged) followed by the nb x 4 fp16 scales block-major
// (scale of row i, block b at b*8 + i*2), padded to 16 bytes.  A CTA owns a
// contiguous range of tiles of each matrix, so a ring stage is one bulk copy.
//
// Inner product.  As in gemv.cuh: activations in block fixed point (23 bits
// per 32-element block, three signed byte planes), weights' nibbles / bytes
// multiplied with dp4a, exact in int32, combined in fp32.  At the start of a
// matvec phase each consumer thread reads its 32 input values from L2 and
// converts them (RMSNorm first where the reference has one: ss = sum x^2,
// scale = 1 / sqrtf(ss / n + eps), x * scale * w, SlipStream/src/backends/
// cpu_neon.c:109-115); every CTA does this from the same data in the same
// order, so all use identical activations.  Epilogues only write the phase's
// output vector.
//
// All waits are bounded (about one second of SM clocks); on expiry a CTA sets
// an error bit and a global abort flag that every other wait also watches, the
// producer drains its outstanding copies, and the kernel returns.
//
// Tensor parallelism (the TP instantiation; one process per GPU): each rank
// runs the step on its shard -- its q / kv heads and FFN rows, the matching
// columns of O and down, its slice of the vocabulary -- and the exchanges run
// inside the kernel over NVLink, through one exchange block per rank that
// every peer has mapped (StepXchg):
//   * QKV: each CTA stores its (max |k|, max |v|) into every rank's block; the
//     int8 scales use the maximum over all ranks' CTAs (one scale over the
//     whole kv_dim, layer_scheduler.c:101-111);
//   * O, DOWN (row-parallel): each CTA stores its rows' partial sums into every
//     rank's block (rank 0's carries the residual); the next phases read h as
//     the sum of the tp partials in rank order, so every rank holds the same h;
//   * HEAD: each rank's best (value, index) goes to every rank; all pick the
//     same token.
// The barrier after QKV, O and DOWN counts the arrivals of every rank's CTAs
// on a monotonic 64-bit counter in each rank's block (system-scope release /
// acquire); the other barriers stay local.
#pragma once
#include "attention.cuh"
#include "gemv.cuh"

namespace ss {

constexpr int kStepTileRows = 4;
constexpr int kStepConsumerWarps = 16;
constexpr int kStepConsumers = kStepConsumerWarps * 32;  // 512
// Warpgroup 0 (warp 0: the producer; warps 1-3 exit at once) gives registers
// to the four consumer warpgroups: launched at kStepLaunchRegs per thread, it
// drops to kStepProducerRegs and the consumers rise to kStepConsumerRegs, so
// 128 * producer + 512 * consumer == 640 * launch -- the host launches only
// when the compiled kernel's launch register count is exactly kStepLaunchRegs.
constexpr int kStepProducerThreads = 128;
constexpr int kStepThreads = kStepProducerThreads + kStepConsumers;  // 640
constexpr int kStepLaunchRegs = 96;
constexpr int kStepProducerRegs = 32;
constexpr int kStepConsumerRegs = 112;
static_assert(kStepProducerThreads * kStepProducerRegs + kStepConsumers * kStepConsumerRegs ==
                  kStepThreads * kStepLaunchRegs,
              "register split must equal the launch allocation");
constexpr int kStepMaxNb = kStepConsumers;               // <= 16384 columns
constexpr int kStepMaxSplit = 4;                         // attention position splits per kv head
constexpr int kStepMaxTp = 8;                            // tensor-parallel ranks

// Tensor parallelism: the group and every rank's exchange block.
struct StepTp {
  int tp, rank;
  int vocab_off;                 // global index of this rank's first lm_head row
  int pad;
  uint8_t* xpeer[kStepMaxTp];    // [rank] is this rank's own block
#ifdef SS_STEP_CHECKS
  long long xbytes;              // bytes of one exchange block
  unsigned* dbg;                 // host-mapped record (StepDbg)
#endif
};

// Checks builds (compiled with -DSS_STEP_CHECKS, never the shipped library):
// the tensor-parallel step records its progress into host-mapped memory, which
// the host can read after a fault, and checks every peer store against the
// exchange block's bounds (skipping and recording a bad one).  Word offsets:
struct StepDbg {
  static constexpr int kCons = 0;     // [cta] consumer thread 0: 16 * (1 + phase) + sub-step
  static constexpr int kProd = 256;   // [cta] producer: 1 + phase being issued
  static constexpr int kBad = 512;    // [cta][4] last violation: code, where, rank, offset
  static constexpr int kHead = 1536;  // argmax exchange stage of the last CTA
  static constexpr int kWords = 2048;
};

// Exchange block of one rank, same layout on every rank (byte offsets).
struct StepXchg {
  static constexpr int kBar = 0;     // u64: arrivals of all ranks' CTAs at cross-rank barriers
  static constexpr int kHead = 64;   // u64: arrivals of all ranks' argmax
  static constexpr int kStep = 128;  // u64: steps this rank has run (read only by it)
  static constexpr int kBest = 256;  // u64 [tp]: each rank's best (value, index) of this step
  static constexpr int kAm = 512;    // float2 [tp][grid]: each rank's CTAs' (max |k|, max |v|)
  static constexpr int kCounters = 512;  // bytes ss_cuda_reset zeroes
  // float [2][tp][d]: partial h of the O (slot 0) and DOWN (slot 1) phases
  __host__ __device__ static size_t h_off(int tp, int grid) {
    return ((size_t)kAm + (size_t)tp * grid * 8 + 255) / 256 * 256;
  }
  __host__ __device__ static size_t bytes(int tp, int grid, int d) {
    return h_off(tp, grid) + 2 * (size_t)tp * d * sizeof(float);
  }
};

// One activation block in block fixed point in shared memory: 112 bytes (7 x
// 16), no padding -- consumer lane j reads block j with 16-byte loads, and the
// odd stride spreads a warp's lanes over all banks.
struct PlaneBlock {
  int pl[3][8];  // word w of plane p: digits p of elements 4w .. 4w+3
  int nsum[3];   // -sum_j digit_pj (times the weights' zero point: accumulator start)
  float c0;      // 2^(e-22): value of one unit of plane 0
};
static_assert(sizeof(PlaneBlock) == 112, "PlaneBlock must be 112 bytes");

struct TMat {
  const uint8_t* w;
  int nb;          // 32-column blocks per row
  int ntiles;      // 4-row tiles
  int tile_bytes;  // bytes per tile (multiple of 16)
  int type;        // kQ4_0 / kQ8_0
  int rows;        // real rows (the last tile may carry zero padding rows)
};

struct StepParams {
  // layer 0's matrices; layer l's start layer_stride * l bytes further (all
  // layers live in one allocation), so no descriptor is read from memory
  TMat qkv0, o0, gu0, down0;  // gu rows interleave gate (even) and up (odd)
  long long layer_stride;
  const float* attn_norm;  // [L][d]
  const float* ffn_norm;   // [L][d]
  int L;
  TMat head;
  const float* out_norm;
  const float* embd;  // [vocab][d] fp32
  int d, qd, kvd, ff, vocab, nh, nkv, hd, rope_dim, ctx;
  float eps, attn_scale;
  const float2* rope_tab;
  int8_t* kc;  // [L][nkv][ctx][hd] (head-major: a head's positions are contiguous)
  int8_t* vc;
  float* ks;   // [L][ctx]
  float* vs;
  int* d_pos;          // position of this step; advanced by one at the end
  const int* fixed_until;
  int* err;
  int* seq_tokens;     // [ctx + 1]
  float* h;            // residual stream [d]
  float* qkv_out;      // q | k | v
  float* attn_out;     // [qd]
  float* act;          // [ff]
  float* logits;       // [vocab]
  float2* amax_part;   // [grid] (max |k|, max |v|) of this position
  float* att_part;     // [nh][nsplit][hd + 4]: m, l, -, -, o[hd] (merged by the O phase)
  unsigned* grid_bar;  // [1]
  unsigned* abort_flag;  // [1]
  unsigned long long* am_part;  // [grid]
  unsigned* am_cnt;    // [1]
  int nsplit;          // attention position splits per kv head
  int slot_bytes, nslots;
  int inflight;        // weight stages a producer keeps in flight (not yet landed)
  int split_rows;      // cached positions per attention split (see step_nsplit)
  int prefetch;        // weight stages the L2 prefetch runs ahead of the bulk copies (0: off)
  // optional timeline (measurement aid): [phase][cta][8] global-timer ns --
  // 0 input ready (grid barrier passed), 1 main work done, 2 arrival at the
  // next barrier, 3 producer issued the phase's last weight stage, 4 first
  // stage's weights ready, 5 last stage's weights ready, 6 consumer warp 0
  // done with its rows, 7 producer issued the phase's first stage
  long long* trace;
  // every bounded wait gives up after this many SM clocks (kWaitBudget; the
  // cross-rank waits 4x); a failure-path test shortens it for one step
  long long wait_budget;
  // test aid (ss_cuda_test_fail_next_step): the producer issues no copy for
  // the first weight stage of phase `test_withhold` (-1: off), so that stage's
  // consumers wait until their budget runs out and the step reports an error
  int test_withhold;
};

// ---------------------------------------------------------------- helpers

SS_DEVINL unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SS_DEVINL unsigned ld_volatile_u32(const unsigned* p) {
  return *reinterpret_cast<const volatile unsigned*>(p);
}

SS_DEVINL long long global_ns() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
SS_DEVINL void trace_mark(const StepParams& p, int phase, int what) {
  if (p.trace) p.trace[((size_t)phase * gridDim.x + blockIdx.x) * 8 + what] = global_ns();
}

// Balanced contiguous split of n items over g parts.
SS_DEVINL void part_range(int n, int i, int g, int& a, int& b) {
  a = (int)(((long long)n * i) / g);
  b = (int)(((long long)n * (i + 1)) / g);
}

// Warps per row and row groups of a matrix with nb blocks.
SS_DEVINL int step_wpr(int nb) { return (nb + 31) >> 5; }
SS_DEVINL int step_rg(int nb) { return kStepConsumerWarps / step_wpr(nb); }

// Q4_0 row block: sum_j (q_j - 8) * m_j with m in three planes (exact int32),
// returned as fp32 units of plane 0.  |a0 + 256 a1| < 2^24, so its conversion
// is exact; one rounding in the final fma.
SS_DEVINL float step_dot_q4(const uint4 q, const int (&pl)[3][8], const int (&init)[3]) {
  int a0 = init[0], a1 = init[1], a2 = init[2];
  const unsigned wq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const unsigned lo = wq[t] & 0x0F0F0F0Fu;
    const unsigned hi = (wq[t] >> 4) & 0x0F0F0F0Fu;
    a0 = dp4a_us(lo, pl[0][t], a0);
    a1 = dp4a_us(lo, pl[1][t], a1);
    a2 = dp4a_us(lo, pl[2][t], a2);
    a0 = dp4a_us(hi, pl[0][4 + t], a0);
    a1 = dp4a_us(hi, pl[1][4 + t], a1);
    a2 = dp4a_us(hi, pl[2][4 + t], a2);
  }
  return fmaf((float)a2, 65536.0f, (float)(a0 + a1 * 256));
}

SS_DEVINL float step_dot_q8(const uint4 qa, const uint4 qb, const int (&pl)[3][8]) {
  int a0 = 0, a1 = 0, a2 = 0;
  const unsigned wa[4] = {qa.x, qa.y, qa.z, qa.w};
  const unsigned wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    a0 = dp4a_ss((int)wa[t], pl[0][t], a0);
    a1 = dp4a_ss((int)wa[t], pl[1][t], a1);
    a2 = dp4a_ss((int)wa[t], pl[2][t], a2);
    a0 = dp4a_ss((int)wb[t], pl[0][4 + t], a0);
    a1 = dp4a_ss((int)wb[t], pl[1][4 + t], a1);
    a2 = dp4a_ss((int)wb[t], pl[2][4 + t], a2);
  }
  return fmaf((float)a2, 65536.0f, fmaf((float)a1, 256.0f, (float)a0));
}

// Phases of one step: 0 EMBED, then per layer QKV ATT O GU DOWN, then HEAD.
enum StepPhase : int { kPhEmbed = 0, kPhQKV, kPhAtt, kPhO, kPhGU, kPhDown, kPhHead };

SS_DEVINL int step_phase_count(int L) { return 2 + 5 * L; }
SS_DEVINL void step_phase(int k, int L, int& kind, int& layer) {
  if (k == 0) { kind = kPhEmbed; layer = 0; return; }
  if (k == 1 + 5 * L) { kind = kPhHead; layer = L - 1; return; }
  layer = (k - 1) / 5;
  kind = kPhQKV + (k - 1) % 5;
}
SS_DEVINL bool step_phase_has_mat(int kind) { return kind != kPhEmbed && kind != kPhAtt; }
// Weights a phase streams (kinds with step_phase_has_mat only).
SS_DEVINL TMat step_phase_mat(const StepParams& p, int kind, int layer) {
  TMat m;
  switch (kind) {
    case kPhQKV: m = p.qkv0; break;
    case kPhO: m = p.o0; break;
    case kPhGU: m = p.gu0; break;
    case kPhDown: m = p.down0; break;
    default: return p.head;
  }
  m.w += (size_t)layer * (size_t)p.layer_stride;
  return m;
}

// Shared memory (dynamic): [ring][full][empty barriers][scratch].  The
// scratch holds, one use at a time, a phase's activation planes, the matvec
// partial sums, or an attention task's buffers.
struct StepSmem {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  float* scratch;
};

// Attention-stage geometry (shared by producer and consumers; layout in the
// attention section below).
__host__ __device__ __forceinline__ int step_att_rows(int slot_bytes, int hd) {
  return (slot_bytes - 96) / (2 * hd + 8);
}
// Shared-memory scratch of an attention task (layout in step_attention_task):
// q[G][hd] | scores[max(G * rows per stage, consumers)] | m, l, corr [24] |
// int8 K and V rows of this position.  One function for host and kernel.
__host__ __device__ __forceinline__ size_t step_att_scratch_bytes(int G, int hd, int slot_bytes) {
  const int sc = G * step_att_rows(slot_bytes, hd);
  return sizeof(float) * ((size_t)G * hd + (size_t)(sc > kStepConsumers ? sc : kStepConsumers) + 24) +
         2 * (size_t)hd;
}
// Position splits of this step: one per p.split_rows cached positions, at most
// p.nsplit (more splits: shorter attention tasks; fewer: less for the O phase
// to merge).
SS_DEVINL int step_nsplit(const StepParams& p, int pos) {
  return max(1, min(p.nsplit, (pos + p.split_rows) / p.split_rows));
}
SS_DEVINL void step_att_task(const StepParams& p, int task, int pos, int& kvh, int& split, int& t0,
                             int& t1) {
  const int ns = step_nsplit(p, pos);
  kvh = task / ns;
  split = task - kvh * ns;
  const int seq = pos + 1;
  const int chunk = (seq + ns - 1) / ns;
  t0 = min(split * chunk, seq);
  t1 = min(t0 + chunk, seq);
}
// Byte offsets of the scale blocks inside an attention stage.
SS_DEVINL int step_att_ks_off(int rows, int hd) { return 2 * rows * hd; }
SS_DEVINL int step_att_vs_off(int rows, int hd) { return 2 * rows * hd + ((rows + 8) * 4 + 15) / 16 * 16; }

// ---------------------------------------------------------------- producer

// `s_cabort` is written by consumers only; the producer just watches it.
SS_DEVINL void step_producer(const StepParams& p, const StepSmem& sm, const volatile int* s_cabort,
                             int lane, int pos) {
  if (lane != 0) return;
  const int ncta = gridDim.x, cta = blockIdx.x;
  const int nph = step_phase_count(p.L);
  const int nslots = p.nslots;
  const uint32_t ring0 = smem_addr(sm.ring), slot_bytes = (uint32_t)p.slot_bytes;
  int issued = 0;          // stages issued so far
  int slot = 0;            // issued % nslots
  uint32_t wraps = 0;      // issued / nslots
  // landing cursor: the stage `inflight` behind `issued` must have landed
  // before the next copy is issued, so at most `inflight` copies per SM queue
  // in the memory system -- more only delays every other load (the
  // consumers' activations, the grid barrier) without adding bandwidth
  const int inflight = p.inflight;
  int lslot = 0;
  uint32_t lwraps = 0;
  // L2 prefetch `p.prefetch` weight stages ahead of the bulk copies, across
  // phase boundaries (0: off): while the consumers sit at a barrier and the
  // ring is full, HBM keeps loading the stages after the ring into L2, a
  // stage at a time, so no large burst queues ahead of the consumers' loads
  struct Ahead {
    int k = 0, t = 0, t1 = 0, rg = 1;
    TMat m;
  } ah;
  auto ahead_next = [&](const uint8_t*& ptr, uint32_t& bytes) -> bool {
    while (ah.t >= ah.t1) {
      if (++ah.k >= nph) return false;
      int kind, layer;
      step_phase(ah.k, p.L, kind, layer);
      if (!step_phase_has_mat(kind)) continue;
      ah.m = step_phase_mat(p, kind, layer);
      part_range(ah.m.ntiles, cta, ncta, ah.t, ah.t1);
      ah.rg = step_rg(ah.m.nb);
    }
    const int nt = min(ah.rg, ah.t1 - ah.t);
    ptr = ah.m.w + (size_t)ah.t * ah.m.tile_bytes;
    bytes = (uint32_t)(nt * ah.m.tile_bytes);
    ah.t += ah.rg;
    return true;
  };
  auto prefetch_one = [&]() {
    const uint8_t* ptr;
    uint32_t bytes;
    if (ahead_next(ptr, bytes)) prefetch_l2_bulk(ptr, bytes);
  };
  for (int i = 0; i < p.prefetch; i++) prefetch_one();  // the window's first stages
  bool aborted = false;
  // Waits until the next slot may be filled (its previous stage released, and
  // the stage `inflight` back landed); returns its full barrier, or 0 on abort.
  auto acquire_slot = [&]() -> uint32_t {
    const uint32_t fb = smem_addr(sm.full + slot), eb = smem_addr(sm.empty + slot);
    auto wait = [&](uint32_t bar, uint32_t par) {
      if (mbar_try_wait(bar, par)) return true;
      const long long c0 = clock64();
      while (!mbar_try_wait(bar, par)) {
        if (*s_cabort || ld_volatile_u32(p.abort_flag)) return false;
        if (clock64() - c0 > p.wait_budget) {
          atomicOr(p.err, 4);
          atomicExch(p.abort_flag, 1u);
          return false;
        }
      }
      return true;
    };
    if (wraps > 0 && !wait(eb, (wraps - 1) & 1u)) return 0u;
    if (issued >= inflight) {
      if (!wait(smem_addr(sm.full + lslot), lwraps & 1u)) return 0u;
      if (++lslot == nslots) { lslot = 0; lwraps++; }
    }
    return fb;
  };
  auto advance = [&]() {
    issued++;
    if (++slot == nslots) { slot = 0; wraps++; }
  };
  for (int k = 1; k < nph && !aborted; k++) {
    int kind, layer;
    step_phase(k, p.L, kind, layer);
    if (kind == kPhAtt) {
      // this CTA's attention task(s): the cached K / V rows and scales
      const int R = step_att_rows(p.slot_bytes, p.hd);
      const size_t lrow = (size_t)layer * p.ctx;
      for (int task = cta; task < p.nkv * step_nsplit(p, pos) && !aborted; task += ncta) {
        int kvh, split, t0, t1;
        step_att_task(p, task, pos, kvh, split, t0, t1);
        const int tend = min(t1, pos);
        for (int ts = t0; ts < tend; ts += R) {
          const int te = min(ts + R, tend), nr = te - ts;
          const uint32_t fb = acquire_slot();
          if (!fb) { aborted = true; break; }
          const int sa = ts & ~3, sb = (te + 3) & ~3;
          const uint32_t sbytes = (uint32_t)((sb - sa) * 4);
          mbar_expect_tx(fb, (uint32_t)(2 * nr * p.hd) + 2 * sbytes);
          const uint32_t dst = ring0 + (uint32_t)slot * slot_bytes;
          const size_t row0 = lrow * p.kvd + ((size_t)kvh * p.ctx + ts) * p.hd;  // head-major
          bulk_g2s(dst, p.kc + row0, (uint32_t)(nr * p.hd), fb);
          bulk_g2s(dst + (uint32_t)(R * p.hd), p.vc + row0, (uint32_t)(nr * p.hd), fb);
          bulk_g2s(dst + (uint32_t)step_att_ks_off(R, p.hd), p.ks + lrow + sa, sbytes, fb);
          bulk_g2s(dst + (uint32_t)step_att_vs_off(R, p.hd), p.vs + lrow + sa, sbytes, fb);
          advance();
        }
      }
      trace_mark(p, k, 3);
      continue;
    }
    if (!step_phase_has_mat(kind)) continue;
    const TMat mv = step_phase_mat(p, kind, layer);
    const TMat* m = &mv;
    int t0, t1;
    part_range(m->ntiles, cta, ncta, t0, t1);
    const int rg = step_rg(m->nb);
    for (int t = t0; t < t1; t += rg) {
      if (t == t0) trace_mark(p, k, 7);
      const uint32_t fb = acquire_slot();
      if (!fb) { aborted = true; break; }
      const int nt = min(rg, t1 - t);
      const uint32_t bytes = (uint32_t)(nt * m->tile_bytes);
      if (k == p.test_withhold && t == t0) {  // test aid: this stage never lands
        advance();
        continue;
      }
      mbar_expect_tx(fb, bytes);
      bulk_g2s(ring0 + (uint32_t)slot * slot_bytes, m->w + (size_t)t * m->tile_bytes, bytes, fb);
      advance();
      if (p.prefetch) prefetch_one();  // keep the L2 window p.prefetch stages ahead
    }
    trace_mark(p, k, 3);
  }
  if (aborted) {
    // drain: the copies of the last nslots stages may still be in flight
    for (int g = max(0, issued - nslots); g < issued; g++)
      mbar_wait_bounded(smem_addr(sm.full + g % nslots), (uint32_t)((g / nslots) & 1), p.wait_budget);
  }
}

// ---------------------------------------------------------------- consumers

struct ConsumerCtx {
  int ctid, lane, cw;  // consumer thread id 0..511, lane, consumer warp 0..15
  int slot;            // ring slot of the next stage
  uint32_t phase;      // its full-barrier parity
  volatile int* s_abort;  // set by consumers when they give up; read by the producer only
  float* s_red;        // 32 floats of reduction scratch
  int* s_flag;
};

SS_DEVINL void cbar() { named_bar_sync(1, kStepConsumers); }
// Consumer barrier that also ORs a predicate over all consumers: every consumer
// gets the same answer, so abort decisions never diverge between warps.
SS_DEVINL bool cbar_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n"
      " barrier.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(kStepConsumers)
      : "memory");
  return r != 0;
}

SS_DEVINL float cblock_max(float v, ConsumerCtx& cc) {
  v = warp_max(v);
  if (cc.lane == 0) cc.s_red[cc.cw] = v;
  cbar();
  float t = cc.s_red[0];
  for (int w = 1; w < kStepConsumerWarps; w++) t = fmaxf(t, cc.s_red[w]);
  cbar();
  return t;
}

// Grid barrier: wait until `target` CTA-phase completions were counted.
SS_DEVINL bool step_grid_wait(const StepParams& p, ConsumerCtx& cc, unsigned target) {
  bool bad = false;
  if (cc.ctid == 0) {
    const long long c0 = clock64();
    while (true) {
      const unsigned v = ld_acquire_u32(p.grid_bar);
      if ((int)(v - target) >= 0) break;
      if (ld_volatile_u32(p.abort_flag)) { bad = true; break; }
      if (clock64() - c0 > p.wait_budget) {
        atomicOr(p.err, 8);
        atomicExch(p.abort_flag, 1u);
        bad = true;
        break;
      }
    }
  }
  bad = cbar_any(bad);  // the acquire above, then this barrier, order the CTA's reads
  if (bad && cc.ctid == 0) *cc.s_abort = 1;
  return !bad;
}
// Called by every consumer thread after its last global write of the phase:
// the consumer barrier orders those writes before thread 0's release-add.
SS_DEVINL void step_grid_arrive(const StepParams& p, ConsumerCtx& cc) {
  cbar();
  if (cc.ctid == 0)
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.grid_bar) : "memory");
}

// ---- cross-rank barrier and exchange blocks (tensor parallelism)
SS_DEVINL unsigned long long ld_relaxed_sys_u64(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
SS_DEVINL void red_relaxed_sys_add_u64(unsigned long long* a, unsigned long long v) {
  asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
SS_DEVINL void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
SS_DEVINL unsigned long long* xchg_u64(const StepTp& t, int rank, int off) {
  return reinterpret_cast<unsigned long long*>(t.xpeer[rank] + off);
}
SS_DEVINL float2* xchg_am(const StepTp& t, int rank) {
  return reinterpret_cast<float2*>(t.xpeer[rank] + StepXchg::kAm);
}
#ifdef SS_STEP_CHECKS
SS_DEVINL void dbg_mark(const StepTp& t, int word, unsigned v) {
  if (!t.dbg) return;
  *reinterpret_cast<volatile unsigned*>(t.dbg + word) = v;
  __threadfence_system();
}
// A store of `bytes` at `ptr` into rank `rank`'s block must land inside it.
SS_DEVINL bool xchg_ok(const StepTp& t, int rank, const void* ptr, int bytes, unsigned where) {
  const long long off = reinterpret_cast<const uint8_t*>(ptr) - t.xpeer[rank];
  if (rank >= 0 && rank < t.tp && t.xpeer[rank] != nullptr && off >= 0 && off + bytes <= t.xbytes &&
      (off % bytes) == 0)
    return true;
  if (t.dbg) {
    volatile unsigned* e = t.dbg + StepDbg::kBad + 4 * blockIdx.x;
    e[1] = where;
    e[2] = (unsigned)rank;
    e[3] = (unsigned)off;
    e[0] = 2u;
    __threadfence_system();
  }
  return false;
}
#define SS_TP_MARK(t, word, v) dbg_mark((t), (word), (v))
#define SS_TP_OK(t, rank, ptr, bytes, where) xchg_ok((t), (rank), (ptr), (bytes), (where))
#else
#define SS_TP_MARK(t, word, v) ((void)0)
#define SS_TP_OK(t, rank, ptr, bytes, where) true
#endif
// Partial-h slot `s` (0: O, 1: DOWN) of rank `rank`'s block: [tp][d].
SS_DEVINL float* xchg_h(const StepTp& t, int rank, int s, int d) {
  return reinterpret_cast<float*>(t.xpeer[rank] + StepXchg::h_off(t.tp, gridDim.x)) + (size_t)s * t.tp * d;
}
// Peers may still be launching their step: the cross-rank waits get a longer
// budget than the local ones.
SS_DEVINL long long xwait_budget(const StepParams& p) { return 4 * p.wait_budget; }

// Waits until this rank's counter holds the arrivals of the `ncross` cross
// phases of this step after the `epoch` earlier steps (3 per layer each), every
// CTA of every rank arriving once per phase.
SS_DEVINL bool step_xwait(const StepParams& p, const StepTp& t, ConsumerCtx& cc, unsigned long long epoch,
                          unsigned ncross) {
  bool bad = false;
  if (cc.ctid == 0) {
    const unsigned long long per = (unsigned long long)gridDim.x * (unsigned long long)t.tp;
    const unsigned long long target = (epoch * 3ull * (unsigned long long)p.L + ncross) * per;
    const unsigned long long* ctr = xchg_u64(t, t.rank, StepXchg::kBar);
    SS_TP_MARK(t, StepDbg::kCons + blockIdx.x, 0x80000000u | (ncross << 8) | 5u);
    const long long c0 = clock64();
    while (true) {
      // relaxed polling; one acquire fence once the count is there
      if ((long long)(ld_relaxed_sys_u64(ctr) - target) >= 0) break;
      if (ld_volatile_u32(p.abort_flag)) { bad = true; break; }
      if (clock64() - c0 > xwait_budget(p)) {
        atomicOr(p.err, 32);
        atomicExch(p.abort_flag, 1u);
        bad = true;
        break;
      }
    }
    fence_acq_rel_sys();
  }
  bad = cbar_any(bad);
  if (bad && cc.ctid == 0) *cc.s_abort = 1;
  return !bad;
}
// Arrival at a cross-rank barrier: after the consumer barrier, thread 0's
// system-scope fence and then its adds (one per rank) publish every consumer's
// stores of the phase -- the peer stores included -- to all ranks (a release
// made of one fence and relaxed adds).
SS_DEVINL void step_xarrive(const StepTp& t, ConsumerCtx& cc) {
  cbar();
  if (cc.ctid == 0) {
    fence_acq_rel_sys();
    for (int r = 0; r < t.tp; r++)
      if (SS_TP_OK(t, r, xchg_u64(t, r, StepXchg::kBar), 8, 50u))
        red_relaxed_sys_add_u64(xchg_u64(t, r, StepXchg::kBar), 1ull);
  }
}
// Phases whose outputs other ranks read: their CTAs arrive at the cross-rank
// counter (QKV: its K/V maxima, and also at the local barrier, since the
// attention phase needs only this rank's q / k / v).  The phases after O and
// DOWN wait at the cross-rank counter; every other phase at the local barrier.
SS_DEVINL bool step_cross(int kind) { return kind == kPhQKV || kind == kPhO || kind == kPhDown; }
SS_DEVINL bool step_cross_wait(int prev_kind) { return prev_kind == kPhO || prev_kind == kPhDown; }
// Arrivals before phase k: local (EMBED, then QKV, ATT, GU of each layer) and
// cross-rank (QKV, O, DOWN of each layer).
SS_DEVINL void step_bar_counts(int k, unsigned& nloc, unsigned& ncross) {
  const unsigned f = (unsigned)(k - 1) / 5, rr = (unsigned)(k - 1) % 5;
  nloc = 1 + 3 * f + (rr > 0) + (rr > 1) + (rr > 3);
  ncross = 3 * f + (rr > 0) + (rr > 2);
}
// Where h lives for phase (kind, layer) under tensor parallelism: p.h (the
// embedding, before layer 0's O), else the tp partials of the last O (slot 0)
// or DOWN (slot 1) exchange -- the h that QKV / GU / lm_head normalise and that
// the O / DOWN epilogues add to.
SS_DEVINL const float* step_hsrc(const StepParams& p, const StepTp& t, int kind, int layer, int& n) {
  n = t.tp;
  if (kind == kPhGU || kind == kPhDown) return xchg_h(t, t.rank, 0, p.d);
  if (kind == kPhHead || layer > 0) return xchg_h(t, t.rank, 1, p.d);
  n = 1;
  return p.h;
}

// Bounded wait on an mbarrier phase by a whole warp: every lane waits (each
// needs the barrier's acquire); giving up is a warp vote, so the warp never
// splits.  Returns false on timeout or when another CTA aborted.
SS_DEVINL bool warp_wait_phase(const StepParams& p, uint32_t bar, uint32_t par) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, par))) return true;
  const long long w0 = clock64();
  while (true) {
    const bool ok = mbar_try_wait(bar, par);
    if (__all_sync(0xffffffffu, ok)) return true;
    const bool late = !ok && (ld_volatile_u32(p.abort_flag) != 0u || clock64() - w0 > p.wait_budget);
    if (__any_sync(0xffffffffu, late)) {
      if ((threadIdx.x & 31) == 0) {
        atomicOr(p.err, 4);
        atomicExch(p.abort_flag, 1u);
      }
      return false;
    }
  }
}

// Block fixed point of the phase's input vector src[nb * 32] into shared
// memory.  Four consecutive consumer threads build one block together, each
// converting 8 elements (the block maximum and the digit sums are combined
// over the four with shuffles); with more than 128 blocks the consumers take
// R rounds of 128 blocks, every load issued before any conversion.  No block
// is built twice.  With norm_w, RMSNorm (cpu_neon.c:109-115): the planes hold
// x = src * w, and the returned scale = 1 / sqrtf(ss / n + eps) multiplies each
// block's unit in the matvec instead (it is uniform over the vector), so the
// sum of squares ss = sum src^2 (each thread over its elements in order, then a
// warp tree, then the warps in order -- the same in every CTA) needs no
// barrier before the conversion: the warps' sums are added after the closing
// one.  The digits are those of make_planes (gemv.cuh).  Ends with a consumer
// barrier; returns 1 without norm_w.
//
// With `att` (the O phase), the input is the attention output, merged here
// from the position splits' partials (m, l, o): M = max m_s, f_s = e^(m_s-M),
// out = sum_s f_s o_s / sum_s f_s l_s.  MULTI (tensor parallelism): the input
// is the sum of nsrc vectors sstride apart, added in order.
template <int R, bool MULTI>
SS_DEVINL float build_block_planes_r(const float* src, int nsrc, int sstride, const float* norm_w,
                                    const float* att, int nsplit, int hd, int nb, float eps,
                                    PlaneBlock* dst, ConsumerCtx& cc) {
  constexpr int EPT = 8;
  const int q = cc.ctid & 3;
  float xv[R][EPT];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int b = (cc.ctid + r * kStepConsumers) >> 2;
    const bool mine = b < nb;
    const int base = b * 32 + q * EPT;
#pragma unroll
    for (int j = 0; j < EPT; j++) xv[r][j] = 0.0f;
    if (!mine) continue;
    if (R <= 2 && att) {  // the attention output: qd <= 8192
      const int qh = base / hd, i0 = base - qh * hd;  // 8 elements of one head
      const float* pb = att + (size_t)qh * nsplit * (hd + 4);
      float ms[kStepMaxSplit], ls[kStepMaxSplit];
      float4 ov[kStepMaxSplit][2];
#pragma unroll
      for (int sp = 0; sp < kStepMaxSplit; sp++) {
        const float* ps = pb + (size_t)sp * (hd + 4);
        ms[sp] = sp < nsplit ? __ldcg(ps) : -INFINITY;
        ls[sp] = sp < nsplit ? __ldcg(ps + 1) : 0.0f;
#pragma unroll
        for (int j = 0; j < 2; j++)
          ov[sp][j] = sp < nsplit ? __ldcg(reinterpret_cast<const float4*>(ps + 4 + i0) + j)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float M = -INFINITY;
#pragma unroll
      for (int sp = 0; sp < kStepMaxSplit; sp++) M = fmaxf(M, ms[sp]);
      float L = 0.0f;
#pragma unroll
      for (int sp = 0; sp < kStepMaxSplit; sp++) {
        if (ms[sp] == -INFINITY) continue;
        const float f = expf(ms[sp] - M);
        L = fmaf(ls[sp], f, L);
#pragma unroll
        for (int j = 0; j < 2; j++) {
          xv[r][4 * j] = fmaf(ov[sp][j].x, f, xv[r][4 * j]);
          xv[r][4 * j + 1] = fmaf(ov[sp][j].y, f, xv[r][4 * j + 1]);
          xv[r][4 * j + 2] = fmaf(ov[sp][j].z, f, xv[r][4 * j + 2]);
          xv[r][4 * j + 3] = fmaf(ov[sp][j].w, f, xv[r][4 * j + 3]);
        }
      }
      const float inv = 1.0f / L;
#pragma unroll
      for (int j = 0; j < EPT; j++) xv[r][j] = xv[r][j] * inv;
    } else {
#pragma unroll
      for (int i = 0; i < EPT; i += 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + base + i));
        xv[r][i] = v.x; xv[r][i + 1] = v.y; xv[r][i + 2] = v.z; xv[r][i + 3] = v.w;
      }
      if constexpr (MULTI) {
        for (int s2 = 1; s2 < nsrc; s2++) {
#pragma unroll
          for (int i = 0; i < EPT; i += 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (size_t)s2 * sstride + base + i));
            xv[r][i] = __fadd_rn(xv[r][i], v.x);
            xv[r][i + 1] = __fadd_rn(xv[r][i + 1], v.y);
            xv[r][i + 2] = __fadd_rn(xv[r][i + 2], v.z);
            xv[r][i + 3] = __fadd_rn(xv[r][i + 3], v.w);
          }
        }
      }
    }
  }
  if (R <= 2 && norm_w) {  // RMSNorm inputs: d <= 8192
    // the weights are requested before the reduction, so both loads overlap
    float wv[R][EPT];
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int b = (cc.ctid + r * kStepConsumers) >> 2;
#pragma unroll
      for (int i = 0; i < EPT; i += 4) {
        const float4 w = b < nb ? __ldg(reinterpret_cast<const float4*>(norm_w + b * 32 + q * EPT + i))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        wv[r][i] = w.x; wv[r][i + 1] = w.y; wv[r][i + 2] = w.z; wv[r][i + 3] = w.w;
      }
    }
    float ss = 0.0f;
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int i = 0; i < EPT; i++) ss = fmaf(xv[r][i], xv[r][i], ss);
    ss = warp_sum(ss);
    if (cc.lane == 0) cc.s_red[cc.cw] = ss;  // added up after the closing barrier
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int i = 0; i < EPT; i++) xv[r][i] = __fmul_rn(xv[r][i], wv[r][i]);
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int b = (cc.ctid + r * kStepConsumers) >> 2;
    const bool mine = b < nb;
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < EPT; j++) amax = fmaxf(amax, fabsf(xv[r][j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const bool live = amax >= 1e-30f;
    const int e = (int)((__float_as_uint(amax) >> 23) & 255u) - 126;
    const float sc = live ? pow2i(22 - e) : 0.0f;
    int s0 = 0, s1 = 0, s2 = 0;
    PlaneBlock* d = dst + b;
#pragma unroll
    for (int w = 0; w < 2; w++) {
      int d0[4], d1[4], d2[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int m = __float2int_rn(xv[r][4 * w + i] * sc);
        d0[i] = sext8(m);
        const int m1 = (m - d0[i]) >> 8;
        d1[i] = sext8(m1);
        d2[i] = (m1 - d1[i]) >> 8;
        s0 += d0[i];
        s1 += d1[i];
        s2 += d2[i];
      }
      if (mine) {
        d->pl[0][q * 2 + w] = (int)pack_low_bytes(d0[0], d0[1], d0[2], d0[3]);
        d->pl[1][q * 2 + w] = (int)pack_low_bytes(d1[0], d1[1], d1[2], d1[3]);
        d->pl[2][q * 2 + w] = (int)pack_low_bytes(d2[0], d2[1], d2[2], d2[3]);
      }
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (mine && q == 0) {
      d->nsum[0] = -s0;
      d->nsum[1] = -s1;
      d->nsum[2] = -s2;
      d->c0 = live ? pow2i(e - 22) : 0.0f;
    }
  }
  cbar();
  if (R <= 2 && norm_w) {
    float t = 0.0f;
    for (int w = 0; w < kStepConsumerWarps; w++) t += cc.s_red[w];
    return 1.0f / sqrtf(t / (float)(nb * 32) + eps);
  }
  return 1.0f;
}
template <bool MULTI>
SS_DEVINL float build_block_planes(const float* src, int nsrc, int sstride, const float* norm_w,
                                   const float* att, int nsplit, int hd, int nb, float eps,
                                   PlaneBlock* dst, ConsumerCtx& cc) {
  constexpr int per = kStepConsumers / 4;  // blocks per round
  if (nb <= per)
    return build_block_planes_r<1, MULTI>(src, nsrc, sstride, norm_w, att, nsplit, hd, nb, eps, dst, cc);
  else if (nb <= 2 * per)
    return build_block_planes_r<2, MULTI>(src, nsrc, sstride, norm_w, att, nsplit, hd, nb, eps, dst, cc);
  else if (nb <= 3 * per)
    return build_block_planes_r<3, MULTI>(src, nsrc, sstride, norm_w, att, nsplit, hd, nb, eps, dst, cc);
  else
    return build_block_planes_r<4, MULTI>(src, nsrc, sstride, norm_w, att, nsplit, hd, nb, eps, dst, cc);
}

// Consumes this CTA's tiles of `m` from the ring: red[wl * rows_cta + lr] gets
// the partial sum of local row lr over the 32 blocks of consumer warp wl of a
// row group.  Returns rows_cta, or -1 on abort.
template <int TYPE, bool MULTI>
SS_DEVINL int step_gemv(const StepParams& p, const StepSmem& sm, ConsumerCtx& cc, const TMat& m,
                        const float* src, int nsrc, const float* norm_w, float* red, int phase,
                        int pos) {
  const int ncta = gridDim.x, cta = blockIdx.x;
  constexpr int QB = TYPE == kQ4_0 ? 16 : 32;
  const int nb = m.nb, wpr = step_wpr(nb), RG = kStepConsumerWarps / wpr;
  const int rg = cc.cw / wpr, wl = cc.cw - rg * wpr;
  const int blk = wl * 32 + cc.lane;
  const bool active = rg < RG && blk < nb;
  int t0, t1;
  part_range(m.ntiles, cta, ncta, t0, t1);
  const int rows_cta = (t1 - t0) * kStepTileRows;

  // this thread's block of the input planes, built in shared memory; the
  // RMSNorm scale (1 without a norm) joins each block's unit
  const float nscale =
      build_block_planes<MULTI>(src, nsrc, p.d, norm_w, src == nullptr ? p.att_part : nullptr,
                                step_nsplit(p, pos), p.hd, nb, p.eps, reinterpret_cast<PlaneBlock*>(red), cc);
  int pl[3][8];
  int init[3];
  float c0;
  {
    const int4* sp = reinterpret_cast<const int4*>(reinterpret_cast<const PlaneBlock*>(red) +
                                                   (active ? blk : 0));
#pragma unroll
    for (int p4 = 0; p4 < 6; p4++) {
      const int4 v = active ? sp[p4] : make_int4(0, 0, 0, 0);
      pl[p4 >> 1][(p4 & 1) * 4 + 0] = v.x;
      pl[p4 >> 1][(p4 & 1) * 4 + 1] = v.y;
      pl[p4 >> 1][(p4 & 1) * 4 + 2] = v.z;
      pl[p4 >> 1][(p4 & 1) * 4 + 3] = v.w;
    }
    const int4 v = active ? sp[6] : make_int4(0, 0, 0, 0);
    const int zp = TYPE == kQ4_0 ? 8 : 0;
    init[0] = zp * v.x;  // stored: -sum_j digit_pj
    init[1] = zp * v.y;
    init[2] = zp * v.z;
    c0 = __int_as_float(v.w) * nscale;
  }
  cbar();  // every consumer has its planes before the scratch turns into partial sums
  bool bad = false;

  const int bsafe = active ? blk : 0;
  const uint32_t q_off = (uint32_t)(rg * m.tile_bytes + bsafe * QB);
  const uint32_t s_off = (uint32_t)(rg * m.tile_bytes + kStepTileRows * nb * QB + bsafe * 8);
  const uint32_t rstride = (uint32_t)(nb * QB);
  const uint32_t ring0 = smem_addr(sm.ring);
  const uint32_t slot_bytes = (uint32_t)p.slot_bytes;
  const int nslots = p.nslots;
  const bool writer = (cc.lane & 7) == 0;
  const int my_row = row_of_lane<4>(cc.lane);
  float* red_w = red + wl * rows_cta + my_row;

  for (int s = 0; t0 + s * RG < t1; s++) {
    const int slot = cc.slot;
    const uint32_t par = cc.phase;
    const uint32_t fb = smem_addr(sm.full + slot);
    if (!warp_wait_phase(p, fb, par)) {  // leave the loop; every warp still meets the barrier below
      bad = true;
      break;
    }
    if (cc.ctid == 0 && p.trace) {
      if (s == 0) trace_mark(p, phase, 4);
      if (t0 + (s + 1) * RG >= t1) trace_mark(p, phase, 5);
    }
    const int tl = s * RG + rg;  // tile of this row group, local to the CTA range
    const bool has = rg < RG && t0 + tl < t1;
    const uint32_t st = ring0 + (uint32_t)slot * slot_bytes;
    uint4 qa[4], qb[4];
    uint2 scv = make_uint2(0u, 0u);
    if (has) {
      asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(scv.x), "=r"(scv.y) : "r"(st + s_off));
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t a = st + q_off + (uint32_t)i * rstride;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(qa[i].x), "=r"(qa[i].y), "=r"(qa[i].z), "=r"(qa[i].w) : "r"(a));
        if constexpr (TYPE == kQ8_0)
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(qb[i].x), "=r"(qb[i].y), "=r"(qb[i].z), "=r"(qb[i].w) : "r"(a + 16));
      }
    }
    __syncwarp();
    if (cc.lane == 0) mbar_arrive(smem_addr(sm.empty + slot));
    if (++cc.slot == nslots) { cc.slot = 0; cc.phase ^= 1u; }
    if (has) {
      const __half2 h01 = *reinterpret_cast<const __half2*>(&scv.x);
      const __half2 h23 = *reinterpret_cast<const __half2*>(&scv.y);
      const float2 d01 = __half22float2(h01), d23 = __half22float2(h23);
      const float dsc[4] = {d01.x, d01.y, d23.x, d23.y};
      float acc[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float r;
        if constexpr (TYPE == kQ4_0) r = step_dot_q4(qa[i], pl, init);
        else r = step_dot_q8(qa[i], qb[i], pl);
        acc[i] = r * (c0 * dsc[i]);
      }
      const float v = warp_reduce_rows<4>(acc, cc.lane);
      if (writer) red_w[tl * kStepTileRows] = v;
    }
  }
  if (cc.ctid == 0) trace_mark(p, phase, 6);
  bad = cbar_any(bad);  // also: every warp's partial sums are in `red`
  if (bad) {
    if (cc.ctid == 0) *cc.s_abort = 1;
    return -1;
  }
  return rows_cta;
}

SS_DEVINL float row_total(const float* red, int wpr, int rows_cta, int lr) {
  float s = 0.0f;
  for (int w = 0; w < wpr; w++) s += red[w * rows_cta + lr];
  return s;
}


// Residual h of row r under tensor parallelism: the sum of nsrc partials
// (stride d) in rank order.
SS_DEVINL float h_sum(const float* hs, int nsrc, int d, int r) {
  float v = __ldcg(hs + r);
  for (int q = 1; q < nsrc; q++) v = __fadd_rn(v, __ldcg(hs + (size_t)q * d + r));
  return v;
}
// Tensor parallelism: this rank's partial rows of the CTA (rank 0 adds the old
// h, read from (hs, nsrc); h_pre is its value at the thread's first row) go to
// slot `xs` of every rank's exchange block.
SS_DEVINL void epi_residual_tp(const StepParams& p, const StepTp& t, ConsumerCtx& cc, const float* red,
                               int wpr, int rows_cta, int r0, float h_pre, const float* hs, int nsrc, int xs) {
  const int r1 = min(r0 + rows_cta, p.d);
  for (int r = r0 + cc.ctid; r < r1; r += kStepConsumers) {
    float v = row_total(red, wpr, rows_cta, r - r0);
    if (t.rank == 0) v = __fadd_rn(v, r == r0 + cc.ctid ? h_pre : h_sum(hs, nsrc, p.d, r));
    for (int q = 0; q < t.tp; q++) {
      float* dst = xchg_h(t, q, xs, p.d) + (size_t)t.rank * p.d + r;
      if (SS_TP_OK(t, q, dst, 4, 20u + xs)) __stcg(dst, v);
    }
  }
}

// h[r] += v[r] for the CTA's rows (layer_scheduler.c:484, :566).
SS_DEVINL void epi_residual(const StepParams& p, ConsumerCtx& cc, const float* red, int wpr,
                            int rows_cta, int r0, float h_pre) {
  const int r1 = min(r0 + rows_cta, p.d);
  for (int r = r0 + cc.ctid; r < r1; r += kStepConsumers)
    __stcg(p.h + r, __fadd_rn(row_total(red, wpr, rows_cta, r - r0),
                              r == r0 + cc.ctid ? h_pre : __ldcg(p.h + r)));
}

// ---------------------------------------------------------------- attention
//
// Task (kv head kvh, position split): positions [t0, t1) of 0..pos split
// evenly over nsplit tasks.  The cached rows t < pos of the split never change
// during a step, so the producer streams them into the ring while the QKV
// phase runs, in "attention stages" of up to step_att_rows rows:
//   [K rows: rows x HD int8][V rows][K scales][V scales]
// each scale block covering positions ts & ~3 .. (te + 3) & ~3 (16-byte aligned
// copies).  Row `pos` is this step's own K/V, encoded from the QKV output.

// Scores, online-softmax update and PV for `nr` rows whose int8 K / V (row
// stride HD) and scales are in shared memory (layer_scheduler.c:415-468,
// softmax tensor.c:154-173 in online form: running max m, sum l, o).  Every
// consumer calls it; `sc` holds the group's scores, `ml` m[8], l[8], corr[8].
template <int HD>
SS_DEVINL void att_rows(const StepParams& p, ConsumerCtx& cc, const int8_t* K, const int8_t* V,
                        const float* ksc, const float* vsc, int nr, const float* q, float* sc,
                        int scs, float* ml, int G, float (&o)[2]) {
  constexpr int DPL = HD / 32;
  constexpr int U = 4;  // rows per warp at a time: their shuffle reductions overlap
  for (int rb = cc.cw; rb < nr; rb += U * kStepConsumerWarps) {
    float kd[U][DPL];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int r = rb + u * kStepConsumerWarps;
      const float s = r < nr ? ksc[r] : 0.0f;
#pragma unroll
      for (int i = 0; i < DPL; i++)
        kd[u][i] = r < nr ? __fmul_rn((float)K[r * HD + cc.lane * DPL + i], s) : 0.0f;
    }
    for (int g = 0; g < G; g++) {
      float ds[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        ds[u] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; i++) ds[u] = fmaf(q[g * HD + cc.lane * DPL + i], kd[u][i], ds[u]);
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1)
#pragma unroll
        for (int u = 0; u < U; u++) ds[u] += __shfl_xor_sync(0xffffffffu, ds[u], o2);
      if (cc.lane == 0) {
#pragma unroll
        for (int u = 0; u < U; u++) {
          const int r = rb + u * kStepConsumerWarps;
          if (r < nr) sc[g * scs + r] = __fmul_rn(ds[u], p.attn_scale);
        }
      }
    }
  }
  cbar();
  if (cc.cw < G) {
    const int g = cc.cw;
    float mt = -INFINITY;
    for (int r = cc.lane; r < nr; r += 32) mt = fmaxf(mt, sc[g * scs + r]);
    mt = warp_max(mt);
    const float mold = ml[g];
    const float mnew = fmaxf(mold, mt);
    float lt = 0.0f;
    for (int r = cc.lane; r < nr; r += 32) {
      const float e = expf(sc[g * scs + r] - mnew);
      sc[g * scs + r] = e;
      lt += e;
    }
    lt = warp_sum(lt);
    if (cc.lane == 0) {
      const float c = mold == -INFINITY ? 0.0f : expf(mold - mnew);
      ml[16 + g] = c;
      ml[8 + g] = fmaf(ml[8 + g], c, lt);
      ml[g] = mnew;
    }
  }
  cbar();
  // PV: item (g, i) of the group's outputs; with fewer items than consumers,
  // `ngrp` thread groups take interleaved rows (reduced at the end of the task)
  const int items = G * HD;
  const int ngrp = items >= kStepConsumers ? 1 : kStepConsumers / items;
  const int grp = items >= kStepConsumers ? 0 : cc.ctid / items;
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int item = items >= kStepConsumers ? cc.ctid + k * kStepConsumers : cc.ctid % items;
    if (item < items && (k == 0 || items > kStepConsumers)) {
      const int g = item / HD, i = item - g * HD;
      float acc = o[k] * ml[16 + g];
      for (int r = grp; r < nr; r += ngrp)
        acc = fmaf(sc[g * scs + r], __fmul_rn((float)V[r * HD + i], vsc[r]), acc);
      o[k] = acc;
    }
  }
}

// One task: append this token's K/V slice of the kv head when the split holds
// `pos`, attention over the split's positions (ring stages, then row pos) for
// the group's query heads, partial (m, l, o) to att_part.  The O phase merges
// the splits.  Returns false on abort.
// This thread's share of a task's inputs, loaded before the k / v maxima are
// known: q items ctid and ctid + 512 of the group, and element ctid of the kv
// head's current k and v rows.
struct AttInputs {
  float q[2];
  float k, v;
};
SS_DEVINL AttInputs att_load_inputs(const StepParams& p, const ConsumerCtx& cc, int task, int pos,
                                    int hd) {
  AttInputs in;
  in.q[0] = in.q[1] = in.k = in.v = 0.0f;
  const int G = p.nh / p.nkv;
  if (task >= p.nkv * step_nsplit(p, pos)) return in;  // this CTA has no task: nothing to load
  int kvh, split, t0, t1;
  step_att_task(p, task, pos, kvh, split, t0, t1);
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int item = cc.ctid + k * kStepConsumers;
    in.q[k] = item < G * hd ? __ldcg(p.qkv_out + (size_t)kvh * G * hd + item) : 0.0f;
  }
  const bool has_pos = pos >= t0 && pos < t1;
  in.k = has_pos && cc.ctid < hd ? __ldcg(p.qkv_out + p.qd + kvh * hd + cc.ctid) : 0.0f;
  in.v = has_pos && cc.ctid < hd ? __ldcg(p.qkv_out + p.qd + p.kvd + kvh * hd + cc.ctid) : 0.0f;
  return in;
}

template <int HD>
SS_DEVINL bool step_attention_task(const StepParams& p, const StepSmem& sm, ConsumerCtx& cc,
                                   float* scratch, int layer, int pos, int task, float k_scale,
                                   float v_scale, int phase, const AttInputs& in) {
  const int G = p.nh / p.nkv;
  int kvh, split, t0, t1;
  step_att_task(p, task, pos, kvh, split, t0, t1);
  const int tend = min(t1, pos);  // cached rows [t0, tend); row pos separately
  const int R = step_att_rows(p.slot_bytes, HD);
  const size_t lrow = (size_t)layer * p.ctx;

  // scratch: q[G][HD] | sc[max(G * R, consumers)] (scores, then the row-group
  // reduction) | ml[24] | kcur[HD], vcur[HD] (int8)
  float* q = scratch;
  float* sc = q + G * HD;
  float* ml = sc + max(G * R, kStepConsumers);
  int8_t* kcur = reinterpret_cast<int8_t*>(ml + 24);
  int8_t* vcur = kcur + HD;
#pragma unroll
  for (int k = 0; k < 2; k++)
    if (cc.ctid + k * kStepConsumers < G * HD) q[cc.ctid + k * kStepConsumers] = in.q[k];
  if (cc.ctid < 8) {
    ml[cc.ctid] = -INFINITY;
    ml[8 + cc.ctid] = 0.0f;
  }
  const bool has_pos = pos >= t0 && pos < t1;
  if (has_pos) {
    // kv_turboquant_encode (layer_scheduler.c:101-118) of this kv head's slice
    const float kinv = k_scale > 0.0f ? 1.0f / k_scale : 0.0f;
    const float vinv = v_scale > 0.0f ? 1.0f / v_scale : 0.0f;
    if (cc.ctid < HD) {
      const int i = cc.ctid;
      const int8_t kq = kv_encode(in.k, kinv), vq = kv_encode(in.v, vinv);
      kcur[i] = kq;
      vcur[i] = vq;
      p.kc[lrow * p.kvd + ((size_t)kvh * p.ctx + pos) * HD + i] = kq;
      p.vc[lrow * p.kvd + ((size_t)kvh * p.ctx + pos) * HD + i] = vq;
    }
    if (cc.ctid == 0 && kvh == 0) {
      p.ks[lrow + pos] = k_scale;
      p.vs[lrow + pos] = v_scale;
    }
  }
  cbar();

  float o[2] = {0.0f, 0.0f};
  const uint32_t ring0 = smem_addr(sm.ring);
  bool bad = false;
  bool pos_done = false;
  for (int ts = t0; ts < tend; ts += R) {
    const int nr = min(R, tend - ts);
    // every warp agrees before att_rows (which has consumer barriers)
    if (cbar_any(!warp_wait_phase(p, smem_addr(sm.full + cc.slot), cc.phase))) {
      bad = true;
      break;
    }
    if (cc.ctid == 0 && ts == t0) trace_mark(p, phase, 4);
    uint8_t* st = sm.ring + (size_t)cc.slot * p.slot_bytes;
    int8_t* K = reinterpret_cast<int8_t*>(st);
    int8_t* V = K + R * HD;
    const int sa = ts & ~3;
    float* ksc = reinterpret_cast<float*>(st + step_att_ks_off(R, HD)) + (ts - sa);
    float* vsc = reinterpret_cast<float*>(st + step_att_vs_off(R, HD)) + (ts - sa);
    int n = nr;
    if (has_pos && ts + nr == tend && nr < R) {
      // row pos joins the last stage (the slot is ours until released; the
      // scale blocks have room past the copied range)
      for (int i = cc.ctid; i < HD; i += kStepConsumers) {
        K[nr * HD + i] = kcur[i];
        V[nr * HD + i] = vcur[i];
      }
      if (cc.ctid == 0) {
        ksc[nr] = k_scale;
        vsc[nr] = v_scale;
      }
      // these generic writes must be ordered before the producer's next bulk
      // copy (async proxy) into this slot
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      pos_done = true;
      n = nr + 1;
      cbar();
    }
    att_rows<HD>(p, cc, K, V, ksc, vsc, n, q, sc, R, ml, G, o);
    __syncwarp();
    if (cc.lane == 0) mbar_arrive(smem_addr(sm.empty + cc.slot));
    if (++cc.slot == p.nslots) { cc.slot = 0; cc.phase ^= 1u; }
    cbar();  // scores of this stage consumed before the next overwrites them
  }
  (void)ring0;
  if (bad) return false;
  if (cc.ctid == 0) trace_mark(p, phase, 5);
  if (has_pos && !pos_done) {
    att_rows<HD>(p, cc, kcur, vcur, &k_scale, &v_scale, 1, q, sc, R, ml, G, o);
    cbar();
  }
  const int items = G * HD;
  if (items < kStepConsumers) {
    // sum the row groups' partial outputs (groups in order)
    float* red = sc;  // scores are consumed; [ngrp][items]
    red[cc.ctid] = o[0];
    cbar();
    if (cc.ctid < items) {
      float t = 0.0f;
      for (int j = 0; j < kStepConsumers / items; j++) t += red[j * items + cc.ctid];
      o[0] = t;
    }
  }
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int item = cc.ctid + k * kStepConsumers;
    if (item < items) {
      const int g = item / HD, i = item - g * HD;
      float* part = p.att_part + ((size_t)(kvh * G + g) * step_nsplit(p, pos) + split) * (HD + 4);
      __stcg(part + 4 + i, o[k]);
      if (i == 0) {
        __stcg(part, ml[g]);
        __stcg(part + 1, ml[8 + g]);
      }
    }
  }
  if (cc.ctid == 0) trace_mark(p, phase, 6);
  return true;
}

// ---------------------------------------------------------------- kernel

template <int TYPE, int HTYPE, int HD, bool TP>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepParams p, const StepTp t) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ int s_cabort_v;
  __shared__ float s_red[32];
  __shared__ int s_flag[4];
  __shared__ unsigned long long s_best[kStepConsumerWarps];
  __shared__ unsigned long long s_epoch;  // tensor parallelism: steps this rank ran before
  volatile int* s_cabort = &s_cabort_v;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ncta = gridDim.x, cta = blockIdx.x;

  StepSmem sm;
  sm.ring = smem_raw;
  sm.full = reinterpret_cast<uint64_t*>(smem_raw + (size_t)p.nslots * p.slot_bytes);
  sm.empty = sm.full + p.nslots;
  sm.scratch = reinterpret_cast<float*>(smem_raw + (size_t)p.nslots * p.slot_bytes + 128);

  const int pos = *reinterpret_cast<volatile int*>(p.d_pos);
  if (pos < 0 || pos >= p.ctx) {
    if (tid == 0 && cta == 0) atomicOr(p.err, 1);
    return;  // uniform across the grid: nothing started
  }
  {
    // the scratch must hold the attention task's buffers (the host sizes it
    // with the same function); uniform across the grid
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    const size_t need = (size_t)p.nslots * p.slot_bytes + 128 +
                        step_att_scratch_bytes(p.nh / p.nkv, HD, p.slot_bytes);
    if (need > dyn) {
      if (tid == 0 && cta == 0) atomicOr(p.err, 16);
      return;
    }
  }
  if (tid == 0) {
    s_cabort_v = 0;
    for (int i = 0; i < p.nslots; i++) {
      mbar_init(smem_addr(sm.full + i), 1);
      mbar_init(smem_addr(sm.empty + i), kStepConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp < kStepProducerThreads / 32) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kStepProducerRegs));
    if (warp == 0) step_producer(p, sm, s_cabort, lane, pos);
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kStepConsumerRegs));

  ConsumerCtx cc;
  cc.ctid = tid - kStepProducerThreads;
  cc.lane = lane;
  cc.cw = warp - kStepProducerThreads / 32;
  cc.slot = 0;
  cc.phase = 0;
  cc.s_abort = s_cabort;
  cc.s_red = s_red;
  cc.s_flag = s_flag;
  float* red = sm.scratch;
  const int nph = step_phase_count(p.L);
  if constexpr (TP) {
    if (cc.ctid == 0)  // read by consumer thread 0 only (its barrier waits, the argmax)
      s_epoch = *reinterpret_cast<volatile unsigned long long*>(xchg_u64(t, t.rank, StepXchg::kStep));
  }

  for (int k = 0; k < nph; k++) {
    int kind, layer;
    step_phase(k, p.L, kind, layer);
    if constexpr (TP) {
      if (cc.ctid == 0) SS_TP_MARK(t, StepDbg::kCons + cta, 16u * (unsigned)(k + 1) + 0u);
      if (k > 0) {
        int pkind, player;
        step_phase(k - 1, p.L, pkind, player);
        unsigned nloc, ncross;
        step_bar_counts(k, nloc, ncross);
        if (!(step_cross_wait(pkind) ? step_xwait(p, t, cc, s_epoch, ncross)
                                     : step_grid_wait(p, cc, nloc * (unsigned)ncta)))
          return;
      }
      if (cc.ctid == 0) SS_TP_MARK(t, StepDbg::kCons + cta, 16u * (unsigned)(k + 1) + 1u);
    } else {
      if (k > 0 && !step_grid_wait(p, cc, (unsigned)(k * ncta))) return;
    }
    if (cc.ctid == 0) trace_mark(p, k, 0);

    if (kind == kPhEmbed) {
      // h = token_embd[token] (layer_scheduler.c:584-587)
      int tok = p.seq_tokens[pos];
      if (tok < 0 || tok >= p.vocab) {
        if (cc.ctid == 0 && cta == 0) atomicOr(p.err, 2);
        tok = 0;
      }
      const float* row = p.embd + (size_t)tok * p.d;
      for (int i = cta * kStepConsumers + cc.ctid; i < p.d; i += ncta * kStepConsumers)
        __stcg(p.h + i, row[i]);
      if (cc.ctid == 0) trace_mark(p, k, 2);
      step_grid_arrive(p, cc);
      continue;
    }

    if (kind == kPhAtt) {
      // this step's q / k / v of the CTA's task, requested before the maxima
      const AttInputs ain = att_load_inputs(p, cc, cta, pos, HD);
      // this position's int8 scales need max |k| / |v| over the whole kv_dim
      // (tensor parallelism: over every rank's CTAs; only a CTA whose task
      // holds this position encodes a K/V row, so only such a CTA waits for
      // the other ranks' QKV phase -- the phase started at a local barrier)
      float mk = 0.0f, mv = 0.0f;
      const float2* amp = p.amax_part;
      int nam = ncta;
      bool need_scale = true;
      if constexpr (TP) {
        amp = xchg_am(t, t.rank);
        nam = ncta * t.tp;
        need_scale = false;
        for (int task = cta; task < p.nkv * step_nsplit(p, pos); task += ncta) {
          int kvh, split, a0, a1;
          step_att_task(p, task, pos, kvh, split, a0, a1);
          need_scale = need_scale || (pos >= a0 && pos < a1);
        }
        if (need_scale) {  // uniform across the CTA
          unsigned nloc, ncross;
          step_bar_counts(k, nloc, ncross);  // ncross counts this layer's QKV
          if (!step_xwait(p, t, cc, s_epoch, ncross)) return;
        }
      }
      if (need_scale) {
        for (int i = cc.ctid; i < nam; i += kStepConsumers) {
          const float2 a = __ldcg(amp + i);
          mk = fmaxf(mk, a.x);
          mv = fmaxf(mv, a.y);
        }
        mk = warp_max(mk);
        mv = warp_max(mv);
        if (cc.lane == 0) { s_red[cc.cw] = mk; s_red[16 + cc.cw] = mv; }
        cbar();
        mk = 0.0f;
        mv = 0.0f;
        for (int w = 0; w < kStepConsumerWarps; w++) {
          mk = fmaxf(mk, s_red[w]);
          mv = fmaxf(mv, s_red[16 + w]);
        }
      }
      const float k_scale = mk / 127.0f, v_scale = mv / 127.0f;  // layer_scheduler.c:109-110
      bool ok = true;
      for (int task = cta; ok && task < p.nkv * step_nsplit(p, pos); task += ncta) {
        ok = step_attention_task<HD>(p, sm, cc, sm.scratch, layer, pos, task, k_scale, v_scale, k,
                                     task == cta ? ain : att_load_inputs(p, cc, task, pos, HD));
        cbar();
      }
      if (!ok) {
        if (cc.ctid == 0) *s_cabort = 1;
        return;
      }
      if (cc.ctid == 0) trace_mark(p, k, 2);
      step_grid_arrive(p, cc);
      continue;
    }

    // ---- matvec phases
    const TMat m = step_phase_mat(p, kind, layer);
    // this phase's input: RMSNorm(h) for QKV / GU / lm_head, else the
    // attention output (O: merged from the split partials, src == nullptr) or
    // the SwiGLU activations (down)
    const float* hin = p.h;
    int nsrc = 1;
    if constexpr (TP) hin = step_hsrc(p, t, kind, layer, nsrc);
    const float* src = kind == kPhO ? nullptr : kind == kPhDown ? p.act : hin;
    if (kind == kPhO || kind == kPhDown) nsrc = 1;
    const float* nw = kind == kPhQKV  ? p.attn_norm + (size_t)layer * p.d
                      : kind == kPhGU ? p.ffn_norm + (size_t)layer * p.d
                      : kind == kPhHead ? p.out_norm : nullptr;
    int t0, t1;
    part_range(m.ntiles, cta, ncta, t0, t1);
    const int r0 = t0 * kStepTileRows;
    // the epilogue's other inputs (this thread's first row or row pair), requested
    // now so they arrive while the weights stream: the RoPE cos/sin (QKV) and the
    // residual h (O, DOWN -- no phase writes h between here and the epilogue)
    float2 cs_pre = make_float2(1.0f, 0.0f);
    float h_pre = 0.0f;
    {
      const int rows = (t1 - t0) * kStepTileRows;
      if (kind == kPhQKV) {
        const int r = r0 + 2 * cc.ctid, i = r % p.hd;
        if (2 * cc.ctid < rows && r < p.qd + p.kvd && i < p.rope_dim)
          cs_pre = __ldg(p.rope_tab + (size_t)pos * (p.rope_dim >> 1) + (i >> 1));
      } else if (kind == kPhO || kind == kPhDown) {
        if constexpr (TP) {
          if (t.rank == 0 && cc.ctid < rows && r0 + cc.ctid < p.d) {
            int nres;
            const float* hres = step_hsrc(p, t, kind, layer, nres);
            h_pre = h_sum(hres, nres, p.d, r0 + cc.ctid);
          }
        } else {
          if (cc.ctid < rows && r0 + cc.ctid < p.d) h_pre = __ldcg(p.h + r0 + cc.ctid);
        }
      }
    }
    int rows_cta;
    if (kind == kPhHead) rows_cta = step_gemv<HTYPE, TP>(p, sm, cc, m, src, nsrc, nw, red, k, pos);
    else rows_cta = step_gemv<TYPE, TP>(p, sm, cc, m, src, nsrc, nw, red, k, pos);
    if (rows_cta < 0) return;
    if constexpr (TP) {
      if (cc.ctid == 0) SS_TP_MARK(t, StepDbg::kCons + cta, 16u * (unsigned)(k + 1) + 2u);
    }
    if (cc.ctid == 0) trace_mark(p, k, 1);
    const int wpr = step_wpr(m.nb);

    if (kind == kPhQKV) {
      // RoPE (non-NeoX, tensor.c:249-274) on q and k rows; |k|, |v| maxima
      float mk = 0.0f, mv = 0.0f;
      const int qkv_rows = p.qd + 2 * p.kvd;
      for (int lp = cc.ctid; 2 * lp < rows_cta; lp += kStepConsumers) {
        const int r = r0 + 2 * lp;
        if (r >= qkv_rows) break;
        float a = row_total(red, wpr, rows_cta, 2 * lp);
        float b = row_total(red, wpr, rows_cta, 2 * lp + 1);
        if (r < p.qd + p.kvd) {
          const int i = r % p.hd;
          if (i < p.rope_dim) {
            const float2 cs = lp == cc.ctid ? cs_pre : p.rope_tab[(size_t)pos * (p.rope_dim >> 1) + (i >> 1)];
            const float na = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
            const float nb2 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
            a = na;
            b = nb2;
          }
          if (r >= p.qd) mk = fmaxf(mk, fmaxf(fabsf(a), fabsf(b)));
        } else {
          mv = fmaxf(mv, fmaxf(fabsf(a), fabsf(b)));
        }
        __stcg(p.qkv_out + r, a);
        __stcg(p.qkv_out + r + 1, b);
      }
      mk = warp_max(mk);
      mv = warp_max(mv);
      if (lane == 0) { s_red[cc.cw] = mk; s_red[16 + cc.cw] = mv; }
      cbar();
      if (cc.ctid == 0) {
        for (int w = 1; w < kStepConsumerWarps; w++) {
          mk = fmaxf(mk, s_red[w]);
          mv = fmaxf(mv, s_red[16 + w]);
        }
        if constexpr (TP) {
          for (int q = 0; q < t.tp; q++) {
            float2* dst = xchg_am(t, q) + t.rank * ncta + cta;
            if (SS_TP_OK(t, q, dst, 8, 30u)) __stcg(dst, make_float2(mk, mv));
          }
        } else {
          __stcg(p.amax_part + cta, make_float2(mk, mv));
        }
      }
    } else if (kind == kPhO) {
      if constexpr (TP) {
        int nres;
        const float* hres = step_hsrc(p, t, kind, layer, nres);
        epi_residual_tp(p, t, cc, red, wpr, rows_cta, r0, h_pre, hres, nres, 0);
      } else {
        epi_residual(p, cc, red, wpr, rows_cta, r0, h_pre);
      }
    } else if (kind == kPhGU) {
      // act = up * g / (1 + expf(-g)) (layer_scheduler.c:533-549)
      const int a0 = r0 / 2, a1 = min((r0 + rows_cta) / 2, p.ff);
      for (int j = a0 + cc.ctid; j < a1; j += kStepConsumers) {
        const int lr = 2 * (j - a0);
        const float g = row_total(red, wpr, rows_cta, lr);
        const float u = row_total(red, wpr, rows_cta, lr + 1);
        __stcg(p.act + j, __fmul_rn(u, __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)))));
      }
    } else if (kind == kPhDown) {
      if constexpr (TP) {
        int nres;
        const float* hres = step_hsrc(p, t, kind, layer, nres);
        epi_residual_tp(p, t, cc, red, wpr, rows_cta, r0, h_pre, hres, nres, 1);
      } else {
        epi_residual(p, cc, red, wpr, rows_cta, r0, h_pre);
      }
    } else {  // kPhHead: logits, greedy argmax (tensor.c:318-328), next token
      unsigned long long best = 0;
      // tensor parallelism: this rank's vocabulary rows, global indices
      const int r1 = min(r0 + rows_cta, TP ? m.rows : p.vocab);
      for (int r = r0 + cc.ctid; r < r1; r += kStepConsumers) {
        const float v = row_total(red, wpr, rows_cta, r - r0);
        __stcg(p.logits + r, v);
        const unsigned long long pk = pack_argmax(v, TP ? t.vocab_off + r : r);
        best = pk > best ? pk : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      if (lane == 0) s_best[cc.cw] = best;
      cbar();
      if (cc.ctid == 0) {
        unsigned long long b = 0;
        for (int w = 0; w < kStepConsumerWarps; w++) b = s_best[w] > b ? s_best[w] : b;
        __stcg(p.am_part + cta, b);
        __threadfence();
        s_flag[1] = atomicAdd(p.am_cnt, 1u) == (unsigned)(ncta - 1);
      }
      cbar();
      if (s_flag[1] && cc.cw == 0) {
        __threadfence();
        unsigned long long b = 0;
        for (int i = lane; i < ncta; i += 32) {
          const unsigned long long v = __ldcg(p.am_part + i);
          b = v > b ? v : b;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
          b = other > b ? other : b;
        }
        bool ok = true;
        if constexpr (TP) {
          if (lane == 0) {
            // every rank's best to every rank, then the best of the tp
            SS_TP_MARK(t, StepDbg::kHead, 1u);
            for (int q = 0; q < t.tp; q++) {
              unsigned long long* dst = xchg_u64(t, q, StepXchg::kBest) + t.rank;
              if (SS_TP_OK(t, q, dst, 8, 40u)) __stcg(dst, b);
            }
            fence_acq_rel_sys();
            for (int q = 0; q < t.tp; q++)
              if (SS_TP_OK(t, q, xchg_u64(t, q, StepXchg::kHead), 8, 41u))
                red_relaxed_sys_add_u64(xchg_u64(t, q, StepXchg::kHead), 1ull);
            SS_TP_MARK(t, StepDbg::kHead, 2u);
            const unsigned long long epoch = s_epoch;
            const unsigned long long target = (epoch + 1ull) * (unsigned long long)t.tp;
            const unsigned long long* ctr = xchg_u64(t, t.rank, StepXchg::kHead);
            const long long c0 = clock64();
            while ((long long)(ld_relaxed_sys_u64(ctr) - target) < 0) {
              if (clock64() - c0 > xwait_budget(p)) {
                atomicOr(p.err, 32);
                atomicExch(p.abort_flag, 1u);
                ok = false;
                break;
              }
            }
            fence_acq_rel_sys();
            if (ok) {
              const unsigned long long* bs = xchg_u64(t, t.rank, StepXchg::kBest);
              for (int q = 0; q < t.tp; q++) {
                const unsigned long long v = __ldcg(bs + q);
                b = v > b ? v : b;
              }
              *xchg_u64(t, t.rank, StepXchg::kStep) = epoch + 1ull;
            }
            SS_TP_MARK(t, StepDbg::kHead, ok ? 3u : 4u);
          }
        }
        if (lane == 0 && ok) {
          const int tok = unpack_argmax_index(b);
          if (pos + 1 < p.ctx && pos + 1 >= *p.fixed_until) p.seq_tokens[pos + 1] = tok;
          p.seq_tokens[p.ctx] = tok;
          *p.d_pos = pos + 1;
          *p.am_cnt = 0u;
          *p.grid_bar = 0u;  // every CTA has passed its last grid barrier
        }
      }
      if (cc.ctid == 0) trace_mark(p, k, 2);
      return;
    }
    if (cc.ctid == 0) trace_mark(p, k, 2);
    if constexpr (TP) {
      if (cc.ctid == 0) SS_TP_MARK(t, StepDbg::kCons + cta, 16u * (unsigned)(k + 1) + 3u);
      if (kind != kPhO && kind != kPhDown) step_grid_arrive(p, cc);
      if (step_cross(kind)) step_xarrive(t, cc);
      if (cc.ctid == 0) SS_TP_MARK(t, StepDbg::kCons + cta, 16u * (unsigned)(k + 1) + 4u);
    } else {
      step_grid_arrive(p, cc);
    }
  }
}

}  // namespace ss
