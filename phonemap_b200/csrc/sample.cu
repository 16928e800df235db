// sample.cu -- ss_sample (SlipStream/src/core/tensor.c:363-451) on the device.
//
// The reference draws a token from a logits vector with four sequential fp32
// running sums in a fixed order: the softmax denominator (index order,
// tensor.c:161-165), the top-p walk over the probabilities sorted high to low
// (tensor.c:404-421), the renormalisation (index order, :426-433) and the CDF
// walk (index order, :437-448).  Each running sum rounds after every addition,
// and on a near-flat distribution a different summation order moves the top-p
// cutoff or the drawn index often, so this kernel keeps the reference's order
// exactly: one thread adds, in order, while the rest of the CTA produces the
// next tile of addends (the exponentials, the sorted keys, the filtered
// probabilities) in shared memory.  Everything else is parallel and exact: the
// maximum, the element-wise steps (IEEE division and multiplication, no
// contraction), and the ordering for top-k / top-p: with top-k a radix select
// of the k-th largest probability, then a shared-memory sort of the values at
// or above it (the only ones the top-p walk can add); with top-p alone a
// stable LSD radix sort of all of them.  Equal probabilities add the same
// values in any order, so ties need no particular order.
//
// One CTA of 1024 threads does the whole draw -- the running sums are the
// critical path and a single SM keeps the vectors (at most a few MB) in L2.
// The exponential is e^x evaluated in double precision and rounded once to
// float (the oracle restates the same steps); libm's expf, which the reference
// calls, rounds differently in about one input in 1,600, which reaches a drawn
// token only when that last bit moves a running sum across a threshold.
#include "sample.h"

#include <cfloat>
#include <cstdint>

namespace ss {
namespace {

constexpr int kSmpThreads = 1024;
constexpr int kSmpWarps = kSmpThreads / 32;
constexpr int kSmpTile = 4096;  // floats per tile of addends
constexpr int kSmpBins = 256;   // radix digit: 8 bits

struct SmpSmem {
  float tile[2][kSmpTile];              // addends: tile k in tile[k & 1]
  unsigned hist[kSmpWarps][kSmpBins];   // per-warp digit counts, then scatter cursors
  unsigned digit_base[kSmpBins];
  float redf[kSmpWarps];
  int redi[kSmpWarps];
  float bcast[4];
  int bcasti[4];
};

__host__ __device__ __forceinline__ size_t pad_n(int n) { return ((size_t)n + 63) & ~(size_t)63; }

// 1/i! for i = 0..13, each rounded to double.
__constant__ double kSmpInvFact[14] = {
    0x1.0000000000000p+0,  0x1.0000000000000p+0,  0x1.0000000000000p-1,  0x1.5555555555555p-3,
    0x1.5555555555555p-5,  0x1.1111111111111p-7,  0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13,
    0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22, 0x1.ae64567f544e4p-26,
    0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33};

// e^x rounded to float: k = rint(x log2 e); r = x - k ln2 with ln2 split into
// a 33-bit head (k * head exact for |k| < 2^20) and a tail; e^r by its Taylor
// series to degree 13 (truncation < 5e-18 for |r| <= ln2 / 2); times 2^k from
// the exponent bits; one rounding to float (float subnormals included).  Only
// IEEE basic operations and fma, so the oracle's C restatement rounds
// identically.
__device__ __forceinline__ float smp_exp(float xf) {
  if (xf != xf) return xf;
  if (xf < -200.0f) return 0.0f;
  if (xf > 200.0f) return __int_as_float(0x7f800000);
  const double x = (double)xf;
  const double k = rint(__dmul_rn(x, 0x1.71547652b82fep+0));
  double r = __fma_rn(-k, 0x1.62e42ff000000p-1, x);
  r = __fma_rn(-k, -0x1.718432a1b0e26p-35, r);
  double p = kSmpInvFact[13];
#pragma unroll
  for (int i = 12; i >= 0; i--) p = __fma_rn(p, r, kSmpInvFact[i]);
  const double s = __longlong_as_double((long long)((int)k + 1023) << 52);
  return __double2float_rn(__dmul_rn(p, s));
}

// Streams the addends fill(0..n-1) through shared memory to thread 0: warps
// 1..31 produce tile k + 1 while thread 0 runs eat(tile, first index, count)
// over tile k, in order.  eat returning true ends the stream (every thread
// leaves together: the end-of-tile barrier ORs the flag).
template <class Fill, class Eat>
__device__ __forceinline__ void smp_stream(int n, SmpSmem& sm, Fill fill, Eat eat) {
  const int tid = threadIdx.x;
  const int nt = (n + kSmpTile - 1) / kSmpTile;
  if (tid >= 32) {
    const int cnt = min(kSmpTile, n);
    for (int j = tid - 32; j < cnt; j += kSmpThreads - 32) sm.tile[0][j] = fill(j);
  }
  __syncthreads();
  for (int k = 0; k < nt; k++) {
    bool stop = false;
    if (tid >= 32) {
      if (k + 1 < nt) {
        const int base = (k + 1) * kSmpTile, cnt = min(kSmpTile, n - base);
        float* t = sm.tile[(k + 1) & 1];
        for (int j = tid - 32; j < cnt; j += kSmpThreads - 32) t[j] = fill(base + j);
      }
    } else if (tid == 0) {
      const int base = k * kSmpTile;
      stop = eat(sm.tile[k & 1], base, min(kSmpTile, n - base));
    }
    if (__syncthreads_or(stop)) break;
  }
}

// The sequential walks below read their tile 16 values at a time and issue the
// next 16 values' loads before the current 16 additions, so each addition
// waits only for the previous one.
struct Smp16 {
  float4 a, b, c, d;
};
__device__ __forceinline__ Smp16 smp_ld16(const float* t, int g) {
  const float4* t4 = reinterpret_cast<const float4*>(t) + 4 * g;
  return {t4[0], t4[1], t4[2], t4[3]};
}
__device__ __forceinline__ float smp_at(const Smp16& v, int k) {
  const float4& q = k < 4 ? v.a : k < 8 ? v.b : k < 12 ? v.c : v.d;
  const int r = k & 3;
  return r == 0 ? q.x : r == 1 ? q.y : r == 2 ? q.z : q.w;
}

// s + t[0] + t[1] + ... in order, each addition rounded.
__device__ __forceinline__ float smp_seq_sum(float s, const float* t, int cnt) {
  const int ng = cnt >> 4;
  Smp16 cur = ng > 0 ? smp_ld16(t, 0) : Smp16{};
  for (int g = 0; g < ng; g++) {
    const Smp16 nxt = smp_ld16(t, min(g + 1, ng - 1));
#pragma unroll
    for (int k = 0; k < 16; k++) s = __fadd_rn(s, smp_at(cur, k));
    cur = nxt;
  }
  for (int j = ng * 16; j < cnt; j++) s = __fadd_rn(s, t[j]);
  return s;
}

// The top-p walk over sorted probabilities (tensor.c:408-416): acc adds each
// positive value in order; the first value at which acc >= top_p is the
// cutoff.  Adding 0 in place of a non-positive (or NaN) value leaves acc
// unchanged, and acc never decreases, so 16 additions run back to back and one
// comparison of the last finds whether any reached top_p (the group is then
// walked again one value at a time).
__device__ __forceinline__ bool smp_topp_walk(float& acc, float& cut, const float* t, int cnt, float top_p) {
  auto pos = [](float v) { return v > 0.0f ? v : 0.0f; };
  const int ng = cnt >> 4;
  Smp16 cur = ng > 0 ? smp_ld16(t, 0) : Smp16{};
  for (int g = 0; g < ng; g++) {
    const Smp16 nxt = smp_ld16(t, min(g + 1, ng - 1));
    float a = acc;
#pragma unroll
    for (int k = 0; k < 16; k++) a = __fadd_rn(a, pos(smp_at(cur, k)));
    if (a >= top_p) {
      float b = acc;
#pragma unroll
      for (int k = 0; k < 16; k++) {
        b = __fadd_rn(b, pos(smp_at(cur, k)));
        if (b >= top_p) {
          cut = smp_at(cur, k);
          acc = b;
          return true;
        }
      }
    }
    acc = a;
    cur = nxt;
  }
  for (int j = ng * 16; j < cnt; j++) {
    acc = __fadd_rn(acc, pos(t[j]));
    if (acc >= top_p) {
      cut = t[j];
      return true;
    }
  }
  return false;
}

// The CDF walk (tensor.c:440-446): the first index whose running sum exceeds
// r, or -1.  The addends are non-negative, so a group of 16 can hold the first
// such index only if its last sum is not <= r (which also catches a NaN sum,
// which the per-value walk of the group then compares false, as the reference
// does).
__device__ __forceinline__ int smp_cdf_walk(float& cdf, const float* t, int cnt, float r) {
  const int ng = cnt >> 4;
  Smp16 cur = ng > 0 ? smp_ld16(t, 0) : Smp16{};
  for (int g = 0; g < ng; g++) {
    const Smp16 nxt = smp_ld16(t, min(g + 1, ng - 1));
    float c = cdf;
#pragma unroll
    for (int k = 0; k < 16; k++) c = __fadd_rn(c, smp_at(cur, k));
    if (!(c <= r)) {
      float b = cdf;
#pragma unroll
      for (int k = 0; k < 16; k++) {
        b = __fadd_rn(b, smp_at(cur, k));
        if (r < b) return 16 * g + k;
      }
    }
    cdf = c;
    cur = nxt;
  }
  for (int j = ng * 16; j < cnt; j++) {
    cdf = __fadd_rn(cdf, t[j]);
    if (r < cdf) return j;
  }
  return -1;
}

// Order-preserving compaction of the filtered probabilities that are not 0
// (NaN included) into cv / ci (value, index); returns their count.  A running
// sum in index order skips exactly these zeros: every addend is +0 or
// positive, so adding +0 leaves the sum's bits unchanged, and the CDF walk can
// first exceed r only where its sum grows.
template <class Filter>
__device__ int smp_compact(int n, Filter filter, float* cv, int* ci, SmpSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  int total = 0;
  for (int base = 0; base < n; base += 8 * kSmpThreads) {
    const int i0 = base + 8 * tid;
    float q[8];
    int c = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      q[j] = i0 + j < n ? filter(i0 + j) : 0.0f;
      c += q[j] != 0.0f;
    }
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    if (lane == 31) sm.redi[w] = inc;
    __syncthreads();
    if (w == 0) {
      const int v = sm.redi[lane];
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
      }
      sm.redi[lane] = x - v;
      if (lane == 31) sm.bcasti[0] = x;
    }
    __syncthreads();
    int off = total + sm.redi[w] + inc - c;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (q[j] != 0.0f) {
        cv[off] = q[j];
        ci[off] = i0 + j;
        off++;
      }
    total += sm.bcasti[0];
    __syncthreads();
  }
  return total;
}

// Descending sort of n keys (non-negative floats' bits) from ka, result in ka
// (kb is the other buffer): four stable passes of 8-bit digits, lowest first.
// Warp w owns the contiguous keys [w * seg, (w + 1) * seg); within a warp the
// keys go in index order, 32 at a time, ranked among equal digits with
// __match_any_sync, so every pass keeps the order of equal digits.
__device__ void smp_sort_desc(unsigned* ka, unsigned* kb, int n, SmpSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int seg = ((n + kSmpWarps - 1) / kSmpWarps + 31) & ~31;
  const int lo = min(n, w * seg), hi = min(n, lo + seg);
  const unsigned lt = (1u << lane) - 1u;
  unsigned* src = ka;
  unsigned* dst = kb;
  for (int pass = 0; pass < 4; pass++) {
    const int sh = 8 * pass;
    for (int i = tid; i < kSmpWarps * kSmpBins; i += kSmpThreads) (&sm.hist[0][0])[i] = 0u;
    __syncthreads();
    for (int base = lo; base < hi; base += 8 * 32) {
      unsigned d[8];
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const int i = base + r * 32 + lane;
        d[r] = i < hi ? 255u - ((src[i] >> sh) & 255u) : 256u;
      }
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const unsigned peers = __match_any_sync(0xffffffffu, d[r]);
        if (d[r] < 256u && lane == __ffs(peers) - 1) sm.hist[w][d[r]] += (unsigned)__popc(peers);
        __syncwarp();
      }
    }
    __syncthreads();
    if (tid < kSmpBins) {
      unsigned tot = 0;
      for (int ww = 0; ww < kSmpWarps; ww++) tot += sm.hist[ww][tid];
      sm.digit_base[tid] = tot;
    }
    __syncthreads();
    if (w == 0) {  // exclusive scan of the 256 digit totals, 8 per lane
      unsigned v[8], s = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        v[j] = sm.digit_base[lane * 8 + j];
        s += v[j];
      }
      unsigned inc = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      unsigned run = inc - s;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        sm.digit_base[lane * 8 + j] = run;
        run += v[j];
      }
    }
    __syncthreads();
    if (tid < kSmpBins) {  // cursors: digit-major, then warp order
      unsigned run = sm.digit_base[tid];
      for (int ww = 0; ww < kSmpWarps; ww++) {
        const unsigned h = sm.hist[ww][tid];
        sm.hist[ww][tid] = run;
        run += h;
      }
    }
    __syncthreads();
    for (int base = lo; base < hi; base += 8 * 32) {
      unsigned key[8], d[8];
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const int i = base + r * 32 + lane;
        key[r] = i < hi ? src[i] : 0u;
        d[r] = i < hi ? 255u - ((key[r] >> sh) & 255u) : 256u;
      }
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const unsigned peers = __match_any_sync(0xffffffffu, d[r]);
        const unsigned b = d[r] < 256u ? sm.hist[w][d[r]] : 0u;
        if (d[r] < 256u) dst[b + (unsigned)__popc(peers & lt)] = key[r];
        __syncwarp();
        if (d[r] < 256u && lane == __ffs(peers) - 1) sm.hist[w][d[r]] = b + (unsigned)__popc(peers);
        __syncwarp();
      }
    }
    __syncthreads();
    unsigned* t = src;
    src = dst;
    dst = t;
  }
}

// The key of rank k (1 = largest) among n keys: four 8-bit digit passes from
// the top, each counting the digits of the keys that match the digits chosen
// so far (warp-aggregated shared-memory atomics) and choosing the digit whose
// cumulative count from the top reaches the remaining rank.  Exact; the
// result is what ka[k - 1] would be after the descending sort.
__device__ unsigned smp_select_kth(const unsigned* keys, int n, int k, SmpSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31;
  unsigned prefix = 0u, pmask = 0u;
  int kk = k;
  for (int b = 3; b >= 0; b--) {
    const int sh = 8 * b;
    if (tid < kSmpBins) sm.digit_base[tid] = 0u;
    __syncthreads();
    for (int base = 0; base < n; base += 8 * kSmpThreads) {
      unsigned d[8];
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const int i = base + r * kSmpThreads + tid;
        const unsigned key = i < n ? keys[i] : 0u;
        d[r] = (i < n && (key & pmask) == prefix) ? (key >> sh) & 255u : 256u;
      }
#pragma unroll
      for (int r = 0; r < 8; r++) {
        const unsigned peers = __match_any_sync(0xffffffffu, d[r]);
        if (d[r] < 256u && lane == __ffs(peers) - 1) atomicAdd(&sm.digit_base[d[r]], (unsigned)__popc(peers));
      }
    }
    __syncthreads();
    if (tid < 32) {
      // lane l holds digits 255 - 8 l - j (j = 0..7, high to low); the lane
      // whose range holds the kk-th key from the top finds the digit in it
      unsigned c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        c[j] = sm.digit_base[255 - 8 * lane - j];
        tot += c[j];
      }
      unsigned inc = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      unsigned cum = inc - tot;
      if (cum < (unsigned)kk && (unsigned)kk <= inc) {
        for (int j = 0; j < 8; j++) {
          if (cum + c[j] >= (unsigned)kk) {
            sm.bcasti[2] = (int)(prefix | ((unsigned)(255 - 8 * lane - j) << sh));
            sm.bcasti[3] = kk - (int)cum;
            break;
          }
          cum += c[j];
        }
      }
    }
    __syncthreads();
    prefix = (unsigned)sm.bcasti[2];
    kk = sm.bcasti[3];
    pmask |= 255u << sh;
    __syncthreads();  // digit_base and bcasti are reused by the next pass
  }
  return prefix;
}

constexpr int kSmpSmall = 2 * kSmpTile;  // keys the shared-memory sort takes (the two tiles)

// The keys >= tk, gathered (in any order) into shared memory and sorted there
// high to low (bitonic, padded with 0 to a power of two), then copied to
// out[0, count).  Returns their count, or -1 (nothing written) when there are
// more than kSmpSmall of them.
__device__ int smp_gather_sort(const unsigned* keys, int n, unsigned tk, unsigned* out, SmpSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31;
  unsigned* sk = reinterpret_cast<unsigned*>(&sm.tile[0][0]);
  if (tid == 0) sm.bcasti[0] = 0;
  __syncthreads();
  for (int base = 0; base < n; base += 4 * kSmpThreads) {
    unsigned key[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int i = base + r * kSmpThreads + tid;
      key[r] = i < n ? keys[i] : 0u;
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const bool take = base + r * kSmpThreads + tid < n && key[r] >= tk;
      const unsigned bal = __ballot_sync(0xffffffffu, take);
      int first = 0;
      if (lane == 0 && bal) first = atomicAdd(&sm.bcasti[0], __popc(bal));
      first = __shfl_sync(0xffffffffu, first, 0);
      const int slot = first + __popc(bal & ((1u << lane) - 1u));
      if (take && slot < kSmpSmall) sk[slot] = key[r];
    }
  }
  __syncthreads();
  const int cnt = sm.bcasti[0];
  if (cnt > kSmpSmall) return -1;  // uniform
  int np2 = 2;
  while (np2 < cnt) np2 <<= 1;
  for (int i = cnt + tid; i < np2; i += kSmpThreads) sk[i] = 0u;
  __syncthreads();
  for (int kq = 2; kq <= np2; kq <<= 1)
    for (int j = kq >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += kSmpThreads) {
        const int ij = i ^ j;
        if (ij > i) {
          const unsigned x = sk[i], y = sk[ij];
          if ((i & kq) == 0 ? x < y : x > y) {
            sk[i] = y;
            sk[ij] = x;
          }
        }
      }
      __syncthreads();
    }
  for (int i = tid; i < cnt; i += kSmpThreads) out[i] = sk[i];
  __syncthreads();
  return cnt;
}

// Largest of v over the CTA (no NaN reaches it).
__device__ __forceinline__ float smp_block_max(float v, SmpSmem& sm) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm.redf[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = sm.redf[0];
  for (int w = 1; w < kSmpWarps; w++) m = fmaxf(m, sm.redf[w]);
  __syncthreads();
  return m;
}

// ss_argmax (tensor.c:318-328): the first index of the largest value, comparing
// with '>' from x[0] -- so NaN entries are never chosen, and a NaN x[0] wins.
__device__ int smp_argmax(const float* x, int n, SmpSmem& sm) {
  float bv = -__int_as_float(0x7f800000);
  int bi = -1;
  for (int i = threadIdx.x; i < n; i += kSmpThreads) {
    const float v = x[i];
    if (v > bv) {
      bv = v;
      bi = i;
    }
  }
  auto better = [](float v, int i, float bv2, int bi2) {
    return i >= 0 && (bi2 < 0 || v > bv2 || (v == bv2 && i < bi2));
  };
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sm.redf[threadIdx.x >> 5] = bv;
    sm.redi[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  float v0 = sm.redf[0];
  int i0 = sm.redi[0];
  for (int w = 1; w < kSmpWarps; w++)
    if (better(sm.redf[w], sm.redi[w], v0, i0)) {
      v0 = sm.redf[w];
      i0 = sm.redi[w];
    }
  const float x0 = x[0];
  return (x0 != x0 || i0 < 0) ? 0 : i0;
}

__global__ void __launch_bounds__(kSmpThreads, 1) sample_kernel(SampleArgs a) {
  extern __shared__ __align__(16) unsigned char smp_raw[];
  SmpSmem& sm = *reinterpret_cast<SmpSmem*>(smp_raw);
  const int n = a.n, tid = threadIdx.x;
  if (blockIdx.x > 0) {  // draw b of a batch: its own logits, RNG state, token and scratch
    const int b = blockIdx.x;
    a.logits += (size_t)b * a.logits_stride;
    if (a.rng) a.rng += b;
    a.token += (size_t)b * a.token_stride;
    a.scratch = static_cast<unsigned char*>(a.scratch) + (size_t)b * a.scratch_stride;
  }
  int tok = 0;
  if (a.temperature <= 0.0f) {
    tok = smp_argmax(a.logits, n, sm);  // tensor.c:367-369
  } else {
    float* pr = reinterpret_cast<float*>(a.scratch);
    unsigned* ka = reinterpret_cast<unsigned*>(pr + pad_n(n));
    unsigned* kb = ka + pad_n(n);
    const float T = a.temperature;
    // logits / temperature, NaN -> -FLT_MAX (tensor.c:372-379), and the maximum
    float m = -FLT_MAX;
    for (int i = tid; i < n; i += kSmpThreads) {
      const float l = a.logits[i];
      const float v = l != l ? -FLT_MAX : __fdiv_rn(l, T);
      pr[i] = v;
      if (v > m) m = v;
    }
    m = smp_block_max(m, sm);
    // softmax (tensor.c:154-173): e_i = exp(x_i - max) and their sum in order
    float sum = 0.0f;
    smp_stream(
        n, sm,
        [&](int i) {
          const float e = smp_exp(__fsub_rn(pr[i], m));
          pr[i] = e;
          return e;
        },
        [&](const float* t, int, int cnt) {
          sum = smp_seq_sum(sum, t, cnt);
          return false;
        });
    if (tid == 0) sm.bcast[0] = sum;
    __syncthreads();
    const float inv = __fdiv_rn(1.0f, sm.bcast[0]);
    const bool use_k = a.top_k > 0 && a.top_k < n;
    const bool use_p = a.top_p > 0.0f && a.top_p < 1.0f;
    for (int i = tid; i < n; i += kSmpThreads) {
      const float p = __fmul_rn(pr[i], inv);
      pr[i] = p;
      if (use_k || use_p) ka[i] = p != p ? 0u : __float_as_uint(p);  // NaN sorts as 0 (tensor.c:386-390)
    }
    __syncthreads();
    float thr = 0.0f, cutoff = 0.0f;
    // the probabilities high to low for the top-p walk: sorted[0, nw)
    const unsigned* sorted = ka;
    int nw = n;
    if (use_k) {
      // the threshold is the k-th largest probability (tensor.c:396-401)
      const unsigned tk = smp_select_kth(ka, n, a.top_k, sm);
      thr = __uint_as_float(tk);
      if (use_p) {
        // past the values >= the threshold everything is zeroed and cannot
        // move the walk's sum: only those need sorting
        nw = smp_gather_sort(ka, n, tk, kb, sm);
        sorted = kb;
        if (nw < 0) {  // too many for shared memory: the full sort
          smp_sort_desc(ka, kb, n, sm);
          sorted = ka;
          if (tid == 0) {
            int lo = a.top_k, hi = n;
            while (lo < hi) {
              const int mid = (lo + hi) >> 1;
              if (ka[mid] < tk) hi = mid;
              else lo = mid + 1;
            }
            sm.bcasti[1] = lo;
          }
          __syncthreads();
          nw = sm.bcasti[1];
        }
      }
    } else if (use_p) {
      smp_sort_desc(ka, kb, n, sm);
    }
    if (use_p) {  // tensor.c:404-421
      float acc = 0.0f, cut = 0.0f;
      smp_stream(
          nw, sm,
          [&](int i) {
            const float v = __uint_as_float(sorted[i]);
            return use_k && v < thr ? 0.0f : v;
          },
          [&](const float* t, int, int cnt) { return smp_topp_walk(acc, cut, t, cnt, a.top_p); });
      if (tid == 0) sm.bcast[1] = cut;
      __syncthreads();
      cutoff = sm.bcast[1];
    }
    auto filtered = [&](int i) {
      float p = pr[i];
      if (use_k && p < thr) p = 0.0f;
      if (use_p && p < cutoff) p = 0.0f;
      return p;
    };
    // the non-zero filtered probabilities in index order (the sort's keys are
    // no longer needed: values into ka, indices into kb)
    float* cv = reinterpret_cast<float*>(ka);
    int* ci = reinterpret_cast<int*>(kb);
    const int nz = smp_compact(n, filtered, cv, ci, sm);
    // renormalisation (tensor.c:426-433)
    float tot = 0.0f;
    smp_stream(nz, sm, [&](int i) { return cv[i]; }, [&](const float* t, int, int cnt) {
      tot = smp_seq_sum(tot, t, cnt);
      return false;
    });
    if (tid == 0) sm.bcast[2] = tot;
    __syncthreads();
    tot = sm.bcast[2];
    const bool renorm = tot > 0.0f;
    const float rinv = renorm ? __fdiv_rn(1.0f, tot) : 1.0f;
    // the draw (tensor.c:331-342, 437-448)
    float r = 0.0f;
    if (tid == 0) {
      unsigned long long s = *a.rng;
      s ^= s << 13;
      s ^= s >> 7;
      s ^= s << 17;
      *a.rng = s;
      r = __fdiv_rn(__ull2float_rn(s >> 11), 9007199254740992.0f);
    }
    int pick = n - 1;
    float cdf = 0.0f;
    smp_stream(
        nz, sm, [&](int i) { return renorm ? __fmul_rn(cv[i], rinv) : cv[i]; },
        [&](const float* t, int base, int cnt) {
          const int j = smp_cdf_walk(cdf, t, cnt, r);
          if (j >= 0) pick = ci[base + j];
          return j >= 0;
        });
    tok = pick;
  }
  if (tid == 0) {
    *a.token = tok;
    if (a.seq_tokens) {
      const int pos = *a.d_pos;
      if (pos >= 0 && pos < a.ctx && pos >= *a.fixed_until) a.seq_tokens[pos] = tok;
      a.seq_tokens[a.ctx] = tok;
    }
  }
}

}  // namespace

size_t sample_scratch_bytes(int n) { return 3 * pad_n(n) * sizeof(float); }

cudaError_t sample_launch(const SampleArgs& a, cudaStream_t s) {
  // the RNG is read whenever the greedy branch is not taken (NaN included)
  if (a.n < 1 || a.n > kSampleMaxN || !a.logits || !a.token || !a.scratch || (!(a.temperature <= 0.0f) && !a.rng))
    return cudaErrorInvalidValue;
  if (a.batch < 1 || (a.batch > 1 && (a.seq_tokens || a.logits_stride < (size_t)a.n || a.token_stride < 1 ||
                                      a.scratch_stride < sample_scratch_bytes(a.n))))
    return cudaErrorInvalidValue;
  const cudaError_t e =
      cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SmpSmem));
  if (e != cudaSuccess) return e;
  sample_kernel<<<a.batch, kSmpThreads, sizeof(SmpSmem), s>>>(a);
  return cudaGetLastError();
}

}  // namespace ss
