// ss_cuda_api.cu -- the C ABI of the CUDA backend (include/slipstream_cuda.h).
//
// Host side of SlipStream's decode path on sm_100a: parses the GGUF, uploads
// and repacks the weights, allocates the int8 KV cache, and runs one decode
// step as a CUDA graph of 5 kernels per layer plus the embedding gather and
// the lm_head (RMSNorm + GEMV + greedy argmax), chained with programmatic
// dependent launch.  The position and the token of every position live on the
// device, so consecutive steps need no host round trip.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

#include "gguf_view.h"
#include "slipstream_cuda.h"
#include "ss_cuda_internal.h"

#define SS_API extern "C" __attribute__((visibility("default")))

namespace ss {
namespace {

thread_local std::string g_err;

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  throw Error(code, buf);
}

#define CK(call)                                                                          \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess) {                                                              \
      fail(e_ == cudaErrorMemoryAllocation ? SS_CUDA_ERROR_OUT_OF_MEMORY                  \
                                           : SS_CUDA_ERROR_BACKEND,                       \
           "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__);   \
    }                                                                                     \
  } while (0)

#define NK(call)                                                                          \
  do {                                                                                    \
    ncclResult_t r_ = (call);                                                             \
    if (r_ != ncclSuccess)                                                                \
      fail(SS_CUDA_ERROR_BACKEND, "%s failed: %s (%s:%d)", #call,                         \
           nccl_api().GetErrorString(r_), __FILE__, __LINE__);                            \
  } while (0)

template <typename F>
int guard(F&& f) {
  try {
    f();
    return SS_CUDA_OK;
  } catch (const Error& e) {
    g_err = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_err = e.what();
    return SS_CUDA_ERROR_BACKEND;
  }
}

template <typename T>
T* dev_alloc(Context* c, size_t n) {
  void* p = nullptr;
  if (n == 0) n = 1;
  CK(cudaMalloc(&p, n * sizeof(T)));
  c->allocations.push_back(p);
  return static_cast<T*>(p);
}

int round_up(int a, int b) { return (a + b - 1) / b * b; }
size_t round_up_sz(size_t a, size_t b) { return (a + b - 1) / b * b; }

// ---------------------------------------------------------------- launches

template <typename... KArgs, typename... Args>
void launch(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  CK(cudaLaunchKernelEx(&cfg, fn, std::forward<Args>(args)...));
}

using GemvFn = void (*)(const GemvParams);

template <XSrc XS, Epi EPI, int RG>
GemvFn gemv_fn_rg(int type) {
  if (type == kQ4_0) return &gemv_kernel<kQ4_0, XS, EPI, RG>;
  if (type == kQ8_0) return &gemv_kernel<kQ8_0, XS, EPI, RG>;
  fail(SS_CUDA_ERROR_INVALID_MODEL, "unsupported weight type %d (Q4_0 and Q8_0 only)", type);
}

template <XSrc XS, Epi EPI>
GemvFn gemv_fn_type(int type, int rg) {
  switch (rg) {
    case 1: return gemv_fn_rg<XS, EPI, 1>(type);
    case 2: return gemv_fn_rg<XS, EPI, 2>(type);
    case 4: return gemv_fn_rg<XS, EPI, 4>(type);
    case 8: return gemv_fn_rg<XS, EPI, 8>(type);
    default: fail(SS_CUDA_ERROR_BACKEND, "row groups %d", rg);
  }
}

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

GemvTuning read_tuning() {
  GemvTuning t;
  t.target_threads = env_int("SS_GEMV_THREADS", t.target_threads);
  t.ring_bytes = (size_t)env_int("SS_GEMV_RING_KB", (int)(t.ring_bytes / 1024)) * 1024;
  t.prefetch = env_int("SS_GEMV_PREFETCH", t.prefetch);
  t.max_ctas_per_sm = env_int("SS_GEMV_CTAS_PER_SM", t.max_ctas_per_sm);
  return t;
}

// Row-groups of threads per CTA: as many as fit in the target thread count.
int gemv_row_groups(const GemvTuning& tu, int cols) {
  const int nbt = round_up(cols / 32, 32);
  int rg = 1;
  while (rg < 8 && nbt * rg * 2 <= tu.target_threads) rg *= 2;  // consumer threads
  return rg;
}

// Geometry (see gemv.cuh): one thread per 32-column block in each of RG
// row-groups; a weight ring of `nstage` stages of 2*RG rows; as many CTAs as
// are co-resident (capped by the row count), each owning a contiguous, even
// range of rows.
GemvLaunch plan_gemv(Context* c, GemvFn fn, const DevMatrix& m, int rg) {
  const GemvTuning& tu = c->tuning;
  GemvLaunch g;
  g.fn = (const void*)fn;
  const int nb = m.cols / 32;
  if (nb < 1 || nb > kGemvMaxNb)
    fail(SS_CUDA_ERROR_INVALID_MODEL, "matrix with %d columns is outside 32..%d", m.cols, 32 * kGemvMaxNb);
  const int nbt = round_up(nb, 32);
  g.threads = 32 + nbt * rg;  // producer warp + consumer row-groups
  g.stage_rows = kGemvG * rg;
  const size_t stage_bytes = (size_t)g.stage_rows * m.row_stride;
  g.nstage = (int)std::max<size_t>(2, std::min<size_t>(16, tu.ring_bytes / stage_bytes));
  const int nwb = nbt / 32;
  auto smem_for = [&](int rpc) {
    return (size_t)g.nstage * stage_bytes + (size_t)g.nstage * 16 + (size_t)nwb * rpc * 4 + 64 * 4;
  };
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, g.threads, smem_for(256)));
  occ = std::max(occ, 1);
  if (tu.max_ctas_per_sm > 0) occ = std::min(occ, tu.max_ctas_per_sm);
  const int ctas = std::min((m.rows + 1) / 2, c->sm_count * occ);
  g.rows_per_cta = round_up((m.rows + ctas - 1) / ctas, 2);
  g.ctas = (m.rows + g.rows_per_cta - 1) / g.rows_per_cta;
  g.smem = smem_for(g.rows_per_cta);
  if (g.smem > 220 * 1024) fail(SS_CUDA_ERROR_INVALID_MODEL, "GEMV shared memory too large");
  return g;
}

GemvLaunch plan_gemv_for(Context* c, XSrc xs, Epi epi, const DevMatrix& m) {
  const int rg = gemv_row_groups(c->tuning, m.cols);
  GemvFn fn = nullptr;
  if (xs == XSrc::RmsNorm && epi == Epi::QKV) fn = gemv_fn_type<XSrc::RmsNorm, Epi::QKV>(m.type, rg);
  else if (xs == XSrc::RmsNorm && epi == Epi::SwiGLU) fn = gemv_fn_type<XSrc::RmsNorm, Epi::SwiGLU>(m.type, rg);
  else if (xs == XSrc::RmsNorm && epi == Epi::Argmax) fn = gemv_fn_type<XSrc::RmsNorm, Epi::Argmax>(m.type, rg);
  else if (xs == XSrc::Plain && epi == Epi::Residual) fn = gemv_fn_type<XSrc::Plain, Epi::Residual>(m.type, rg);
  else if (xs == XSrc::Plain && epi == Epi::Store) fn = gemv_fn_type<XSrc::Plain, Epi::Store>(m.type, rg);
  else fail(SS_CUDA_ERROR_BACKEND, "GEMV variant not built");
  return plan_gemv(c, fn, m, rg);
}

void run_gemv(Context* c, const GemvLaunch& g, GemvParams p, bool pdl) {
  p.rows_per_cta = g.rows_per_cta;
  p.nstage = g.nstage;
  p.stage_rows = g.stage_rows;
  launch((GemvFn)g.fn, dim3(g.ctas), dim3(g.threads), g.smem, c->stream, pdl, p);
}

// ------------------------------------------------------------- weight upload

DevMatrix layout(int rows, int cols, int type) {
  DevMatrix m;
  m.rows = rows;
  m.cols = cols;
  m.type = type;
  const int nb = cols / 32;
  const int qsz = type == kQ4_0 ? 16 : 32;
  m.scale_off = nb * qsz;
  m.row_stride = m.scale_off + round_up(nb * 2, 16);
  return m;
}

// Tiled layout of the persistent step kernel (step_kernel.cuh).
DevMatrix layout_tiled(int rows, int cols, int type) {
  DevMatrix m;
  m.rows = rows;
  m.cols = cols;
  m.type = type;
  m.tiled = true;
  const int nb = cols / 32;
  const int qsz = type == kQ4_0 ? 16 : 32;
  m.tile_bytes = kStepTileRows * nb * qsz + round_up(nb * 8, 16);
  m.ntiles = (rows + kStepTileRows - 1) / kStepTileRows;
  return m;
}

size_t matrix_bytes(const DevMatrix& m) {
  return m.tiled ? (size_t)m.ntiles * m.tile_bytes : (size_t)m.rows * m.row_stride;
}

// Repacks nrows GGUF rows (src_nb blocks each, already in device memory) into
// rows dst_row_mul*r + dst_row_add of `dst`, taking blocks [b0, b0 + dst.cols/32).
void repack_into(const uint8_t* src, int nrows, int src_nb, int b0, int type, const DevMatrix& dst,
                 int dst_row_mul, int dst_row_add, cudaStream_t stream) {
  const long long blocks = (long long)nrows * (dst.cols / 32);
  const int threads = 256;
  const int grid = (int)std::min<long long>((blocks + threads - 1) / threads, 65535);
  if (dst.tiled)
    repack_tiled_kernel<<<grid, threads, 0, stream>>>(src, nrows, dst.cols, type, dst.data, dst.tile_bytes,
                                                      dst_row_mul, dst_row_add, src_nb, b0);
  else
    repack_kernel<<<grid, threads, 0, stream>>>(src, nrows, dst.cols, type, dst.data, dst.row_stride,
                                                dst.scale_off, dst_row_mul, dst_row_add, src_nb, b0);
  CK(cudaGetLastError());
}

// Uploads rows [row0, row0 + nrows) of one GGUF matrix through the staging
// buffer, and of each row the 32-column blocks [b0, b0 + dst.cols / 32) (the
// whole row when not sharded), repacked into rows dst_row_mul*r + dst_row_add
// of `dst`.  nrows < 0: all rows.
void upload_matrix(Context* c, const GgufTensor& t, const DevMatrix& dst, int dst_row_mul,
                   int dst_row_add, uint8_t* stage, size_t stage_cap, int row0 = 0, int nrows = -1,
                   int b0 = 0) {
  if (t.type != dst.type)
    fail(SS_CUDA_ERROR_INVALID_MODEL, "tensor %s has type %d, expected %d", t.name.c_str(), t.type,
         dst.type);
  const int src_nb = (int)(t.cols() / 32), nb = dst.cols / 32;
  if (nrows < 0) nrows = (int)t.rows() - row0;
  if (b0 < 0 || b0 + nb > src_nb || row0 < 0 || row0 + nrows > (int)t.rows())
    fail(SS_CUDA_ERROR_INVALID_MODEL, "tensor %s: slice rows %d+%d blocks %d+%d outside %llu x %d",
         t.name.c_str(), row0, nrows, b0, nb, (unsigned long long)t.rows(), src_nb);
  const size_t row_bytes = (size_t)src_nb * ggml_type_size(t.type);
  const size_t bytes = (size_t)nrows * row_bytes;
  if (bytes > stage_cap) fail(SS_CUDA_ERROR_BACKEND, "staging buffer too small");
  CK(cudaMemcpyAsync(stage, t.data + (size_t)row0 * row_bytes, bytes, cudaMemcpyHostToDevice,
                     c->stream));
  repack_into(stage, nrows, src_nb, b0, t.type, dst, dst_row_mul, dst_row_add, c->stream);
}

const GgufTensor& need(const GgufModel& m, const std::string& name) {
  const GgufTensor* t = m.find(name);
  if (!t) fail(SS_CUDA_ERROR_INVALID_MODEL, "GGUF has no tensor %s", name.c_str());
  return *t;
}

void upload_f32_into(Context* c, const GgufTensor& t, size_t n, float* dst) {
  if (t.type != kF32) fail(SS_CUDA_ERROR_INVALID_MODEL, "%s must be F32", t.name.c_str());
  if (t.bytes < n * 4) fail(SS_CUDA_ERROR_INVALID_MODEL, "%s is too small", t.name.c_str());
  CK(cudaMemcpyAsync(dst, t.data, n * 4, cudaMemcpyHostToDevice, c->stream));
}

float* upload_f32(Context* c, const GgufTensor& t, size_t n) {
  float* p = dev_alloc<float>(c, n);
  upload_f32_into(c, t, n, p);
  return p;
}

// ------------------------------------------------------ persistent step plan

using StepFn = void (*)(const StepParams, const StepTp);

template <int T, int H, bool TP>
StepFn step_fn_hd(int hd) {
  switch (hd) {
    case 32: return &decode_step_kernel<T, H, 32, TP>;
    case 64: return &decode_step_kernel<T, H, 64, TP>;
    case 128: return &decode_step_kernel<T, H, 128, TP>;
    case 256: return &decode_step_kernel<T, H, 256, TP>;
    default: return nullptr;
  }
}
template <bool TP>
StepFn step_fn_tp(int type, int htype, int hd) {
  if (type == kQ4_0 && htype == kQ4_0) return step_fn_hd<kQ4_0, kQ4_0, TP>(hd);
  if (type == kQ4_0 && htype == kQ8_0) return step_fn_hd<kQ4_0, kQ8_0, TP>(hd);
  if (type == kQ8_0 && htype == kQ8_0) return step_fn_hd<kQ8_0, kQ8_0, TP>(hd);
  return nullptr;
}
// The single-GPU step, or (tp) the tensor-parallel one with its exchanges
// inside the kernel.
StepFn step_fn_for(int type, int htype, int hd, bool tp) {
  return tp ? step_fn_tp<true>(type, htype, hd) : step_fn_tp<false>(type, htype, hd);
}

// Decides whether the persistent step kernel can run this model on this GPU
// and sizes it: one CTA per SM; the weight ring gets what shared memory is left
// after the consumers' scratch (row partial sums or the attention task's
// buffers).  Returns false (multi-kernel step) when a shape is outside what the
// kernel supports.  SS_STEP_SLOTS caps the ring slots (tuning sweeps).
bool plan_step(Context* c, int htype) {
  const int qd = c->nh * c->hd, kvd = c->nkv * c->hd;
  const int G = c->nh / c->nkv;
  StepFn fn = step_fn_for(c->wtype, htype, c->hd, c->tp_size > 1);
  if (!fn || G > kAttnMaxG) return false;
  const int cols[3] = {c->d, qd, c->ff};
  for (int x : cols)
    if (x % 32 || x / 32 > kStepMaxNb) return false;
  if (c->d % 32 || c->ff % 32 || qd % 32) return false;
  int coop = 0;
  CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->device));
  if (!coop) return false;
  const int ncta = c->sm_count;
  const int nsplit = std::max(1, std::min(ncta / c->nkv, kStepMaxSplit));
  if (c->nkv > ncta || G * c->hd > 2 * kStepConsumers || c->ctx % 4) return false;
  if (qd / 32 > kStepConsumers / 2) return false;    // attention output merged in <= 2 rounds
  if (c->d / 32 > kStepConsumers / 2) return false;  // RMSNorm inputs converted in <= 2 rounds
  struct Shape { int rows, cols, type; };
  const Shape shapes[5] = {{qd + 2 * kvd, c->d, c->wtype}, {c->d, qd, c->wtype},
                           {2 * c->ff, c->d, c->wtype}, {c->d, c->ff, c->wtype},
                           {c->vocab_l, c->d, htype}};
  int slot = 0;
  size_t red = 0;
  for (const Shape& sh : shapes) {
    const DevMatrix m = layout_tiled(sh.rows, sh.cols, sh.type);
    const int nb = sh.cols / 32, wpr = (nb + 31) / 32, rg = kStepConsumerWarps / wpr;
    slot = std::max(slot, rg * m.tile_bytes);
    const size_t rows_cta = (size_t)((m.ntiles + ncta - 1) / ncta) * kStepTileRows;
    red = std::max(red, (size_t)wpr * rows_cta * sizeof(float));
  }
  slot = round_up(slot, 128);
  const size_t att = step_att_scratch_bytes(G, c->hd, slot);
  // the scratch also holds a phase's activation planes
  const size_t planes = (size_t)(std::max(std::max(c->d, qd), c->ff) / 32) * sizeof(PlaneBlock);
  const size_t scratch = (std::max(std::max(red, att), planes) + 127) / 128 * 128;
  cudaFuncAttributes fa;
  CK(cudaFuncGetAttributes(&fa, fn));
  // the kernel hands registers from its producer warpgroup to its consumers
  // (setmaxnreg); that split is exact for this launch count only
  if (fa.numRegs != kStepLaunchRegs) return false;
  int optin = 0;
  CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device));
  // [ring][128 B of mbarriers: full, empty per slot + the plane barrier][scratch]
  const long long avail = (long long)optin - (long long)fa.sharedSizeBytes - (long long)scratch - 128;
  int nslots = (int)std::min<long long>(7, avail / slot);
  nslots = std::min(nslots, env_int("SS_STEP_SLOTS", 7));
  if (nslots < 2) return false;
  const size_t smem = (size_t)nslots * slot + 128 + scratch;
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kStepThreads, smem));
  if (occ < 1) return false;
  c->step_fn = (const void*)fn;
  c->step_grid = ncta;
  c->step_nslots = nslots;
  c->step_slot_bytes = slot;
  c->step_nsplit = nsplit;
  c->step_smem = smem;
  return true;
}

void load_model(Context* c, const uint8_t* base, uint64_t size, uint32_t ctx_opt) {
  GgufModel g;
  std::string err;
  if (!gguf_parse(base, size, &g, &err)) fail(SS_CUDA_ERROR_INVALID_MODEL, "%s", err.c_str());
  if (g.arch.find("llama") == std::string::npos)
    fail(SS_CUDA_ERROR_INVALID_MODEL, "architecture '%s' is not llama", g.arch.c_str());
  c->d = (int)g.hidden;
  c->L = (int)g.n_layers;
  c->nh = (int)g.n_heads;
  c->nkv = g.n_kv_heads ? (int)g.n_kv_heads : c->nh;
  c->ff = (int)g.ffn;
  c->eps = g.rms_eps;
  c->theta = g.rope_theta;
  if (c->d <= 0 || c->L <= 0 || c->nh <= 0 || c->ff <= 0)
    fail(SS_CUDA_ERROR_INVALID_MODEL, "missing llama dimensions in GGUF metadata");
  const GgufTensor& wq0 = need(g, "blk.0.attn_q.weight");
  // head_dim, rope_dim, vocab clamp: SlipStream/src/core/layer_scheduler.c:161-197
  c->hd = g.key_length ? (int)g.key_length : (int)(wq0.rows() / (uint64_t)c->nh);
  c->rope_dim = g.rope_dim ? (int)g.rope_dim : c->hd;
  const GgufTensor& embd = need(g, "token_embd.weight");
  const GgufTensor* out = g.find("output.weight");
  int vocab = (int)g.vocab;
  if (out && (int)out->rows() < vocab) vocab = (int)out->rows();
  if ((int)embd.rows() < vocab) vocab = (int)embd.rows();
  c->vocab = vocab;
  if (c->nh % c->nkv) fail(SS_CUDA_ERROR_INVALID_MODEL, "heads %% kv_heads != 0");
  // tensor parallelism: this rank keeps nh/tp q heads, nkv/tp kv heads, ff/tp
  // FFN rows and vocab/tp lm_head rows; c->nh, c->nkv, c->ff become the local
  // counts (the full ones stay in *_full)
  c->nh_full = c->nh;
  c->nkv_full = c->nkv;
  c->ff_full = c->ff;
  c->vocab_l = c->vocab;
  c->vocab_off = 0;
  if (c->tp_size > 1) {
    const int tp = c->tp_size;
    if (c->nh % tp || c->nkv % tp || c->ff % (32 * tp) || c->vocab % tp)
      fail(SS_CUDA_ERROR_INVALID_MODEL,
           "tensor parallelism %d needs heads (%d), kv heads (%d), ffn/32 (%d) and vocab (%d) divisible by it",
           tp, c->nh, c->nkv, c->ff / 32, c->vocab);
    c->nh /= tp;
    c->nkv /= tp;
    c->ff /= tp;
    c->vocab_l = c->vocab / tp;
    c->vocab_off = c->tp_rank * c->vocab_l;
  }
  if (c->nh / c->nkv > 8) fail(SS_CUDA_ERROR_INVALID_MODEL, "GQA group above 8 is not supported");
  if (c->hd % 32 || c->hd > 256 || c->rope_dim > c->hd || c->rope_dim % 2)
    fail(SS_CUDA_ERROR_INVALID_MODEL, "head_dim %d / rope_dim %d unsupported", c->hd, c->rope_dim);
  // context: engine.c:99-106 (default from the file, capped at 8192)
  uint32_t ctx = ctx_opt ? ctx_opt : g.context_length;
  if (ctx == 0 || ctx > 8192) ctx = 8192;
  c->ctx = (int)ctx;
  c->wtype = wq0.type;
  if (c->wtype != kQ4_0 && c->wtype != kQ8_0)
    fail(SS_CUDA_ERROR_INVALID_MODEL, "weight type %d unsupported (Q4_0 / Q8_0)", c->wtype);
  c->attn_scale = 1.0f / sqrtf((float)c->hd);  // layer_scheduler.c:421

  const int qd = c->nh * c->hd, kvd = c->nkv * c->hd;  // this rank's
  const int r = c->tp_rank;
  if (!out) fail(SS_CUDA_ERROR_INVALID_MODEL, "tied embeddings (no output.weight) unsupported");
  if (out->type != kQ4_0 && out->type != kQ8_0)
    fail(SS_CUDA_ERROR_INVALID_MODEL, "output.weight type %d unsupported", out->type);
  // layer streaming: the layers' GGUF bytes exceed the HBM budget
  {
    uint64_t raw = 0;
    for (const char* nm : {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"})
      raw += need(g, std::string("blk.0.") + nm + ".weight").bytes;
    if (c->hbm_budget && raw * (uint64_t)c->L > c->hbm_budget) {
      if (c->tp_size > 1)
        fail(SS_CUDA_ERROR_INVALID_PARAMS, "layer streaming with tensor parallelism is not supported");
      c->streaming = true;
    }
  }
  // layer streaming runs the multi-kernel step
  c->mega = c->mega && !c->streaming && plan_step(c, out->type);
  // several sequences decode through the many-token step, which reads the
  // tiled layout; without the persistent step it then runs every step
  if (c->max_batch > 1 && (c->streaming || c->tp_size > 1))
    fail(SS_CUDA_ERROR_INVALID_PARAMS, "max_batch %d: batched decode runs on one GPU with the weights resident",
         c->max_batch);
  c->tiled = c->mega || c->max_batch > 1;
  auto mat_layout = [&](int rows, int cols, int type) {
    return c->tiled ? layout_tiled(rows, cols, type) : layout(rows, cols, type);
  };
  size_t max_bytes = 0;
  for (const auto& t : g.tensors) max_bytes = std::max<size_t>(max_bytes, t.bytes);
  uint8_t* stage = nullptr;
  CK(cudaMalloc(&stage, max_bytes));

  try {
    // embeddings: F32 rows (layer_scheduler.c:585-587)
    if (embd.type != kF32) fail(SS_CUDA_ERROR_INVALID_MODEL, "token_embd.weight must be F32");
    if ((int)embd.cols() != c->d) fail(SS_CUDA_ERROR_INVALID_MODEL, "token_embd width mismatch");
    c->embd = upload_f32(c, embd, (size_t)embd.rows() * c->d);
    c->weight_bytes += (size_t)embd.rows() * c->d * 4;
    c->layers.resize((size_t)c->L);
    // every layer's four matrices in one allocation at a fixed stride (the
    // persistent step addresses layer l as layer 0 + l * stride), and the
    // norm weights as [L][d] arrays
    // an FFN wider than one GEMV's columns: down as two column halves
    const bool split_down = !c->tiled && c->ff / 32 > kGemvMaxNb;
    if (split_down && (c->tp_size > 1 || c->streaming || c->ff % 64 || c->ff / 64 > kGemvMaxNb))
      fail(SS_CUDA_ERROR_INVALID_MODEL,
           "FFN width %d needs the down projection split in two, which supports one GPU without "
           "streaming and widths up to %d", c->ff, 64 * kGemvMaxNb);
    const int down_cols = split_down ? c->ff / 2 : c->ff;
    const DevMatrix s_qkv = mat_layout(qd + 2 * kvd, c->d, c->wtype), s_o = mat_layout(c->d, qd, c->wtype),
                    s_gu = mat_layout(2 * c->ff, c->d, c->wtype), s_down = mat_layout(c->d, down_cols, c->wtype);
    const size_t o_o = round_up_sz(matrix_bytes(s_qkv), 256);
    const size_t o_gu = o_o + round_up_sz(matrix_bytes(s_o), 256);
    const size_t o_down = o_gu + round_up_sz(matrix_bytes(s_gu), 256);
    const size_t o_down2 = o_down + round_up_sz(matrix_bytes(s_down), 256);
    c->layer_stride = split_down ? o_down2 + round_up_sz(matrix_bytes(s_down), 256) : o_down2;
    // streaming: the budget holds the resident layers, two slots and the raw
    // bytes of the layer being repacked (about one more layer)
    int hbm_layers = c->L;
    c->n_resident = c->L;
    if (c->streaming) {
      const uint64_t fit = c->hbm_budget / c->layer_stride;
      if (fit < 3)
        fail(SS_CUDA_ERROR_INVALID_PARAMS,
             "HBM budget of %llu bytes holds %llu layers of %zu bytes; streaming needs 3 (two slots and "
             "the staging of one layer)",
             (unsigned long long)c->hbm_budget, (unsigned long long)fit, c->layer_stride);
      c->n_resident = (int)std::min<uint64_t>(fit - 3, (uint64_t)c->L - 2);
      hbm_layers = c->n_resident + 2;
      c->stream_src.resize((size_t)c->L);
    }
    uint8_t* slab = dev_alloc<uint8_t>(c, c->layer_stride * (size_t)hbm_layers);
    CK(cudaMemsetAsync(slab, 0, c->layer_stride * (size_t)hbm_layers, c->stream));
    c->attn_norm_all = dev_alloc<float>(c, (size_t)c->L * c->d);
    c->ffn_norm_all = dev_alloc<float>(c, (size_t)c->L * c->d);
    for (int l = 0; l < c->L; l++) {
      Layer& ly = c->layers[(size_t)l];
      auto nm = [&](const char* s) { return "blk." + std::to_string(l) + "." + s; };
      const GgufTensor& wq = need(g, nm("attn_q.weight"));
      const GgufTensor& wk = need(g, nm("attn_k.weight"));
      const GgufTensor& wv = need(g, nm("attn_v.weight"));
      const GgufTensor& wo = need(g, nm("attn_output.weight"));
      const GgufTensor& wg = need(g, nm("ffn_gate.weight"));
      const GgufTensor& wu = need(g, nm("ffn_up.weight"));
      const GgufTensor& wd = need(g, nm("ffn_down.weight"));
      const int qd_f = c->nh_full * c->hd, kvd_f = c->nkv_full * c->hd;
      if ((int)wq.rows() != qd_f || (int)wk.rows() != kvd_f || (int)wv.rows() != kvd_f ||
          (int)wo.rows() != c->d || (int)wo.cols() != qd_f || (int)wg.rows() != c->ff_full ||
          (int)wu.rows() != c->ff_full || (int)wd.rows() != c->d || (int)wd.cols() != c->ff_full ||
          (int)wq.cols() != c->d || (int)wg.cols() != c->d)
        fail(SS_CUDA_ERROR_INVALID_MODEL, "layer %d tensor shapes do not match the metadata", l);
      ly.qkv = s_qkv;
      ly.o = s_o;
      ly.gu = s_gu;
      ly.down = s_down;
      const int place = l < c->n_resident ? l : c->n_resident + (l - c->n_resident) % 2;
      ly.block = slab + (size_t)place * c->layer_stride;
      ly.qkv.data = ly.block;
      ly.o.data = ly.block + o_o;
      ly.gu.data = ly.block + o_gu;
      ly.down.data = ly.block + o_down;
      if (split_down) {
        ly.down2 = s_down;
        ly.down2.data = ly.block + o_down2;
      }
      if (l < c->n_resident || !c->streaming)
        c->weight_bytes += matrix_bytes(s_qkv) + matrix_bytes(s_o) + matrix_bytes(s_gu) +
                           (split_down ? 2 : 1) * matrix_bytes(s_down);
      ly.attn_norm = c->attn_norm_all + (size_t)l * c->d;
      ly.ffn_norm = c->ffn_norm_all + (size_t)l * c->d;
      upload_f32_into(c, need(g, nm("attn_norm.weight")), (size_t)c->d, ly.attn_norm);
      upload_f32_into(c, need(g, nm("ffn_norm.weight")), (size_t)c->d, ly.ffn_norm);
      if (l >= c->n_resident) {
        // streamed: remember where its bytes are; every step copies them in
        auto& src = c->stream_src[(size_t)l];
        const GgufTensor* ts[7] = {&wq, &wk, &wv, &wo, &wg, &wu, &wd};
        const int which[7] = {0, 0, 0, 1, 2, 2, 3}, mul[7] = {1, 1, 1, 1, 2, 2, 1},
                  add[7] = {0, qd, qd + kvd, 0, 0, 1, 0};
        size_t off = 0;
        for (int i = 0; i < 7; i++) {
          Context::StreamTensor st;
          st.t = *ts[i];
          st.raw_off = off;
          st.which = which[i];
          st.mul = mul[i];
          st.add = add[i];
          src.push_back(st);
          off += round_up_sz(ts[i]->bytes, 256);
        }
        c->stream_raw_bytes = std::max(c->stream_raw_bytes, off);
        c->streamed_bytes += off;
        CK(cudaStreamSynchronize(c->stream));
        continue;
      }
      // rank r's shard (the whole matrix without tensor parallelism): rows of
      // its heads / FFN rows, and for O and down the matching column blocks
      upload_matrix(c, wq, ly.qkv, 1, 0, stage, max_bytes, r * qd, qd);
      upload_matrix(c, wk, ly.qkv, 1, qd, stage, max_bytes, r * kvd, kvd);
      upload_matrix(c, wv, ly.qkv, 1, qd + kvd, stage, max_bytes, r * kvd, kvd);
      upload_matrix(c, wo, ly.o, 1, 0, stage, max_bytes, 0, -1, r * qd / 32);
      upload_matrix(c, wg, ly.gu, 2, 0, stage, max_bytes, r * c->ff, c->ff);
      upload_matrix(c, wu, ly.gu, 2, 1, stage, max_bytes, r * c->ff, c->ff);
      upload_matrix(c, wd, ly.down, 1, 0, stage, max_bytes, 0, -1, r * c->ff / 32);
      if (split_down) upload_matrix(c, wd, ly.down2, 1, 0, stage, max_bytes, 0, -1, down_cols / 32);
      CK(cudaStreamSynchronize(c->stream));  // staging buffer reuse
    }
    c->out_norm = upload_f32(c, need(g, "output_norm.weight"), (size_t)c->d);
    c->lm_head = mat_layout(c->vocab_l, c->d, out->type);
    c->lm_block = dev_alloc<uint8_t>(c, matrix_bytes(c->lm_head));
    c->lm_head.data = c->lm_block;
    c->weight_bytes += matrix_bytes(c->lm_head);
    if (c->streaming) {
      c->stream_raw = dev_alloc<uint8_t>(c, c->stream_raw_bytes);
      c->weight_bytes += 2 * c->layer_stride + c->stream_raw_bytes;  // the slots and the staging
    }
    // only the first `vocab` rows are addressable (layer_scheduler.c:189-197);
    // this rank's slice of them
    upload_matrix(c, *out, c->lm_head, 1, 0, stage, max_bytes, c->vocab_off, c->vocab_l);
    CK(cudaStreamSynchronize(c->stream));
  } catch (...) {
    cudaFree(stage);
    throw;
  }
  CK(cudaFree(stage));
}

void alloc_step_state(Context* c);

void alloc_state(Context* c) {
  const int kvd = c->nkv * c->hd, qd = c->nh * c->hd;
  const size_t rows = (size_t)c->max_batch * c->L * c->ctx;  // sequence 0 first
  c->kc = dev_alloc<int8_t>(c, rows * kvd);
  c->vc = dev_alloc<int8_t>(c, rows * kvd);
  c->ks = dev_alloc<float>(c, rows);
  c->vs = dev_alloc<float>(c, rows);
  c->amax = dev_alloc<unsigned int>(c, 2 * (size_t)c->L);
  c->kv_bytes = rows * (2 * (size_t)kvd + 16);
  c->h = dev_alloc<float>(c, (size_t)c->d);
  c->qkv = dev_alloc<float>(c, (size_t)qd + 2 * kvd);
  c->attn_out = dev_alloc<float>(c, (size_t)std::max(qd, c->d));
  c->act = dev_alloc<float>(c, (size_t)c->ff);
  c->logits = dev_alloc<float>(c, (size_t)c->vocab_l);
  if (c->tp_size > 1) {
    c->hpart = dev_alloc<float>(c, (size_t)c->d);
    c->tp_best = dev_alloc<unsigned long long>(c, 1);
    c->logits_full = dev_alloc<float>(c, (size_t)c->vocab);
  }
  // attention: position splits of one kv head form a thread-block cluster
  // (at most 8, the portable cluster size); ~2 CTAs per SM over the kv heads
  c->attn_nsplit = std::max(1, std::min(8, (2 * c->sm_count + c->nkv - 1) / c->nkv));
  switch (c->hd) {
    case 32: c->attn_smem = sizeof(AttnSmem<32>); break;
    case 64: c->attn_smem = sizeof(AttnSmem<64>); break;
    case 128: c->attn_smem = sizeof(AttnSmem<128>); break;
    case 256: c->attn_smem = sizeof(AttnSmem<256>); break;
    default: fail(SS_CUDA_ERROR_INVALID_MODEL, "head_dim %d unsupported (32, 64, 128, 256)", c->hd);
  }
  c->am_part = dev_alloc<unsigned long long>(c, 4096);
  c->am_cnt = dev_alloc<unsigned int>(c, 1);
  c->seq_tokens = dev_alloc<int>(c, (size_t)c->ctx + 1);
  c->ctrl = dev_alloc<Ctrl>(c, 1);
  CK(cudaMemsetAsync(c->am_cnt, 0, sizeof(unsigned), c->stream));
  CK(cudaMemsetAsync(c->seq_tokens, 0, sizeof(int) * (c->ctx + 1), c->stream));
  CK(cudaMemsetAsync(c->ctrl, 0, sizeof(Ctrl), c->stream));
  // RoPE table, computed with the reference's float expressions
  // (SlipStream/src/core/tensor.c:250-254) so cos/sin match it exactly.
  const int half = c->rope_dim / 2;
  std::vector<float2> tab((size_t)c->ctx * half);
  for (int pos = 0; pos < c->ctx; pos++)
    for (int j = 0; j < half; j++) {
      const float freq = 1.0f / powf(c->theta, (float)(2 * j) / (float)c->rope_dim);
      const float angle = (float)pos * freq;
      tab[(size_t)pos * half + j] = make_float2(cosf(angle), sinf(angle));
    }
  c->rope_tab = dev_alloc<float2>(c, tab.size());
  CK(cudaMemcpy(c->rope_tab, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
  CK(cudaMallocHost(&c->h_logits, sizeof(float) * (size_t)c->vocab));
  CK(cudaMallocHost(&c->h_small, sizeof(int) * 64));
  c->embed_blocks = std::max(1, std::min(16, (c->d + 255) / 256));
  if (c->mega) alloc_step_state(c);
}

// Buffers of the persistent step kernel and its parameter block.
void alloc_step_state(Context* c) {
  const int qd = c->nh * c->hd, kvd = c->nkv * c->hd, ncta = c->step_grid;
  StepParams& p = c->step_params;
  p = StepParams{};
  const Layer& l0 = c->layers[0];
  p.qkv0 = l0.qkv.t();
  p.o0 = l0.o.t();
  p.gu0 = l0.gu.t();
  p.down0 = l0.down.t();
  p.layer_stride = (long long)c->layer_stride;
  p.attn_norm = c->attn_norm_all;
  p.ffn_norm = c->ffn_norm_all;
  p.L = c->L;
  p.head = c->lm_head.t();
  p.out_norm = c->out_norm;
  p.embd = c->embd;
  p.d = c->d;
  p.qd = qd;
  p.kvd = kvd;
  p.ff = c->ff;
  p.vocab = c->vocab;
  p.nh = c->nh;
  p.nkv = c->nkv;
  p.hd = c->hd;
  p.rope_dim = c->rope_dim;
  p.ctx = c->ctx;
  p.eps = c->eps;
  p.attn_scale = c->attn_scale;
  p.rope_tab = c->rope_tab;
  p.kc = c->kc;
  p.vc = c->vc;
  p.ks = c->ks;
  p.vs = c->vs;
  p.d_pos = &c->ctrl->pos;
  p.fixed_until = &c->ctrl->fixed_until;
  p.err = &c->ctrl->err;
  p.seq_tokens = c->seq_tokens;
  p.h = c->h;
  p.qkv_out = c->qkv;
  p.attn_out = c->attn_out;
  p.act = c->act;
  p.logits = c->logits;
  p.amax_part = dev_alloc<float2>(c, (size_t)ncta);
  p.att_part = dev_alloc<float>(c, (size_t)c->nh * c->step_nsplit * (c->hd + 4));
  // counters, zeroed here and by ss_cuda_reset: grid barrier, abort flag
  c->step_sync_words = 4;
  c->step_sync = dev_alloc<unsigned>(c, c->step_sync_words);
  CK(cudaMemset(c->step_sync, 0, sizeof(unsigned) * c->step_sync_words));
  p.grid_bar = c->step_sync;
  p.abort_flag = c->step_sync + 1;
  p.am_part = c->am_part;
  p.am_cnt = c->am_cnt;
  p.nsplit = c->step_nsplit;
  p.slot_bytes = c->step_slot_bytes;
  p.nslots = c->step_nslots;
  // producer pacing (measured on B200): a few stages in flight per SM keep HBM
  // busy; SS_STEP_INFLIGHT / SS_STEP_PREFETCH override for tuning sweeps
  p.inflight = std::max(1, std::min(c->step_nslots, env_int("SS_STEP_INFLIGHT", c->step_nslots)));
  p.prefetch = env_int("SS_STEP_PREFETCH", 0);
  p.split_rows = std::max(16, env_int("SS_STEP_SPLIT_ROWS", 64));
  p.wait_budget = kWaitBudget;
  p.test_withhold = -1;
  if (c->trace) {
    const size_t n = (size_t)(2 + 5 * c->L) * ncta * 8;
    c->step_trace = dev_alloc<long long>(c, n);
    CK(cudaMemset(c->step_trace, 0, n * sizeof(long long)));
    p.trace = c->step_trace;
  }
}

void launch_step(Context* c) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c->step_grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = c->step_smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  StepParams p = c->step_params;
  if (c->test_fail_phase > 0) {
    // one step of the failure-path test (ss_cuda_test_fail_next_step)
    p.test_withhold = c->test_fail_phase;
    p.wait_budget = kTestWaitBudget;
    c->test_fail_phase = 0;
  }
  void* args[2] = {&p, &c->step_tp};
  CK(cudaLaunchKernelExC(&cfg, c->step_fn, args));
}

using AttnFn = void (*)(const AttnParams);
AttnFn attn_fn(int hd) {
  switch (hd) {
    case 32: return &attention_kernel<32>;
    case 64: return &attention_kernel<64>;
    case 128: return &attention_kernel<128>;
    case 256: return &attention_kernel<256>;
    default: fail(SS_CUDA_ERROR_INVALID_MODEL, "head_dim %d", hd);
  }
}

void plan_all(Context* c) {
  CK(cudaFuncSetAttribute(attn_fn(c->hd), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->attn_smem));
  if (c->tiled) return;  // the persistent step was planned before the upload; no GEMV step
  const Layer& l0 = c->layers[0];
  c->g_qkv = plan_gemv_for(c, XSrc::RmsNorm, Epi::QKV, l0.qkv);
  c->g_o = plan_gemv_for(c, XSrc::Plain, Epi::Residual, l0.o);
  c->g_gu = plan_gemv_for(c, XSrc::RmsNorm, Epi::SwiGLU, l0.gu);
  c->g_down = plan_gemv_for(c, XSrc::Plain, Epi::Residual, l0.down);
  c->g_head = plan_gemv_for(c, XSrc::RmsNorm, Epi::Argmax, c->lm_head);
  if (c->g_head.ctas > 4096) fail(SS_CUDA_ERROR_INVALID_MODEL, "lm_head grid too large");
}

GemvParams base_params(Context* c) {
  GemvParams p = {};
  p.eps = c->eps;
  p.d_pos = &c->ctrl->pos;
  p.ctx = c->ctx;
  p.err = &c->ctrl->err;
  p.prefetch = c->tuning.prefetch;
  return p;
}

// ---- the kernels of one decode step ------------------------------------

void launch_embed(Context* c, bool pdl) {
  EmbedParams e{c->embd, c->d, c->vocab, c->L, c->ctx, c->seq_tokens, &c->ctrl->pos,
                c->h, c->amax, &c->ctrl->err};
  launch(embed_kernel, dim3(c->embed_blocks), dim3(256), 0, c->stream, pdl, e);
}

// RMSNorm(h) -> [Wq;Wk;Wv] -> RoPE(q, k), |k| / |v| maxima of this position.
void launch_qkv(Context* c, int l, bool pdl) {
  const Layer& ly = c->layers[(size_t)l];
  GemvParams p = base_params(c);
  p.w = ly.qkv.q();
  p.x = c->h;
  p.norm_w = ly.attn_norm;
  p.out = c->qkv;
  p.q_rows = c->nh * c->hd;
  p.kv_rows = c->nkv * c->hd;
  p.head_dim = c->hd;
  p.rope_dim = c->rope_dim;
  p.rope_tab = c->rope_tab;
  p.amax_k = c->amax + 2 * (size_t)l;
  p.amax_v = c->amax + 2 * (size_t)l + 1;
  run_gemv(c, c->g_qkv, p, pdl);
}

// int8 K/V append + GQA attention over positions 0..pos.
void launch_attn(Context* c, int l, bool pdl) {
  const int kvd = c->nkv * c->hd;
  const size_t lo = (size_t)l * c->ctx;
  AttnParams a{};
  a.qkv = c->qkv;
  a.kc = c->kc + lo * kvd;
  a.vc = c->vc + lo * kvd;
  a.ks = c->ks + lo;
  a.vs = c->vs + lo;
  a.amax_k = c->amax + 2 * (size_t)l;
  a.amax_v = c->amax + 2 * (size_t)l + 1;
  a.d_pos = &c->ctrl->pos;
  a.out = c->attn_out;
  a.nh = c->nh;
  a.nkv = c->nkv;
  a.hd = c->hd;
  a.ctx = c->ctx;
  a.nsplit = c->attn_nsplit;
  a.scale = c->attn_scale;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c->attn_nsplit, c->nkv);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = c->attn_smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = c->attn_nsplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  CK(cudaLaunchKernelEx(&cfg, attn_fn(c->hd), a));
}

// Tensor parallelism: sum of the ranks' row-parallel partials into h.  Rank
// 0's partial already holds the residual, so the sum is h + W . x.
void tp_reduce_h(Context* c) {
  NK(nccl_api().AllReduce(c->hpart, c->h, (size_t)c->d, ncclFloat32, ncclSum, c->comm, c->stream));
}

// h = Wo . attn + h  (tensor parallelism: this rank's heads' columns, then the
// all-reduce)
void launch_o(Context* c, int l, bool pdl) {
  GemvParams p = base_params(c);
  p.w = c->layers[(size_t)l].o.q();
  p.x = c->attn_out;
  const bool tp = c->tp_size > 1;
  p.out = tp ? c->hpart : c->h;
  p.residual = (!tp || c->tp_rank == 0) ? c->h : nullptr;
  run_gemv(c, c->g_o, p, pdl);
  if (tp) tp_reduce_h(c);
}

// act = up * silu(gate) of RMSNorm(h)
void launch_gu(Context* c, int l, bool pdl) {
  const Layer& ly = c->layers[(size_t)l];
  GemvParams p = base_params(c);
  p.w = ly.gu.q();
  p.x = c->h;
  p.norm_w = ly.ffn_norm;
  p.out = c->act;
  run_gemv(c, c->g_gu, p, pdl);
}

// h = Wdown . act + h  (tensor parallelism: this rank's FFN columns, then
// the all-reduce)
void launch_down(Context* c, int l, bool pdl) {
  const Layer& ly = c->layers[(size_t)l];
  GemvParams p = base_params(c);
  p.w = ly.down.q();
  p.x = c->act;
  const bool tp = c->tp_size > 1;
  p.out = tp ? c->hpart : c->h;
  p.residual = (!tp || c->tp_rank == 0) ? c->h : nullptr;
  run_gemv(c, c->g_down, p, pdl);
  if (ly.down2.cols) {
    // the second half of the FFN columns adds to the h the first half wrote
    // (one GPU only: the split is refused with tensor parallelism)
    p.w = ly.down2.q();
    p.x = c->act + ly.down.cols;
    run_gemv(c, c->g_down, p, pdl);
  }
  if (tp) tp_reduce_h(c);
}

// logits = W_out . RMSNorm(h); greedy argmax -> token of pos + 1; pos += 1.
void launch_head(Context* c, bool pdl) {
  GemvParams p = base_params(c);
  p.w = c->lm_head.q();
  p.x = c->h;
  p.norm_w = c->out_norm;
  p.out = c->logits;
  p.am_part = c->am_part;
  p.am_count = c->am_cnt;
  p.seq_tokens = c->seq_tokens;
  p.fixed_until = &c->ctrl->fixed_until;
  p.d_pos_rw = &c->ctrl->pos;
  if (c->tp_size > 1) {
    // this rank's vocab slice: its best (value, global index) -> max over the
    // ranks -> the token of pos + 1 (the same packed order as one GPU's)
    p.index_base = c->vocab_off;
    p.tp_best = c->tp_best;
    run_gemv(c, c->g_head, p, pdl);
    NK(nccl_api().AllReduce(c->tp_best, c->tp_best, 1, ncclUint64, ncclMax, c->comm, c->stream));
    launch(tp_finish_kernel, dim3(1), dim3(1), 0, c->stream, false, (const unsigned long long*)c->tp_best,
           &c->ctrl->pos, (const int*)&c->ctrl->fixed_until, c->seq_tokens, c->ctx);
    return;
  }
  run_gemv(c, c->g_head, p, pdl);
}

// Layer streaming: copies streamed layer l's GGUF bytes from host memory into
// the staging buffer and repacks them into the layer's slot, on the copy
// stream, then marks the slot ready.  The copy stream runs these in layer
// order, so the staging buffer is free again when the next copy starts.
void enqueue_layer_copy(Context* c, int l) {
  const Layer& ly = c->layers[(size_t)l];
  const int slot = (l - c->n_resident) % 2;
  for (const Context::StreamTensor& st : c->stream_src[(size_t)l])
    CK(cudaMemcpyAsync(c->stream_raw + st.raw_off, st.t.data, st.t.bytes, cudaMemcpyHostToDevice,
                       c->copy_stream));
  for (const Context::StreamTensor& st : c->stream_src[(size_t)l]) {
    const DevMatrix& dst = st.which == 0 ? ly.qkv : st.which == 1 ? ly.o : st.which == 2 ? ly.gu : ly.down;
    const int src_nb = (int)(st.t.cols() / 32);
    repack_into(c->stream_raw + st.raw_off, (int)st.t.rows(), src_nb, 0, st.t.type, dst, st.mul, st.add,
                c->copy_stream);
  }
  CK(cudaEventRecord(c->ev_ready[slot], c->copy_stream));
}

#include "qgemm_host.inc"
#include "batch_host.inc"

// Enqueues one decode step (embedding -> L layers -> lm_head + argmax).
// Streaming: the first two streamed layers' copies start with the step (their
// slots were last used by the previous step, which is complete in stream
// order); every later one starts when the layer two before it, which used the
// same slot, has finished its kernels.
void enqueue_step(Context* c, bool pdl) {
  if (c->mega) {
    launch_step(c);
    return;
  }
  if (bt_only(c)) {
    bt_dev_step(c);
    return;
  }
  const int R = c->n_resident;
  if (c->streaming) {
    CK(cudaEventRecord(c->ev_fork, c->stream));
    CK(cudaStreamWaitEvent(c->copy_stream, c->ev_fork, 0));
    enqueue_layer_copy(c, R);
    enqueue_layer_copy(c, R + 1);
  }
  launch_embed(c, pdl);
  for (int l = 0; l < c->L; l++) {
    const bool streamed = c->streaming && l >= R;
    if (streamed) CK(cudaStreamWaitEvent(c->stream, c->ev_ready[(l - R) % 2], 0));
    launch_qkv(c, l, pdl);
    if (c->tp_size > 1)  // one int8 scale over the whole kv_dim: max over the ranks' slices
      NK(nccl_api().AllReduce(c->amax + 2 * (size_t)l, c->amax + 2 * (size_t)l, 2, ncclUint32, ncclMax,
                              c->comm, c->stream));
    launch_attn(c, l, pdl);
    launch_o(c, l, pdl);
    launch_gu(c, l, pdl);
    launch_down(c, l, pdl);
    if (streamed && l + 2 < c->L) {
      const int slot = (l - R) % 2;
      CK(cudaEventRecord(c->ev_free[slot], c->stream));
      CK(cudaStreamWaitEvent(c->copy_stream, c->ev_free[slot], 0));
      enqueue_layer_copy(c, l + 2);
    }
  }
  launch_head(c, pdl);
}

void build_graph(Context* c) {
  // one launch per step needs no graph; the many-token step keeps its own
  if (c->step_exec || !c->use_graph || c->tiled) return;
  for (int attempt = 0; attempt < 2; attempt++) {
    const bool pdl = c->use_pdl && attempt == 0;
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    try {
      enqueue_step(c, pdl);
    } catch (...) {
      cudaStreamEndCapture(c->stream, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    CK(cudaStreamEndCapture(c->stream, &graph));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e == cudaSuccess) {
      c->step_exec = exec;
      c->graph_pdl = pdl;
      return;
    }
    cudaGetLastError();
    if (!pdl) fail(SS_CUDA_ERROR_BACKEND, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
  }
}

void run_steps(Context* c, int n) {
  if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
  if (n <= 0) return;
  if (c->host_pos + n > c->ctx)
    fail(SS_CUDA_ERROR_INVALID_PARAMS, "positions %d..%d exceed the context of %d", c->host_pos,
         c->host_pos + n - 1, c->ctx);
  build_graph(c);
  for (int i = 0; i < n; i++) {
    if (c->step_exec) CK(cudaGraphLaunch(c->step_exec, c->stream));
    else enqueue_step(c, c->use_pdl);
  }
  c->host_pos += n;
  c->steps_run += n;
}

void set_position(Context* c, int pos, int fixed_until) {
  if (pos < 0 || pos >= c->ctx) fail(SS_CUDA_ERROR_INVALID_PARAMS, "position %d outside 0..%d", pos, c->ctx - 1);
  c->h_small[0] = pos;
  c->h_small[1] = fixed_until;
  CK(cudaMemcpyAsync(c->ctrl, c->h_small, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
  c->host_pos = pos;
}

void put_tokens(Context* c, const int32_t* toks, int n, int pos) {
  for (int i = 0; i < n; i++)
    if (toks[i] < 0 || toks[i] >= c->vocab)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "token %d outside 0..%d", toks[i], c->vocab - 1);
  if (pos < 0 || pos + n > c->ctx) fail(SS_CUDA_ERROR_INVALID_PARAMS, "tokens past the context");
  CK(cudaMemcpyAsync(c->seq_tokens + pos, toks, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream));
}

// The prompt of sequence 0 (ss_scheduler_prefill, layer_scheduler.c:681-803):
// through the tensor-core product, 32 tokens per pass, where the weights are
// in its layout; otherwise the decode step replayed once per prompt token.
// Afterwards the last token's logits and greedy token are the context's.
void ingest_prompt(Context* c, const int32_t* tokens, int n, int start_pos) {
  put_tokens(c, tokens, n, start_pos);
  if (bt_eligible(c)) {
    bt_prefill(c, 0, tokens, n, start_pos);
  } else {
    set_position(c, start_pos, start_pos + n);
    run_steps(c, n);
  }
}

// Checks builds: the tensor-parallel step's record, to stderr.
void dump_step_dbg(Context* c) {
  const unsigned* d = c->dbg_host;
  if (!d) return;
  fprintf(stderr, "[step checks rank %d] consumer thread 0 per CTA (16 * (1 + phase) + sub-step, "
          "0x8...05: in a cross-rank wait):", c->tp_rank);
  for (int i = 0; i < c->step_grid; i++) fprintf(stderr, "%s%x", i % 16 ? " " : "\n  ", d[StepDbg::kCons + i]);
  fprintf(stderr, "\n[step checks rank %d] argmax exchange stage %u\n", c->tp_rank, d[StepDbg::kHead]);
  for (int i = 0; i < c->step_grid; i++) {
    const unsigned* e = d + StepDbg::kBad + 4 * i;
    if (e[0]) fprintf(stderr, "[step checks rank %d] cta %d violation %u at %u: rank %u offset %u\n",
                      c->tp_rank, i, e[0], e[1], e[2], e[3]);
  }
}

void check_device_error(Context* c) {
  int err = 0;
  CK(cudaMemcpyAsync(&c->h_small[8], &c->ctrl->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  {
    const cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
      dump_step_dbg(c);
      fail(SS_CUDA_ERROR_BACKEND, "cudaStreamSynchronize failed: %s", cudaGetErrorString(e));
    }
  }
  err = c->h_small[8];
  if (err) {
    CK(cudaMemsetAsync(&c->ctrl->err, 0, sizeof(int), c->stream));
    fail(SS_CUDA_ERROR_BACKEND,
         "device reported error bits 0x%x (1: position, 2: token, 4: ring wait, 8: grid barrier, "
         "16: shared-memory plan, 32: cross-GPU barrier)", err);
  }
}

void read_logits(Context* c, float* dst) {
  const float* src = c->logits;
  if (c->tp_size > 1) {  // every rank gathers the full logits (a collective: all ranks call it)
    NK(nccl_api().AllGather(c->logits, c->logits_full, (size_t)c->vocab_l, ncclFloat32, c->comm, c->stream));
    src = c->logits_full;
  }
  CK(cudaMemcpyAsync(c->h_logits, src, sizeof(float) * c->vocab, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaMemcpyAsync(&c->h_small[16], c->seq_tokens + c->ctx, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  check_device_error(c);
  if (dst && dst != c->h_logits) memcpy(dst, c->h_logits, sizeof(float) * c->vocab);
}

// Tensor parallelism: all ranks have reached this point (a collective on the
// library's communicator, then a host wait).
void tp_barrier(Context* c) {
  NK(nccl_api().AllReduce(c->tp_best, c->tp_best, 1, ncclUint64, ncclMax, c->comm, c->stream));
  CK(cudaStreamSynchronize(c->stream));
}

// Tensor parallelism, after the model is loaded on every rank: every rank
// must have planned the same step (an all-gather of the plan), then a barrier.
void tp_setup(Context* c) {
  const int tp = c->tp_size;
  int* dv = dev_alloc<int>(c, 2 * (size_t)tp);
  c->h_small[0] = c->mega ? 1 : 0;
  c->h_small[1] = c->mega ? c->step_grid : 0;
  CK(cudaMemcpyAsync(dv + 2 * c->tp_rank, c->h_small, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
  NK(nccl_api().AllGather(dv + 2 * c->tp_rank, dv, 2, ncclInt32, c->comm, c->stream));
  CK(cudaMemcpyAsync(c->h_small, dv, 2 * sizeof(int) * tp, cudaMemcpyDeviceToHost, c->stream));
  CK(cudaStreamSynchronize(c->stream));
  for (int r = 1; r < tp; r++)
    if (c->h_small[2 * r] != c->h_small[0] || c->h_small[2 * r + 1] != c->h_small[1])
      fail(SS_CUDA_ERROR_BACKEND, "tensor-parallel ranks planned different steps (rank 0: %d/%d, rank %d: %d/%d)",
           c->h_small[0], c->h_small[1], r, c->h_small[2 * r], c->h_small[2 * r + 1]);
  if (c->mega) {
    // the persistent step's exchange block, mapped by every peer (CUDA IPC;
    // the 64-byte handles travel by an NCCL all-gather)
    if (tp > kStepMaxTp) fail(SS_CUDA_ERROR_INVALID_PARAMS, "tensor parallelism above %d", kStepMaxTp);
    const size_t xb = StepXchg::bytes(tp, c->step_grid, c->d);
    c->xchg = dev_alloc<uint8_t>(c, xb);
    CK(cudaMemsetAsync(c->xchg, 0, xb, c->stream));
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, c->xchg));
    uint8_t* dh = dev_alloc<uint8_t>(c, sizeof(mine) * (size_t)tp);
    std::vector<cudaIpcMemHandle_t> all((size_t)tp);
    CK(cudaMemcpyAsync(dh + sizeof(mine) * c->tp_rank, &mine, sizeof(mine), cudaMemcpyHostToDevice, c->stream));
    NK(nccl_api().AllGather(dh + sizeof(mine) * c->tp_rank, dh, sizeof(mine), ncclUint8, c->comm, c->stream));
    CK(cudaMemcpyAsync(all.data(), dh, sizeof(mine) * tp, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    StepTp& t = c->step_tp;
    t = StepTp{};
    t.tp = tp;
    t.rank = c->tp_rank;
    t.vocab_off = c->vocab_off;
#ifdef SS_STEP_CHECKS
    t.xbytes = (long long)xb;
    CK(cudaHostAlloc(&c->dbg_host, sizeof(unsigned) * StepDbg::kWords, cudaHostAllocMapped));
    memset(c->dbg_host, 0, sizeof(unsigned) * StepDbg::kWords);
    CK(cudaHostGetDevicePointer(&t.dbg, c->dbg_host, 0));
#endif
    for (int r = 0; r < tp; r++) {
      if (r == c->tp_rank) {
        t.xpeer[r] = c->xchg;
        continue;
      }
      void* ptr = nullptr;
      CK(cudaIpcOpenMemHandle(&ptr, all[(size_t)r], cudaIpcMemLazyEnablePeerAccess));
      c->xpeer_open.push_back(ptr);
      t.xpeer[r] = static_cast<uint8_t*>(ptr);
    }
  }
  tp_barrier(c);  // every block zeroed and mapped before any rank's first step
}

// Copies n bytes with a few host threads (a one-time copy of the streamed
// layers into pinned memory).
void parallel_memcpy(uint8_t* dst, const uint8_t* src, size_t n) {
  const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  const size_t chunk = (n + hw - 1) / hw;
  std::vector<std::thread> ts;
  for (unsigned i = 0; i < hw; i++) {
    const size_t a = (size_t)i * chunk, e = std::min(n, a + chunk);
    if (a >= e) break;
    ts.emplace_back([=] { memcpy(dst + a, src + a, e - a); });
  }
  for (auto& t : ts) t.join();
}

// Layer streaming: the copy stream and its events, and DMA-able sources for
// the copies, so that they run at the host link's rate and can sit in the
// step's CUDA graph: the model's bytes registered with CUDA (read-only), or,
// where the platform does not register a read-only file mapping, the streamed
// layers' bytes copied once into pinned host memory.  Only when neither is
// possible do the copies come from pageable memory, which a graph cannot hold:
// the step then runs without one.  The bytes must stay mapped while the
// context lives (the registered case reads them every step).
void setup_streaming(Context* c, const uint8_t* base, uint64_t size) {
  c->use_pdl = false;  // the step is bound by the host link; plain stream order around the copies
  CK(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking));
  CK(cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming));
  for (int i = 0; i < 2; i++) {
    CK(cudaEventCreateWithFlags(&c->ev_ready[i], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&c->ev_free[i], cudaEventDisableTiming));
  }
  int ro = 0;
  cudaDeviceGetAttribute(&ro, cudaDevAttrHostRegisterReadOnlySupported, c->device);
  const uintptr_t page = (uintptr_t)sysconf(_SC_PAGESIZE);
  const uintptr_t a = (uintptr_t)base & ~(page - 1);
  const uintptr_t e = ((uintptr_t)base + size + page - 1) & ~(page - 1);
  // SS_STREAM_SOURCE=pinned / pageable skips the better sources (test coverage
  // of the fallbacks)
  const char* force = getenv("SS_STREAM_SOURCE");
  const bool allow_reg = !force || !strcmp(force, "registered");
  const bool allow_pin = !force || strcmp(force, "pageable") != 0;
  if (allow_reg && ro && cudaHostRegister((void*)a, e - a, cudaHostRegisterReadOnly) == cudaSuccess) {
    c->host_reg = (void*)a;
    return;
  }
  cudaGetLastError();
  if (!allow_pin || cudaHostAlloc(&c->host_pinned, c->streamed_bytes, cudaHostAllocDefault) != cudaSuccess) {
    cudaGetLastError();
    c->host_pinned = nullptr;
    c->use_graph = false;
    return;
  }
  size_t at = 0;
  for (auto& layer : c->stream_src) {
    if (layer.empty()) continue;
    size_t span = 0;
    for (Context::StreamTensor& st : layer) {
      parallel_memcpy(c->host_pinned + at + st.raw_off, st.t.data, st.t.bytes);
      st.t.data = c->host_pinned + at + st.raw_off;
      span = std::max(span, st.raw_off + round_up_sz(st.t.bytes, 256));
    }
    at += span;
  }
}

Context* create(const uint8_t* base, uint64_t size, const ss_cuda_options_t* o) {
  ss_cuda_options_t opts;
  ss_cuda_default_options(&opts);
  if (o) memcpy(&opts, o, std::min<size_t>(sizeof(opts), o->struct_size ? o->struct_size : sizeof(opts)));
  if (opts.max_batch == 0) opts.max_batch = 1;
  if (opts.max_batch > (uint32_t)kQgMaxT)
    fail(SS_CUDA_ERROR_INVALID_PARAMS, "max_batch %u: at most %d sequences decode together", opts.max_batch,
         kQgMaxT);
  int dev = opts.device;
  if (dev < 0) {
    const char* e = getenv("SS_CUDA_DEVICE");
    dev = e ? atoi(e) : 0;
  }
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (dev >= ndev) fail(SS_CUDA_ERROR_INVALID_PARAMS, "device %d of %d", dev, ndev);
  CK(cudaSetDevice(dev));
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, dev));
  if (prop.major < 10) fail(SS_CUDA_ERROR_BACKEND, "device %s is sm_%d%d; sm_100a required", prop.name, prop.major, prop.minor);
  auto* c = new Context();
  c->device = dev;
  c->sm_count = prop.multiProcessorCount;
  c->max_batch = (int)opts.max_batch;
  c->use_pdl = !(opts.flags & SS_CUDA_FLAG_NO_PDL) && !getenv("SS_CUDA_NO_PDL");
  c->use_graph = !(opts.flags & SS_CUDA_FLAG_NO_GRAPH);
  c->tuning = read_tuning();
  c->mega = !(opts.flags & SS_CUDA_FLAG_MULTI_KERNEL) && !getenv("SS_CUDA_MULTI_KERNEL");
  c->trace = (opts.flags & SS_CUDA_FLAG_TRACE) != 0;
  c->flags = opts.flags;
  c->tp_size = opts.tp_size > 1 ? opts.tp_size : 1;
  c->tp_rank = c->tp_size > 1 ? opts.tp_rank : 0;
  c->hbm_budget = opts.hbm_budget_bytes;
  try {
    if (c->tp_size > 1) {
      if (c->tp_rank < 0 || c->tp_rank >= c->tp_size)
        fail(SS_CUDA_ERROR_INVALID_PARAMS, "tp_rank %d outside 0..%d", c->tp_rank, c->tp_size - 1);
      if (!nccl_api().ok) fail(SS_CUDA_ERROR_BACKEND, "tensor parallelism needs libnccl.so.2 (not found)");
      // the multi-kernel step's collectives sit between its kernels; a graph
      // with NCCL inside is built without programmatic dependent launch.  The
      // persistent step exchanges inside the kernel (tp_setup).
      c->use_pdl = false;
      ncclUniqueId id;
      static_assert(sizeof(id) == sizeof(opts.tp_nccl_id), "NCCL unique id size");
      memcpy(&id, opts.tp_nccl_id, sizeof(id));
      NK(nccl_api().CommInitRank(&c->comm, c->tp_size, id, c->tp_rank));
    }
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    if (base) {
      load_model(c, base, size, opts.context_size);
      if (c->max_batch > 1 && !bt_shapes_ok(c))
        fail(SS_CUDA_ERROR_INVALID_MODEL, "max_batch %d: the weights' blocks do not fit the batched product",
             c->max_batch);
      if (c->streaming) setup_streaming(c, base, size);
      alloc_state(c);
      plan_all(c);
      if (c->tp_size > 1) tp_setup(c);
      CK(cudaStreamSynchronize(c->stream));
      c->has_model = true;
    }
  } catch (...) {
    ss_cuda_free(reinterpret_cast<ss_cuda_ctx_t*>(c));
    throw;
  }
  return c;
}

Context* need_model(ss_cuda_ctx_t* ctx) {
  auto* c = reinterpret_cast<Context*>(ctx);
  if (!c) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null context");
  if (!c->has_model) fail(SS_CUDA_ERROR_INVALID_PARAMS, "context has no model");
  CK(cudaSetDevice(c->device));
  return c;
}

// ------------------------------------------------- op-level (Metal twin) path

OpCacheEntry& op_weights(Context* c, const void* mat, int rows, int cols, int type) {
  auto it = c->op_cache.find(mat);
  if (it != c->op_cache.end()) {
    const OpCacheEntry& e = it->second;
    const int r = e.f32 ? e.m.rows : e.m.rows, cc = e.m.cols;
    if (r == rows && cc == cols && e.m.type == type) return it->second;
    fail(SS_CUDA_ERROR_INVALID_PARAMS, "weight pointer reused with a different shape");
  }
  OpCacheEntry e;
  e.m.rows = rows;
  e.m.cols = cols;
  e.m.type = type;
  if (type == kF32) {
    e.f32 = dev_alloc<float>(c, (size_t)rows * cols);
    CK(cudaMemcpyAsync(e.f32, mat, sizeof(float) * (size_t)rows * cols, cudaMemcpyHostToDevice, c->stream));
  } else if (type == kQ4_K) {
    const size_t bytes = (size_t)rows * (cols / 256) * 144;
    e.raw = dev_alloc<uint8_t>(c, bytes);
    CK(cudaMemcpyAsync(e.raw, mat, bytes, cudaMemcpyHostToDevice, c->stream));
  } else {
    e.m = layout(rows, cols, type);
    e.m.data = dev_alloc<uint8_t>(c, matrix_bytes(e.m));
    CK(cudaMemsetAsync(e.m.data, 0, matrix_bytes(e.m), c->stream));
    GgufTensor t;
    t.name = "matvec operand";
    t.n_dims = 2;
    t.dims[0] = (uint64_t)cols;
    t.dims[1] = (uint64_t)rows;
    t.type = type;
    t.bytes = (uint64_t)rows * (cols / 32) * ggml_type_size(type);
    t.data = static_cast<const uint8_t*>(mat);
    if (c->op_stage_cap < t.bytes) {
      if (c->op_stage) CK(cudaFree(c->op_stage));
      c->op_stage = nullptr;
      CK(cudaMalloc(&c->op_stage, t.bytes));
      c->op_stage_cap = t.bytes;
    }
    upload_matrix(c, t, e.m, 1, 0, c->op_stage, c->op_stage_cap);
  }
  return c->op_cache.emplace(mat, e).first->second;
}

bool op_matvec(ss_cuda_ctx_t* ctx, float* out, const void* mat, const float* vec, int rows, int cols,
               int type) {
  return guard([&] {
           auto* c = reinterpret_cast<Context*>(ctx);
           if (!c || !out || !mat || !vec || rows <= 0 || cols <= 0)
             fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad matvec arguments");
           if (type != kF32 && cols % (type == kQ4_K ? 256 : 32))
             fail(SS_CUDA_ERROR_INVALID_PARAMS, "cols %d not a multiple of the block size", cols);
           CK(cudaSetDevice(c->device));
           OpCacheEntry& w = op_weights(c, mat, rows, cols, type);
           const int slot = c->in_batch ? c->batch_count : 0;
           if (c->in_batch && slot >= 64) fail(SS_CUDA_ERROR_INVALID_PARAMS, "more than 64 matvecs in a batch");
           if ((int)c->op_slots.size() <= slot) c->op_slots.resize((size_t)slot + 1);
           auto& s = c->op_slots[(size_t)slot];
           if (s.x_cap < (size_t)cols) {
             if (s.d_x) CK(cudaFree(s.d_x));
             s.d_x = nullptr;
             CK(cudaMalloc(&s.d_x, sizeof(float) * cols));
             s.x_cap = (size_t)cols;
           }
           if (s.out_cap < (size_t)rows) {
             if (s.d_out) CK(cudaFree(s.d_out));
             s.d_out = nullptr;
             CK(cudaMalloc(&s.d_out, sizeof(float) * rows));
             s.out_cap = (size_t)rows;
           }
           CK(cudaMemcpyAsync(s.d_x, vec, sizeof(float) * cols, cudaMemcpyHostToDevice, c->stream));
           if (type == kF32) {
             const int threads = 256;
             const int grid = (rows * 32 + threads - 1) / threads;
             matvec_f32_kernel<<<grid, threads, 0, c->stream>>>(w.f32, s.d_x, s.d_out, rows, cols);
             CK(cudaGetLastError());
           } else if (type == kQ4_K) {
             CK(matvec_q4k_launch(w.raw, s.d_x, s.d_out, rows, cols, c->stream));
           } else {
             GemvLaunch g = plan_gemv_for(c, XSrc::Plain, Epi::Store, w.m);
             GemvParams p = base_params(c);
             p.w = w.m.q();
             p.x = s.d_x;
             p.out = s.d_out;
             p.prefetch = 0;
             run_gemv(c, g, p, false);
           }
           if (c->in_batch) {
             s.host_out = out;
             s.out_n = (size_t)rows;
             c->batch_count++;
           } else {
             CK(cudaMemcpyAsync(out, s.d_out, sizeof(float) * rows, cudaMemcpyDeviceToHost, c->stream));
             CK(cudaStreamSynchronize(c->stream));
           }
           c->ops_run++;
         }) == SS_CUDA_OK;
}


// A quantized weight tensor by GGUF name: its device matrix and where its rows
// sit there (row r of the tensor is matrix row r * mul + add).
const DevMatrix* find_named(Context* c, const std::string& s, int& rows, int& mul, int& add) {
  mul = 1;
  add = 0;
  rows = 0;
  const int qd = c->nh * c->hd, kvd = c->nkv * c->hd;
  if (s == "output.weight") { rows = c->vocab_l; return &c->lm_head; }
  if (s.rfind("blk.", 0) != 0) return nullptr;
  const int l = atoi(s.c_str() + 4);
  const size_t dot = s.find('.', 4);
  if (l < 0 || l >= c->L || dot == std::string::npos) return nullptr;
  const std::string suf = s.substr(dot + 1);
  const Layer& ly = c->layers[(size_t)l];
  if (suf == "attn_q.weight") { rows = qd; return &ly.qkv; }
  if (suf == "attn_k.weight") { rows = kvd; add = qd; return &ly.qkv; }
  if (suf == "attn_v.weight") { rows = kvd; add = qd + kvd; return &ly.qkv; }
  if (suf == "attn_output.weight") { rows = c->d; return &ly.o; }
  if (suf == "ffn_gate.weight") { rows = c->ff; mul = 2; return &ly.gu; }
  if (suf == "ffn_up.weight") { rows = c->ff; mul = 2; add = 1; return &ly.gu; }
  if (suf == "ffn_down.weight") { rows = c->d; return ly.down2.cols ? nullptr : &ly.down; }
  return nullptr;
}

}  // namespace
}  // namespace ss

using namespace ss;

SS_API int ss_cuda_matmul_batch(ss_cuda_ctx_t* ctx, const char* name, const float* x, int32_t n_tokens,
                                float* out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!name || !x || !out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    if (n_tokens < 1 || n_tokens > kQgMaxT) fail(SS_CUDA_ERROR_INVALID_PARAMS, "n_tokens must be 1..%d", kQgMaxT);
    int rows, mul, add;
    const DevMatrix* m = find_named(c, name, rows, mul, add);
    if (!m) fail(SS_CUDA_ERROR_INVALID_PARAMS, "no quantized tensor %s", name);
    if (!m->tiled) fail(SS_CUDA_ERROR_INVALID_PARAMS, "the many-token product needs the persistent step's layout");
    const int T = n_tokens, K = m->cols, R = m->rows;
    float* d_x = nullptr;
    float* d_y = nullptr;
    CK(cudaMalloc(&d_x, sizeof(float) * (size_t)T * K));
    cudaError_t e = cudaMalloc(&d_y, sizeof(float) * (size_t)T * R);
    std::vector<float> y((size_t)T * R);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_x, x, sizeof(float) * (size_t)T * K, cudaMemcpyHostToDevice, c->stream);
    int nsplit = 0;
    if (e == cudaSuccess) {
      try {
        nsplit = qg_product(c, *m, d_x, K, nullptr, T);
      } catch (...) {
        cudaFree(d_x);
        cudaFree(d_y);
        throw;
      }
      qg_sum_kernel<<<256, 256, 0, c->stream>>>(c->qg_out, nsplit, T, R, d_y);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(y.data(), d_y, sizeof(float) * y.size(), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(d_x);
    cudaFree(d_y);
    CK(e);
    check_device_error(c);
    for (int t = 0; t < T; t++)
      for (int r = 0; r < rows; r++) out[(size_t)t * rows + r] = y[(size_t)t * R + (size_t)r * mul + add];
  });
}

// ======================================================================= C ABI

SS_API void ss_cuda_default_options(ss_cuda_options_t* o) {
  if (!o) return;
  memset(o, 0, sizeof(*o));
  o->struct_size = sizeof(*o);
  o->device = -1;
  o->max_batch = 1;
}

SS_API int ss_cuda_abi_version(void) { return SS_CUDA_ABI_VERSION; }

SS_API const char* ss_cuda_last_error(void) { return g_err.c_str(); }

SS_API ss_cuda_ctx_t* ss_cuda_init(const void* gguf_base, uint64_t gguf_size, const ss_cuda_options_t* opts) {
  Context* c = nullptr;
  const int rc = guard([&] { c = create(static_cast<const uint8_t*>(gguf_base), gguf_size, opts); });
  return rc == SS_CUDA_OK ? reinterpret_cast<ss_cuda_ctx_t*>(c) : nullptr;
}

SS_API ss_cuda_ctx_t* ss_cuda_init_file(const char* path, const ss_cuda_options_t* opts) {
  Context* c = nullptr;
  const int rc = guard([&] {
    if (!path) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null path");
    const int fd = open(path, O_RDONLY);
    if (fd < 0) fail(SS_CUDA_ERROR_FILE_NOT_FOUND, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); fail(SS_CUDA_ERROR_FILE_NOT_FOUND, "cannot stat %s", path); }
    void* map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (map == MAP_FAILED) fail(SS_CUDA_ERROR_INVALID_MODEL, "mmap of %s failed", path);
    madvise(map, (size_t)st.st_size, MADV_SEQUENTIAL);
    try {
      c = create(static_cast<const uint8_t*>(map), (uint64_t)st.st_size, opts);
    } catch (...) {
      munmap(map, (size_t)st.st_size);
      throw;
    }
    if (c->streaming) {  // streamed layers are read from the mapping every step
      c->owned_map = map;
      c->owned_map_bytes = (size_t)st.st_size;
    } else {
      munmap(map, (size_t)st.st_size);
    }
  });
  return rc == SS_CUDA_OK ? reinterpret_cast<ss_cuda_ctx_t*>(c) : nullptr;
}

SS_API void ss_cuda_free(ss_cuda_ctx_t* ctx) {
  auto* c = reinterpret_cast<Context*>(ctx);
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->step_exec) cudaGraphExecDestroy(c->step_exec);  // before the communicator it uses
  for (auto& g : c->bt_graphs)
    if (g.second) cudaGraphExecDestroy(g.second);
  if (c->bt_dev_exec) cudaGraphExecDestroy(c->bt_dev_exec);
  if (c->bt_meta_host) cudaFreeHost(c->bt_meta_host);
  if (c->comm) {
    // no rank unmaps or frees an exchange block while a peer may still use it
    if (c->has_model && c->xchg) guard([&] { tp_barrier(c); });
    for (void* ptr : c->xpeer_open) cudaIpcCloseMemHandle(ptr);
    if (c->has_model && c->xchg) guard([&] { tp_barrier(c); });
    nccl_api().CommDestroy(c->comm);
  }
  for (void* p : c->allocations) cudaFree(p);
  for (auto& s : c->op_slots) {
    if (s.d_x) cudaFree(s.d_x);
    if (s.d_out) cudaFree(s.d_out);
  }
  if (c->op_stage) cudaFree(c->op_stage);
  if (c->smp_dev) cudaFree(c->smp_dev);
  if (c->smp_host) cudaFreeHost(c->smp_host);
  if (c->h_logits) cudaFreeHost(c->h_logits);
  if (c->h_small) cudaFreeHost(c->h_small);
  if (c->dbg_host) cudaFreeHost(c->dbg_host);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
  for (cudaEvent_t ev : {c->ev_fork, c->ev_ready[0], c->ev_ready[1], c->ev_free[0], c->ev_free[1]})
    if (ev) cudaEventDestroy(ev);
  if (c->host_reg) cudaHostUnregister(c->host_reg);
  if (c->host_pinned) cudaFreeHost(c->host_pinned);
  if (c->owned_map) munmap(c->owned_map, c->owned_map_bytes);
  delete c;
}

SS_API int ss_cuda_tp_unique_id(uint8_t* id_out) {
  return guard([&] {
    if (!id_out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    if (!nccl_api().ok) fail(SS_CUDA_ERROR_BACKEND, "libnccl.so.2 not found");
    ncclUniqueId id;
    NK(nccl_api().GetUniqueId(&id));
    memcpy(id_out, &id, sizeof(id));
  });
}

SS_API int ss_cuda_model_dims(const ss_cuda_ctx_t* ctx, int32_t* dims) {
  return guard([&] {
    auto* c = reinterpret_cast<const Context*>(ctx);
    if (!c || !dims) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    // the whole model's dimensions, also under tensor parallelism
    const int32_t v[12] = {c->vocab, c->d, c->L, c->nh_full, c->nkv_full, c->hd, c->ff_full, c->ctx, c->rope_dim,
                           c->wtype, c->max_batch, c->device};
    memcpy(dims, v, sizeof(v));
  });
}

SS_API int ss_cuda_stats(const ss_cuda_ctx_t* ctx, int64_t* out, int32_t n) {
  return guard([&] {
    auto* c = reinterpret_cast<const Context*>(ctx);
    if (!c || !out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    // architecture the loaded kernels were compiled for (100 = sm_100a)
    cudaFuncAttributes fa{};
    const int64_t arch = cudaFuncGetAttributes(&fa, embed_kernel) == cudaSuccess ? fa.binaryVersion : -1;
    cudaGetLastError();
    const int64_t v[17] = {c->has_model ? (c->mega ? 1 : bt_only(c) ? bt_launches(c, 1) + 2 : 2 + 5LL * c->L + (c->tp_size > 1) +
                                                   (c->layers[0].down2.cols ? (int64_t)c->L : 0) +
                                                   (c->streaming ? 7LL * (c->L - c->n_resident) : 0))
                                       : 0,
                           (int64_t)c->weight_bytes,
                           (int64_t)c->kv_bytes,
                           c->mega ? c->step_nsplit : c->attn_nsplit,
                           c->graph_pdl ? 1 : 0,
                           c->steps_run,
                           c->mega ? c->step_grid : c->g_qkv.ctas,
                           c->mega ? c->step_grid : c->g_down.ctas,
                           c->mega ? 1 : 0,
                           c->mega ? c->step_nslots : 0,
                           c->n_resident,
                           (int64_t)c->streamed_bytes,
                           (int64_t)c->layer_stride,
                           !c->streaming ? 0 : c->host_reg ? 1 : c->host_pinned ? 2 : 3,
                           arch,
                           c->has_model && c->tiled ? bt_launches(c, 1) + 1 : 0,
                           c->ops_run};
    for (int i = 0; i < n && i < 17; i++) out[i] = v[i];
  });
}

SS_API bool ss_cuda_should_use_gpu(int32_t rows, int32_t cols) {
  (void)rows;
  (void)cols;
  return true;  // every matvec runs on the GPU; there is no CPU fallback
}

SS_API bool ss_cuda_matvec(ss_cuda_ctx_t* ctx, float* out, const float* mat, const float* vec, int32_t rows, int32_t cols) {
  return op_matvec(ctx, out, mat, vec, rows, cols, kF32);
}
SS_API bool ss_cuda_matvec_q4_0(ss_cuda_ctx_t* ctx, float* out, const void* mat, const float* vec, int32_t rows, int32_t cols) {
  return op_matvec(ctx, out, mat, vec, rows, cols, kQ4_0);
}
SS_API bool ss_cuda_matvec_q8_0(ss_cuda_ctx_t* ctx, float* out, const void* mat, const float* vec, int32_t rows, int32_t cols) {
  return op_matvec(ctx, out, mat, vec, rows, cols, kQ8_0);
}
SS_API bool ss_cuda_matvec_q4_K(ss_cuda_ctx_t* ctx, float* out, const void* mat, const float* vec, int32_t rows, int32_t cols) {
  return op_matvec(ctx, out, mat, vec, rows, cols, kQ4_K);
}

SS_API void ss_cuda_begin_batch(ss_cuda_ctx_t* ctx) {
  auto* c = reinterpret_cast<Context*>(ctx);
  if (!c || c->in_batch) return;
  c->in_batch = true;
  c->batch_count = 0;
}

SS_API void ss_cuda_end_batch(ss_cuda_ctx_t* ctx) {
  auto* c = reinterpret_cast<Context*>(ctx);
  if (!c || !c->in_batch) return;
  guard([&] {
    CK(cudaSetDevice(c->device));
    for (int i = 0; i < c->batch_count; i++) {
      auto& s = c->op_slots[(size_t)i];
      CK(cudaMemcpyAsync(s.host_out, s.d_out, sizeof(float) * s.out_n, cudaMemcpyDeviceToHost, c->stream));
    }
    CK(cudaStreamSynchronize(c->stream));
  });
  c->in_batch = false;
  c->batch_count = 0;
}

SS_API float* ss_cuda_scheduler_forward(ss_cuda_ctx_t* ctx, int32_t token_id, int32_t pos) {
  float* res = nullptr;
  guard([&] {
    Context* c = need_model(ctx);
    if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
    put_tokens(c, &token_id, 1, pos);
    set_position(c, pos, pos + 1);
    run_steps(c, 1);
    read_logits(c, nullptr);
    res = c->h_logits;
  });
  return res;
}

SS_API float* ss_cuda_scheduler_prefill(ss_cuda_ctx_t* ctx, const int32_t* tokens, int32_t n, int32_t start_pos) {
  float* res = nullptr;
  guard([&] {
    Context* c = need_model(ctx);
    if (!tokens || n <= 0) fail(SS_CUDA_ERROR_INVALID_PARAMS, "empty prompt");
    if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
    ingest_prompt(c, tokens, n, start_pos);
    read_logits(c, nullptr);
    res = c->h_logits;
  });
  return res;
}

SS_API void ss_cuda_reset(ss_cuda_ctx_t* ctx) {
  guard([&] {
    Context* c = need_model(ctx);
    const size_t rows = (size_t)c->max_batch * c->L * c->ctx, kvd = (size_t)c->nkv * c->hd;
    CK(cudaMemsetAsync(c->kc, 0, rows * kvd, c->stream));
    CK(cudaMemsetAsync(c->vc, 0, rows * kvd, c->stream));
    CK(cudaMemsetAsync(c->ks, 0, rows * 4, c->stream));
    CK(cudaMemsetAsync(c->vs, 0, rows * 4, c->stream));
    CK(cudaMemsetAsync(c->amax, 0, 2 * sizeof(unsigned) * c->L, c->stream));
    CK(cudaMemsetAsync(c->h, 0, sizeof(float) * c->d, c->stream));
    CK(cudaMemsetAsync(c->ctrl, 0, sizeof(Ctrl), c->stream));
    CK(cudaMemsetAsync(c->am_cnt, 0, sizeof(unsigned), c->stream));
    if (c->step_sync)
      CK(cudaMemsetAsync(c->step_sync, 0, sizeof(unsigned) * c->step_sync_words, c->stream));
    if (c->xchg) CK(cudaMemsetAsync(c->xchg, 0, StepXchg::kCounters, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    // tensor parallelism: every rank's counters are zero before any rank's next step
    if (c->xchg) tp_barrier(c);
    c->host_pos = 0;
    c->cancelled.store(false);
  });
}

SS_API void ss_cuda_scheduler_reset(ss_cuda_ctx_t* ctx) { ss_cuda_reset(ctx); }

SS_API int ss_cuda_test_fail_next_step(ss_cuda_ctx_t* ctx, int32_t phase) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!c->mega) fail(SS_CUDA_ERROR_INVALID_PARAMS, "only the persistent step has this test aid");
    if (c->tp_size > 1) fail(SS_CUDA_ERROR_INVALID_PARAMS, "single-GPU contexts only");
    if (phase < 1 || phase > 1 + 5 * c->L) fail(SS_CUDA_ERROR_INVALID_PARAMS, "phase %d", phase);
    if ((phase - 1) % 5 == 1) fail(SS_CUDA_ERROR_INVALID_PARAMS, "phase %d streams no weights", phase);
    c->test_fail_phase = phase;
  });
}

SS_API void ss_cuda_cancel(ss_cuda_ctx_t* ctx) {
  auto* c = reinterpret_cast<Context*>(ctx);
  if (c) c->cancelled.store(true);
}

SS_API int ss_cuda_forward(ss_cuda_ctx_t* ctx, const int32_t* token_ids, int32_t n_seq, int32_t pos,
                           float* logits_out, int32_t* argmax_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!token_ids || n_seq < 1) fail(SS_CUDA_ERROR_INVALID_PARAMS, "no tokens");
    if (n_seq > 1) {
      // sequences 0..n_seq-1 together, one token each at position pos
      if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
      if (!bt_eligible(c)) fail(SS_CUDA_ERROR_INVALID_PARAMS, "n_seq %d: the context decodes one sequence", n_seq);
      bt_decode(c, token_ids, n_seq, pos);
      if (logits_out)
        CK(cudaMemcpyAsync(logits_out, c->bt_logits, sizeof(float) * (size_t)n_seq * c->vocab_l,
                           cudaMemcpyDeviceToHost, c->stream));
      CK(cudaMemcpyAsync(&c->h_small[32], c->bt_meta + 3 * kQgMaxT, sizeof(int) * n_seq, cudaMemcpyDeviceToHost,
                         c->stream));
      check_device_error(c);
      if (argmax_out) memcpy(argmax_out, &c->h_small[32], sizeof(int) * n_seq);
      return;
    }
    put_tokens(c, token_ids, 1, pos);
    set_position(c, pos, pos + 1);
    run_steps(c, 1);
    if (logits_out) {
      read_logits(c, logits_out);
    } else {
      CK(cudaMemcpyAsync(&c->h_small[16], c->seq_tokens + c->ctx, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
      check_device_error(c);
    }
    if (argmax_out) *argmax_out = c->h_small[16];
  });
}

SS_API int ss_cuda_prefill(ss_cuda_ctx_t* ctx, const int32_t* tokens, int32_t n, int32_t start_pos, float* logits_out) {
  int tok = -1;
  const int rc = guard([&] {
    Context* c = need_model(ctx);
    if (!tokens || n <= 0) fail(SS_CUDA_ERROR_INVALID_PARAMS, "empty prompt");
    if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
    ingest_prompt(c, tokens, n, start_pos);
    read_logits(c, logits_out ? logits_out : nullptr);
    tok = c->h_small[16];
  });
  return rc == SS_CUDA_OK ? tok : rc;
}

SS_API int ss_cuda_prefill_batch(ss_cuda_ctx_t* ctx, const int32_t* tokens, int32_t n_seq, int32_t n,
                                 int32_t start_pos, float* logits_out, int32_t* argmax_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!tokens || n <= 0 || n_seq < 1) fail(SS_CUDA_ERROR_INVALID_PARAMS, "empty prompt");
    if (n_seq > c->max_batch)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "n_seq %d outside 1..%d (max_batch)", n_seq, c->max_batch);
    if (!bt_eligible(c)) fail(SS_CUDA_ERROR_INVALID_PARAMS, "the batched prompt needs the many-token step");
    for (int s = 0; s < n_seq; s++) {
      if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
      const int32_t* t = tokens + (size_t)s * n;
      if (s == 0) put_tokens(c, t, n, start_pos);
      bt_prefill(c, s, t, n, start_pos);
      if (logits_out)
        CK(cudaMemcpyAsync(logits_out + (size_t)s * c->vocab_l, c->bt_logits, sizeof(float) * c->vocab_l,
                           cudaMemcpyDeviceToHost, c->stream));
      CK(cudaMemcpyAsync(&c->h_small[32 + s], c->bt_meta + 3 * kQgMaxT, sizeof(int), cudaMemcpyDeviceToHost,
                         c->stream));
    }
    check_device_error(c);
    if (argmax_out) memcpy(argmax_out, &c->h_small[32], sizeof(int) * n_seq);
  });
}

SS_API int ss_cuda_decode_greedy_batch(ss_cuda_ctx_t* ctx, const int32_t* tokens, int32_t n_seq,
                                      int32_t start_pos, int32_t n_steps, int32_t* ids_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!tokens || !ids_out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    if (!bt_eligible(c)) fail(SS_CUDA_ERROR_INVALID_PARAMS, "batched decode needs the many-token step");
    bt_decode_greedy(c, tokens, n_seq, start_pos, n_steps);
    check_device_error(c);
    std::vector<int> rows((size_t)n_steps * kQgMaxT);
    CK(cudaMemcpy(rows.data(), c->bt_ids + (size_t)(start_pos + 1) * kQgMaxT, sizeof(int) * rows.size(),
                  cudaMemcpyDeviceToHost));
    for (int k = 0; k < n_steps; k++)
      for (int s = 0; s < n_seq; s++) ids_out[(size_t)k * n_seq + s] = rows[(size_t)k * kQgMaxT + s];
  });
}

SS_API int ss_cuda_embed(ss_cuda_ctx_t* ctx, const int32_t* tokens, int32_t n, float* out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!tokens || !out || n <= 0) fail(SS_CUDA_ERROR_INVALID_PARAMS, "empty prompt");
    if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
    if (!bt_eligible(c)) fail(SS_CUDA_ERROR_INVALID_PARAMS, "the embedding needs the many-token step");
    put_tokens(c, tokens, n, 0);
    bt_embed(c, tokens, n);
    CK(cudaMemcpyAsync(out, c->bt_emb + c->d, sizeof(float) * c->d, cudaMemcpyDeviceToHost, c->stream));
    check_device_error(c);
  });
}

SS_API float* ss_cuda_scheduler_embed(ss_cuda_ctx_t* ctx, const int32_t* tokens, int32_t n) {
  auto* c = reinterpret_cast<Context*>(ctx);
  if (!c || !c->has_model) return nullptr;
  float* e = static_cast<float*>(malloc(sizeof(float) * (size_t)c->d));
  if (!e) return nullptr;
  if (ss_cuda_embed(ctx, tokens, n, e) != SS_CUDA_OK) {
    free(e);
    return nullptr;
  }
  return e;
}

SS_API int ss_cuda_decode_begin(ss_cuda_ctx_t* ctx, int32_t token, int32_t pos) {
  return guard([&] {
    Context* c = need_model(ctx);
    put_tokens(c, &token, 1, pos);
    set_position(c, pos, pos + 1);
  });
}

SS_API int ss_cuda_decode_steps(ss_cuda_ctx_t* ctx, int32_t n_steps) {
  return guard([&] {
    Context* c = need_model(ctx);
    run_steps(c, n_steps);
  });
}

SS_API int ss_cuda_decode_read(ss_cuda_ctx_t* ctx, int32_t first_pos, int32_t n, int32_t* ids_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!ids_out || n < 0 || first_pos < 0 || first_pos + n > c->ctx + 1)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad token range");
    check_device_error(c);
    CK(cudaMemcpy(ids_out, c->seq_tokens + first_pos, sizeof(int) * n, cudaMemcpyDeviceToHost));
  });
}

SS_API int ss_cuda_decode_greedy(ss_cuda_ctx_t* ctx, int32_t token, int32_t start_pos, int32_t n_steps, int32_t* ids_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!ids_out || n_steps <= 0) fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad arguments");
    if (start_pos + n_steps >= c->ctx + 1) fail(SS_CUDA_ERROR_INVALID_PARAMS, "decode runs past the context");
    put_tokens(c, &token, 1, start_pos);
    set_position(c, start_pos, start_pos + 1);
    run_steps(c, n_steps);
    check_device_error(c);
    // tokens of positions start_pos+1 .. start_pos+n_steps; the last one may sit
    // at index ctx (the last-argmax slot) when it falls past the context
    const int in_ctx = std::min(n_steps, c->ctx - 1 - start_pos);
    if (in_ctx > 0)
      CK(cudaMemcpy(ids_out, c->seq_tokens + start_pos + 1, sizeof(int) * in_ctx, cudaMemcpyDeviceToHost));
    if (in_ctx < n_steps)
      CK(cudaMemcpy(ids_out + in_ctx, c->seq_tokens + c->ctx, sizeof(int), cudaMemcpyDeviceToHost));
  });
}

// ------------------------------------------------------------ sampling
// ss_sample (SlipStream/src/core/tensor.c:363-451) on the device: the
// context's sampler buffers, one draw, and the generation loop of ss_generate
// (engine.c:233-289) with the draw between decode steps on the device.

constexpr int kSmpMaxDraws = kQgMaxT;                   // draws per launch (the batch limit)
constexpr size_t kSmpTokOff = 8 * kSmpMaxDraws;          // tokens after the RNG states
constexpr size_t kSmpInOff = 512;                        // caller logits after the header

size_t smp_slice(int n) { return round_up_sz(sample_scratch_bytes(n), 256); }

void smp_reserve(Context* c, int n, int batch = 1) {
  if (n < 1 || n > kSampleMaxN) fail(SS_CUDA_ERROR_INVALID_PARAMS, "vocabulary size %d outside 1..%d", n, kSampleMaxN);
  if (!c->smp_host) CK(cudaHostAlloc(reinterpret_cast<void**>(&c->smp_host), kSmpInOff, cudaHostAllocDefault));
  if (n <= c->smp_cap && batch <= c->smp_batch) return;
  n = std::max(n, c->smp_cap);
  batch = std::max(batch, c->smp_batch);
  CK(cudaStreamSynchronize(c->stream));
  if (c->smp_dev) {
    CK(cudaFree(c->smp_dev));
    c->smp_dev = nullptr;
    c->smp_cap = c->smp_batch = 0;
  }
  const size_t bytes = kSmpInOff + round_up_sz((size_t)n * sizeof(float), 256) + (size_t)batch * smp_slice(n);
  CK(cudaMalloc(reinterpret_cast<void**>(&c->smp_dev), bytes));
  c->smp_cap = n;
  c->smp_batch = batch;
}
unsigned long long* smp_rng(Context* c) { return reinterpret_cast<unsigned long long*>(c->smp_dev); }
int* smp_token(Context* c) { return reinterpret_cast<int*>(c->smp_dev + kSmpTokOff); }
float* smp_input(Context* c) { return reinterpret_cast<float*>(c->smp_dev + kSmpInOff); }
void* smp_scratch(Context* c) {
  return c->smp_dev + kSmpInOff + round_up_sz((size_t)c->smp_cap * sizeof(float), 256);
}

// One draw from d_logits[n] on the context's stream; with to_seq the token
// also becomes seq_tokens[ctrl->pos] (and the last-token slot), the input of
// the next decode step.
void smp_draw(Context* c, const float* d_logits, int n, float temperature, float top_p, int top_k, bool to_seq) {
  SampleArgs a;
  a.logits = d_logits;
  a.n = n;
  a.temperature = temperature;
  a.top_p = top_p;
  a.top_k = top_k;
  a.rng = smp_rng(c);
  a.token = smp_token(c);
  if (to_seq) {
    a.seq_tokens = c->seq_tokens;
    a.d_pos = &c->ctrl->pos;
    a.fixed_until = &c->ctrl->fixed_until;
    a.ctx = c->ctx;
  }
  a.scratch = smp_scratch(c);
  const cudaError_t e = sample_launch(a, c->stream);
  if (e != cudaSuccess) fail(SS_CUDA_ERROR_BACKEND, "sampler launch: %s", cudaGetErrorString(e));
}

// `batch` draws at once, one per row of d_logits ([batch][stride]), with RNG
// states smp_rng(c)[0..batch); the tokens go to tokens[b * token_stride].
void smp_draw_batch(Context* c, const float* d_logits, size_t stride, int n, int batch, float temperature,
                    float top_p, int top_k, int* tokens, int token_stride) {
  SampleArgs a;
  a.logits = d_logits;
  a.n = n;
  a.temperature = temperature;
  a.top_p = top_p;
  a.top_k = top_k;
  a.rng = smp_rng(c);
  a.token = tokens;
  a.scratch = smp_scratch(c);
  a.batch = batch;
  a.logits_stride = stride;
  a.token_stride = token_stride;
  a.scratch_stride = smp_slice(c->smp_cap);
  const cudaError_t e = sample_launch(a, c->stream);
  if (e != cudaSuccess) fail(SS_CUDA_ERROR_BACKEND, "sampler launch: %s", cudaGetErrorString(e));
}

// RNG states of draws 0..n-1 to the device (NULL: zeros; greedy draws never
// read them).
void smp_put_states(Context* c, const uint64_t* states, int n) {
  for (int i = 0; i < n; i++) c->smp_host[i] = states ? (unsigned long long)states[i] : 0ull;
  CK(cudaMemcpyAsync(smp_rng(c), c->smp_host, 8 * (size_t)n, cudaMemcpyHostToDevice, c->stream));
}
void smp_put_state(Context* c, const uint64_t* rng_state) { smp_put_states(c, rng_state, 1); }
// Reads the header (RNG states, tokens) back, synchronously; copies n states
// out when `states` is not NULL and returns draw 0's token.
int smp_get_n(Context* c, uint64_t* states, int n) {
  CK(cudaMemcpyAsync(c->smp_host, c->smp_dev, kSmpInOff, cudaMemcpyDeviceToHost, c->stream));
  if (c->has_model) check_device_error(c);
  else CK(cudaStreamSynchronize(c->stream));
  if (states)
    for (int i = 0; i < n; i++) states[i] = (uint64_t)c->smp_host[i];
  int tok;
  memcpy(&tok, reinterpret_cast<const uint8_t*>(c->smp_host) + kSmpTokOff, sizeof(int));
  return tok;
}
int smp_get(Context* c, uint64_t* rng_state) { return smp_get_n(c, rng_state, 1); }

// The context's full-vocabulary logits of the last single-sequence step
// (tensor parallelism: every rank gathers them; a collective).
const float* smp_logits(Context* c) {
  if (c->tp_size > 1) {
    NK(nccl_api().AllGather(c->logits, c->logits_full, (size_t)c->vocab_l, ncclFloat32, c->comm, c->stream));
    return c->logits_full;
  }
  return c->logits;
}

bool smp_needs_rng(float temperature) { return !(temperature <= 0.0f); }

SS_API int ss_cuda_sample_logits(ss_cuda_ctx_t* ctx, const float* logits, int32_t n, float temperature,
                                 float top_p, int32_t top_k, uint64_t* rng_state, int32_t* token_out) {
  return guard([&] {
    auto* c = reinterpret_cast<Context*>(ctx);
    if (!c) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null context");
    if (!logits || !token_out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    if (smp_needs_rng(temperature) && !rng_state) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null RNG state");
    CK(cudaSetDevice(c->device));
    smp_reserve(c, n);
    CK(cudaMemcpyAsync(smp_input(c), logits, sizeof(float) * (size_t)n, cudaMemcpyHostToDevice, c->stream));
    smp_put_state(c, rng_state);
    smp_draw(c, smp_input(c), n, temperature, top_p, top_k, false);
    *token_out = smp_get(c, smp_needs_rng(temperature) ? rng_state : nullptr);
  });
}

SS_API int ss_cuda_sample(ss_cuda_ctx_t* ctx, float temperature, float top_p, int32_t top_k, uint64_t* rng_state,
                          int32_t* token_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!token_out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    if (smp_needs_rng(temperature) && !rng_state) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null RNG state");
    smp_reserve(c, c->vocab);
    smp_put_state(c, rng_state);
    smp_draw(c, smp_logits(c), c->vocab, temperature, top_p, top_k, false);
    *token_out = smp_get(c, smp_needs_rng(temperature) ? rng_state : nullptr);
  });
}

SS_API int ss_cuda_decode_sample(ss_cuda_ctx_t* ctx, int32_t start_pos, int32_t n_tokens, float temperature,
                                 float top_p, int32_t top_k, uint64_t* rng_state, int32_t* ids_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!ids_out || n_tokens <= 0) fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad arguments");
    if (smp_needs_rng(temperature) && !rng_state) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null RNG state");
    if (start_pos < 0 || start_pos + n_tokens - 1 > c->ctx)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "tokens %d..%d past the context of %d", start_pos, start_pos + n_tokens - 1,
           c->ctx);
    if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
    smp_reserve(c, c->vocab);
    // the draws fill seq_tokens[start_pos ...] (start_pos == ctx: one draw into
    // the last-token slot, no step); afterwards the position is the last
    // draw's, so ss_cuda_decode_steps continues from it
    c->h_small[0] = start_pos;
    c->h_small[1] = start_pos;
    CK(cudaMemcpyAsync(c->ctrl, c->h_small, 2 * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    c->host_pos = start_pos;
    smp_put_state(c, rng_state);
    for (int t = 0; t < n_tokens; t++) {
      smp_draw(c, smp_logits(c), c->vocab, temperature, top_p, top_k, true);
      if (t + 1 < n_tokens) run_steps(c, 1);  // forward(token, start_pos + t)
    }
    smp_get(c, smp_needs_rng(temperature) ? rng_state : nullptr);
    // tokens of positions start_pos .. start_pos + n_tokens - 1; one at index
    // ctx (past the context) sits in the last-token slot
    const int in_ctx = std::max(0, std::min(n_tokens, c->ctx - start_pos));
    if (in_ctx > 0)
      CK(cudaMemcpy(ids_out, c->seq_tokens + start_pos, sizeof(int) * in_ctx, cudaMemcpyDeviceToHost));
    if (in_ctx < n_tokens)
      CK(cudaMemcpy(ids_out + in_ctx, c->seq_tokens + c->ctx, sizeof(int), cudaMemcpyDeviceToHost));
  });
}

// Sampled decode of sequences 0..n_seq-1 for n_steps, the batched twin of
// the greedy loop (bt_decode_greedy): after each many-token step one sampler
// launch draws every sequence's token from its row of logits with its own RNG
// state (smp_rng(c)[s]), into the greedy-token row the feedback kernel reads.
void bt_decode_sample(Context* c, const int32_t* tok, int n_seq, int start_pos, int n_steps, float temperature,
                      float top_p, int top_k) {
  if (n_steps < 1 || start_pos + n_steps > c->ctx)
    fail(SS_CUDA_ERROR_INVALID_PARAMS, "decode runs past the context");
  if (n_seq < 1 || n_seq > c->max_batch)
    fail(SS_CUDA_ERROR_INVALID_PARAMS, "n_seq %d outside 1..%d (max_batch)", n_seq, c->max_batch);
  std::vector<int> ps((size_t)n_seq, start_pos), sq((size_t)n_seq);
  for (int s = 0; s < n_seq; s++) sq[(size_t)s] = s;
  bt_stage(c, tok, ps.data(), sq.data(), n_seq);
  for (int k = 0; k < n_steps; k++) {
    if (c->cancelled.load()) fail(SS_CUDA_ERROR_CANCELLED, "cancelled");
    bt_launch(c, n_seq, n_seq);
    smp_draw_batch(c, c->bt_logits, (size_t)c->vocab_l, c->vocab, n_seq, temperature, top_p, top_k,
                   c->bt_meta + 3 * kQgMaxT, 1);
    bt_feed_kernel<<<1, kQgMaxT, 0, c->stream>>>(c->bt_meta, kQgMaxT, n_seq, c->bt_ids, kQgMaxT, c->ctx);
    CK(cudaGetLastError());
  }
  c->steps_run += (long long)n_seq * n_steps;
}

SS_API int ss_cuda_decode_sample_batch(ss_cuda_ctx_t* ctx, const int32_t* tokens, int32_t n_seq, int32_t start_pos,
                                       int32_t n_steps, float temperature, float top_p, int32_t top_k,
                                       uint64_t* rng_states, int32_t* ids_out) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!tokens || !ids_out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    if (smp_needs_rng(temperature) && !rng_states) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null RNG states");
    if (!bt_eligible(c)) fail(SS_CUDA_ERROR_INVALID_PARAMS, "batched decode needs the many-token step");
    if (n_seq < 1 || n_seq > c->max_batch)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "n_seq %d outside 1..%d (max_batch)", n_seq, c->max_batch);
    smp_reserve(c, c->vocab, n_seq);
    smp_put_states(c, smp_needs_rng(temperature) ? rng_states : nullptr, n_seq);
    bt_decode_sample(c, tokens, n_seq, start_pos, n_steps, temperature, top_p, top_k);
    smp_get_n(c, smp_needs_rng(temperature) ? rng_states : nullptr, n_seq);
    std::vector<int> rows((size_t)n_steps * kQgMaxT);
    CK(cudaMemcpy(rows.data(), c->bt_ids + (size_t)(start_pos + 1) * kQgMaxT, sizeof(int) * rows.size(),
                  cudaMemcpyDeviceToHost));
    for (int k = 0; k < n_steps; k++)
      for (int s = 0; s < n_seq; s++) ids_out[(size_t)k * n_seq + s] = rows[(size_t)k * kQgMaxT + s];
  });
}

SS_API void* ss_cuda_stream(ss_cuda_ctx_t* ctx) {
  auto* c = reinterpret_cast<Context*>(ctx);
  return c ? (void*)c->stream : nullptr;
}

SS_API int ss_cuda_dequantize_tensor(ss_cuda_ctx_t* ctx, const char* name, float* out, int64_t n) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!name || !out) fail(SS_CUDA_ERROR_INVALID_PARAMS, "null argument");
    std::string s(name);
    const DevMatrix* m = nullptr;
    int mul = 1, add = 0, rows = 0;
    const int qd = c->nh * c->hd, kvd = c->nkv * c->hd;
    if (s == "output.weight") { m = &c->lm_head; rows = c->vocab; }
    else if (s.rfind("blk.", 0) == 0) {
      const int l = atoi(s.c_str() + 4);
      const size_t dot = s.find('.', 4);
      if (l < 0 || l >= c->L || dot == std::string::npos) fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad tensor %s", name);
      const std::string suf = s.substr(dot + 1);
      const Layer& ly = c->layers[(size_t)l];
      if (suf == "attn_q.weight") { m = &ly.qkv; rows = qd; }
      else if (suf == "attn_k.weight") { m = &ly.qkv; rows = kvd; add = qd; }
      else if (suf == "attn_v.weight") { m = &ly.qkv; rows = kvd; add = qd + kvd; }
      else if (suf == "attn_output.weight") { m = &ly.o; rows = c->d; }
      else if (suf == "ffn_gate.weight") { m = &ly.gu; rows = c->ff; mul = 2; }
      else if (suf == "ffn_up.weight") { m = &ly.gu; rows = c->ff; mul = 2; add = 1; }
      else if (suf == "ffn_down.weight") {
        m = &ly.down;
        rows = c->d;
        if (ly.down2.cols) {
          // the two column halves, each dequantised and placed side by side
          if (n != (int64_t)rows * 2 * m->cols) fail(SS_CUDA_ERROR_INVALID_PARAMS, "n must be rows*cols");
          const size_t half = (size_t)rows * m->cols;
          float* d_tmp = nullptr;
          CK(cudaMalloc(&d_tmp, sizeof(float) * half));
          cudaError_t e = cudaSuccess;
          for (int k = 0; k < 2 && e == cudaSuccess; k++) {
            const DevMatrix& mk = k ? ly.down2 : ly.down;
            dequant_rows_kernel<<<1024, 256, 0, c->stream>>>(mk.data, rows, mk.cols, mk.type, mk.row_stride,
                                                            mk.scale_off, 1, 0, d_tmp);
            e = cudaGetLastError();
            if (e == cudaSuccess)
              e = cudaMemcpy2DAsync(out + (size_t)k * mk.cols, sizeof(float) * 2 * mk.cols, d_tmp,
                                    sizeof(float) * mk.cols, sizeof(float) * mk.cols, rows,
                                    cudaMemcpyDeviceToHost, c->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
          }
          cudaFree(d_tmp);
          CK(e);
          return;
        }
      }
    }
    if (!m) fail(SS_CUDA_ERROR_INVALID_PARAMS, "no quantized tensor %s", name);
    if (n != (int64_t)rows * m->cols) fail(SS_CUDA_ERROR_INVALID_PARAMS, "n must be rows*cols = %lld", (long long)rows * m->cols);
    if (c->streaming && s.rfind("blk.", 0) == 0) {
      const int l = atoi(s.c_str() + 4);
      if (l >= c->n_resident) {  // a streamed layer: bring it into its slot first
        CK(cudaStreamSynchronize(c->stream));
        enqueue_layer_copy(c, l);
        CK(cudaStreamWaitEvent(c->stream, c->ev_ready[(l - c->n_resident) % 2], 0));
      }
    }
    float* d_out = nullptr;
    CK(cudaMalloc(&d_out, sizeof(float) * (size_t)n));
    if (m->tiled)
      dequant_tiled_kernel<<<1024, 256, 0, c->stream>>>(m->data, rows, m->cols, m->type, m->tile_bytes,
                                                       mul, add, d_out);
    else
      dequant_rows_kernel<<<1024, 256, 0, c->stream>>>(m->data, rows, m->cols, m->type, m->row_stride,
                                                      m->scale_off, mul, add, d_out);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d_out, sizeof(float) * (size_t)n, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(d_out);
    CK(e);
  });
}

SS_API int ss_cuda_dequantize(int32_t type, const void* blocks, int64_t n, float* out) {
  return guard([&] {
    if (!blocks || !out || n <= 0) fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad arguments");
    if (!quant_type_size(type)) fail(SS_CUDA_ERROR_INVALID_PARAMS, "type %d", type);
    const int bs = quant_block_size(type);
    if (n % bs) fail(SS_CUDA_ERROR_INVALID_PARAMS, "n %lld not a multiple of the block size %d", (long long)n, bs);
    const size_t in_bytes = (size_t)(n / bs) * quant_type_size(type);
    uint8_t* d_in = nullptr;
    float* d_out = nullptr;
    CK(cudaMalloc(&d_in, in_bytes));
    cudaError_t e = cudaMalloc(&d_out, sizeof(float) * (size_t)n);
    if (e == cudaSuccess) e = cudaMemcpy(d_in, blocks, in_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = dequant_launch(d_in, n, type, d_out, nullptr);
    if (e == cudaSuccess) e = cudaMemcpy(out, d_out, sizeof(float) * (size_t)n, cudaMemcpyDeviceToHost);
    cudaFree(d_in);
    if (d_out) cudaFree(d_out);
    CK(e);
  });
}

SS_API int ss_cuda_time_kernel(ss_cuda_ctx_t* ctx, int32_t which, int32_t iters, float* ms_per_launch) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (which < 0 || which > 10 || iters <= 0 || !ms_per_launch) fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad arguments");
    if (c->tiled && which < 6)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "per-kernel timing needs the multi-kernel step (SS_CUDA_FLAG_MULTI_KERNEL)");
    if (which == 7 || which == 8) {
      if (!bt_eligible(c)) fail(SS_CUDA_ERROR_INVALID_PARAMS, "the tensor-core product needs the tiled layout");
      bt_prepare(c);
      const DevMatrix& m0 = which == 7 ? c->layers[0].gu : c->layers[0].qkv;
      qg_product(c, m0, c->bt_h, c->d, nullptr, c->max_batch, true, false);
    }
    if (which >= 9) {  // the sampler over the last step's logits
      smp_reserve(c, c->vocab);
      const uint64_t seed = 0x9E3779B97F4A7C15ull;
      smp_put_state(c, &seed);
    }
    const int pos0 = c->host_pos;
    if (which == 6 && pos0 + iters + 3 > c->ctx)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "%d steps from position %d exceed the context", iters + 3, pos0);
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    auto one = [&](int i) {
      const int l = i % c->L;
      switch (which) {
        case 6: enqueue_step(c, c->use_pdl); break;
        case 7: qg_product(c, c->layers[(size_t)l].gu, c->bt_h, c->d, nullptr, c->max_batch, false, true); break;
        case 8: qg_product(c, c->layers[0].qkv, c->bt_h, c->d, nullptr, c->max_batch, false, true); break;
        case 9: smp_draw(c, smp_logits(c), c->vocab, 0.7f, 0.9f, 40, false); break;  // ss_default_params
        case 10: smp_draw(c, smp_logits(c), c->vocab, 1.0f, 0.95f, 0, false); break;  // the longest walks
        case 0: launch_qkv(c, l, false); break;
        case 1: launch_attn(c, l, false); break;
        case 2: launch_o(c, l, false); break;
        case 3: launch_gu(c, l, false); break;
        case 4: launch_down(c, l, false); break;
        default: launch_head(c, false); break;
      }
    };
    for (int i = 0; i < 3; i++) one(i);  // warm-up
    CK(cudaEventRecord(e0, c->stream));
    for (int i = 0; i < iters; i++) one(i);
    CK(cudaEventRecord(e1, c->stream));
    CK(cudaEventSynchronize(e1));
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms_per_launch = ms / (float)iters;
    if (which >= 5 && which <= 8) {  // the lm_head advanced the device position; restore it
      CK(cudaMemcpyAsync(c->ctrl, &c->host_pos, sizeof(int), cudaMemcpyHostToDevice, c->stream));
      CK(cudaStreamSynchronize(c->stream));
      check_device_error(c);
    }
  });
}

SS_API int64_t ss_cuda_kernel_bytes(const ss_cuda_ctx_t* ctx, int32_t which) {
  auto* c = reinterpret_cast<const Context*>(ctx);
  if (!c || !c->has_model) return -1;
  const Layer& l0 = c->layers[0];
  switch (which) {
    case 0: return (int64_t)matrix_bytes(l0.qkv);
    case 2: return (int64_t)matrix_bytes(l0.o);
    case 3: return (int64_t)matrix_bytes(l0.gu);
    case 4: return (int64_t)(matrix_bytes(l0.down) + (l0.down2.cols ? matrix_bytes(l0.down2) : 0));
    case 7: return (int64_t)matrix_bytes(l0.gu);
    case 8: return (int64_t)matrix_bytes(l0.qkv);
    case 5: return (int64_t)matrix_bytes(c->lm_head);
    case 6: {
      int64_t b = (int64_t)matrix_bytes(c->lm_head);
      for (const Layer& ly : c->layers)
        b += (int64_t)(matrix_bytes(ly.qkv) + matrix_bytes(ly.o) + matrix_bytes(ly.gu) + matrix_bytes(ly.down) +
                       (ly.down2.cols ? matrix_bytes(ly.down2) : 0));
      return b;
    }
    default: return -1;
  }
}

SS_API int ss_cuda_step_trace(ss_cuda_ctx_t* ctx, int64_t* out, int64_t n) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (!c->step_trace) fail(SS_CUDA_ERROR_INVALID_PARAMS, "no trace: create the context with SS_CUDA_FLAG_TRACE");
    const int64_t total = (int64_t)(2 + 5 * c->L) * c->step_grid * 8;
    if (!out || n != total) fail(SS_CUDA_ERROR_INVALID_PARAMS, "n must be %lld", (long long)total);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(out, c->step_trace, sizeof(int64_t) * (size_t)n, cudaMemcpyDeviceToHost));
  });
}

SS_API int ss_cuda_kv_row(ss_cuda_ctx_t* ctx, int32_t layer, int32_t pos, int8_t* k, int8_t* v,
                          float* k_scale, float* v_scale) {
  return guard([&] {
    Context* c = need_model(ctx);
    if (layer < 0 || layer >= c->L || pos < 0 || pos >= c->ctx || !k || !v || !k_scale || !v_scale)
      fail(SS_CUDA_ERROR_INVALID_PARAMS, "bad kv_row arguments");
    // the device cache is head-major ([L][nkv][ctx][hd]); gather the row
    const size_t kvd = (size_t)c->nkv * c->hd, vi = (size_t)layer * c->ctx + pos;
    const size_t off = (size_t)layer * c->ctx * kvd + (size_t)pos * c->hd;
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy2D(k, (size_t)c->hd, c->kc + off, (size_t)c->ctx * c->hd, (size_t)c->hd, (size_t)c->nkv,
                    cudaMemcpyDeviceToHost));
    CK(cudaMemcpy2D(v, (size_t)c->hd, c->vc + off, (size_t)c->ctx * c->hd, (size_t)c->hd, (size_t)c->nkv,
                    cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(k_scale, c->ks + vi, 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(v_scale, c->vs + vi, 4, cudaMemcpyDeviceToHost));
  });
}
