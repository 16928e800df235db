// ss_cuda_internal.h -- context state of the CUDA backend (host side).
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "attention.cuh"
#include "batch_kernels.cuh"
#include "gemv.cuh"
#include "gguf_view.h"
#include "misc_kernels.cuh"
#include "qgemm.cuh"
#include "quant.h"
#include "sample.h"
#include "step_kernel.cuh"
#include "tp_nccl.h"

namespace ss {

// A repacked quantized matrix in device memory: row-interleaved (gemv.cuh,
// the multi-kernel step and the op-level matvecs) or tiled (step_kernel.cuh).
struct DevMatrix {
  uint8_t* data = nullptr;
  int rows = 0, cols = 0, row_stride = 0, scale_off = 0, type = 0;
  bool tiled = false;
  int ntiles = 0, tile_bytes = 0;
  QMatrix q() const { return QMatrix{data, rows, cols, row_stride, scale_off, type}; }
  TMat t() const { return TMat{data, cols / 32, ntiles, tile_bytes, type, rows}; }
};

// Launch geometry of one GEMV (see gemv.cuh for the work split).
struct GemvLaunch {
  const void* fn = nullptr;
  int threads = 0, ctas = 0, rows_per_cta = 0;
  int nstage = 0, stage_rows = 0;
  size_t smem = 0;
};

struct Layer {
  DevMatrix qkv, o, gu, down;  // gu rows interleave gate (even) and up (odd)
  // FFN widths beyond one GEMV's 16384 columns (the 70B shape on one GPU, the
  // multi-kernel step): `down` holds the first half of the FFN columns and
  // `down2` the second; both GEMVs add into h in turn.  down2.cols == 0: unsplit.
  DevMatrix down2;
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  uint8_t* block = nullptr;    // one allocation holding the four matrices
};

// Device control block of the decode step.
struct Ctrl {
  int pos;          // position processed by the next step
  int fixed_until;  // positions below this hold caller-provided tokens
  int err;          // sticky device error bits
  int pad;
};

struct OpCacheEntry {
  DevMatrix m;
  float* f32 = nullptr;    // F32 matrices stay row-major
  uint8_t* raw = nullptr;  // Q4_K matrices keep their GGUF bytes
};

// GEMV geometry knobs (defaults measured on B200; the SS_GEMV_* environment
// variables override them at context creation, for tuning sweeps).
struct GemvTuning {
  int target_threads = 256;        // threads per CTA
  size_t ring_bytes = 100 * 1024;  // shared memory for the weight ring
  int prefetch = 1;                // bulk L2 prefetch of the rest of the CTA's rows
  int max_ctas_per_sm = 0;         // 0 = as many as are co-resident
};

struct Context {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  bool has_model = false;
  bool use_pdl = true;
  bool use_graph = true;
  bool trace = false;
  int test_fail_phase = 0;  // > 0: the next persistent step runs the failure-path test
  // many-token tensor-core product (qgemm.cuh): tensor maps per weight
  // matrix, activation planes, partial sums
  std::unordered_map<const void*, QgMaps> qg_maps;
  __half* qg_xq = nullptr;
  size_t qg_xq_bytes = 0;
  float* qg_scale = nullptr;
  float* qg_out = nullptr;
  size_t qg_out_floats = 0;
  // the many-token step (batch_kernels.cuh): hidden states, q, attention
  // output, SwiGLU activations, logits of up to 32 tokens; token metadata
  uint32_t flags = 0;
  float* bt_h = nullptr;
  float* bt_h2 = nullptr;       // the residual stream alternates between bt_h and bt_h2
  int bt_zero_words = 0;        // words of bt_amax (+ bt_best) the pass's first kernel zeroes
  bool bt_pdl = true;           // programmatic dependent launches in the many-token step
  float* bt_q = nullptr;
  float* bt_att = nullptr;
  float* bt_act = nullptr;
  float* bt_logits = nullptr;
  int* bt_meta = nullptr;       // [4][32]: token, position, sequence, greedy token
  int* bt_meta_host = nullptr;  // pinned staging
  float* bt_kv = nullptr;       // [32][2 kvd]: k | v of each token before encoding
  unsigned* bt_amax = nullptr;  // [32][2]: largest |k|, |v| (float bits)
  unsigned long long* bt_best = nullptr;  // [32]: packed greedy choice
  int* bt_ids = nullptr;                   // [ctx + 1][32]: batched greedy tokens by position
  float* bt_emb = nullptr;                 // [d] embedding sum | [d] result | [32] norm scales
  float* bt_apart = nullptr;               // attention partials [32][nh][slots][hd + 2]
  bool bt_ready = false;                   // scratch reserved for 32 tokens, tensor maps built
  // captured many-token steps: key 2 * T + (head of the last token only);
  // bt_dev_exec is the single-sequence step that reads its token and position
  // from the device (contexts without the persistent step)
  std::map<int, cudaGraphExec_t> bt_graphs;
  cudaGraphExec_t bt_dev_exec = nullptr;
  GemvTuning tuning;
  std::atomic<bool> cancelled{false};

  // model dims (nh, nkv, ff: this rank's under tensor parallelism)
  int vocab = 0, d = 0, L = 0, nh = 0, nkv = 0, hd = 0, rope_dim = 0, ff = 0, ctx = 0, wtype = 0;
  int nh_full = 0, nkv_full = 0, ff_full = 0;
  int vocab_l = 0, vocab_off = 0;  // this rank's lm_head rows

  // tensor parallelism (multi-kernel step + NCCL)
  int tp_rank = 0, tp_size = 1;
  ncclComm_t comm = nullptr;
  float* hpart = nullptr;               // row-parallel partial outputs [d]
  unsigned long long* tp_best = nullptr;  // packed (value, index) of the argmax
  float* logits_full = nullptr;         // gathered logits [vocab]
  int max_batch = 1;
  float eps = 1e-5f, theta = 10000.0f, attn_scale = 1.0f;

  // weights
  float* embd = nullptr;
  float* out_norm = nullptr;
  DevMatrix lm_head;
  uint8_t* lm_block = nullptr;
  std::vector<Layer> layers;
  size_t layer_stride = 0;           // bytes between layers in the weight slab
  float* attn_norm_all = nullptr;    // [L][d]
  float* ffn_norm_all = nullptr;     // [L][d]
  size_t weight_bytes = 0;

  // layer streaming (hbm_budget_bytes below the layers' size; multi-kernel
  // step): layers [n_resident, L) stay in host memory and pass through two HBM
  // slots every step -- layer l uses slot (l - n_resident) % 2.  Their GGUF
  // bytes are copied by DMA into `stream_raw` on `copy_stream` and repacked
  // into the slot; events order copy, repack and the layer's kernels.
  struct StreamTensor {
    GgufTensor t;          // the GGUF tensor (host pointer into the file)
    size_t raw_off = 0;    // its place in stream_raw
    int which = 0;         // 0 qkv, 1 o, 2 gu, 3 down (destination matrix)
    int mul = 1, add = 0;  // destination rows mul * r + add
  };
  bool streaming = false;
  int n_resident = 0;
  uint64_t hbm_budget = 0;
  std::vector<std::vector<StreamTensor>> stream_src;  // [layer] (empty for resident layers)
  uint8_t* stream_raw = nullptr;
  size_t stream_raw_bytes = 0;      // one layer's GGUF bytes (padded per tensor)
  size_t streamed_bytes = 0;        // host-to-device bytes per step
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_ready[2] = {nullptr, nullptr}, ev_free[2] = {nullptr, nullptr};
  void* host_reg = nullptr;         // the model file's range registered with CUDA (read-only)
  uint8_t* host_pinned = nullptr;   // else: the streamed layers' bytes copied into pinned memory
  void* owned_map = nullptr;        // ss_cuda_init_file's mapping, kept while streaming
  size_t owned_map_bytes = 0;

  // KV cache [L][nkv][ctx][hd] (head-major; the reference's is [L][ctx][kvd],
  // ss_cuda_kv_row gathers a position) + scales/maxima [L][ctx]
  int8_t* kc = nullptr;
  int8_t* vc = nullptr;
  float* ks = nullptr;
  float* vs = nullptr;
  unsigned int* amax = nullptr;  // [L][2] |k|, |v| maxima of the current position
  size_t kv_bytes = 0;

  // activations / scratch
  float* h = nullptr;
  float* qkv = nullptr;
  float* attn_out = nullptr;
  float* act = nullptr;
  float* logits = nullptr;
  unsigned long long* am_part = nullptr;
  unsigned int* am_cnt = nullptr;
  int* seq_tokens = nullptr;  // [ctx + 1]; [ctx] = last argmax
  Ctrl* ctrl = nullptr;
  float2* rope_tab = nullptr;

  // pinned host staging
  float* h_logits = nullptr;
  int* h_small = nullptr;  // 64 ints

  // launch geometry
  GemvLaunch g_qkv, g_o, g_gu, g_down, g_head;
  int attn_nsplit = 1;
  size_t attn_smem = 0;
  int embed_blocks = 1;

  // persistent single-kernel step (step_kernel.cuh)
  bool mega = false;
  // matrices in the tiled layout (the persistent step's, which the many-token
  // product reads): the persistent step, or several sequences decoded together
  bool tiled = false;
  const void* step_fn = nullptr;
  int step_grid = 0, step_nslots = 0, step_slot_bytes = 0, step_nsplit = 1;
  size_t step_smem = 0;
  StepParams step_params{};
  StepTp step_tp{};                     // tensor parallelism (TP instantiation of the step)
  uint8_t* xchg = nullptr;              // its exchange block (StepXchg), mapped by the peers
  std::vector<void*> xpeer_open;        // the peers' blocks mapped here (CUDA IPC)
  unsigned* dbg_host = nullptr;         // checks builds: the TP step's record (host-mapped)
  unsigned* step_sync = nullptr;  // counters zeroed by reset (see alloc_step_state)
  long long* step_trace = nullptr;  // per-phase timeline of the last step (SS_CUDA_FLAG_TRACE)
  size_t step_sync_words = 0;

  cudaGraphExec_t step_exec = nullptr;
  bool graph_pdl = false;
  int host_pos = 0;  // host shadow of ctrl->pos for bounds checks
  long long steps_run = 0;
  long long ops_run = 0;  // op-level matvecs served (ss_cuda_matvec*)

  // op-level (Metal-twin) state
  std::unordered_map<const void*, OpCacheEntry> op_cache;
  struct BatchSlot {
    float* d_x = nullptr;
    float* d_out = nullptr;
    size_t x_cap = 0, out_cap = 0;
    float* host_out = nullptr;
    size_t out_n = 0;
  };
  std::vector<BatchSlot> op_slots;
  bool in_batch = false;
  int batch_count = 0;
  uint8_t* op_stage = nullptr;
  size_t op_stage_cap = 0;

  // on-device sampling (sample.cu), grown on demand for smp_cap logits and
  // smp_batch draws at once: [32 RNG states u64][32 drawn tokens int] |
  // caller logits | smp_batch scratch slices
  uint8_t* smp_dev = nullptr;
  int smp_cap = 0, smp_batch = 0;
  unsigned long long* smp_host = nullptr;  // pinned copy of the header

  std::vector<void*> allocations;
};

}  // namespace ss
