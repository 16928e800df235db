/*
 * slipstream_cuda.h -- CUDA (sm_100a) backend for SlipStream's decode path.
 *
 * A sibling of SlipStream's Metal backend (SlipStream/src/backends/
 * metal_backend.h:21-75), reached from the same call sites:
 *   - ss_model_load creates it next to ss_metal_init (SlipStream/src/core/
 *     engine.c:87-96) and ss_model_free frees it (engine.c:467-469);
 *   - ss_matmul_dispatch calls the op-level matvecs (SlipStream/src/core/
 *     layer_scheduler.c:248-279), with the begin/end batch brackets of
 *     layer_scheduler.c:352-362 and :508-517;
 *   - ss_scheduler_forward / _prefill / _reset (layer_scheduler.h:107-132)
 *     hand whole tokens to ss_cuda_scheduler_* so activations stay on the GPU.
 *
 * Plain C types only.  Every entry point is synchronous unless it says
 * otherwise.  On failure the bool/pointer entry points return false/NULL and
 * the int ones a negative SS_CUDA_ERROR_* code (the values of ss_error_t,
 * SlipStream/include/slipstream.h:32-43); ss_cuda_last_error() describes the
 * most recent failure on the calling thread.  There is no CPU fallback: a
 * failure is reported, never silently computed elsewhere.
 *
 * Threading: one caller thread per context (as the reference's scheduler).
 * ss_cuda_cancel may be called from any thread.
 */
#ifndef SLIPSTREAM_CUDA_H
#define SLIPSTREAM_CUDA_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SS_CUDA_ABI_VERSION 1

/* Error codes: same values as ss_error_t (SlipStream/include/slipstream.h:32-43). */
#define SS_CUDA_OK 0
#define SS_CUDA_ERROR_FILE_NOT_FOUND (-1)
#define SS_CUDA_ERROR_INVALID_MODEL (-2)
#define SS_CUDA_ERROR_OUT_OF_MEMORY (-3)
#define SS_CUDA_ERROR_INVALID_PARAMS (-5)
#define SS_CUDA_ERROR_CANCELLED (-6)
#define SS_CUDA_ERROR_BACKEND (-7)

/* Backend id to add to ss_backend_t (slipstream.h:47-51). */
#define SS_BACKEND_CUDA 3

typedef struct ss_cuda_ctx ss_cuda_ctx_t;

typedef struct {
    uint32_t struct_size;      /* sizeof(ss_cuda_options_t) */
    int32_t device;            /* CUDA ordinal; -1 = $SS_CUDA_DEVICE or 0 */
    uint32_t context_size;     /* positions (0 = GGUF context_length), capped at 8192 as engine.c:103-106 */
    /* Sequences decoded together (1..32; 0 = 1).  Above 1 each sequence has its
     * own KV cache (sequence 0's is the single-sequence one), the matrices take
     * the tiled layout the tensor-core product reads, and ss_cuda_forward /
     * ss_cuda_prefill_batch accept n_seq > 1; one GPU, no layer streaming. */
    uint32_t max_batch;
    /* Bytes of HBM for the layers' weights; 0 = every layer resident.  When the
     * layers need more, layers past the first (budget / layer bytes - 3) stay in
     * host memory and are copied into two HBM slots every step (layer
     * streaming; needs room for 3 layers, single GPU, multi-kernel step).  The
     * GGUF bytes given to ss_cuda_init must then stay mapped while the context
     * lives (ss_cuda_init_file keeps its own mapping). */
    uint64_t hbm_budget_bytes;
    uint32_t flags;            /* SS_CUDA_FLAG_* */
    /* Tensor parallelism (one process per GPU): tp_size GPUs share one model,
     * Q/K/V and gate/up sharded by heads / rows, O and down by columns (an
     * all-reduce after each), lm_head by vocabulary rows.  0 or 1 = off. */
    int32_t tp_rank;
    int32_t tp_size;
    uint8_t tp_nccl_id[128];   /* from ss_cuda_tp_unique_id on rank 0, the same on every rank */
} ss_cuda_options_t;

#define SS_CUDA_FLAG_NO_PDL 1u   /* launch without programmatic dependent launch */
#define SS_CUDA_FLAG_NO_GRAPH 2u /* launch kernels one by one instead of a CUDA graph */
/* Run the decode step as 2 + 5 * layers kernels (a CUDA graph) instead of the
 * default single persistent kernel; also used automatically when a model's
 * shapes exceed what the persistent kernel supports. */
#define SS_CUDA_FLAG_MULTI_KERNEL 4u
/* Record a per-phase timeline of every persistent step (measurement aid). */
#define SS_CUDA_FLAG_TRACE 8u
/* Ingest prompts by replaying the decode step once per token (the reference's
 * token-by-token order) instead of the many-token tensor-core step. */
#define SS_CUDA_FLAG_STEP_PREFILL 16u

/* Fills defaults: device -1, context 0, batch 1, no budget, no flags, no
 * tensor parallelism. */
void ss_cuda_default_options(ss_cuda_options_t *opts);

/* An NCCL unique id (128 bytes) for a tensor-parallel group: call on rank 0,
 * hand the bytes to every rank's ss_cuda_options_t.tp_nccl_id. */
int ss_cuda_tp_unique_id(uint8_t *id_out);

/* ---- lifecycle (twin of ss_metal_init / ss_metal_free, metal_backend.h:21,75) ----
 * Uploads and repacks every weight tensor of the llama GGUF held in
 * [gguf_base, gguf_base + gguf_size) (the loader's mmap: ss_gguf_file_t
 * mmap_base / file_size, SlipStream/src/core/gguf_loader.h:84-85) and
 * allocates the int8 KV cache.  The mapping may be unmapped afterwards.
 * Returns NULL on failure. */
ss_cuda_ctx_t *ss_cuda_init(const void *gguf_base, uint64_t gguf_size,
                            const ss_cuda_options_t *opts);
/* Same, mapping the file itself. */
ss_cuda_ctx_t *ss_cuda_init_file(const char *gguf_path, const ss_cuda_options_t *opts);
void ss_cuda_free(ss_cuda_ctx_t *ctx);

const char *ss_cuda_last_error(void);
int ss_cuda_abi_version(void);

/* dims[0..11] = vocab, hidden, layers, heads, kv_heads, head_dim, ffn,
 * context (positions), rope_dim, weight type, max_batch, device (the whole
 * model's, also under tensor parallelism). */
int ss_cuda_model_dims(const ss_cuda_ctx_t *ctx, int32_t *dims);

/* Counters (no reference counterpart; profiling aid like the recap at
 * engine.c:291-302): out[0] kernels launched per decode step, [1] device weight
 * bytes, [2] device KV-cache bytes, [3] attention position splits, [4] 1 when
 * the step graph chains kernels with programmatic dependent launch, [5] decode
 * steps run, [6] CTAs of the QKV GEMV, [7] CTAs of the down GEMV (both: the
 * grid of the persistent step), [8] 1 when the step is the single persistent
 * kernel, [9] its weight-ring slots, [10] layers resident in HBM (all of them
 * unless streaming), [11] bytes copied from host memory per step (layer
 * streaming), [12] device bytes of one layer's four matrices, [13] where
 * streamed layers are copied from: 1 the registered model mapping, 2 a pinned
 * host copy, 3 pageable memory (0: not streaming), [14] the binary version the
 * loaded kernels were compiled for (cudaFuncAttributes::binaryVersion; 100 =
 * sm_100a), [15] kernels launched per step of several sequences decoded
 * together (the many-token step with every token's lm_head and the greedy
 * feedback; 0 where the matrices are not in the tiled layout), [16] op-level
 * matvecs served (ss_cuda_matvec*). */
int ss_cuda_stats(const ss_cuda_ctx_t *ctx, int64_t *out, int32_t n);

/* Measurement aid, no reference counterpart: times `iters` back-to-back
 * launches (no programmatic overlap) of one kernel of the decode step --
 * which = 0 QKV GEMV, 1 attention, 2 O GEMV, 3 gate/up GEMV, 4 down GEMV,
 * 5 lm_head GEMV -- cycling through the layers so weights stream from HBM --
 * or 6 the whole decode step (steps at the current position onwards), or 7
 * the tensor-core gate/up product of max_batch tokens (the kernel alone, its
 * activation pieces built once before), or 8 the same for layer 0's Q/K/V
 * matrix at every launch (L2-resident where it fits), or 9 / 10 one sampler
 * draw (ss_cuda_sample) over the last step's logits with the reference's
 * default settings (temperature 0.7, top_p 0.9, top_k 40: ss_default_params,
 * engine.c:42-51) / temperature 1, top_p 0.95, no top-k, and writes the
 * average milliseconds per launch.  0..5 exist only in the multi-kernel step,
 * 7 and 8 only where the matrices are in the tiled layout.  Clobbers the
 * activations and the K/V rows it passes over; call ss_cuda_reset before
 * decoding again. */
int ss_cuda_time_kernel(ss_cuda_ctx_t *ctx, int32_t which, int32_t iters, float *ms_per_launch);
/* Device bytes of the weights one launch of kernel `which` streams (layer 0;
 * repacked layout, i.e. the GGUF bytes plus row padding; 6: every weight
 * matrix of the step; 7: the gate/up matrix; 8: the Q/K/V matrix); -1 if not
 * a GEMV. */
int64_t ss_cuda_kernel_bytes(const ss_cuda_ctx_t *ctx, int32_t which);

/* Measurement aid, no reference counterpart: the timeline of the last
 * persistent step (context created with SS_CUDA_FLAG_TRACE).  out[n] with
 * n = (2 + 5 * layers) * grid * 4, indexed [phase][cta][event]; phases are
 * 0 embedding, then per layer QKV, attention, O, gate/up, down, then lm_head;
 * events are global-timer nanoseconds: 0 the phase's input ready, 1 the CTA's
 * matvec rows done, 2 the CTA done with the phase, 3 the CTA's producer issued
 * the phase's last weight copy (0 where an event does not apply). */
int ss_cuda_step_trace(ss_cuda_ctx_t* ctx, int64_t* out, int64_t n);

/* ---- op level: twins of ss_metal_should_use_gpu / ss_metal_matvec* ----
 * (metal_backend.h:27-58).  out[rows] = W[rows x cols] . vec[cols] with host
 * pointers.  W is a GGUF tensor's bytes (Q4_0: 18 B per 32 weights, Q8_0: 34 B,
 * F32: 4 B per weight); its device copy is cached by host address, as the
 * Metal backend caches its zero-copy buffers (metal_backend.m:190-235).
 * Returns true when `out` has been written (at ss_cuda_end_batch when called
 * inside a batch). */
bool ss_cuda_should_use_gpu(int32_t rows, int32_t cols);
bool ss_cuda_matvec(ss_cuda_ctx_t *ctx, float *out, const float *mat, const float *vec,
                    int32_t rows, int32_t cols);
bool ss_cuda_matvec_q4_0(ss_cuda_ctx_t *ctx, float *out, const void *mat, const float *vec,
                         int32_t rows, int32_t cols);
bool ss_cuda_matvec_q8_0(ss_cuda_ctx_t *ctx, float *out, const void *mat, const float *vec,
                         int32_t rows, int32_t cols);
/* Twin of ss_metal_matvec_q4_K (metal_backend.h:44-49, kernel metal_backend.m:
 * 111-154; called from ss_matmul_dispatch, layer_scheduler.c:255-256): W in
 * Q4_K super-blocks (144 B per 256 weights), cols a multiple of 256.  Each
 * weight is dequantized as ss_dequantize does (bit-identical); the dot
 * product is summed in fp32 in the GPU's order (one warp per row). */
bool ss_cuda_matvec_q4_K(ss_cuda_ctx_t *ctx, float *out, const void *mat, const float *vec,
                         int32_t rows, int32_t cols);
/* Twins of ss_metal_begin_batch / ss_metal_end_batch (metal_backend.h:64-70). */
void ss_cuda_begin_batch(ss_cuda_ctx_t *ctx);
void ss_cuda_end_batch(ss_cuda_ctx_t *ctx);

/* ---- scheduler level: twins of ss_scheduler_forward / _prefill / _reset ----
 * (layer_scheduler.h:107-132).  The returned fp32 logits[vocab] live in a host
 * buffer owned by the context and stay valid until the next call; NULL on
 * error or cancellation.  Positions must satisfy 0 <= pos < context. */
float *ss_cuda_scheduler_forward(ss_cuda_ctx_t *ctx, int32_t token_id, int32_t pos);
float *ss_cuda_scheduler_prefill(ss_cuda_ctx_t *ctx, const int32_t *tokens, int32_t n,
                                 int32_t start_pos);
void ss_cuda_scheduler_reset(ss_cuda_ctx_t *ctx);
/* ss_scheduler_embed (layer_scheduler.c:805-915): the tokens at positions
 * 0..n-1 (sequence 0's cache rows overwritten), every token's final hidden
 * state RMSNormed with output_norm, mean-pooled and L2-normalised; returns a
 * malloc'd float[hidden] the caller frees, as the reference's does (engine.c
 * ss_embed hands it out), or NULL on error (ss_cuda_last_error). */
float *ss_cuda_scheduler_embed(ss_cuda_ctx_t *ctx, const int32_t *tokens, int32_t n);

/* ---- coarse entry points (activations and tokens stay on the device) ----
 * One decode step at `pos` (ss_scheduler_forward, layer_scheduler.c:571-679):
 * n_seq = 1 runs sequence 0 with token_ids[0]; optional logits out (host,
 * vocab floats) and greedy argmax out (host, lowest index wins ties as
 * ss_argmax, SlipStream/src/core/tensor.c:318-328).  n_seq > 1 (up to the
 * context's max_batch) steps sequences 0..n_seq-1 together, token_ids[s] at
 * position pos of sequence s, through one pass of the tensor-core product:
 * logits_out [n_seq][vocab] (nullable), argmax_out [n_seq] (nullable); the
 * single-sequence decode state (ss_cuda_decode_*) is left unchanged. */
int ss_cuda_forward(ss_cuda_ctx_t *ctx, const int32_t *token_ids, int32_t n_seq, int32_t pos,
                    float *logits_out, int32_t *argmax_out);
/* The prompts of sequences 0..n_seq-1 (tokens [n_seq][n], all at positions
 * start_pos..start_pos+n-1), each as ss_cuda_prefill ingests one: the last
 * token's logits to logits_out [n_seq][vocab] (nullable), its greedy token to
 * argmax_out [n_seq] (nullable).  Sequence 0 then continues with
 * ss_cuda_decode_* as after ss_cuda_prefill.  Needs max_batch >= n_seq. */
int ss_cuda_prefill_batch(ss_cuda_ctx_t *ctx, const int32_t *tokens, int32_t n_seq, int32_t n,
                          int32_t start_pos, float *logits_out, int32_t *argmax_out);
/* Prompt ingestion at positions start_pos..start_pos+n-1; logits of the last
 * token to logits_out (nullable); returns the greedy next token (>= 0). */
int ss_cuda_prefill(ss_cuda_ctx_t *ctx, const int32_t *tokens, int32_t n, int32_t start_pos,
                    float *logits_out);
/* The same embedding into out[hidden] (host); the prompt runs through the
 * tensor-core product, 32 tokens per pass (single-GPU contexts with the
 * weights resident and in the tiled layout: the default, or max_batch > 1). */
int ss_cuda_embed(ss_cuda_ctx_t *ctx, const int32_t *tokens, int32_t n, float *out);
/* Greedy decode of sequences 0..n_seq-1 together for n_steps (n_seq <=
 * max_batch), each step's tokens fed back on the device without a host round
 * trip: tokens[s] is sequence s's token at start_pos; ids_out [n_steps][n_seq]
 * receives the tokens generated at positions start_pos + 1 .. start_pos +
 * n_steps.  The single-sequence decode state is left unchanged. */
int ss_cuda_decode_greedy_batch(ss_cuda_ctx_t *ctx, const int32_t *tokens, int32_t n_seq,
                                int32_t start_pos, int32_t n_steps, int32_t *ids_out);
/* Greedy decode of n_steps tokens, each fed back on the device without a host
 * round trip: the token at start_pos is `token`, ids_out[i] receives the token
 * generated at position start_pos + 1 + i. */
int ss_cuda_decode_greedy(ss_cuda_ctx_t *ctx, int32_t token, int32_t start_pos, int32_t n_steps,
                          int32_t *ids_out);
/* Asynchronous pieces of ss_cuda_decode_greedy, for timing with events on
 * ss_cuda_stream(): begin (host->device of the token and position), steps
 * (enqueue n replays of the step graph, no synchronisation), read (wait, then
 * copy the tokens of positions [first_pos, first_pos + n) to the host). */
int ss_cuda_decode_begin(ss_cuda_ctx_t *ctx, int32_t token, int32_t pos);
int ss_cuda_decode_steps(ss_cuda_ctx_t *ctx, int32_t n_steps);
int ss_cuda_decode_read(ss_cuda_ctx_t *ctx, int32_t first_pos, int32_t n, int32_t *ids_out);
/* ---- sampling on the device: ss_sample (SlipStream/src/core/tensor.c:363-451)
 * temperature <= 0: the greedy argmax (tensor.c:318-328) and the RNG state is
 * neither read nor changed (rng_state may be NULL).  Otherwise: logits /
 * temperature (NaN logits as -FLT_MAX), softmax, top-k (top_k in 1..n-1: the
 * probabilities below the k-th largest are zeroed), top-p (top_p in (0, 1):
 * the sorted probabilities are added high to low until the sum reaches top_p,
 * those below the one reached are zeroed), renormalisation, and a draw with
 * xorshift64 (tensor.c:331-342) that advances *rng_state once -- every
 * running sum in the reference's order, so the result is the reference's
 * token for the same logits and state (the exponential is evaluated in double
 * precision; libm's expf differs in the last bit for about 1 input in 1,600).
 * One CTA on the context's stream; scratch of 3 floats per logit, grown on
 * first use.  Synchronous. */
/* ss_sample over caller logits (host memory, n floats; 1 <= n <= 16,777,216);
 * works on a context without a model too. */
int ss_cuda_sample_logits(ss_cuda_ctx_t *ctx, const float *logits, int32_t n, float temperature, float top_p,
                          int32_t top_k, uint64_t *rng_state, int32_t *token_out);
/* ss_sample over the logits of the context's last single-sequence step
 * (ss_cuda_forward / _prefill / _decode_*), which stay on the device.  Tensor
 * parallelism: every rank calls it (the logits are gathered) and all draw the
 * same token. */
int ss_cuda_sample(ss_cuda_ctx_t *ctx, float temperature, float top_p, int32_t top_k, uint64_t *rng_state,
                   int32_t *token_out);
/* The generation loop of ss_generate (engine.c:233-289) without a host round
 * trip per token: ids_out[0] is drawn from the context's current logits (those
 * for position start_pos, e.g. after a prefill of start_pos tokens), and for
 * t >= 1 ids_out[t] is drawn from the logits of the decode step that took
 * ids_out[t - 1] at position start_pos + t - 1.  n_tokens draws and n_tokens - 1
 * steps (start_pos + n_tokens - 1 <= ctx); *rng_state advances once per draw.
 * The caller ends the text at an EOS or stop string itself.  Afterwards the
 * context's position is the last draw's, so ss_cuda_decode_steps continues
 * from that token. */
int ss_cuda_decode_sample(ss_cuda_ctx_t *ctx, int32_t start_pos, int32_t n_tokens, float temperature,
                          float top_p, int32_t top_k, uint64_t *rng_state, int32_t *ids_out);
/* Several sequences sampled together (no reference counterpart: the reference
 * decodes one sequence; contexts with max_batch > 1): the sampled twin of
 * ss_cuda_decode_greedy_batch.  tokens[s] is sequence s's token at start_pos;
 * each of n_steps steps runs sequences 0..n_seq-1 through the many-token step,
 * draws every sequence's next token from its own logits with ss_sample's rule
 * and its own RNG state rng_states[s] (one draw each, one CTA per sequence, all
 * in one launch), and feeds the draws back on the device.  ids_out is
 * [n_steps][n_seq] (positions start_pos + 1 ..); rng_states is updated. */
int ss_cuda_decode_sample_batch(ss_cuda_ctx_t *ctx, const int32_t *tokens, int32_t n_seq, int32_t start_pos,
                                int32_t n_steps, float temperature, float top_p, int32_t top_k,
                                uint64_t *rng_states, int32_t *ids_out);

/* The cudaStream_t all work of this context runs on. */
void *ss_cuda_stream(ss_cuda_ctx_t *ctx);
/* Clears the KV cache (ss_scheduler_reset, layer_scheduler.c:917-936). */
void ss_cuda_reset(ss_cuda_ctx_t *ctx);
/* Thread-safe; the next scheduler/forward call returns SS_CUDA_ERROR_CANCELLED
 * (ss_cancel, engine.c:372-379). */
void ss_cuda_cancel(ss_cuda_ctx_t *ctx);

/* Test aid, no reference counterpart: makes the next persistent decode step
 * fail on the device without faulting -- its producer issues no copy for the
 * first weight stage of `phase` (1 = layer 0's QKV, 5 l + 1 + {0 QKV, 2 O, 3
 * gate/up, 4 down} = layer l's phases, 5 L + 1 = the lm_head), and every wait
 * of that step gives up after ~2 ms of clocks instead of ~1 s.  The step then
 * returns SS_CUDA_ERROR_BACKEND (device error bit 4, a ring wait ran out);
 * ss_cuda_reset makes the context usable again.  Single-GPU persistent step
 * only (SS_CUDA_ERROR_INVALID_PARAMS otherwise). */
int ss_cuda_test_fail_next_step(ss_cuda_ctx_t *ctx, int32_t phase);

/* ---- allocation-free greedy argmax (no counterpart in the reference) ----
 * For callers that cannot allocate device memory where they need a greedy
 * token -- e.g. while a stream is being captured into a CUDA graph, where
 * cudaMalloc is not allowed, or inside a host that only hands out buffers from
 * its own pool.  Writes to *d_index (device memory) the index of the first
 * maximum of d_values[0..n) (device memory).  The rule: scanning from index 0,
 * the answer moves only to a strictly greater value, so the first maximum wins
 * ties, -0.0 and +0.0 tie, a NaN after index 0 never wins, and a NaN at index 0
 * makes the answer 0.  Enqueued on `stream` (a cudaStream_t, NULL for the
 * legacy default stream) and asynchronous; calls no cudaMalloc/cudaFree.  n
 * must be 1 .. 4,194,304 and both pointers non-NULL
 * (SS_CUDA_ERROR_INVALID_PARAMS otherwise, nothing enqueued).  Its scratch is a
 * fixed 8 KiB array in the library's device image, shared by all calls: calls
 * that overlap on the GPU race, calls ordered on one stream do not.  The first
 * call on each device looks the array's address up (cudaGetSymbolAddress)
 * with that device current and keeps it for the life of the process; make that
 * first call before any stream capture begins, and do not reset the device
 * (cudaDeviceReset) after it -- the kept address would be stale. */
int ss_cuda_argmax_noalloc(const float *d_values, int32_t n, int32_t *d_index, void *stream);

/* Many-token twin of the op-level matvec (ss_cuda_matvec_q4_0 / _q8_0 for
 * n_tokens vectors at once, the pass over the weights shared): out[t] = W . x[t]
 * for the uploaded quantized tensor `name` (GGUF name, this rank's rows under
 * tensor parallelism), x as [n_tokens][cols] and out as [n_tokens][rows], host
 * memory, n_tokens 1..32.  Runs on the tensor cores (tcgen05, int8 planes of
 * the activations against the weights' int8 values, per-block fp16 scales in
 * fp32) -- the product the prompt and multi-sequence paths use.  Needs the
 * persistent step's weight layout (SS_CUDA_ERROR_INVALID_PARAMS otherwise). */
int ss_cuda_matmul_batch(ss_cuda_ctx_t *ctx, const char *name, const float *x, int32_t n_tokens, float *out);

/* ---- inspection (parity tests) ----
 * fp32 dequantisation of an uploaded weight tensor by GGUF name, rows in GGUF
 * order (n = rows * cols floats), computed on the device from the repacked
 * layout -- bit-identical to ss_dequantize (SlipStream/src/core/quantize.c:
 * 389-442) for Q4_0 / Q8_0. */
int ss_cuda_dequantize_tensor(ss_cuda_ctx_t *ctx, const char *name, float *out, int64_t n);
/* Device dequantisation of raw GGUF blocks (host in, host out); no context.
 * Every type of ss_dequantize (SlipStream/src/core/quantize.c:389-442): F32,
 * F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1 (blocks of 32) and Q2_K, Q3_K, Q4_K,
 * Q5_K, Q6_K (super-blocks of 256), bit-identical to the reference; n a
 * multiple of the block size.  Other types: SS_CUDA_ERROR_INVALID_PARAMS (the
 * reference zero-fills them). */
int ss_cuda_dequantize(int32_t type, const void *blocks, int64_t n, float *out);
/* int8 K/V row and scales of (layer, pos) (layer_scheduler.h:19-34 layout).
 * Under tensor parallelism: this rank's kv heads (n_kv_heads / tp_size * head_dim
 * bytes each), with the group-wide scale. */
int ss_cuda_kv_row(ss_cuda_ctx_t *ctx, int32_t layer, int32_t pos, int8_t *k, int8_t *v,
                   float *k_scale, float *v_scale);

#ifdef __cplusplus
}
#endif
#endif /* SLIPSTREAM_CUDA_H */
