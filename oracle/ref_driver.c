/*
 * ref_driver.c -- flat C entry points into the reference SlipStream CPU path.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled by oracle/build_ref.py together with a
 * temporary copy of the reference sources into oracle/_ref/libss_ref*.so; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Random-init GGUF files carry no tokenizer vocabulary, so the driver skips
 * ss_generate/ss_embed's tokenizer step and calls the scheduler directly, the
 * same calls engine.c makes (engine.c:211 prefill, :284 forward, :339 embed).
 */
#include "core/engine.h"
#include "core/layer_scheduler.h"
#include "core/quantize.h"
#include "core/tensor.h"

#include <stdlib.h>
#include <string.h>

/* ss_model_load with the CPU backend (engine.c:56-137). */
void *ssr_load(const char *path, uint32_t context_size) {
    ss_model_config_t cfg = ss_default_config();
    cfg.backend = SS_BACKEND_CPU;
    cfg.context_size = context_size;
    cfg.prefetch = false;
    return ss_model_load(path, &cfg);
}

void ssr_free(void *m) { ss_model_free((ss_model_t *)m); }

#ifdef SS_HAS_CUDA
/* The integration build (build_ref.py, libss_ref_cuda.so): hand the
 * scheduler a CUDA context, as ss_model_load would next to the Metal one
 * (engine.c:87-96); ss_matmul_dispatch then sends the projections to it. */
void ssr_attach_cuda(void *m, void *cuda_ctx) { ((ss_model_t *)m)->scheduler->cuda_ctx = cuda_ctx; }
#endif

/* dims[0..7] = vocab, hidden, layers, heads, kv_heads, head_dim, ffn, max_seq */
void ssr_dims(void *m, int32_t *dims) {
    ss_scheduler_t *s = ((ss_model_t *)m)->scheduler;
    dims[0] = s->state.vocab_size;
    dims[1] = s->state.hidden_size;
    dims[2] = s->num_layers;
    dims[3] = s->state.num_heads;
    dims[4] = s->state.num_kv_heads;
    dims[5] = s->state.head_dim;
    dims[6] = s->state.intermediate_size;
    dims[7] = s->kv_cache.max_seq_len;
}

void ssr_reset(void *m) { ss_scheduler_reset(((ss_model_t *)m)->scheduler); }

/* ss_scheduler_prefill (layer_scheduler.c:681-803); copies the logits out. */
int ssr_prefill(void *m, const int32_t *tokens, int32_t n, int32_t start_pos,
                float *logits_out) {
    ss_scheduler_t *s = ((ss_model_t *)m)->scheduler;
    float *lg = ss_scheduler_prefill(s, tokens, n, start_pos);
    if (!lg) return -1;
    if (logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)s->state.vocab_size);
    return 0;
}

/* ss_scheduler_forward (layer_scheduler.c:571-679); copies the logits out. */
int ssr_forward(void *m, int32_t token, int32_t pos, float *logits_out) {
    ss_scheduler_t *s = ((ss_model_t *)m)->scheduler;
    float *lg = ss_scheduler_forward(s, token, pos);
    if (!lg) return -1;
    if (logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)s->state.vocab_size);
    return 0;
}

/* ss_scheduler_embed (layer_scheduler.c:805-915). */
int ssr_embed(void *m, const int32_t *tokens, int32_t n, float *out) {
    ss_scheduler_t *s = ((ss_model_t *)m)->scheduler;
    float *e = ss_scheduler_embed(s, tokens, n);
    if (!e) return -1;
    memcpy(out, e, sizeof(float) * (size_t)s->state.hidden_size);
    free(e);
    return 0;
}

/* int8 K/V row and scales written by kv_turboquant_encode (layer_scheduler.c:409-413). */
void ssr_kv_row(void *m, int32_t layer, int32_t pos, int8_t *k_out, int8_t *v_out,
                float *k_scale, float *v_scale) {
    ss_kv_cache_t *c = &((ss_model_t *)m)->scheduler->kv_cache;
    size_t vi = (size_t)layer * c->max_seq_len + pos;
    memcpy(k_out, c->q_key_cache + vi * c->kv_dim, (size_t)c->kv_dim);
    memcpy(v_out, c->q_val_cache + vi * c->kv_dim, (size_t)c->kv_dim);
    *k_scale = c->k_scales[vi];
    *v_scale = c->v_scales[vi];
}

/* ---- single ops, for op-level parity ---- */
void ssr_dequantize(const void *src, float *dst, int32_t n, int32_t type) {
    ss_dequantize(src, dst, n, (ggml_type_t)type);
}
void ssr_dequant_matvec(float *out, const void *w, const float *x, int32_t rows,
                        int32_t cols, int32_t type) {
    ss_dequant_matvec(out, w, x, rows, cols, (ggml_type_t)type);
}
void ssr_matvec_f32(float *out, const float *w, const float *x, int32_t rows, int32_t cols) {
    ss_matvec(out, w, x, rows, cols);
}
void ssr_rmsnorm(float *out, const float *x, const float *w, int32_t n, float eps) {
    ss_rmsnorm(out, x, w, n, eps, 0);
}
void ssr_rope(float *q, float *k, int32_t nh, int32_t nkv, int32_t hd, int32_t rope_dim,
              int32_t pos, float theta) {
    ss_rope(q, k, nh, nkv, hd, rope_dim, pos, theta, false);
}
void ssr_softmax(float *x, int32_t n) { ss_softmax(x, n); }
int32_t ssr_argmax(const float *x, int32_t n) { return ss_argmax(x, n); }
float ssr_f16_to_f32(uint16_t h) { return ss_f16_to_f32(h); }
