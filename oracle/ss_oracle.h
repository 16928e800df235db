/*
 * ss_oracle.h -- CPU restatement of SlipStream's decode path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA backend.  Nothing in
 * phonemap_b200/ includes or links this.  Every function restates the
 * reference function cited beside it (paths relative to the PhoneMap repo) in
 * the same arithmetic order, so that with gcc -O2 it reproduces the
 * reference's results bit for bit (tests/test_oracle_ref.py checks this).
 */
#ifndef SS_ORACLE_H
#define SS_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sso_model sso_model_t;

/* dims: vocab, hidden, layers, heads, kv_heads, head_dim, ffn, max_seq */
sso_model_t *sso_load(const char *gguf_path, uint32_t context_size, int cap512);
void sso_free(sso_model_t *m);
void sso_dims(const sso_model_t *m, int32_t *dims);
void sso_reset(sso_model_t *m);
int sso_forward(sso_model_t *m, int32_t token, int32_t pos, float *logits_out);
int sso_prefill(sso_model_t *m, const int32_t *tokens, int32_t n, int32_t start_pos,
                float *logits_out);
int sso_embed(sso_model_t *m, const int32_t *tokens, int32_t n, float *out);
void sso_kv_row(const sso_model_t *m, int32_t layer, int32_t pos, int8_t *k, int8_t *v,
                float *ks, float *vs);

/* Summation order of this model's quantized matvecs: 0 = the reference's
 * sequential fp32 sum (default), 1 = a GPU-shaped blocked order (per-block FMA
 * chains, a 32-way butterfly).  Used to measure a configuration's parity noise
 * floor.  The single-op sso_dequant_matvec always uses order 0. */
void sso_set_dot_order(sso_model_t *m, int mode);

/* single ops */
float sso_f16_to_f32(uint16_t h);
void sso_dequantize(const void *src, float *dst, int32_t n, int32_t type);
void sso_dequant_matvec(float *out, const void *w, const float *x, int32_t rows,
                        int32_t cols, int32_t type);
void sso_rmsnorm(float *out, const float *x, const float *w, int32_t n, float eps);
void sso_rope(float *q, float *k, int32_t nh, int32_t nkv, int32_t hd, int32_t rope_dim,
              int32_t pos, float theta);
void sso_kv_encode(const float *src, int8_t *dst, float *scale, int32_t n);
void sso_softmax(float *x, int32_t n);
int32_t sso_argmax(const float *x, int32_t n);

/* ss_sample (SlipStream/src/core/tensor.c:363-451); exp_mode 0: libm expf as
 * the reference, 1: sso_exp_dd, the GPU sampler's exponential. */
int32_t sso_sample(const float *logits, int32_t n, float temperature, float top_p, int32_t top_k,
                   uint64_t *rng_state, int exp_mode);
float sso_exp_dd(float x);
void sso_exp_dd_array(const float *x, float *out, int32_t n);
float sso_rand_float(uint64_t *state);

#ifdef __cplusplus
}
#endif
#endif
