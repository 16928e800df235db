/*
 * synth_gguf.c -- deterministic random-init llama GGUF writer.
 *
 * Writes the seeded synthetic models the benchmark configurations name:
 * weights drawn from N(0, stddev) (Box-Muller over a counter-based hash, so the
 * bytes depend only on (seed, tensor index, element index) and not on thread
 * count or host), quantized to Q4_0 or Q8_0 blocks of 32 with an fp16 scale,
 * fp32 token embeddings, fp32 norm weights.
 *
 * File format: GGUF v3 as read by SlipStream's loader
 * (SlipStream/src/core/gguf_loader.c:210-485): little-endian header, KV
 * metadata, tensor infos with dims [ne0 = cols, ne1 = rows], then the data
 * section starting at the next 32-byte boundary, each tensor 32-byte aligned.
 * Block layouts follow SlipStream/src/core/quantize.h:13-17 (Q4_0: fp16 d then
 * 16 bytes, byte j = q[j] | q[j+16] << 4) and the Q8_0 struct in the same file
 * (fp16 d then 32 int8).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    uint32_t n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn, vocab, ctx;
    float rope_theta, rms_eps;
    int32_t wtype;       /* 2 = Q4_0, 8 = Q8_0 */
    int32_t out_type;    /* type of output.weight (2, 8) */
    uint64_t seed;
    float stddev;
    float norm_jitter;   /* 0 -> norm weights exactly 1.0; else 1 + N(0, jitter) */
} ss_synth_config_t;

enum { T_F32 = 0, T_Q4_0 = 2, T_Q8_0 = 8 };

static uint64_t mix64(uint64_t x) {
    x ^= x >> 30; x *= 0xbf58476d1ce4e5b9ULL;
    x ^= x >> 27; x *= 0x94d049bb133111ebULL;
    x ^= x >> 31;
    return x;
}

/* Normal sample for element i of tensor t. */
static float gauss(uint64_t seed, uint64_t t, uint64_t i) {
    uint64_t pair = i >> 1;
    uint64_t h = mix64(seed * 0x9e3779b97f4a7c15ULL + mix64(t * 0xd1b54a32d192ed03ULL + pair));
    double u1 = ((double)(h >> 32) + 0.5) * (1.0 / 4294967296.0);
    double u2 = ((double)(h & 0xffffffffULL) + 0.5) * (1.0 / 4294967296.0);
    double r = sqrt(-2.0 * log(u1));
    double a = 6.283185307179586 * u2;
    return (float)((i & 1) ? r * sin(a) : r * cos(a));
}

static uint16_t f32_to_f16(float f) {
    _Float16 h = (_Float16)f;  /* round-to-nearest-even */
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

static size_t type_row_bytes(int type, uint64_t cols) {
    if (type == T_F32) return cols * 4;
    if (type == T_Q4_0) return cols / 32 * 18;
    return cols / 32 * 34;
}

/* Q4_0 block: d = signed absmax / -8, q = clamp(trunc(x/d + 8.5), 0, 15). */
static void quant_q4_0(const float *x, uint8_t *out) {
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < 32; j++) {
        float a = fabsf(x[j]);
        if (a > amax) { amax = a; mx = x[j]; }
    }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = f32_to_f16(d);
    memcpy(out, &dh, 2);
    for (int j = 0; j < 16; j++) {
        int q0 = (int)(x[j] * id + 8.5f);
        int q1 = (int)(x[j + 16] * id + 8.5f);
        q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
        q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
        out[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* Q8_0 block: d = absmax / 127, q = round(x / d). */
static void quant_q8_0(const float *x, uint8_t *out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) {
        float a = fabsf(x[j]);
        if (a > amax) amax = a;
    }
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = f32_to_f16(d);
    memcpy(out, &dh, 2);
    for (int j = 0; j < 32; j++) {
        int q = (int)roundf(x[j] * id);
        q = q < -128 ? -128 : (q > 127 ? 127 : q);
        out[2 + j] = (uint8_t)(int8_t)q;
    }
}

typedef struct {
    char name[64];
    uint64_t cols, rows;  /* rows = 1 for vectors */
    int n_dims;
    int type;
    int kind;             /* 0 = gaussian weight, 1 = norm */
    uint64_t offset;      /* relative to data section */
    uint64_t bytes;
} tdesc_t;

static void fill_tensor(const ss_synth_config_t *c, uint64_t tidx, const tdesc_t *t,
                        uint8_t *buf) {
    uint64_t n = t->cols * t->rows;
    if (t->type == T_F32) {
        float *f = (float *)buf;
        if (t->kind == 1) {
            #pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++)
                f[i] = c->norm_jitter == 0.0f ? 1.0f
                     : 1.0f + c->norm_jitter * gauss(c->seed, tidx, (uint64_t)i);
        } else {
            #pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++)
                f[i] = c->stddev * gauss(c->seed, tidx, (uint64_t)i);
        }
        return;
    }
    int64_t nblk = (int64_t)(n / 32);
    size_t bb = t->type == T_Q4_0 ? 18 : 34;
    #pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblk; b++) {
        float x[32];
        for (int j = 0; j < 32; j++)
            x[j] = c->stddev * gauss(c->seed, tidx, (uint64_t)b * 32 + j);
        if (t->type == T_Q4_0) quant_q4_0(x, buf + b * bb);
        else quant_q8_0(x, buf + b * bb);
    }
}

/* ---- GGUF writing ---- */
static void w_u32(FILE *f, uint32_t v) { fwrite(&v, 4, 1, f); }
static void w_u64(FILE *f, uint64_t v) { fwrite(&v, 8, 1, f); }
static void w_f32(FILE *f, float v) { fwrite(&v, 4, 1, f); }
static void w_str(FILE *f, const char *s) { w_u64(f, strlen(s)); fwrite(s, 1, strlen(s), f); }
static void kv_u32(FILE *f, const char *k, uint32_t v) { w_str(f, k); w_u32(f, 4); w_u32(f, v); }
static void kv_f32(FILE *f, const char *k, float v) { w_str(f, k); w_u32(f, 6); w_f32(f, v); }
static void kv_str(FILE *f, const char *k, const char *v) { w_str(f, k); w_u32(f, 8); w_str(f, v); }

static int add(tdesc_t *t, int *n, const char *name, uint64_t cols, uint64_t rows,
               int type, int kind) {
    tdesc_t *d = &t[(*n)++];
    memset(d, 0, sizeof(*d));
    snprintf(d->name, sizeof(d->name), "%s", name);
    d->cols = cols; d->rows = rows; d->n_dims = rows > 1 ? 2 : 1;
    d->type = type; d->kind = kind;
    d->bytes = type_row_bytes(type, cols) * rows;
    return 0;
}

/* Returns 0 on success, negative on error. */
int ss_synth_write_gguf(const char *path, const ss_synth_config_t *c) {
    if (!path || !c || c->d_model % 32 || c->ffn % 32) return -1;
    if (c->wtype != T_Q4_0 && c->wtype != T_Q8_0) return -1;
    uint64_t d = c->d_model, hd = c->head_dim;
    uint64_t qd = (uint64_t)c->n_heads * hd, kvd = (uint64_t)c->n_kv_heads * hd;
    int cap = 3 + 9 * (int)c->n_layers;
    tdesc_t *t = (tdesc_t *)calloc((size_t)cap, sizeof(tdesc_t));
    if (!t) return -3;
    int n = 0;
    char nm[64];
    add(t, &n, "token_embd.weight", d, c->vocab, T_F32, 0);
    for (uint32_t l = 0; l < c->n_layers; l++) {
        snprintf(nm, 64, "blk.%u.attn_norm.weight", l);   add(t, &n, nm, d, 1, T_F32, 1);
        snprintf(nm, 64, "blk.%u.attn_q.weight", l);      add(t, &n, nm, d, qd, c->wtype, 0);
        snprintf(nm, 64, "blk.%u.attn_k.weight", l);      add(t, &n, nm, d, kvd, c->wtype, 0);
        snprintf(nm, 64, "blk.%u.attn_v.weight", l);      add(t, &n, nm, d, kvd, c->wtype, 0);
        snprintf(nm, 64, "blk.%u.attn_output.weight", l); add(t, &n, nm, qd, d, c->wtype, 0);
        snprintf(nm, 64, "blk.%u.ffn_norm.weight", l);    add(t, &n, nm, d, 1, T_F32, 1);
        snprintf(nm, 64, "blk.%u.ffn_gate.weight", l);    add(t, &n, nm, d, c->ffn, c->wtype, 0);
        snprintf(nm, 64, "blk.%u.ffn_up.weight", l);      add(t, &n, nm, d, c->ffn, c->wtype, 0);
        snprintf(nm, 64, "blk.%u.ffn_down.weight", l);    add(t, &n, nm, c->ffn, d, c->wtype, 0);
    }
    add(t, &n, "output_norm.weight", d, 1, T_F32, 1);
    add(t, &n, "output.weight", d, c->vocab, c->out_type ? c->out_type : c->wtype, 0);

    uint64_t off = 0;
    for (int i = 0; i < n; i++) {
        t[i].offset = off;
        off += (t[i].bytes + 31) & ~(uint64_t)31;
    }

    FILE *f = fopen(path, "wb");
    if (!f) { free(t); return -2; }
    w_u32(f, 0x46554747u);
    w_u32(f, 3);
    w_u64(f, (uint64_t)n);
    w_u64(f, 12);
    kv_str(f, "general.architecture", "llama");
    kv_u32(f, "general.alignment", 32);
    kv_u32(f, "llama.block_count", c->n_layers);
    kv_u32(f, "llama.context_length", c->ctx);
    kv_u32(f, "llama.embedding_length", c->d_model);
    kv_u32(f, "llama.feed_forward_length", c->ffn);
    kv_u32(f, "llama.attention.head_count", c->n_heads);
    kv_u32(f, "llama.attention.head_count_kv", c->n_kv_heads);
    kv_u32(f, "llama.rope.dimension_count", c->head_dim);
    kv_f32(f, "llama.rope.freq_base", c->rope_theta);
    kv_f32(f, "llama.attention.layer_norm_rms_epsilon", c->rms_eps);
    kv_u32(f, "llama.vocab_size", c->vocab);
    for (int i = 0; i < n; i++) {
        w_str(f, t[i].name);
        w_u32(f, (uint32_t)t[i].n_dims);
        w_u64(f, t[i].cols);
        if (t[i].n_dims == 2) w_u64(f, t[i].rows);
        w_u32(f, (uint32_t)t[i].type);
        w_u64(f, t[i].offset);
    }
    long pos = ftell(f);
    static const uint8_t zeros[32] = {0};
    fwrite(zeros, 1, (size_t)(((pos + 31) & ~31L) - pos), f);

    int rc = 0;
    for (int i = 0; i < n && rc == 0; i++) {
        uint64_t padded = (t[i].bytes + 31) & ~(uint64_t)31;
        uint8_t *buf = (uint8_t *)calloc(1, padded);
        if (!buf) { rc = -3; break; }
        fill_tensor(c, (uint64_t)i, &t[i], buf);
        if (fwrite(buf, 1, padded, f) != padded) rc = -4;
        free(buf);
    }
    if (fclose(f) != 0 && rc == 0) rc = -4;
    free(t);
    return rc;
}
