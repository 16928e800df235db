/*
 * ss_oracle.c -- CPU restatement of SlipStream's decode path (llama variant).
 *
 * TEST INFRASTRUCTURE ONLY (see ss_oracle.h).  Reference = harrisonfar123/
 * PhoneMap, SlipStream/ (abbreviated SS/ below).  Scope is the path the CUDA
 * backend replaces: embedding -> L x (RMSNorm, Q/K/V GEMV, RoPE, int8 KV
 * encode, GQA attention, O GEMV + residual, RMSNorm, gate/up GEMV, SwiGLU, down
 * GEMV + residual) -> final RMSNorm -> lm_head, plus greedy argmax.  The
 * Gemma/Qwen/Phi/NeoX branches of the reference are out of scope.
 *
 * Arithmetic order is the reference's: every dot product is one sequential
 * fp32 sum (the Accelerate stand-in used to build the reference on Linux),
 * every product and sum is rounded separately (gcc -O2, no FMA), and libm's
 * expf/powf/cosf/sinf/roundf/sqrtf are called as the reference calls them.
 * Rows of a matvec and heads of attention are independent, so they run on
 * OpenMP threads without changing any result.
 */
#include "ss_oracle.h"

#include <fcntl.h>
#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

enum {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q8_1 = 9,
    T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14
};

/* ---------------------------------------------------------------- numerics */

/* SS/src/core/quantize.c:20-56 (IEEE half -> float, subnormals normalised). */
float sso_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            e = 1;
            while (!(m & 0x400)) { m <<= 1; e--; }
            m &= 0x3FF;
            bits = sign | ((e + 112) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Bytes per block and values per block (SS/src/core/gguf_loader.c:22-60). */
static size_t type_size(int t) {
    switch (t) {
        case T_F32: return 4;
        case T_F16: return 2;
        case T_Q4_0: return 18;
        case T_Q4_1: return 20;
        case T_Q5_0: return 22;
        case T_Q5_1: return 24;
        case T_Q8_0: return 34;
        case T_Q8_1: return 40;
        case T_Q2_K: return 84;
        case T_Q3_K: return 110;
        case T_Q4_K: return 144;
        case T_Q5_K: return 176;
        case T_Q6_K: return 210;
        default: return 0;
    }
}
static int block_size(int t) {
    if (t == T_F32 || t == T_F16) return 1;
    return t >= T_Q2_K && t <= T_Q6_K ? 256 : 32;
}

static float half_at(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return sso_f16_to_f32(h);
}

/* The 6-bit scale and min of sub-block j of a Q4_K / Q5_K super-block
 * (quantize.c:268-276): sub-blocks 0-3 in the low 6 bits of bytes j and j + 4,
 * 4-7 split between the nibbles of bytes j + 4 and the top 2 bits of bytes
 * j - 4 and j. */
static void k4_scale_min(int j, const uint8_t *sc, float *s, float *m) {
    int a, b;
    if (j < 4) {
        a = sc[j] & 63;
        b = sc[j + 4] & 63;
    } else {
        a = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        b = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    *s = (float)a;
    *m = (float)b;
}

/* One block of `type` into out[0 .. block_size): the formulas of
 * SS/src/core/quantize.c:58-383, each product and difference rounded on its own
 * (the reference is built without FMA). */
static void dequant_block(int type, const uint8_t *blk, float *out) {
    switch (type) {
        case T_Q4_0: {  /* :60-72 */
            const float d = half_at(blk);
            for (int i = 0; i < 16; i++) {
                out[i] = d * ((int32_t)(blk[2 + i] & 0xF) - 8);
                out[i + 16] = d * ((int32_t)(blk[2 + i] >> 4) - 8);
            }
            break;
        }
        case T_Q4_1: {  /* :76-89 */
            const float d = half_at(blk), mn = half_at(blk + 2);
            for (int i = 0; i < 16; i++) {
                out[i] = d * (blk[4 + i] & 0xF) + mn;
                out[i + 16] = d * (blk[4 + i] >> 4) + mn;
            }
            break;
        }
        case T_Q5_0: {  /* :93-112: the fifth bits in a 32-bit mask */
            const float d = half_at(blk);
            uint32_t hb;
            memcpy(&hb, blk + 2, 4);
            for (int i = 0; i < 16; i++) {
                const int lo = (blk[6 + i] & 0xF) | (int)(((hb >> i) & 1) << 4);
                const int hi = (blk[6 + i] >> 4) | (int)(((hb >> (i + 16)) & 1) << 4);
                out[i] = (lo - 16) * d;
                out[i + 16] = (hi - 16) * d;
            }
            break;
        }
        case T_Q5_1: {  /* :116-135 */
            const float d = half_at(blk), mn = half_at(blk + 2);
            uint32_t hb;
            memcpy(&hb, blk + 4, 4);
            for (int i = 0; i < 16; i++) {
                const int lo = (blk[8 + i] & 0xF) | (int)(((hb >> i) & 1) << 4);
                const int hi = (blk[8 + i] >> 4) | (int)(((hb >> (i + 16)) & 1) << 4);
                out[i] = lo * d + mn;
                out[i + 16] = hi * d + mn;
            }
            break;
        }
        case T_Q8_0: {  /* :139-149 */
            const float d = half_at(blk);
            for (int i = 0; i < 32; i++) out[i] = d * (int8_t)blk[2 + i];
            break;
        }
        case T_Q8_1: {  /* :153-163: an fp32 scale (and an unused fp32 sum) */
            float d;
            memcpy(&d, blk, 4);
            for (int i = 0; i < 32; i++) out[i] = d * (int8_t)blk[8 + i];
            break;
        }
        case T_Q2_K: {  /* :180-215: 16-value groups, 4-bit scale and min each */
            const uint8_t *sc = blk, *qs = blk + 16;
            const float d = half_at(blk + 80), mn = half_at(blk + 82);
            for (int e = 0; e < 256; e++) {
                const int h = e >> 7, r = e & 31, j = (e & 127) >> 5;
                const uint8_t s8 = sc[8 * h + 2 * j + (r >> 4)];
                const float dl = d * (s8 & 0xF), ml = mn * (s8 >> 4);
                out[e] = dl * ((int8_t)((qs[32 * h + r] >> (2 * j)) & 3)) - ml;
            }
            break;
        }
        case T_Q3_K: {  /* :219-263: 6-bit scales unpacked from 12 bytes */
            const uint8_t *hm = blk, *qs = blk + 32;
            const float d = half_at(blk + 108);
            int8_t s6[16];
            for (int i = 0; i < 16; i++) {
                const int low = i < 8 ? (blk[96 + i] & 0xF) : (blk[96 + i - 8] >> 4);
                const int top = (blk[104 + (i & 3)] >> (2 * (i >> 2))) & 3;
                s6[i] = (int8_t)(low | (top << 4));
            }
            for (int e = 0; e < 256; e++) {
                const int h = e >> 7, r = e & 31, j = (e & 127) >> 5;
                const float dl = d * (s6[8 * h + 2 * j + (r >> 4)] - 32);
                const int q = (int8_t)((qs[32 * h + r] >> (2 * j)) & 3) - ((hm[r] & (1 << (4 * h + j))) ? 0 : 4);
                out[e] = dl * q;
            }
            break;
        }
        case T_Q4_K: {  /* :278-308 */
            const float d = half_at(blk), mn = half_at(blk + 2);
            const uint8_t *sc = blk + 4, *qs = blk + 16;
            for (int c = 0; c < 4; c++) {
                float s1, m1, s2, m2;
                k4_scale_min(2 * c, sc, &s1, &m1);
                k4_scale_min(2 * c + 1, sc, &s2, &m2);
                const float d1 = d * s1, n1 = mn * m1, d2 = d * s2, n2 = mn * m2;
                for (int l = 0; l < 32; l++) {
                    out[64 * c + l] = d1 * (qs[32 * c + l] & 0xF) - n1;
                    out[64 * c + 32 + l] = d2 * (qs[32 * c + l] >> 4) - n2;
                }
            }
            break;
        }
        case T_Q5_K: {  /* :312-348 */
            const float d = half_at(blk), mn = half_at(blk + 2);
            const uint8_t *sc = blk + 4, *qh = blk + 16, *qs = blk + 48;
            for (int c = 0; c < 4; c++) {
                float s1, m1, s2, m2;
                k4_scale_min(2 * c, sc, &s1, &m1);
                k4_scale_min(2 * c + 1, sc, &s2, &m2);
                const float d1 = d * s1, n1 = mn * m1, d2 = d * s2, n2 = mn * m2;
                for (int l = 0; l < 32; l++) {
                    out[64 * c + l] = d1 * ((qs[32 * c + l] & 0xF) + ((qh[l] >> (2 * c)) & 1 ? 16 : 0)) - n1;
                    out[64 * c + 32 + l] = d2 * ((qs[32 * c + l] >> 4) + ((qh[l] >> (2 * c + 1)) & 1 ? 16 : 0)) - n2;
                }
            }
            break;
        }
        case T_Q6_K: {  /* :352-383: (d * scale) * q, two roundings */
            const float d = half_at(blk + 208);
            for (int e = 0; e < 256; e++) {
                const int h = e >> 7, g = (e & 127) >> 5, l = e & 31;
                const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
                const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
                const int lo = (g & 1) ? ql[l + 32] : ql[l];
                const int nib = (g & 2) ? (lo >> 4) : (lo & 0xF);
                const int q = (int8_t)(nib | (((qh[l] >> (2 * g)) & 3) << 4)) - 32;
                out[e] = d * sc[(l >> 4) + 2 * g] * q;
            }
            break;
        }
        default:
            memset(out, 0, sizeof(float) * (size_t)block_size(type));
    }
}

/* SS/src/core/quantize.c:389-442 (ss_dequantize): F32 copied, F16 converted,
 * block types block by block; an unknown type gives zeros, as the reference. */
void sso_dequantize(const void *src, float *dst, int32_t n, int32_t type) {
    const uint8_t *p = (const uint8_t *)src;
    if (type == T_F32) { memcpy(dst, src, (size_t)n * 4); return; }
    if (type == T_F16) {
        for (int32_t i = 0; i < n; i++) dst[i] = half_at(p + 2 * i);
        return;
    }
    const size_t ts = type_size(type);
    const int bs = block_size(type);
    if (!ts) {
        memset(dst, 0, (size_t)n * 4);
        return;
    }
    for (int32_t b = 0; b < n / bs; b++) dequant_block(type, p + (size_t)b * ts, dst + (size_t)b * bs);
}

/* Sequential fp32 dot: the order the reference's vDSP_dotpr calls get. */
static float dot_seq(const float *a, const float *b, int32_t n) {
    float s = 0.0f;
    for (int32_t i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* Summation order of the quantized matvecs.  0 (default) is the reference's:
 * one sequential fp32 sum per row.  1 is an equally valid reordering of the
 * same arithmetic -- per 32-weight block a fused multiply-add chain of
 * (q - zp) * x, scaled by the block's d, accumulated per block index modulo 32
 * and combined by a 32-way butterfly (the shape of a GPU reduction) -- used to
 * measure how far the reference's own outputs move under a different fp32
 * rounding order (the parity noise floor of a configuration). */

static float dot_blocked(const uint8_t *row, const float *x, int32_t cols, int32_t type) {
    float lane[32] = {0};
    const size_t bsz = type_size(type);
    for (int32_t b = 0; b < cols / 32; b++) {
        const uint8_t *blk = row + (size_t)b * bsz;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        const float d = sso_f16_to_f32(dh);
        float p = 0.0f;
        for (int j = 0; j < 32; j++) {
            float q;
            if (type == T_Q4_0) q = (float)((j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4)) - 8);
            else q = (float)(int8_t)blk[2 + j];
            p = fmaf(q, x[b * 32 + j], p);
        }
        lane[b % 32] = fmaf(d, p, lane[b % 32]);
    }
    for (int off = 16; off >= 1; off >>= 1)
        for (int l = 0; l < off; l++) lane[l] = lane[l] + lane[l + off];
    return lane[0];
}

/* SS/src/core/quantize.c:446-494: per row, dequantize into a temp, then
 * vDSP_dotpr(tmp, x).  F32 matrices use ss_matvec -> ss_neon_dot scalar
 * (SS/src/backends/cpu_neon.c:55-62), the same sequential sum. */
static void matvec_ordered(float *out, const void *w, const float *x, int32_t rows,
                           int32_t cols, int32_t type, int order) {
    size_t row_bytes = (size_t)(cols / block_size(type)) * type_size(type);
    const int blocked = order == 1 && (type == T_Q4_0 || type == T_Q8_0);
    #pragma omp parallel
    {
        float *tmp = (float *)malloc((size_t)cols * sizeof(float));
        #pragma omp for schedule(static)
        for (int32_t r = 0; r < rows; r++) {
            const uint8_t *rp = (const uint8_t *)w + (size_t)r * row_bytes;
            if (blocked) {
                out[r] = dot_blocked(rp, x, cols, type);
            } else {
                sso_dequantize(rp, tmp, cols, type);
                out[r] = dot_seq(tmp, x, cols);
            }
        }
        free(tmp);
    }
}

void sso_dequant_matvec(float *out, const void *w, const float *x, int32_t rows,
                        int32_t cols, int32_t type) {
    matvec_ordered(out, w, x, rows, cols, type, 0);
}

/* SS/src/backends/cpu_neon.c:109-115 (scalar ss_neon_rmsnorm, reached from
 * ss_rmsnorm SS/src/core/tensor.c:114-118 for F32 weights). */
void sso_rmsnorm(float *out, const float *x, const float *w, int32_t n, float eps) {
    float ss = 0.0f;
    for (int32_t i = 0; i < n; i++) ss += x[i] * x[i];
    float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (int32_t i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

/* SS/src/core/tensor.c:249-274 (non-NeoX RoPE: rotate pairs (i, i+1)). */
void sso_rope(float *q, float *k, int32_t nh, int32_t nkv, int32_t hd, int32_t rope_dim,
              int32_t pos, float theta) {
    for (int32_t i = 0; i < rope_dim; i += 2) {
        float freq = 1.0f / powf(theta, (float)i / (float)rope_dim);
        float angle = (float)pos * freq;
        float c = cosf(angle), s = sinf(angle);
        for (int32_t h = 0; h < nh; h++) {
            float *v = q + h * hd;
            float a = v[i], b = v[i + 1];
            v[i] = a * c - b * s;
            v[i + 1] = a * s + b * c;
        }
        for (int32_t h = 0; h < nkv; h++) {
            float *v = k + h * hd;
            float a = v[i], b = v[i + 1];
            v[i] = a * c - b * s;
            v[i + 1] = a * s + b * c;
        }
    }
}

/* SS/src/core/layer_scheduler.c:101-118 (kv_turboquant_encode): one symmetric
 * int8 scale over the whole kv_dim vector. */
void sso_kv_encode(const float *src, int8_t *dst, float *scale_out, int32_t n) {
    float mx = 0.0f;
    for (int32_t i = 0; i < n; i++) {
        float v = fabsf(src[i]);
        if (v > mx) mx = v;
    }
    float scale = mx / 127.0f;
    *scale_out = scale;
    float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
    for (int32_t i = 0; i < n; i++) dst[i] = (int8_t)roundf(src[i] * inv);
}

/* SS/src/core/tensor.c:154-173. */
void sso_softmax(float *x, int32_t n) {
    float mx = -FLT_MAX;
    for (int32_t i = 0; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int32_t i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    float inv = 1.0f / sum;
    for (int32_t i = 0; i < n; i++) x[i] *= inv;
}

/* SS/src/core/tensor.c:318-328: strict '>' so the lowest index wins ties. */
int32_t sso_argmax(const float *x, int32_t n) {
    int32_t best = 0;
    float mv = x[0];
    for (int32_t i = 1; i < n; i++) if (x[i] > mv) { mv = x[i]; best = i; }
    return best;
}

/* ------------------------------------------------------------------ model */

typedef struct { const uint8_t *data; int type; uint64_t rows, cols; } tref_t;

typedef struct {
    tref_t attn_norm, wq, wk, wv, wo, ffn_norm, wgate, wup, wdown;
} layer_t;

struct sso_model {
    uint8_t *map; size_t map_size;
    int32_t vocab, d, L, nh, nkv, hd, rope_dim, ff, max_seq, kvd;
    float eps, theta;
    tref_t embd, out_norm, out;
    layer_t *layers;
    /* KV cache, SS/src/core/layer_scheduler.h:19-34 */
    int8_t *kc, *vc;
    float *ks, *vs;
    /* working state, SS/src/core/layer_scheduler.h:38-65 */
    float *hidden, *residual, *attn_out, *ffn_buf, *ffn_gate, *q, *k, *v, *logits;
    int dot_order; /* summation order of the quantized matvecs, see matvec_ordered */
};

void sso_set_dot_order(sso_model_t *m, int mode) { m->dot_order = mode; }

typedef struct { const uint8_t *p, *end; int ok; } rd_t;
static uint64_t rd_u(rd_t *r, int n) {
    uint64_t v = 0;
    if (r->p + n > r->end) { r->ok = 0; return 0; }
    memcpy(&v, r->p, (size_t)n);
    r->p += n;
    return v;
}
static const char *rd_s(rd_t *r, uint64_t *len) {
    *len = rd_u(r, 8);
    const char *s = (const char *)r->p;
    if (r->p + *len > r->end) { r->ok = 0; return ""; }
    r->p += *len;
    return s;
}
static void rd_skip(rd_t *r, uint32_t type) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    uint64_t len;
    if (type == 8) { rd_s(r, &len); return; }
    if (type == 9) {
        uint32_t at = (uint32_t)rd_u(r, 4);
        uint64_t n = rd_u(r, 8);
        for (uint64_t i = 0; i < n && r->ok; i++) rd_skip(r, at);
        return;
    }
    if (type < 13) r->p += sz[type]; else r->ok = 0;
}
static int ends_with(const char *s, size_t n, const char *suf) {
    size_t m = strlen(suf);
    return n >= m && memcmp(s + n - m, suf, m) == 0;
}

/* Header/KV/tensor-info walk of SS/src/core/gguf_loader.c:250-431 restated for
 * the keys this path reads; defaults from :370-379. */
sso_model_t *sso_load(const char *path, uint32_t context_size, int cap512) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return NULL; }
    uint8_t *map = (uint8_t *)mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return NULL;
    sso_model_t *m = (sso_model_t *)calloc(1, sizeof(*m));
    m->map = map; m->map_size = (size_t)st.st_size;
    rd_t r = {map, map + st.st_size, 1};
    if (rd_u(&r, 4) != 0x46554747u) goto fail;
    rd_u(&r, 4);
    uint64_t n_t = rd_u(&r, 8), n_kv = rd_u(&r, 8);
    uint32_t ctx_len = 0, vocab_kv = 0, key_len = 0, rope_dim = 0;
    for (uint64_t i = 0; i < n_kv && r.ok; i++) {
        uint64_t kl;
        const char *k = rd_s(&r, &kl);
        uint32_t t = (uint32_t)rd_u(&r, 4);
        #define U32(suf, dst) else if (t == 4 && ends_with(k, kl, suf)) dst = (uint32_t)rd_u(&r, 4)
        if (0) {}
        U32(".embedding_length", m->d);
        U32(".attention.head_count_kv", m->nkv);
        U32(".attention.head_count", m->nh);
        U32(".context_length", ctx_len);
        U32(".feed_forward_length", m->ff);
        U32(".block_count", m->L);
        U32(".vocab_size", vocab_kv);
        U32(".attention.key_length", key_len);
        U32(".rope.dimension_count", rope_dim);
        else if (t == 6 && ends_with(k, kl, ".rope.freq_base")) { uint32_t b = (uint32_t)rd_u(&r, 4); memcpy(&m->theta, &b, 4); }
        else if (t == 6 && ends_with(k, kl, ".attention.layer_norm_rms_epsilon")) { uint32_t b = (uint32_t)rd_u(&r, 4); memcpy(&m->eps, &b, 4); }
        else rd_skip(&r, t);
        #undef U32
    }
    if (m->eps == 0.0f) m->eps = 1e-5f;
    if (m->theta == 0.0f) m->theta = 10000.0f;
    if (ctx_len == 0) ctx_len = 2048;
    if (m->nkv == 0) m->nkv = m->nh;
    m->layers = (layer_t *)calloc((size_t)m->L, sizeof(layer_t));
    typedef struct { const char *name; uint64_t nl; uint64_t d0, d1; int nd, type; uint64_t off; } ti_t;
    ti_t *ti = (ti_t *)calloc((size_t)n_t, sizeof(ti_t));
    for (uint64_t i = 0; i < n_t && r.ok; i++) {
        ti[i].name = rd_s(&r, &ti[i].nl);
        ti[i].nd = (int)rd_u(&r, 4);
        ti[i].d1 = 1;
        for (int j = 0; j < ti[i].nd; j++) {
            uint64_t v = rd_u(&r, 8);
            if (j == 0) ti[i].d0 = v; else if (j == 1) ti[i].d1 = v;
        }
        ti[i].type = (int)rd_u(&r, 4);
        ti[i].off = rd_u(&r, 8);
    }
    if (!r.ok) { free(ti); goto fail; }
    uint64_t data_off = ((uint64_t)(r.p - map) + 31) & ~(uint64_t)31;  /* gguf_loader.c:426 */
    uint32_t vocab = vocab_kv;
    for (uint64_t i = 0; i < n_t; i++) {
        char name[256];
        size_t nl = ti[i].nl < 255 ? ti[i].nl : 255;
        memcpy(name, ti[i].name, nl); name[nl] = 0;
        tref_t tr = {map + data_off + ti[i].off, ti[i].type, ti[i].d1, ti[i].d0};
        if (!strcmp(name, "token_embd.weight")) {
            m->embd = tr;
            if (vocab == 0 && ti[i].nd == 2) vocab = (uint32_t)ti[i].d1;  /* :410-412 */
        } else if (!strcmp(name, "output_norm.weight")) m->out_norm = tr;
        else if (!strcmp(name, "output.weight")) m->out = tr;
        else if (!strncmp(name, "blk.", 4)) {
            int l = atoi(name + 4);
            const char *suf = strchr(name + 4, '.');
            if (l < 0 || l >= m->L || !suf) continue;
            layer_t *ly = &m->layers[l];
            if (!strcmp(suf, ".attn_norm.weight")) ly->attn_norm = tr;
            else if (!strcmp(suf, ".attn_q.weight")) ly->wq = tr;
            else if (!strcmp(suf, ".attn_k.weight")) ly->wk = tr;
            else if (!strcmp(suf, ".attn_v.weight")) ly->wv = tr;
            else if (!strcmp(suf, ".attn_output.weight")) ly->wo = tr;
            else if (!strcmp(suf, ".ffn_norm.weight")) ly->ffn_norm = tr;
            else if (!strcmp(suf, ".ffn_gate.weight")) ly->wgate = tr;
            else if (!strcmp(suf, ".ffn_up.weight")) ly->wup = tr;
            else if (!strcmp(suf, ".ffn_down.weight")) ly->wdown = tr;
        }
    }
    free(ti);
    if (!m->embd.data || !m->L || !m->layers[0].wq.data) goto fail;
    /* head_dim / rope_dim / vocab clamp: SS/src/core/layer_scheduler.c:161-197 */
    m->hd = key_len ? (int32_t)key_len : (int32_t)(m->layers[0].wq.rows / (uint64_t)m->nh);
    m->rope_dim = rope_dim ? (int32_t)rope_dim : m->hd;
    m->vocab = (int32_t)vocab;
    if (m->out.data && (int32_t)m->out.rows < m->vocab) m->vocab = (int32_t)m->out.rows;
    if ((int32_t)m->embd.rows < m->vocab) m->vocab = (int32_t)m->embd.rows;
    /* context: engine.c:99-106 then the scheduler's 512 cap (layer_scheduler.c:199-202) */
    uint32_t ctx = context_size ? context_size : ctx_len;
    if (ctx == 0 || ctx > 8192) ctx = 8192;
    m->max_seq = (int32_t)ctx;
    if (cap512 && m->max_seq > 512) m->max_seq = 512;
    m->kvd = m->nkv * m->hd;
    size_t nv = (size_t)m->L * m->max_seq;
    m->kc = (int8_t *)calloc(nv * m->kvd, 1);
    m->vc = (int8_t *)calloc(nv * m->kvd, 1);
    m->ks = (float *)calloc(nv, 4);
    m->vs = (float *)calloc(nv, 4);
    m->hidden = (float *)calloc((size_t)m->d, 4);
    m->residual = (float *)calloc((size_t)m->d, 4);
    m->attn_out = (float *)calloc((size_t)(m->d > m->nh * m->hd ? m->d : m->nh * m->hd), 4);
    m->ffn_buf = (float *)calloc((size_t)m->ff, 4);
    m->ffn_gate = (float *)calloc((size_t)m->ff, 4);
    m->q = (float *)calloc((size_t)(m->nh * m->hd), 4);
    m->k = (float *)calloc((size_t)m->kvd, 4);
    m->v = (float *)calloc((size_t)m->kvd, 4);
    m->logits = (float *)calloc((size_t)m->vocab, 4);
    return m;
fail:
    sso_free(m);
    return NULL;
}

void sso_free(sso_model_t *m) {
    if (!m) return;
    if (m->map) munmap(m->map, m->map_size);
    free(m->layers); free(m->kc); free(m->vc); free(m->ks); free(m->vs);
    free(m->hidden); free(m->residual); free(m->attn_out); free(m->ffn_buf);
    free(m->ffn_gate); free(m->q); free(m->k); free(m->v); free(m->logits);
    free(m);
}

void sso_dims(const sso_model_t *m, int32_t *dims) {
    dims[0] = m->vocab; dims[1] = m->d; dims[2] = m->L; dims[3] = m->nh;
    dims[4] = m->nkv; dims[5] = m->hd; dims[6] = m->ff; dims[7] = m->max_seq;
}

/* SS/src/core/layer_scheduler.c:917-936 */
void sso_reset(sso_model_t *m) {
    size_t nv = (size_t)m->L * m->max_seq;
    memset(m->kc, 0, nv * m->kvd);
    memset(m->vc, 0, nv * m->kvd);
    memset(m->ks, 0, nv * 4);
    memset(m->vs, 0, nv * 4);
    memset(m->hidden, 0, (size_t)m->d * 4);
}

void sso_kv_row(const sso_model_t *m, int32_t layer, int32_t pos, int8_t *k, int8_t *v,
                float *ks, float *vs) {
    size_t vi = (size_t)layer * m->max_seq + pos;
    memcpy(k, m->kc + vi * m->kvd, (size_t)m->kvd);
    memcpy(v, m->vc + vi * m->kvd, (size_t)m->kvd);
    *ks = m->ks[vi];
    *vs = m->vs[vi];
}

static void matvec(const sso_model_t *m, float *out, const tref_t *w, const float *x,
                   int32_t rows, int32_t cols) {
    matvec_ordered(out, w->data, x, rows, cols, w->type, m->dot_order);
}

/* SS/src/core/layer_scheduler.c:291-567 (process_layer, llama branch). */
static void process_layer(sso_model_t *m, int32_t l, int32_t pos) {
    layer_t *ly = &m->layers[l];
    int32_t d = m->d, hd = m->hd, nh = m->nh, nkv = m->nkv, kvd = m->kvd;
    memcpy(m->residual, m->hidden, (size_t)d * 4);                       /* :325 */
    sso_rmsnorm(m->hidden, m->residual, (const float *)ly->attn_norm.data, d, m->eps);
    matvec(m, m->q, &ly->wq, m->hidden, nh * hd, d);                        /* :356-358 */
    matvec(m, m->k, &ly->wk, m->hidden, kvd, d);
    matvec(m, m->v, &ly->wv, m->hidden, kvd, d);
    sso_rope(m->q, m->k, nh, nkv, hd, m->rope_dim, pos, m->theta);       /* :405 */
    size_t vi = (size_t)l * m->max_seq + pos;                            /* :410-413 */
    sso_kv_encode(m->k, m->kc + vi * kvd, &m->ks[vi], kvd);
    sso_kv_encode(m->v, m->vc + vi * kvd, &m->vs[vi], kvd);
    int32_t seq_len = pos + 1, hpk = nh / nkv;                           /* :416-421 */
    memset(m->attn_out, 0, (size_t)d * 4);
    float scale = 1.0f / sqrtf((float)hd);
    #pragma omp parallel for schedule(static)
    for (int32_t h = 0; h < nh; h++) {                                   /* :424-468 */
        const float *q = m->q + h * hd;
        int32_t kh = h / hpk;
        float *scores = (float *)malloc((size_t)seq_len * 4);
        float *tmp = (float *)malloc((size_t)hd * 4);
        for (int32_t t = 0; t < seq_len; t++) {
            size_t ti = (size_t)l * m->max_seq + t;
            const int8_t *kq = m->kc + ti * kvd + kh * hd;
            float ksc = m->ks[ti];
            for (int32_t i = 0; i < hd; i++) tmp[i] = (float)kq[i] * ksc;
            scores[t] = dot_seq(q, tmp, hd) * scale;
        }
        sso_softmax(scores, seq_len);
        float *dst = m->attn_out + h * hd;
        for (int32_t i = 0; i < hd; i++) dst[i] = 0.0f;
        for (int32_t t = 0; t < seq_len; t++) {
            float w = scores[t];
            size_t ti = (size_t)l * m->max_seq + t;
            const int8_t *vq = m->vc + ti * kvd + kh * hd;
            float vsc = m->vs[ti];
            for (int32_t i = 0; i < hd; i++) tmp[i] = (float)vq[i] * vsc;
            for (int32_t i = 0; i < hd; i++) dst[i] += w * tmp[i];       /* saxpy */
        }
        free(scores);
        free(tmp);
    }
    matvec(m, m->hidden, &ly->wo, m->attn_out, d, nh * hd);                 /* :471-472 */
    for (int32_t i = 0; i < d; i++) m->hidden[i] = m->hidden[i] + m->residual[i];  /* :484 */
    memcpy(m->residual, m->hidden, (size_t)d * 4);                       /* :490 */
    sso_rmsnorm(m->hidden, m->residual, (const float *)ly->ffn_norm.data, d, m->eps);
    matvec(m, m->ffn_gate, &ly->wgate, m->hidden, m->ff, d);                /* :512-513 */
    matvec(m, m->ffn_buf, &ly->wup, m->hidden, m->ff, d);
    for (int32_t i = 0; i < m->ff; i++) {                                /* :533-549 */
        float g = m->ffn_gate[i];
        m->ffn_buf[i] *= g / (1.0f + expf(-g));
    }
    matvec(m, m->hidden, &ly->wdown, m->ffn_buf, d, m->ff);                 /* :553-554 */
    for (int32_t i = 0; i < d; i++) m->hidden[i] = m->hidden[i] + m->residual[i];  /* :566 */
}

static void embed_row(sso_model_t *m, int32_t token, float *dst) {   /* :584-595 */
    size_t rb = (size_t)(m->d / block_size(m->embd.type)) * type_size(m->embd.type);
    sso_dequantize(m->embd.data + (size_t)token * rb, dst, m->d, m->embd.type);
}

static void head(sso_model_t *m, float *logits_out) {                   /* :634-662 */
    if (m->out_norm.data)
        sso_rmsnorm(m->hidden, m->hidden, (const float *)m->out_norm.data, m->d, m->eps);
    const tref_t *lm = m->out.data ? &m->out : &m->embd;
    matvec(m, m->logits, lm, m->hidden, m->vocab, m->d);
    if (logits_out) memcpy(logits_out, m->logits, (size_t)m->vocab * 4);
}

/* SS/src/core/layer_scheduler.c:571-679 */
int sso_forward(sso_model_t *m, int32_t token, int32_t pos, float *logits_out) {
    if (token < 0 || token >= (int32_t)m->embd.rows || pos < 0 || pos >= m->max_seq) return -1;
    embed_row(m, token, m->hidden);
    for (int32_t l = 0; l < m->L; l++) process_layer(m, l, pos);
    head(m, logits_out);
    return 0;
}

/* SS/src/core/layer_scheduler.c:681-803: layer-major over the prompt, final
 * norm and lm_head for the last token only. */
int sso_prefill(sso_model_t *m, const int32_t *tokens, int32_t n, int32_t start_pos,
                float *logits_out) {
    if (n <= 0 || start_pos < 0 || start_pos + n > m->max_seq) return -1;
    float *bh = (float *)malloc((size_t)n * m->d * 4);
    for (int32_t i = 0; i < n; i++) {
        if (tokens[i] < 0 || tokens[i] >= (int32_t)m->embd.rows) { free(bh); return -1; }
        embed_row(m, tokens[i], bh + (size_t)i * m->d);
    }
    for (int32_t l = 0; l < m->L; l++)
        for (int32_t i = 0; i < n; i++) {
            memcpy(m->hidden, bh + (size_t)i * m->d, (size_t)m->d * 4);
            process_layer(m, l, start_pos + i);
            memcpy(bh + (size_t)i * m->d, m->hidden, (size_t)m->d * 4);
        }
    memcpy(m->hidden, bh + (size_t)(n - 1) * m->d, (size_t)m->d * 4);
    free(bh);
    head(m, logits_out);
    return 0;
}

/* SS/src/core/layer_scheduler.c:805-915: positions from 0, final norm on every
 * token, mean pool, L2 normalise. */
int sso_embed(sso_model_t *m, const int32_t *tokens, int32_t n, float *out) {
    if (n <= 0 || n > m->max_seq) return -1;
    int32_t d = m->d;
    float *bh = (float *)malloc((size_t)n * d * 4);
    for (int32_t i = 0; i < n; i++) embed_row(m, tokens[i], bh + (size_t)i * d);
    for (int32_t l = 0; l < m->L; l++)
        for (int32_t i = 0; i < n; i++) {
            memcpy(m->hidden, bh + (size_t)i * d, (size_t)d * 4);
            process_layer(m, l, i);
            memcpy(bh + (size_t)i * d, m->hidden, (size_t)d * 4);
        }
    if (m->out_norm.data)
        for (int32_t i = 0; i < n; i++)
            sso_rmsnorm(bh + (size_t)i * d, bh + (size_t)i * d, (const float *)m->out_norm.data,
                        d, m->eps);
    for (int32_t j = 0; j < d; j++) out[j] = 0.0f;
    for (int32_t i = 0; i < n; i++)
        for (int32_t j = 0; j < d; j++) out[j] += bh[(size_t)i * d + j];
    float inv = 1.0f / (float)n, l2 = 0.0f;
    for (int32_t j = 0; j < d; j++) { out[j] *= inv; l2 += out[j] * out[j]; }
    float sc = 1.0f / (sqrtf(l2) + 1e-12f);
    for (int32_t j = 0; j < d; j++) out[j] *= sc;
    free(bh);
    return 0;
}

/* ---------------------------------------------------------------- sampling */

/* e^x rounded to float from a double-precision evaluation (the sampler's
 * exponential on the GPU, written out the same way here so both round
 * identically): k = rint(x log2 e), r = x - k ln2 in two fma steps (ln2 split
 * into a 33-bit head, so k * head is exact, and a tail), e^r by its Taylor
 * series to degree 13 in Horner form (truncation below 5e-18 for |r| <= ln2/2),
 * times 2^k built from the exponent bits, then one float rounding.  Every step
 * is an IEEE basic operation or fma, so any machine gives the same bits. */
static const double kExpInvFact[14] = {
    0x1.0000000000000p+0,  0x1.0000000000000p+0,  0x1.0000000000000p-1,  0x1.5555555555555p-3,
    0x1.5555555555555p-5,  0x1.1111111111111p-7,  0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13,
    0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22, 0x1.ae64567f544e4p-26,
    0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33};

float sso_exp_dd(float xf) {
    if (xf != xf) return xf;
    if (xf < -200.0f) return 0.0f;
    if (xf > 200.0f) return INFINITY;
    const double x = (double)xf;
    const double k = rint(x * 0x1.71547652b82fep+0);
    double r = fma(-k, 0x1.62e42ff000000p-1, x);
    r = fma(-k, -0x1.718432a1b0e26p-35, r);
    double p = kExpInvFact[13];
    for (int i = 12; i >= 0; i--) p = fma(p, r, kExpInvFact[i]);
    const uint64_t bits = (uint64_t)((int64_t)k + 1023) << 52;
    double s;
    memcpy(&s, &bits, 8);
    return (float)(p * s);
}

void sso_exp_dd_array(const float *x, float *out, int32_t n) {
    for (int32_t i = 0; i < n; i++) out[i] = sso_exp_dd(x[i]);
}

/* SS/src/core/tensor.c:331-342: xorshift64, and the top 53 bits as a float in
 * [0, 1] (the uint64 -> float conversion rounds to nearest). */
static uint64_t sso_xorshift64(uint64_t *s) {
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return x;
}
float sso_rand_float(uint64_t *state) {
    return (float)(sso_xorshift64(state) >> 11) / (float)(1ULL << 53);
}

typedef struct { int32_t id; float p; } sso_cand_t;

/* Descending by probability, NaN read as 0 (tensor.c:350-361). */
static int sso_cand_cmp(const void *a, const void *b) {
    float pa = ((const sso_cand_t *)a)->p, pb = ((const sso_cand_t *)b)->p;
    if (pa != pa) pa = 0.0f;
    if (pb != pb) pb = 0.0f;
    return pa > pb ? -1 : pa < pb ? 1 : 0;
}

/* SS/src/core/tensor.c:363-451 (ss_sample).  temperature <= 0: the greedy
 * argmax.  Otherwise: NaN logits -> -FLT_MAX, logits / temperature, softmax
 * (tensor.c:154-173, one sequential fp32 sum), the candidates sorted by
 * probability (descending), top-k: probabilities below the k-th largest
 * zeroed; top-p: walk the sorted candidates adding the (top-k filtered)
 * positive probabilities in order until the sum reaches top_p, the probability
 * there is the cutoff and those below it are zeroed; renormalise by one more
 * sequential sum when it is positive; draw r and return the first index whose
 * running sum exceeds r (the last index when none does).  exp_mode 0 uses
 * libm's expf as the reference does, 1 sso_exp_dd (the GPU sampler's
 * exponential).  Ties in the sort can be ordered either way: equal
 * probabilities add the same values to the running sum in any order. */
int32_t sso_sample(const float *logits, int32_t n, float temperature, float top_p, int32_t top_k,
                   uint64_t *rng_state, int exp_mode) {
    if (temperature <= 0.0f) return sso_argmax(logits, n);
    float *pr = (float *)malloc((size_t)n * sizeof(float));
    sso_cand_t *cand = (sso_cand_t *)malloc((size_t)n * sizeof(sso_cand_t));
    for (int32_t i = 0; i < n; i++) pr[i] = logits[i] != logits[i] ? -FLT_MAX : logits[i] / temperature;
    float mx = -FLT_MAX;
    for (int32_t i = 0; i < n; i++) if (pr[i] > mx) mx = pr[i];
    float sum = 0.0f;
    for (int32_t i = 0; i < n; i++) {
        pr[i] = exp_mode ? sso_exp_dd(pr[i] - mx) : expf(pr[i] - mx);
        sum += pr[i];
    }
    const float inv = 1.0f / sum;
    for (int32_t i = 0; i < n; i++) pr[i] *= inv;
    for (int32_t i = 0; i < n; i++) {
        cand[i].id = i;
        cand[i].p = pr[i] != pr[i] ? 0.0f : pr[i];
    }
    qsort(cand, (size_t)n, sizeof(sso_cand_t), sso_cand_cmp);
    if (top_k > 0 && top_k < n) {
        const float thr = cand[top_k - 1].p;
        for (int32_t i = 0; i < n; i++) if (pr[i] < thr) pr[i] = 0.0f;
    }
    if (top_p > 0.0f && top_p < 1.0f) {
        float acc = 0.0f, cutoff = 0.0f;
        for (int32_t i = 0; i < n; i++) {
            const float pv = pr[cand[i].id];
            if (pv > 0.0f) acc += pv;
            if (acc >= top_p) { cutoff = pv; break; }
        }
        for (int32_t i = 0; i < n; i++) if (pr[i] < cutoff) pr[i] = 0.0f;
    }
    free(cand);
    float tot = 0.0f;
    for (int32_t i = 0; i < n; i++) tot += pr[i];
    if (tot > 0.0f) {
        const float rinv = 1.0f / tot;
        for (int32_t i = 0; i < n; i++) pr[i] *= rinv;
    }
    const float r = sso_rand_float(rng_state);
    float cdf = 0.0f;
    int32_t pick = n - 1;
    for (int32_t i = 0; i < n; i++) {
        cdf += pr[i];
        if (r < cdf) { pick = i; break; }
    }
    free(pr);
    return pick;
}
