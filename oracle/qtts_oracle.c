/*
 * qtts_oracle.c -- CPU restatement of the per-frame language-model path of
 * mormot2-qwen-tts (Qwen3-TTS talker + code predictor).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: the pytest suite,
 * __graft_entry__.smoke() and the cpu_baseline leg of bench.py load it to
 * compare against the CUDA library.  The product path (libqtts.so) never links
 * or calls it.
 *
 * What it restates (reference = flydev-fr/mormot2-qwen-tts):
 *  - TQwenLm.Forward (src/tts/mormot.ai.tts.qwen.lm.pas:391-408): append `rows`
 *    embedding rows at positions Length..Length+rows-1, return the normed
 *    state of the last row and the logits of head `aOutput` on that row.
 *  - the decoder stack behind ForwardEmbeds (mormot2-ai, absent from the
 *    reference checkout; semantics from the dataset note of
 *    tests/data/infer-ref/qwen3-tts-lm/manifest.json and
 *    tools/tts/make_lm_reference.py:160-168): plain Qwen3 layers, RMSNorm,
 *    per-head q_norm/k_norm, rotate_half RoPE, causal GQA attention, SwiGLU,
 *    no bias, final RMSNorm.
 *  - TQwenLmHeads Q8_0 conversion (lm.pas:244-275) = ggml
 *    quantize_row_q8_0_ref: d = amax/127 stored as fp16, q = roundf(x * (1/d)).
 *  - TQwenTalker.ChooseCode0 (src/tts/mormot.ai.tts.qwen.talker.pas:595-630),
 *    ChooseCode greedy (632-638) and NextFrame (640-681).
 *  - the test's ArgMax (tests/test.tts.qwen.lm.pas:109-117): first maximum.
 *
 * Q8_0 `Linear` activation mode: the mormot2-ai kernel source is absent, so
 * two modes exist.  ORA_ACT_F32 (default): the weights are dequantised per
 * block against float32 activations, y = sum_b d_b * sum_j q_j x_j.
 * ORA_ACT_Q8_0: the activations are quantised to Q8_0 per block as ggml's
 * vec_dot_q8_0_q8_0 does, y = sum_b (d_w,b * d_x,b) * sum_j q_w q_x.
 *
 * Arithmetic: float32 everywhere, AVX2 + FMA dot products, OpenMP over
 * output rows.  Build with -ffp-contract=off so that only the explicit FMAs
 * below are fused.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <immintrin.h>

#define ORA_F32 0
#define ORA_Q8_0 1
#define ORA_ACT_F32 0
#define ORA_ACT_Q8_0 1

static int g_act_mode = ORA_ACT_F32;

void ora_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int ora_get_threads(void) { return omp_get_max_threads(); }
void ora_set_act_mode(int mode) { g_act_mode = mode; }

/* ---------------------------------------------------------------- fp16 */

/* float -> IEEE half, round to nearest even (ggml GGML_FP32_TO_FP16 on F16C
 * hardware is _cvtss_sh(x, 0), the same rounding) */
static uint16_t f32_to_f16(float f) {
    __m128 v = _mm_set_ss(f);
    __m128i h = _mm_cvtps_ph(v, _MM_FROUND_TO_NEAREST_INT);
    return (uint16_t)_mm_extract_epi16(h, 0);
}

static float f16_to_f32(uint16_t h) {
    __m128i v = _mm_cvtsi32_si128(h);
    return _mm_cvtss_f32(_mm_cvtph_ps(v));
}

float ora_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t ora_f32_to_f16(float f) { return f32_to_f16(f); }

/* ---------------------------------------------------------------- Q8_0 */

/* one ggml block_q8_0: fp16 scale then 32 int8, 34 bytes */
#define QK 32
#define QBLOCK 34

/* ggml quantize_row_q8_0_ref, restated: amax over the block, d = amax/127,
 * id = d ? 1/d : 0, q = roundf(x*id) (round half away from zero).
 * Used by TQwenLmHeads.MatrixRows (lm.pas:259-267). */
void ora_quantize_q8_0(const float *x, int64_t n, uint8_t *out) {
    int64_t nb = n / QK;
    for (int64_t i = 0; i < nb; i++) {
        const float *b = x + i * QK;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) {
            float a = fabsf(b[j]);
            amax = amax > a ? amax : a;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = f32_to_f16(d);
        uint8_t *o = out + i * QBLOCK;
        memcpy(o, &dh, 2);
        for (int j = 0; j < QK; j++) {
            float v = b[j] * id;
            o[2 + j] = (uint8_t)(int8_t)roundf(v);
        }
    }
}

void ora_dequantize_q8_0(const uint8_t *in, int64_t n, float *x) {
    int64_t nb = n / QK;
    for (int64_t i = 0; i < nb; i++) {
        uint16_t dh;
        memcpy(&dh, in + i * QBLOCK, 2);
        float d = f16_to_f32(dh);
        const int8_t *q = (const int8_t *)(in + i * QBLOCK + 2);
        for (int j = 0; j < QK; j++) x[i * QK + j] = (float)q[j] * d;
    }
}

/* crc32c (Castagnoli), as mORMot's crc32c used by TQwenLmHeads.Digest
 * (lm.pas:310-317); reflected polynomial 0x82F63B78 */
uint32_t ora_crc32c(uint32_t crc, const void *data, size_t n) {
    static uint32_t table[256];
    static int init = 0;
    if (!init) {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = c & 1 ? (c >> 1) ^ 0x82F63B78u : c >> 1;
            table[i] = c;
        }
        init = 1;
    }
    const uint8_t *p = (const uint8_t *)data;
    crc = ~crc;
    for (size_t i = 0; i < n; i++) crc = table[(crc ^ p[i]) & 0xff] ^ (crc >> 8);
    return ~crc;
}

/* ---------------------------------------------------------------- weights */

typedef struct {
    int dtype;      /* ORA_F32 or ORA_Q8_0 */
    int rows, cols; /* [rows][cols], cols % 32 == 0 for Q8_0 */
    float *f;       /* f32 rows */
    uint8_t *q;     /* ggml blocks, row-major */
} ora_weight;

static void weight_init(ora_weight *w, const float *src, int rows, int cols, int dtype) {
    w->dtype = dtype;
    w->rows = rows;
    w->cols = cols;
    w->f = NULL;
    w->q = NULL;
    size_t n = (size_t)rows * cols;
    if (dtype == ORA_F32) {
        w->f = (float *)malloc(n * sizeof(float));
        memcpy(w->f, src, n * sizeof(float));
    } else {
        w->q = (uint8_t *)malloc(n / QK * QBLOCK);
#pragma omp parallel for schedule(static)
        for (int r = 0; r < rows; r++)
            ora_quantize_q8_0(src + (size_t)r * cols, cols, w->q + (size_t)r * (cols / QK) * QBLOCK);
    }
}

static void weight_free(ora_weight *w) {
    free(w->f);
    free(w->q);
    w->f = NULL;
    w->q = NULL;
}

static inline float hsum256(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    lo = _mm_add_ps(lo, hi);
    lo = _mm_add_ps(lo, _mm_movehl_ps(lo, lo));
    lo = _mm_add_ss(lo, _mm_movehdup_ps(lo));
    return _mm_cvtss_f32(lo);
}

static float dot_f32(const float *w, const float *x, int n) {
    __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(w + i), _mm256_loadu_ps(x + i), a0);
        a1 = _mm256_fmadd_ps(_mm256_loadu_ps(w + i + 8), _mm256_loadu_ps(x + i + 8), a1);
    }
    float s = hsum256(_mm256_add_ps(a0, a1));
    for (; i < n; i++) s += w[i] * x[i];
    return s;
}

/* Q8_0 row . f32 x: sum over blocks of d_b * (q_b . x_b) */
static float dot_q8_f32(const uint8_t *row, const float *x, int n) {
    __m256 acc = _mm256_setzero_ps();
    int nb = n / QK;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = row + (size_t)b * QBLOCK;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        __m256 d = _mm256_set1_ps(f16_to_f32(dh));
        __m128i q16a = _mm_loadu_si128((const __m128i *)(blk + 2));
        __m128i q16b = _mm_loadu_si128((const __m128i *)(blk + 18));
        __m256 q0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q16a));
        __m256 q1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(q16a, 8)));
        __m256 q2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q16b));
        __m256 q3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(q16b, 8)));
        const float *xb = x + b * QK;
        __m256 p = _mm256_mul_ps(q0, _mm256_loadu_ps(xb));
        p = _mm256_fmadd_ps(q1, _mm256_loadu_ps(xb + 8), p);
        p = _mm256_fmadd_ps(q2, _mm256_loadu_ps(xb + 16), p);
        p = _mm256_fmadd_ps(q3, _mm256_loadu_ps(xb + 24), p);
        acc = _mm256_fmadd_ps(d, p, acc);
    }
    return hsum256(acc);
}

/* Q8_0 row . Q8_0 x (ggml vec_dot_q8_0_q8_0): integer block dots */
static float dot_q8_q8(const uint8_t *row, const uint8_t *xq, int n) {
    int nb = n / QK;
    float s = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *w = row + (size_t)b * QBLOCK, *v = xq + (size_t)b * QBLOCK;
        uint16_t dw, dx;
        memcpy(&dw, w, 2);
        memcpy(&dx, v, 2);
        int sumi = 0;
        const int8_t *qw = (const int8_t *)(w + 2), *qx = (const int8_t *)(v + 2);
        for (int j = 0; j < QK; j++) sumi += (int)qw[j] * (int)qx[j];
        s += (float)sumi * (f16_to_f32(dw) * f16_to_f32(dx));
    }
    return s;
}

/* y[rows][w.rows] = x[rows][w.cols] . w^T  (TInferBackend.Linear, no bias) */
static void linear(const float *x, int rows, const ora_weight *w, float *y) {
    int n = w->cols, m = w->rows;
    uint8_t *xq = NULL;
    if (w->dtype == ORA_Q8_0 && g_act_mode == ORA_ACT_Q8_0) {
        xq = (uint8_t *)malloc((size_t)rows * (n / QK) * QBLOCK);
        for (int r = 0; r < rows; r++)
            ora_quantize_q8_0(x + (size_t)r * n, n, xq + (size_t)r * (n / QK) * QBLOCK);
    }
#pragma omp parallel for schedule(static)
    for (int o = 0; o < m; o++) {
        for (int r = 0; r < rows; r++) {
            float v;
            if (w->dtype == ORA_F32)
                v = dot_f32(w->f + (size_t)o * n, x + (size_t)r * n, n);
            else if (xq)
                v = dot_q8_q8(w->q + (size_t)o * (n / QK) * QBLOCK, xq + (size_t)r * (n / QK) * QBLOCK, n);
            else
                v = dot_q8_f32(w->q + (size_t)o * (n / QK) * QBLOCK, x + (size_t)r * n, n);
            y[(size_t)r * m + o] = v;
        }
    }
    free(xq);
}

/* ---------------------------------------------------------------- stack */

typedef struct {
    int layers, hidden, heads, kv_heads, head_dim, inter;
    float eps, theta;
    int dtype;
} ora_config;

/* one layer of a Qwen3 stack, float32 host rows [out][in] */
typedef struct {
    const float *in_norm, *post_norm, *q_norm, *k_norm;
    const float *wq, *wk, *wv, *wo, *wg, *wu, *wd;
} ora_layer_src;

typedef struct {
    float *in_norm, *post_norm, *q_norm, *k_norm;
    ora_weight wq, wk, wv, wo, wg, wu, wd;
} ora_layer;

typedef struct {
    ora_config c;
    ora_layer *layer;
    float *final_norm;
} ora_stack;

static float *dupf(const float *p, size_t n) {
    float *r = (float *)malloc(n * sizeof(float));
    memcpy(r, p, n * sizeof(float));
    return r;
}

/* TQwen3Model.CreateStack (lm.pas:174-179): the layers of one stack, widened
 * to float32 or quantised to Q8_0 */
ora_stack *ora_stack_create(const ora_config *c, const ora_layer_src *src, const float *final_norm) {
    ora_stack *s = (ora_stack *)calloc(1, sizeof(ora_stack));
    s->c = *c;
    int H = c->hidden, q = c->heads * c->head_dim, kv = c->kv_heads * c->head_dim, I = c->inter;
    s->layer = (ora_layer *)calloc(c->layers, sizeof(ora_layer));
    for (int l = 0; l < c->layers; l++) {
        const ora_layer_src *a = src + l;
        ora_layer *L = s->layer + l;
        L->in_norm = dupf(a->in_norm, H);
        L->post_norm = dupf(a->post_norm, H);
        L->q_norm = dupf(a->q_norm, c->head_dim);
        L->k_norm = dupf(a->k_norm, c->head_dim);
        weight_init(&L->wq, a->wq, q, H, c->dtype);
        weight_init(&L->wk, a->wk, kv, H, c->dtype);
        weight_init(&L->wv, a->wv, kv, H, c->dtype);
        weight_init(&L->wo, a->wo, H, q, c->dtype);
        weight_init(&L->wg, a->wg, I, H, c->dtype);
        weight_init(&L->wu, a->wu, I, H, c->dtype);
        weight_init(&L->wd, a->wd, H, I, c->dtype);
    }
    s->final_norm = dupf(final_norm, H);
    return s;
}

void ora_stack_free(ora_stack *s) {
    if (!s) return;
    for (int l = 0; l < s->c.layers; l++) {
        ora_layer *L = s->layer + l;
        free(L->in_norm); free(L->post_norm); free(L->q_norm); free(L->k_norm);
        weight_free(&L->wq); weight_free(&L->wk); weight_free(&L->wv); weight_free(&L->wo);
        weight_free(&L->wg); weight_free(&L->wu); weight_free(&L->wd);
    }
    free(s->layer);
    free(s->final_norm);
    free(s);
}

/* ---------------------------------------------------------------- heads */

/* TQwenLmHeads (lm.pas:64-100): [rows][hidden] matrices in f32 or Q8_0 */
typedef struct {
    int hidden, dtype, count;
    ora_weight *w;
} ora_heads;

ora_heads *ora_heads_create(int hidden, int dtype) {
    ora_heads *h = (ora_heads *)calloc(1, sizeof(ora_heads));
    h->hidden = hidden;
    h->dtype = dtype;
    return h;
}

int ora_heads_add(ora_heads *h, const float *src, int rows) {
    h->w = (ora_weight *)realloc(h->w, (h->count + 1) * sizeof(ora_weight));
    weight_init(h->w + h->count, src, rows, h->hidden, h->dtype);
    return h->count++;
}

/* TQwenLmHeads.Digest (lm.pas:310-317): crc32c of the stored bytes in load
 * order - ggml blocks for Q8_0, float32 rows otherwise */
uint32_t ora_heads_digest(const ora_heads *h) {
    uint32_t crc = 0;
    for (int i = 0; i < h->count; i++) {
        const ora_weight *w = h->w + i;
        if (w->dtype == ORA_F32)
            crc = ora_crc32c(crc, w->f, (size_t)w->rows * w->cols * 4);
        else
            crc = ora_crc32c(crc, w->q, (size_t)w->rows * (w->cols / QK) * QBLOCK);
    }
    return crc;
}

const uint8_t *ora_heads_bytes(const ora_heads *h, int index) {
    return h->w[index].dtype == ORA_F32 ? (const uint8_t *)h->w[index].f : h->w[index].q;
}

void ora_heads_free(ora_heads *h) {
    if (!h) return;
    for (int i = 0; i < h->count; i++) weight_free(h->w + i);
    free(h->w);
    free(h);
}

/* ---------------------------------------------------------------- lm */

/* TQwenLm (lm.pas:102-143): a stack, its KV cache (float32, as the
 * reference's default, talker.pas:188-190) and its length */
typedef struct {
    ora_stack *s;
    int max_pos, len;
    float *k, *v;          /* [layers][max_pos][kv_heads][head_dim] */
    float *rope_cos, *rope_sin; /* [max_pos][head_dim/2] */
    int kv_f16;            /* the cache holds half floats (TQwenLm aKvF16, lm.pas:122-123, 352) */
} ora_lm;

/* RoPE tables as transformers computes them in float32: inv_freq_i =
 * 1/theta^(2i/d), angle = pos * inv_freq_i (one float32 product), cos/sin of
 * that float32 angle */
void ora_rope_table(int max_pos, int head_dim, float theta, float *cos_out, float *sin_out) {
    int half = head_dim / 2;
    for (int i = 0; i < half; i++) {
        float e = (float)(2 * i) / (float)head_dim;
        float inv = 1.0f / powf(theta, e);
        for (int p = 0; p < max_pos; p++) {
            float a = (float)p * inv;
            cos_out[(size_t)p * half + i] = cosf(a);
            sin_out[(size_t)p * half + i] = sinf(a);
        }
    }
}

ora_lm *ora_lm_create(ora_stack *s, int max_pos) {
    ora_lm *m = (ora_lm *)calloc(1, sizeof(ora_lm));
    m->s = s;
    m->max_pos = max_pos;
    size_t n = (size_t)s->c.layers * max_pos * s->c.kv_heads * s->c.head_dim;
    m->k = (float *)calloc(n, sizeof(float));
    m->v = (float *)calloc(n, sizeof(float));
    int half = s->c.head_dim / 2;
    m->rope_cos = (float *)malloc((size_t)max_pos * half * sizeof(float));
    m->rope_sin = (float *)malloc((size_t)max_pos * half * sizeof(float));
    ora_rope_table(max_pos, s->c.head_dim, s->c.theta, m->rope_cos, m->rope_sin);
    return m;
}

void ora_lm_free(ora_lm *m) {
    if (!m) return;
    free(m->k); free(m->v); free(m->rope_cos); free(m->rope_sin);
    free(m);
}

/* TQwenLm.Reset (lm.pas:374-378) */
void ora_lm_reset(ora_lm *m) { m->len = 0; }
/* TQwenLm.Create's aKvF16 (lm.pas:122-123, applied at 352): K and V are kept
 * in half floats (round to nearest even), so every read of a cached position,
 * the current one included, sees the rounded value */
void ora_lm_set_kv_f16(ora_lm *m, int on) { m->kv_f16 = on; }
int ora_lm_length(const ora_lm *m) { return m->len; }

/* Qwen3RMSNorm: x * (1/sqrt(mean(x^2) + eps)), then * weight */
static void rmsnorm(const float *x, const float *w, int n, float eps, float *y) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) y[i] = w[i] * (x[i] * inv);
}

/* rotate_half RoPE at position p: y = x*cos + rotate_half(x)*sin */
static void rope(float *x, int d, const float *cs, const float *sn) {
    int half = d / 2;
    float tmp[512];
    for (int i = 0; i < half; i++) {
        float a = x[i], b = x[i + half];
        tmp[i] = a * cs[i] - b * sn[i];
        tmp[i + half] = b * cs[i] + a * sn[i];
    }
    memcpy(x, tmp, d * sizeof(float));
}

static inline float silu(float v) { return v / (1.0f + expf(-v)); }

/* one pass of the stack over `rows` new rows; x [rows][H] is updated in place
 * to the output of the last layer; states (optional) receives the output of
 * every layer [layers][rows][H] */
static int stack_forward(ora_lm *m, float *x, int rows, float *states) {
    ora_stack *s = m->s;
    const ora_config *c = &s->c;
    int H = c->hidden, D = c->head_dim, Hq = c->heads, Hkv = c->kv_heads, I = c->inter;
    int Q = Hq * D, KV = Hkv * D, half = D / 2, grp = Hq / Hkv;
    int L0 = m->len;
    if (L0 + rows > m->max_pos) return -1;
    float *h = (float *)malloc((size_t)rows * H * sizeof(float));
    float *q = (float *)malloc((size_t)rows * Q * sizeof(float));
    float *k = (float *)malloc((size_t)rows * KV * sizeof(float));
    float *v = (float *)malloc((size_t)rows * KV * sizeof(float));
    float *att = (float *)malloc((size_t)rows * Q * sizeof(float));
    float *o = (float *)malloc((size_t)rows * H * sizeof(float));
    float *g = (float *)malloc((size_t)rows * I * sizeof(float));
    float *u = (float *)malloc((size_t)rows * I * sizeof(float));
    float scale = 1.0f / sqrtf((float)D);
    for (int l = 0; l < c->layers; l++) {
        ora_layer *Ly = s->layer + l;
        for (int r = 0; r < rows; r++) rmsnorm(x + (size_t)r * H, Ly->in_norm, H, c->eps, h + (size_t)r * H);
        linear(h, rows, &Ly->wq, q);
        linear(h, rows, &Ly->wk, k);
        linear(h, rows, &Ly->wv, v);
        for (int r = 0; r < rows; r++) {
            int p = L0 + r;
            const float *cs = m->rope_cos + (size_t)p * half, *sn = m->rope_sin + (size_t)p * half;
            for (int hh = 0; hh < Hq; hh++) {
                float *qh = q + (size_t)r * Q + hh * D;
                float t[512];
                rmsnorm(qh, Ly->q_norm, D, c->eps, t);
                memcpy(qh, t, D * sizeof(float));
                rope(qh, D, cs, sn);
            }
            for (int hh = 0; hh < Hkv; hh++) {
                float *kh = k + (size_t)r * KV + hh * D;
                float t[512];
                rmsnorm(kh, Ly->k_norm, D, c->eps, t);
                memcpy(kh, t, D * sizeof(float));
                rope(kh, D, cs, sn);
            }
            /* KV cache append */
            float *kc = m->k + (((size_t)l * m->max_pos + p) * Hkv) * D;
            float *vc = m->v + (((size_t)l * m->max_pos + p) * Hkv) * D;
            memcpy(kc, k + (size_t)r * KV, KV * sizeof(float));
            memcpy(vc, v + (size_t)r * KV, KV * sizeof(float));
            if (m->kv_f16)
                for (int i = 0; i < KV; i++) {
                    kc[i] = f16_to_f32(f32_to_f16(kc[i]));
                    vc[i] = f16_to_f32(f32_to_f16(vc[i]));
                }
        }
        /* causal GQA attention: query head hh reads kv head hh / grp */
#pragma omp parallel for collapse(2) schedule(static)
        for (int r = 0; r < rows; r++) {
            for (int hh = 0; hh < Hq; hh++) {
                int p = L0 + r, kvh = hh / grp;
                const float *qh = q + (size_t)r * Q + hh * D;
                float *sc = (float *)malloc((size_t)(p + 1) * sizeof(float));
                float mx = -INFINITY;
                for (int t = 0; t <= p; t++) {
                    const float *kt = m->k + (((size_t)l * m->max_pos + t) * Hkv + kvh) * D;
                    float d = 0.0f;
                    for (int i = 0; i < D; i++) d += qh[i] * kt[i];
                    sc[t] = d * scale;
                    if (sc[t] > mx) mx = sc[t];
                }
                float sum = 0.0f;
                for (int t = 0; t <= p; t++) {
                    sc[t] = expf(sc[t] - mx);
                    sum += sc[t];
                }
                float *out = att + (size_t)r * Q + hh * D;
                for (int i = 0; i < D; i++) out[i] = 0.0f;
                for (int t = 0; t <= p; t++) {
                    const float *vt = m->v + (((size_t)l * m->max_pos + t) * Hkv + kvh) * D;
                    float w = sc[t] / sum;
                    for (int i = 0; i < D; i++) out[i] += w * vt[i];
                }
                free(sc);
            }
        }
        linear(att, rows, &Ly->wo, o);
        for (size_t i = 0; i < (size_t)rows * H; i++) x[i] = x[i] + o[i];
        for (int r = 0; r < rows; r++) rmsnorm(x + (size_t)r * H, Ly->post_norm, H, c->eps, h + (size_t)r * H);
        linear(h, rows, &Ly->wg, g);
        linear(h, rows, &Ly->wu, u);
        for (size_t i = 0; i < (size_t)rows * I; i++) g[i] = silu(g[i]) * u[i];
        linear(g, rows, &Ly->wd, o);
        for (size_t i = 0; i < (size_t)rows * H; i++) x[i] = x[i] + o[i];
        if (states) memcpy(states + (size_t)l * rows * H, x, (size_t)rows * H * sizeof(float));
    }
    m->len = L0 + rows;
    free(h); free(q); free(k); free(v); free(att); free(o); free(g); free(u);
    return 0;
}

/* TQwenLm.Forward (lm.pas:391-408): rows appended at Length.., the normed
 * last row in hidden (may be NULL), head `head` of `heads` on it in logits
 * (NULL: none).  states: optional [layers][rows][H] layer outputs; normed:
 * optional [rows][H] final-norm output of every row (the dataset's
 * talker.norm).  Returns 0, or -1 when the cache is full. */
int ora_lm_forward(ora_lm *m, const float *x_in, int rows, const ora_heads *heads, int head,
                   float *logits, float *hidden, float *states, float *normed) {
    if (rows <= 0) return 0;
    int H = m->s->c.hidden;
    float *x = dupf(x_in, (size_t)rows * H);
    if (stack_forward(m, x, rows, states) != 0) {
        free(x);
        return -1;
    }
    float *last = (float *)malloc(H * sizeof(float));
    rmsnorm(x + (size_t)(rows - 1) * H, m->s->final_norm, H, m->s->c.eps, last);
    if (normed)
        for (int r = 0; r < rows; r++)
            rmsnorm(x + (size_t)r * H, m->s->final_norm, H, m->s->c.eps, normed + (size_t)r * H);
    if (hidden) memcpy(hidden, last, H * sizeof(float));
    if (logits && heads) linear(last, 1, heads->w + head, logits);
    free(last);
    free(x);
    return 0;
}

/* ---------------------------------------------------------------- choice */

/* the ArgMax of tests/test.tts.qwen.lm.pas:109-117: strict '>', so the first
 * maximum wins */
int ora_argmax(const float *p, int n) {
    int r = 0;
    for (int i = 1; i < n; i++)
        if (p[i] > p[r]) r = i;
    return r;
}

/* TQwenTalker.ChooseCode0 (talker.pas:595-630) in greedy mode: the last 1024
 * ids forbidden but eos, eos forbidden before 2 frames, repetition penalty
 * once per distinct past code, then the argmax */
int ora_choose_code0(const float *logits, int vocab, int eos, const int *history, int nhist, float penalty,
                     float *work) {
    memcpy(work, logits, vocab * sizeof(float));
    for (int i = vocab - 1024; i < vocab; i++)
        if (i != eos) work[i] = -INFINITY;
    if (nhist < 2) work[eos] = -INFINITY;
    if (penalty != 1.0f)
        for (int j = 0; j < nhist; j++) {
            int i = history[j];
            float s = logits[i];
            if (work[i] != s) continue;
            work[i] = s > 0 ? s / penalty : s * penalty;
        }
    return ora_argmax(work, vocab);
}

/* ---------------------------------------------------------------- text projection */

/* TQwenTalker.TextProject (talker.pas:390-421): for each id, the text
 * embedding row (float32 here; BF16 tables are widened by the caller), then
 * h = fc1 . e + b1 (TInferBackend.Linear with bias), silu as the reference
 * writes it (0 below -80, else v / (1 + exp(-v))), y = fc2 . h + b2. */
void ora_text_project(const float *emb, int vocab, int th, int hidden, const int *ids, int n, const float *w1,
                      const float *b1, const float *w2, const float *b2, float *y) {
    float *e = (float *)malloc((size_t)th * sizeof(float)), *h = (float *)malloc((size_t)th * sizeof(float));
    for (int r = 0; r < n; r++) {
        int id = ids[r] < 0 ? 0 : (ids[r] >= vocab ? vocab - 1 : ids[r]);
        memcpy(e, emb + (size_t)id * th, (size_t)th * sizeof(float));
        for (int o = 0; o < th; o++) {
            float v = dot_f32(w1 + (size_t)o * th, e, th) + b1[o];
            h[o] = v < -80.0f ? 0.0f : v / (1.0f + expf(-v));
        }
        for (int o = 0; o < hidden; o++) y[(size_t)r * hidden + o] = dot_f32(w2 + (size_t)o * th, h, th) + b2[o];
    }
    free(e);
    free(h);
}

/* ---------------------------------------------------------------- sampling */

/* TInferSampler.Next (mormot2-ai, used at talker.pas:626-629 and 632-638;
 * its source is absent here) restated after the logits warpers of
 * transformers' generate, which the reference's options mirror
 * (generation_config: temperature, top_k, top_p; talker.pas:203-229):
 *   z = logit / temperature; keep the values >= the top_k-th largest (ties
 *   kept, -inf never); order them by (z desc, index asc); keep the nucleus
 *   whose probability mass before each kept value is < top_p (at least one);
 *   draw by inverse CDF with u in [0, 1): the first value whose running sum
 *   of exp(z - z_max), in that order, exceeds u * (sum over the nucleus).
 * u comes from a counter-based generator: splitmix64 (Vigna's published
 * finaliser) of seed + (16 * step + group + 1) * golden ratio, top 24 bits.
 * The running sums are sequential in candidate order so that another
 * implementation can repeat them exactly. */
#define ORA_SAMPLE_MAX_K 64
#define ORA_SAMPLE_MAX_CAND 128

static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

float ora_sample_uniform(uint64_t seed, int step, int group) {
    uint64_t c = (uint64_t)step * 16u + (uint64_t)group + 1u;
    uint64_t z = mix64(seed + c * 0x9E3779B97F4A7C15ull);
    return (float)(z >> 40) * (1.0f / 16777216.0f);
}

/* orderable key of a float: larger value, larger key */
static uint32_t okey(float z) {
    uint32_t b;
    memcpy(&b, &z, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

static int cmp_u32_desc(const void *a, const void *b) {
    uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return x < y ? 1 : (x > y ? -1 : 0);
}

/* the index drawn from work[0..n) (logits after the processors) */
int ora_sample(const float *work, int n, float temperature, int top_k, float top_p, float u) {
    if (n <= 0) return 0;
    uint32_t *keys = (uint32_t *)malloc((size_t)n * 4), *sk = (uint32_t *)malloc((size_t)n * 4);
    float *z = (float *)malloc((size_t)n * 4);
    for (int i = 0; i < n; i++) {
        z[i] = work[i] / temperature;
        keys[i] = sk[i] = okey(z[i]);
    }
    int k = top_k < 1 ? 1 : (top_k < n ? top_k : n);
    qsort(sk, n, 4, cmp_u32_desc);
    uint32_t thr = sk[k - 1];
    free(sk);
    int ci[ORA_SAMPLE_MAX_CAND], nc = 0, ncand = 0;
    for (int i = 0; i < n; i++)
        if (keys[i] >= thr && z[i] != -INFINITY) {
            if (nc < ORA_SAMPLE_MAX_CAND) ci[nc++] = i;
            ncand++;
        }
    /* no candidate (all -inf) or more ties than kept: the first maximum of z */
    int code = ora_argmax(z, n);
    if (nc > 0 && ncand <= ORA_SAMPLE_MAX_CAND) {
        /* rank of each candidate under (z desc, index asc) */
        int sidx[ORA_SAMPLE_MAX_CAND];
        float sz[ORA_SAMPLE_MAX_CAND], sw[ORA_SAMPLE_MAX_CAND];
        for (int c = 0; c < nc; c++) {
            int r = 0;
            for (int m = 0; m < nc; m++)
                if (keys[ci[m]] > keys[ci[c]] || (keys[ci[m]] == keys[ci[c]] && ci[m] < ci[c])) r++;
            sidx[r] = ci[c];
            sz[r] = z[ci[c]];
        }
        float mx = sz[0];
        for (int c = 0; c < nc; c++) sw[c] = expf(sz[c] - mx);
        float total = 0.0f;
        for (int c = 0; c < nc; c++) total += sw[c];
        int nk = nc;
        if (top_p < 1.0f) {
            float acc = 0.0f;
            for (int c = 0; c < nc; c++) {
                if (c > 0 && acc / total >= top_p) {
                    nk = c;
                    break;
                }
                acc += sw[c];
            }
        }
        float wsum = 0.0f;
        for (int c = 0; c < nk; c++) wsum += sw[c];
        float target = u * wsum, acc = 0.0f;
        code = sidx[nk - 1];
        for (int c = 0; c < nk; c++) {
            acc += sw[c];
            if (acc > target) {
                code = sidx[c];
                break;
            }
        }
    }
    free(keys);
    free(z);
    return code;
}

/* ---------------------------------------------------------------- talker */

/* the device-side part of TQwenTalker (talker.pas:78-158): both stacks, the
 * code embeddings, the trailing text rows, the greedy choice */
typedef struct {
    ora_lm *talker, *pred;
    const ora_heads *th, *ph;
    int H, vocab, pvocab, groups, eos;
    float penalty;
    float *codec_emb;  /* [vocab][H] */
    float *pred_emb;   /* [groups-1][pvocab][H] */
    float *trailing;   /* [trailing_rows][H] */
    int trailing_rows;
    float *tts_pad;    /* [H] */
    float *logits, *work, *past_hidden, *plogits, *x;
    int *history;
    int nhist, step, cap;
    /* TQwenSampling (talker.pas:59-73): code 0 and the predictor's codes */
    int do_sample, sub_do_sample, top_k, sub_top_k;
    float temperature, top_p, sub_temperature, sub_top_p;
    uint64_t seed;
} ora_talker;

void ora_talker_set_sampling(ora_talker *t, int do_sample, float temperature, int top_k, float top_p,
                             int sub_do_sample, float sub_temperature, int sub_top_k, float sub_top_p,
                             uint64_t seed) {
    t->do_sample = do_sample;
    t->temperature = temperature;
    t->top_k = top_k;
    t->top_p = top_p;
    t->sub_do_sample = sub_do_sample;
    t->sub_temperature = sub_temperature;
    t->sub_top_k = sub_top_k;
    t->sub_top_p = sub_top_p;
    t->seed = seed;
}

ora_talker *ora_talker_create(ora_lm *talker, const ora_heads *th, ora_lm *pred, const ora_heads *ph,
                              const float *codec_emb, int vocab, const float *pred_emb, int pvocab, int groups,
                              int eos, float penalty) {
    ora_talker *t = (ora_talker *)calloc(1, sizeof(ora_talker));
    int H = talker->s->c.hidden;
    t->talker = talker;
    t->pred = pred;
    t->th = th;
    t->ph = ph;
    t->H = H;
    t->vocab = vocab;
    t->pvocab = pvocab;
    t->groups = groups;
    t->eos = eos;
    t->penalty = penalty;
    t->codec_emb = dupf(codec_emb, (size_t)vocab * H);
    t->pred_emb = dupf(pred_emb, (size_t)(groups - 1) * pvocab * H);
    t->logits = (float *)calloc(vocab, sizeof(float));
    t->work = (float *)calloc(vocab, sizeof(float));
    t->plogits = (float *)calloc(pvocab, sizeof(float));
    t->past_hidden = (float *)calloc(H, sizeof(float));
    t->x = (float *)calloc(2 * H, sizeof(float));
    t->tts_pad = (float *)calloc(H, sizeof(float));
    return t;
}

void ora_talker_free(ora_talker *t) {
    if (!t) return;
    free(t->codec_emb); free(t->pred_emb); free(t->trailing); free(t->tts_pad);
    free(t->logits); free(t->work); free(t->plogits); free(t->past_hidden); free(t->x); free(t->history);
    free(t);
}

/* the end of TQwenTalker.Start (talker.pas:561-592): trailing rows, talker
 * reset + prefill, empty history */
int ora_talker_start(ora_talker *t, const float *prefill, int rows, const float *trailing, int trailing_rows,
                     const float *tts_pad) {
    int H = t->H;
    free(t->trailing);
    t->trailing = trailing_rows > 0 ? dupf(trailing, (size_t)trailing_rows * H) : NULL;
    t->trailing_rows = trailing_rows;
    memcpy(t->tts_pad, tts_pad, H * sizeof(float));
    ora_lm_reset(t->talker);
    int rc = ora_lm_forward(t->talker, prefill, rows, t->th, 0, t->logits, t->past_hidden, NULL, NULL);
    t->nhist = 0;
    t->step = 0;
    return rc;
}

static void add_row(float *y, const float *row, int H) {
    for (int c = 0; c < H; c++) y[c] = y[c] + row[c];
}

/* TQwenTalker.NextFrame (talker.pas:640-681), greedy.  force == NULL: the
 * oracle's own choices go to codes[groups].  force != NULL: the frame is
 * driven by the codes force[groups] (another implementation's choices) and
 * gap[g] receives how far force[g] falls below the best value of choice g
 * under the same rule (0 for a first maximum or a tie; +inf for a forbidden
 * id).  Returns 1 after a frame, 0 when code 0 is eos, -1 when a cache is
 * full. */
/* rank of v among x[n]: the values strictly greater */
static int rank_of(const float *x, int n, float v) {
    int r = 0;
    for (int i = 0; i < n; i++) r += x[i] > v;
    return r;
}

/* x[best] minus the largest of the other values: how far the choice is
 * from a tie (0 for a tie, +inf when every other value is -inf) */
static float margin_of(const float *x, int n, int best) {
    float second = -INFINITY;
    for (int i = 0; i < n; i++)
        if (i != best && x[i] > second) second = x[i];
    return x[best] - second;
}

static int talker_frame(ora_talker *t, const int *force, int *codes, float *gap, int *rank, float *margin) {
    int H = t->H;
    int code = ora_choose_code0(t->logits, t->vocab, t->eos, t->history, t->nhist, t->penalty, t->work);
    if (margin) margin[0] = margin_of(t->work, t->vocab, code);
    if (t->do_sample && !force)
        code = ora_sample(t->work, t->vocab, t->temperature, t->top_k, t->top_p,
                          ora_sample_uniform(t->seed, t->step, 0));
    if (force) {
        gap[0] = t->work[code] - t->work[force[0]];
        if (t->work[force[0]] == -INFINITY) gap[0] = INFINITY;
        if (rank) rank[0] = rank_of(t->work, t->vocab, t->work[force[0]]);
        code = force[0];
    }
    if (code == t->eos) return 0;
    codes[0] = code;
    if (t->nhist == t->cap) {
        t->cap = t->cap ? 2 * t->cap : 64;
        t->history = (int *)realloc(t->history, t->cap * sizeof(int));
    }
    t->history[t->nhist++] = code;
    memcpy(t->x, t->past_hidden, H * sizeof(float));
    memcpy(t->x + H, t->codec_emb + (size_t)code * H, H * sizeof(float));
    ora_lm_reset(t->pred);
    if (ora_lm_forward(t->pred, t->x, 2, t->ph, 0, t->plogits, NULL, NULL, NULL)) return -1;
    for (int g = 0; g < t->groups - 1; g++) {
        if (g > 0) {
            memcpy(t->x, t->pred_emb + ((size_t)(g - 1) * t->pvocab + codes[g]) * H, H * sizeof(float));
            if (ora_lm_forward(t->pred, t->x, 1, t->ph, g, t->plogits, NULL, NULL, NULL)) return -1;
        }
        int best = ora_argmax(t->plogits, t->pvocab);
        if (margin) margin[g + 1] = margin_of(t->plogits, t->pvocab, best);
        if (t->sub_do_sample && !force)
            best = ora_sample(t->plogits, t->pvocab, t->sub_temperature, t->sub_top_k, t->sub_top_p,
                              ora_sample_uniform(t->seed, t->step, g + 1));
        if (force) {
            gap[g + 1] = t->plogits[best] - t->plogits[force[g + 1]];
            if (rank) rank[g + 1] = rank_of(t->plogits, t->pvocab, t->plogits[force[g + 1]]);
            best = force[g + 1];
        }
        codes[g + 1] = best;
    }
    memcpy(t->x, t->codec_emb + (size_t)code * H, H * sizeof(float));
    for (int g = 1; g < t->groups; g++)
        add_row(t->x, t->pred_emb + ((size_t)(g - 1) * t->pvocab + codes[g]) * H, H);
    if (t->step < t->trailing_rows)
        add_row(t->x, t->trailing + (size_t)t->step * H, H);
    else
        add_row(t->x, t->tts_pad, H);
    if (ora_lm_forward(t->talker, t->x, 1, t->th, 0, t->logits, t->past_hidden, NULL, NULL)) return -1;
    t->step++;
    return 1;
}

/* returns 1 and fills codes[groups], 0 at eos, -1 when a cache is full */
int ora_talker_next_frame(ora_talker *t, int *codes) { return talker_frame(t, NULL, codes, NULL, NULL, NULL); }

/* as ora_talker_next_frame (greedy), with margin[g]: how far choice g's best
 * value lies above the next one (the room a second implementation has for
 * rounding differences before its first maximum moves) */
int ora_talker_next_frame_margins(ora_talker *t, int *codes, float *margin) {
    return talker_frame(t, NULL, codes, NULL, NULL, margin);
}

/* the frame chosen elsewhere (codes[groups]), with the gaps of its choices */
int ora_talker_check_frame(ora_talker *t, const int *codes, float *gap) {
    int own[64];
    if (t->groups > 64) return -1;
    return talker_frame(t, codes, own, gap, NULL, NULL);
}

/* as ora_talker_check_frame, with rank[g]: how many of choice g's values
 * (after the processors) are strictly above the value of codes[g] */
int ora_talker_check_frame_ranks(ora_talker *t, const int *codes, float *gap, int *rank) {
    int own[64];
    if (t->groups > 64) return -1;
    return talker_frame(t, codes, own, gap, rank, NULL);
}

const float *ora_talker_logits(const ora_talker *t) { return t->logits; }
const float *ora_talker_hidden(const ora_talker *t) { return t->past_hidden; }
