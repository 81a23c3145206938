/* qtts_codec_oracle.c -- CPU restatement of the reference's 12 Hz decoder
 * (TQwenCodec, src/tts/mormot.ai.tts.qwen.codec.pas): 16 codes per frame ->
 * 1920 PCM samples at 24 kHz, frame by frame.
 *
 * TEST INFRASTRUCTURE ONLY (the checker of a device codec); the product
 * library never links it.  Every step cites the reference:
 *   quantizer      codec.pas:667-689 (codebook = embedding_sum / max(usage,
 *                  1e-5)), 886-917 (Quantize)
 *   pre-conv       codec.pas:691, TQwenConv 296-363 (causal, history rows)
 *   transformer    codec.pas:692-716, CacheRoom 919-946, Transformer
 *                  948-1017 (RMSNorm 1e-5, RoPE base 10000 on the frame
 *                  index, 72-frame sliding window, layer scales)
 *   upsampling     codec.pas:717-723, TQwenTransConv 366-428, TQwenConvNeXt
 *                  481-535 (depthwise 7, LayerNorm 1e-6, GELU, gamma)
 *   decoder        codec.pas:724-729, TQwenBlock 592-641 (SnakeBeta,
 *                  transposed conv, residual units with dilations 1, 3, 9),
 *                  TQwenResUnit 538-590, TQwenSnake 431-478, Back and the
 *                  output clamp 1040-1084
 * Weights are looked up by their names in the checkpoint, with the element
 * counts the reference checks (F32(name, dims)).  Dot products are float32
 * with AVX2 FMAs in a fixed order, the same for a row whatever the number of
 * rows decoded at once, so decoding 1 + 3 frames or 4 at once gives the same
 * samples bit for bit (the property the reference states, codec.pas:5-8).
 * The reference's CPU backend (mormot2-ai) is absent: RMSNorm, RoPE
 * (rotate-half pairs i, i + 32), attention softmax, SwiGLU, GELU (erf form)
 * and LayerNorm follow the PyTorch modules the reference mirrors (qwen_tts
 * 0.1.1, Qwen3TTSTokenizerV2Decoder).  The RoPE is the backend's Rope
 * (codec.pas:985-986), the call its Qwen3 stacks make too, whose rotate-half
 * pairs the language-model oracle pins to transformers' Qwen3. */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define CG 16        /* code groups of a frame */
#define CB 2048      /* values of a code */
#define CODE_DIM 256
#define QUANT_DIM 512
#define LATENT 1024
#define TF_DIM 512
#define TF_HEADS 16
#define TF_HD 64
#define TF_QKV (TF_HEADS * TF_HD)
#define TF_MLP 1024
#define TF_LAYERS 8
#define TF_WINDOW 72
#define TF_EPS 1e-5f
#define DEC_DIM 1536
#define FRAME_SAMPLES 1920

static char g_err[512];
const char *ora_codec_error(void) { return g_err; }

static float hsum(__m256 v) {
    __m128 lo = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    lo = _mm_add_ps(lo, _mm_movehl_ps(lo, lo));
    lo = _mm_add_ss(lo, _mm_movehdup_ps(lo));
    return _mm_cvtss_f32(lo);
}

static float dot(const float *a, const float *b, int n) {
    __m256 s0 = _mm256_setzero_ps(), s1 = _mm256_setzero_ps();
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        s0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), s0);
        s1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), s1);
    }
    float s = hsum(_mm256_add_ps(s0, s1));
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

/* y[r][o] = x[r] . w[o] (+ b[o]); w [out][in] (Gemm, codec.pas:830-853) */
static void gemm(const float *x, int rows, int in, const float *w, int out, const float *b, float *y) {
#pragma omp parallel for collapse(2) schedule(static) if ((long long)rows * in * out > 65536)
    for (int r = 0; r < rows; r++)
        for (int o = 0; o < out; o++)
            y[(size_t)r * out + o] = dot(x + (size_t)r * in, w + (size_t)o * in, in) + (b ? b[o] : 0.0f);
}

/* ------------------------------------------------------------- weights */

typedef struct {
    int n;
    const char *const *names;
    const float *const *ptrs;
    const int64_t *counts;
    int bad;
} Table;

static const float *w_get(Table *t, const char *name, int64_t count) {
    for (int i = 0; i < t->n; i++)
        if (strcmp(t->names[i], name) == 0) {
            if (t->counts[i] != count) {
                snprintf(g_err, sizeof g_err, "%s has %lld values instead of %lld", name, (long long)t->counts[i],
                         (long long)count);
                t->bad = 1;
                return NULL;
            }
            return t->ptrs[i];
        }
    snprintf(g_err, sizeof g_err, "no tensor %s", name);
    t->bad = 1;
    return NULL;
}

/* ------------------------------------------------------------- layers */

/* causal convolution, weights [out][in][k] (TQwenConv, codec.pas:296-363):
 * y[t] = b + sum_k W[:, :, k] . x[t - (K-1-k) dil], the rows before the
 * first input from the history (zeros after a reset) */
typedef struct {
    int in, out, k, dil, past;
    const float *w, *b;
    float *hist;
} Conv;

static void conv_init(Conv *c, Table *t, const char *prefix, int in, int out, int k, int dil) {
    char n[512];
    c->in = in, c->out = out, c->k = k, c->dil = dil, c->past = (k - 1) * dil;
    snprintf(n, sizeof n, "%s.weight", prefix);
    c->w = w_get(t, n, (int64_t)out * in * k);
    snprintf(n, sizeof n, "%s.bias", prefix);
    c->b = w_get(t, n, out);
    c->hist = calloc((size_t)(c->past > 0 ? c->past : 1) * in, sizeof(float));
}
static void conv_reset(Conv *c) { memset(c->hist, 0, (size_t)(c->past > 0 ? c->past : 1) * c->in * sizeof(float)); }

static void conv_fwd(Conv *c, const float *x, int rows, float *y) {
    if (c->k == 1) {
        gemm(x, rows, c->in, c->w, c->out, c->b, y);
        return;
    }
    const int in = c->in, K = c->k, cols = in * K;
    float *buf = malloc((size_t)(c->past + rows) * in * sizeof(float));
    memcpy(buf, c->hist, (size_t)c->past * in * sizeof(float));
    memcpy(buf + (size_t)c->past * in, x, (size_t)rows * in * sizeof(float));
    float *col = malloc((size_t)rows * cols * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int k = 0; k < K; k++) {
            const float *src = buf + (size_t)(r + k * c->dil) * in;
            for (int ch = 0; ch < in; ch++) col[(size_t)r * cols + ch * K + k] = src[ch];
        }
    gemm(col, rows, cols, c->w, c->out, c->b, y);
    memcpy(c->hist, buf + (size_t)rows * in, (size_t)c->past * in * sizeof(float));
    free(col);
    free(buf);
}

/* causal transposed convolution, stride s, kernel K = taps * s, cut on the
 * right by K - s (TQwenTransConv, codec.pas:366-428): row t*s + j gets
 * b + sum_{i < taps} x[t - i] . W[:, :, j + i*s]; W [in][out][K] in the file,
 * re-laid as [s*out][taps*in] */
typedef struct {
    int in, out, s, taps;
    float *w, *b, *hist;
} TConv;

static void tconv_init(TConv *c, Table *t, const char *prefix, int in, int out, int k, int s) {
    char n[512];
    c->in = in, c->out = out, c->s = s, c->taps = k / s;
    snprintf(n, sizeof n, "%s.weight", prefix);
    const float *w = w_get(t, n, (int64_t)in * out * k);
    snprintf(n, sizeof n, "%s.bias", prefix);
    const float *b = w_get(t, n, out);
    const int cols = c->taps * in;
    c->w = malloc((size_t)s * out * cols * sizeof(float));
    c->b = malloc((size_t)s * out * sizeof(float));
    c->hist = calloc((size_t)(c->taps > 1 ? c->taps - 1 : 1) * in, sizeof(float));
    if (!w || !b) return;
    for (int j = 0; j < s; j++)
        for (int o = 0; o < out; o++) {
            c->b[j * out + o] = b[o];
            for (int i = 0; i < c->taps; i++)
                for (int ch = 0; ch < in; ch++)
                    c->w[((size_t)j * out + o) * cols + i * in + ch] = w[((size_t)ch * out + o) * k + j + i * s];
        }
}
static void tconv_reset(TConv *c) {
    memset(c->hist, 0, (size_t)(c->taps > 1 ? c->taps - 1 : 1) * c->in * sizeof(float));
}

/* y[rows * s][out]: the s output rows of input row t are one row of
 * [s*out] values of the re-laid product */
static void tconv_fwd(TConv *c, const float *x, int rows, float *y) {
    const int in = c->in, past = c->taps - 1, cols = c->taps * in;
    float *buf = malloc((size_t)(past + rows) * in * sizeof(float));
    memcpy(buf, c->hist, (size_t)past * in * sizeof(float));
    memcpy(buf + (size_t)past * in, x, (size_t)rows * in * sizeof(float));
    float *x2 = malloc((size_t)rows * cols * sizeof(float));
    for (int t = 0; t < rows; t++)
        for (int i = 0; i < c->taps; i++)
            memcpy(x2 + ((size_t)t * c->taps + i) * in, buf + (size_t)(past + t - i) * in, (size_t)in * sizeof(float));
    gemm(x2, rows, cols, c->w, c->s * c->out, c->b, y);
    memcpy(c->hist, buf + (size_t)rows * in, (size_t)past * in * sizeof(float));
    free(x2);
    free(buf);
}

/* SnakeBeta (TQwenSnake, codec.pas:431-478): x + 1/(exp(beta) + 1e-9) *
 * sin(x * exp(alpha))^2, the exps taken once in float32 */
typedef struct {
    int n;
    float *alpha, *inv_beta;
} Snake;

static void snake_init(Snake *s, Table *t, const char *prefix, int n) {
    char nm[512];
    s->n = n;
    snprintf(nm, sizeof nm, "%s.alpha", prefix);
    const float *a = w_get(t, nm, n);
    snprintf(nm, sizeof nm, "%s.beta", prefix);
    const float *b = w_get(t, nm, n);
    s->alpha = malloc((size_t)n * sizeof(float));
    s->inv_beta = malloc((size_t)n * sizeof(float));
    if (!a || !b) return;
    for (int c = 0; c < n; c++) {
        s->alpha[c] = expf(a[c]);
        s->inv_beta[c] = 1.0f / (expf(b[c]) + 1e-9f);
    }
}

static void snake_fwd(const Snake *s, float *x, int rows) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int c = 0; c < s->n; c++) {
            float *v = x + (size_t)r * s->n + c;
            const float q = sinf(*v * s->alpha[c]);
            *v = *v + s->inv_beta[c] * (q * q);
        }
}

/* ConvNeXt block (TQwenConvNeXt, codec.pas:481-535): causal depthwise
 * convolution (7), LayerNorm (1e-6), pwconv1 (4x), GELU, pwconv2, gamma,
 * residual */
typedef struct {
    int dim;
    const float *dw_w, *dw_b, *nw, *nb, *w1, *b1, *w2, *b2, *gamma;
    float *hist;
} Next;

static void next_init(Next *x, Table *t, const char *prefix, int dim) {
    char n[512];
    x->dim = dim;
#define G(field, suffix, count)                          \
    snprintf(n, sizeof n, "%s.%s", prefix, suffix);      \
    x->field = w_get(t, n, count);
    G(dw_w, "dwconv.conv.weight", (int64_t)dim * 7)
    G(dw_b, "dwconv.conv.bias", dim)
    G(nw, "norm.weight", dim)
    G(nb, "norm.bias", dim)
    G(w1, "pwconv1.weight", (int64_t)4 * dim * dim)
    G(b1, "pwconv1.bias", 4 * dim)
    G(w2, "pwconv2.weight", (int64_t)dim * 4 * dim)
    G(b2, "pwconv2.bias", dim)
    G(gamma, "gamma", dim)
#undef G
    x->hist = calloc((size_t)6 * dim, sizeof(float));
}
static void next_reset(Next *x) { memset(x->hist, 0, (size_t)6 * x->dim * sizeof(float)); }

static void next_fwd(Next *x, const float *in, int rows, float *y) {
    const int D = x->dim;
    float *buf = malloc((size_t)(6 + rows) * D * sizeof(float));
    memcpy(buf, x->hist, (size_t)6 * D * sizeof(float));
    memcpy(buf + (size_t)6 * D, in, (size_t)rows * D * sizeof(float));
    float *n = malloc((size_t)rows * D * sizeof(float));
    float *h = malloc((size_t)rows * 4 * D * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int t = 0; t < rows; t++) {
        float *nr = n + (size_t)t * D;
        for (int c = 0; c < D; c++) {
            float acc = x->dw_b[c];
            for (int k = 0; k < 7; k++) acc += x->dw_w[c * 7 + k] * buf[(size_t)(t + k) * D + c];
            nr[c] = acc;
        }
        float mean = 0.0f, var = 0.0f;
        for (int c = 0; c < D; c++) mean += nr[c];
        mean /= (float)D;
        for (int c = 0; c < D; c++) var += (nr[c] - mean) * (nr[c] - mean);
        var /= (float)D;
        const float inv = 1.0f / sqrtf(var + 1e-6f);
        for (int c = 0; c < D; c++) nr[c] = (nr[c] - mean) * inv * x->nw[c] + x->nb[c];
    }
    memcpy(x->hist, buf + (size_t)rows * D, (size_t)6 * D * sizeof(float));
    gemm(n, rows, D, x->w1, 4 * D, x->b1, h);
    for (size_t i = 0; i < (size_t)rows * 4 * D; i++) h[i] = 0.5f * h[i] * (1.0f + erff(h[i] * 0.70710678118654752f));
    gemm(h, rows, 4 * D, x->w2, D, x->b2, n);
    for (size_t i = 0; i < (size_t)rows * D; i++) y[i] = in[i] + x->gamma[i % D] * n[i];
    free(h);
    free(n);
    free(buf);
}

/* residual unit (TQwenResUnit, codec.pas:538-590): x += conv2(snake2(
 * conv1_dil(snake1(x)))) */
typedef struct {
    Snake a1, a2;
    Conv c1, c2;
    int dim;
} Res;

/* decoder block (TQwenBlock, codec.pas:592-641) */
typedef struct {
    int in, out, rate;
    Snake act;
    TConv up;
    Res res[3];
} Block;

typedef struct {
    const float *in_norm, *wq, *wk, *wv, *wo, *post_norm, *wg, *wu, *wd, *attn_scale, *mlp_scale;
} TfLayer;

typedef struct ora_codec {
    float *codebook;  /* [16][2048][256] */
    const float *first_proj, *rest_proj;
    Conv pre;
    const float *tf_in, *tf_in_b, *tf_out, *tf_out_b, *tf_norm;
    TfLayer tf[TF_LAYERS];
    float *keys[TF_LAYERS], *values[TF_LAYERS];  /* [TF_WINDOW + cap][TF_QKV] ring-free: positions base.. */
    int cache_cap;
    long long cache_base;
    float inv_freq[TF_HD / 2];
    TConv up[2];
    Next next[2];
    Conv conv0;
    Block blocks[4];
    Snake act_out;
    Conv conv_out;
    long long frames;
} ora_codec;

static void rmsnorm(const float *x, int rows, int n, const float *w, float eps, float *y) {
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (size_t)r * n;
        float ss = 0.0f;
        for (int i = 0; i < n; i++) ss += xr[i] * xr[i];
        const float inv = 1.0f / sqrtf(ss / (float)n + eps);
        for (int i = 0; i < n; i++) y[(size_t)r * n + i] = xr[i] * inv * w[i];
    }
}

/* rotate-half RoPE over each head: (x_i, x_{i+32}) by angle pos * inv_freq_i */
static void rope(float *x, int rows, const float *cs, const float *sn) {
    for (int r = 0; r < rows; r++)
        for (int h = 0; h < TF_HEADS; h++) {
            float *v = x + (size_t)r * TF_QKV + h * TF_HD;
            for (int i = 0; i < TF_HD / 2; i++) {
                const float c = cs[r * (TF_HD / 2) + i], s = sn[r * (TF_HD / 2) + i];
                const float a = v[i], b = v[i + TF_HD / 2];
                v[i] = a * c - b * s;
                v[i + TF_HD / 2] = b * c + a * s;
            }
        }
}

/* the cache keeps positions cache_base .. frames-1 (CacheRoom, codec.pas:919-946) */
static int cache_room(ora_codec *c, int rows) {
    if (c->frames - c->cache_base + rows <= c->cache_cap) return 0;
    long long keep = c->frames - c->cache_base;
    if (keep > TF_WINDOW - 1) keep = TF_WINDOW - 1;
    const long long from = c->frames - c->cache_base - keep;
    if (keep + rows > c->cache_cap) {
        const int cap = (int)keep + rows + 4 * TF_WINDOW;
        for (int l = 0; l < TF_LAYERS; l++) {
            float *k = realloc(c->keys[l], (size_t)cap * TF_QKV * sizeof(float));
            float *v = realloc(c->values[l], (size_t)cap * TF_QKV * sizeof(float));
            if (!k || !v) return -1;
            c->keys[l] = k, c->values[l] = v;
        }
        c->cache_cap = cap;
    }
    if (keep > 0 && from > 0)
        for (int l = 0; l < TF_LAYERS; l++) {
            memmove(c->keys[l], c->keys[l] + from * TF_QKV, (size_t)keep * TF_QKV * sizeof(float));
            memmove(c->values[l], c->values[l] + from * TF_QKV, (size_t)keep * TF_QKV * sizeof(float));
        }
    c->cache_base = c->frames - keep;
    return 0;
}

static int transformer(ora_codec *c, const float *x, int rows, float *y) {
    const size_t R = (size_t)rows;
    float *h = malloc(R * TF_DIM * 4), *n = malloc(R * TF_DIM * 4), *q = malloc(R * TF_QKV * 4),
          *k = malloc(R * TF_QKV * 4), *v = malloc(R * TF_QKV * 4), *att = malloc(R * TF_QKV * 4),
          *o = malloc(R * TF_DIM * 4), *g = malloc(R * TF_MLP * 4), *u = malloc(R * TF_MLP * 4),
          *cs = malloc(R * (TF_HD / 2) * 4), *sn = malloc(R * (TF_HD / 2) * 4);
    gemm(x, rows, LATENT, c->tf_in, TF_DIM, c->tf_in_b, h);
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < TF_HD / 2; i++) {
            const float f = (float)(c->frames + r) * c->inv_freq[i];  /* float32 product */
            cs[r * (TF_HD / 2) + i] = cosf(f);
            sn[r * (TF_HD / 2) + i] = sinf(f);
        }
    if (cache_room(c, rows)) return -1;
    const long long row0 = c->frames - c->cache_base;
    const float scale = 1.0f / sqrtf((float)TF_HD);
    for (int l = 0; l < TF_LAYERS; l++) {
        const TfLayer *w = &c->tf[l];
        rmsnorm(h, rows, TF_DIM, w->in_norm, TF_EPS, n);
        gemm(n, rows, TF_DIM, w->wq, TF_QKV, NULL, q);
        gemm(n, rows, TF_DIM, w->wk, TF_QKV, NULL, k);
        gemm(n, rows, TF_DIM, w->wv, TF_QKV, NULL, v);
        rope(q, rows, cs, sn);
        rope(k, rows, cs, sn);
        memcpy(c->keys[l] + row0 * TF_QKV, k, R * TF_QKV * 4);
        memcpy(c->values[l] + row0 * TF_QKV, v, R * TF_QKV * 4);
#pragma omp parallel for collapse(2) schedule(static)
        for (int r = 0; r < rows; r++)
            for (int hh = 0; hh < TF_HEADS; hh++) {
                /* frame p sees p - 71 .. p */
                const long long p = c->frames + r;
                long long first = p - (TF_WINDOW - 1);
                if (first < 0) first = 0;
                const int nk = (int)(p - first + 1);
                const float *qr = q + (size_t)r * TF_QKV + hh * TF_HD;
                float sc[TF_WINDOW], mx = -INFINITY;
                for (int j = 0; j < nk; j++) {
                    const float *kr = c->keys[l] + (size_t)(first - c->cache_base + j) * TF_QKV + hh * TF_HD;
                    sc[j] = dot(qr, kr, TF_HD) * scale;
                    mx = sc[j] > mx ? sc[j] : mx;
                }
                float sum = 0.0f;
                for (int j = 0; j < nk; j++) {
                    sc[j] = expf(sc[j] - mx);
                    sum += sc[j];
                }
                float *ar = att + (size_t)r * TF_QKV + hh * TF_HD;
                for (int d = 0; d < TF_HD; d++) ar[d] = 0.0f;
                for (int j = 0; j < nk; j++) {
                    const float *vr = c->values[l] + (size_t)(first - c->cache_base + j) * TF_QKV + hh * TF_HD;
                    const float pj = sc[j] / sum;
                    for (int d = 0; d < TF_HD; d++) ar[d] += pj * vr[d];
                }
            }
        gemm(att, rows, TF_QKV, w->wo, TF_DIM, NULL, o);
        for (size_t i = 0; i < R * TF_DIM; i++) h[i] += w->attn_scale[i % TF_DIM] * o[i];
        rmsnorm(h, rows, TF_DIM, w->post_norm, TF_EPS, n);
        gemm(n, rows, TF_DIM, w->wg, TF_MLP, NULL, g);
        gemm(n, rows, TF_DIM, w->wu, TF_MLP, NULL, u);
        for (size_t i = 0; i < R * TF_MLP; i++) g[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
        gemm(g, rows, TF_MLP, w->wd, TF_DIM, NULL, o);
        for (size_t i = 0; i < R * TF_DIM; i++) h[i] += w->mlp_scale[i % TF_DIM] * o[i];
    }
    rmsnorm(h, rows, TF_DIM, c->tf_norm, TF_EPS, n);
    gemm(n, rows, TF_DIM, c->tf_out, LATENT, c->tf_out_b, y);
    free(h), free(n), free(q), free(k), free(v), free(att), free(o), free(g), free(u), free(cs), free(sn);
    return 0;
}

void ora_codec_free(ora_codec *c);

ora_codec *ora_codec_create(int n, const char *const *names, const float *const *ptrs, const int64_t *counts) {
    Table t = {n, names, ptrs, counts, 0};
    ora_codec *c = calloc(1, sizeof(ora_codec));
    char p[256];
    c->codebook = malloc((size_t)CG * CB * CODE_DIM * sizeof(float));
    for (int g = 0; g < CG && !t.bad; g++) {
        char s[512], u[512];
        if (g == 0)
            snprintf(p, sizeof p, "decoder.quantizer.rvq_first.vq.layers.0._codebook");
        else
            snprintf(p, sizeof p, "decoder.quantizer.rvq_rest.vq.layers.%d._codebook", g - 1);
        snprintf(s, sizeof s, "%s.embedding_sum", p);
        snprintf(u, sizeof u, "%s.cluster_usage", p);
        const float *sum = w_get(&t, s, (int64_t)CB * CODE_DIM), *use = w_get(&t, u, CB);
        if (!sum || !use) break;
        for (int i = 0; i < CB; i++) {
            const float d = use[i] < 1e-5f ? 1e-5f : use[i];
            for (int ch = 0; ch < CODE_DIM; ch++)
                c->codebook[((size_t)g * CB + i) * CODE_DIM + ch] = sum[(size_t)i * CODE_DIM + ch] / d;
        }
    }
    c->first_proj = w_get(&t, "decoder.quantizer.rvq_first.output_proj.weight", (int64_t)QUANT_DIM * CODE_DIM);
    c->rest_proj = w_get(&t, "decoder.quantizer.rvq_rest.output_proj.weight", (int64_t)QUANT_DIM * CODE_DIM);
    conv_init(&c->pre, &t, "decoder.pre_conv.conv", QUANT_DIM, LATENT, 3, 1);
    c->tf_in = w_get(&t, "decoder.pre_transformer.input_proj.weight", (int64_t)TF_DIM * LATENT);
    c->tf_in_b = w_get(&t, "decoder.pre_transformer.input_proj.bias", TF_DIM);
    c->tf_out = w_get(&t, "decoder.pre_transformer.output_proj.weight", (int64_t)LATENT * TF_DIM);
    c->tf_out_b = w_get(&t, "decoder.pre_transformer.output_proj.bias", LATENT);
    c->tf_norm = w_get(&t, "decoder.pre_transformer.norm.weight", TF_DIM);
    for (int l = 0; l < TF_LAYERS; l++) {
        TfLayer *w = &c->tf[l];
#define L(field, suffix, count)                                                     \
    snprintf(p, sizeof p, "decoder.pre_transformer.layers.%d.%s", l, suffix);      \
    w->field = w_get(&t, p, count);
        L(in_norm, "input_layernorm.weight", TF_DIM)
        L(wq, "self_attn.q_proj.weight", (int64_t)TF_QKV * TF_DIM)
        L(wk, "self_attn.k_proj.weight", (int64_t)TF_QKV * TF_DIM)
        L(wv, "self_attn.v_proj.weight", (int64_t)TF_QKV * TF_DIM)
        L(wo, "self_attn.o_proj.weight", (int64_t)TF_DIM * TF_QKV)
        L(post_norm, "post_attention_layernorm.weight", TF_DIM)
        L(wg, "mlp.gate_proj.weight", (int64_t)TF_MLP * TF_DIM)
        L(wu, "mlp.up_proj.weight", (int64_t)TF_MLP * TF_DIM)
        L(wd, "mlp.down_proj.weight", (int64_t)TF_DIM * TF_MLP)
        L(attn_scale, "self_attn_layer_scale.scale", TF_DIM)
        L(mlp_scale, "mlp_layer_scale.scale", TF_DIM)
#undef L
    }
    /* RoPE base 10000: inv_freq_i = 1 / 10000^(2i/64), rounded to float32 */
    for (int i = 0; i < TF_HD / 2; i++) c->inv_freq[i] = (float)(1.0 / exp(log(10000.0) * (2.0 * i / TF_HD)));
    for (int i = 0; i < 2; i++) {
        snprintf(p, sizeof p, "decoder.upsample.%d.0.conv", i);
        tconv_init(&c->up[i], &t, p, LATENT, LATENT, 2, 2);
        snprintf(p, sizeof p, "decoder.upsample.%d.1", i);
        next_init(&c->next[i], &t, p, LATENT);
    }
    conv_init(&c->conv0, &t, "decoder.decoder.0.conv", LATENT, DEC_DIM, 7, 1);
    static const int rates[4] = {8, 5, 4, 3}, dil[3] = {1, 3, 9};
    for (int b = 0; b < 4; b++) {
        Block *k = &c->blocks[b];
        k->in = DEC_DIM >> b, k->out = DEC_DIM >> (b + 1), k->rate = rates[b];
        snprintf(p, sizeof p, "decoder.decoder.%d.block.0", b + 1);
        snake_init(&k->act, &t, p, k->in);
        snprintf(p, sizeof p, "decoder.decoder.%d.block.1.conv", b + 1);
        tconv_init(&k->up, &t, p, k->in, k->out, 2 * k->rate, k->rate);
        for (int r = 0; r < 3; r++) {
            Res *u = &k->res[r];
            u->dim = k->out;
            snprintf(p, sizeof p, "decoder.decoder.%d.block.%d.act1", b + 1, r + 2);
            snake_init(&u->a1, &t, p, k->out);
            snprintf(p, sizeof p, "decoder.decoder.%d.block.%d.conv1.conv", b + 1, r + 2);
            conv_init(&u->c1, &t, p, k->out, k->out, 7, dil[r]);
            snprintf(p, sizeof p, "decoder.decoder.%d.block.%d.act2", b + 1, r + 2);
            snake_init(&u->a2, &t, p, k->out);
            snprintf(p, sizeof p, "decoder.decoder.%d.block.%d.conv2.conv", b + 1, r + 2);
            conv_init(&u->c2, &t, p, k->out, k->out, 1, 1);
        }
    }
    snake_init(&c->act_out, &t, "decoder.decoder.5", DEC_DIM >> 4);
    conv_init(&c->conv_out, &t, "decoder.decoder.6.conv", DEC_DIM >> 4, 1, 7, 1);
    if (t.bad) {
        ora_codec_free(c);
        return NULL;
    }
    return c;
}

void ora_codec_reset(ora_codec *c) {
    c->frames = 0;
    c->cache_base = 0;
    conv_reset(&c->pre);
    for (int i = 0; i < 2; i++) tconv_reset(&c->up[i]), next_reset(&c->next[i]);
    conv_reset(&c->conv0);
    for (int b = 0; b < 4; b++) {
        tconv_reset(&c->blocks[b].up);
        for (int r = 0; r < 3; r++) conv_reset(&c->blocks[b].res[r].c1), conv_reset(&c->blocks[b].res[r].c2);
    }
    conv_reset(&c->conv_out);
}

long long ora_codec_frames(const ora_codec *c) { return c->frames; }

/* TQwenCodec.Decode (codec.pas:1019-1038): codes[frames][16] -> pcm
 * [frames * 1920]; 0 on success, -1 on a code >= 2048 (negative codes
 * clamp to 0) or an allocation failure */
int ora_codec_decode(ora_codec *c, const int32_t *codes, int frames, float *pcm) {
    if (frames <= 0) return 0;
    for (int i = 0; i < frames * CG; i++)
        if (codes[i] >= CB) {
            snprintf(g_err, sizeof g_err, "code %d out of range in group %d", codes[i], i % CG);
            return -1;
        }
    const size_t F = (size_t)frames;
    const size_t big = F * FRAME_SAMPLES * (DEC_DIM >> 4) > F * 4 * DEC_DIM ? F * FRAME_SAMPLES * (DEC_DIM >> 4)
                                                                            : F * 4 * DEC_DIM;
    float *a = malloc(big * 4 * 2), *b = malloc(big * 4 * 2);
    float *q1 = malloc(F * CODE_DIM * 4), *q2 = malloc(F * CODE_DIM * 4), *t = malloc(F * QUANT_DIM * 4);
    /* quantizer: q1 = codebook 0, q2 = the sum of codebooks 1..15 in order */
    for (size_t f = 0; f < F; f++)
        for (int g = 0; g < CG; g++) {
            int code = codes[f * CG + g];
            if (code < 0) code = 0;
            const float *e = c->codebook + ((size_t)g * CB + code) * CODE_DIM;
            if (g == 0)
                memcpy(q1 + f * CODE_DIM, e, CODE_DIM * 4);
            else if (g == 1)
                memcpy(q2 + f * CODE_DIM, e, CODE_DIM * 4);
            else
                for (int ch = 0; ch < CODE_DIM; ch++) q2[f * CODE_DIM + ch] += e[ch];
        }
    gemm(q1, frames, CODE_DIM, c->first_proj, QUANT_DIM, NULL, a);
    gemm(q2, frames, CODE_DIM, c->rest_proj, QUANT_DIM, NULL, t);
    for (size_t i = 0; i < F * QUANT_DIM; i++) a[i] += t[i];
    conv_fwd(&c->pre, a, frames, b);
    if (transformer(c, b, frames, a)) return -1;
    /* the back part (TQwenCodec.Back, codec.pas:1040-1084) */
    int rows = frames;
    for (int i = 0; i < 2; i++) {
        tconv_fwd(&c->up[i], a, rows, b);
        rows *= 2;
        next_fwd(&c->next[i], b, rows, a);
    }
    conv_fwd(&c->conv0, a, rows, b);
    for (int k = 0; k < 4; k++) {
        Block *bl = &c->blocks[k];
        snake_fwd(&bl->act, b, rows);
        tconv_fwd(&bl->up, b, rows, a);
        rows *= bl->rate;
        for (int r = 0; r < 3; r++) {
            Res *u = &bl->res[r];
            const size_t n = (size_t)rows * u->dim;
            float *x1 = malloc(n * 4), *x2 = malloc(n * 4);
            memcpy(x1, a, n * 4);
            snake_fwd(&u->a1, x1, rows);
            conv_fwd(&u->c1, x1, rows, x2);
            snake_fwd(&u->a2, x2, rows);
            conv_fwd(&u->c2, x2, rows, x1);
            for (size_t i = 0; i < n; i++) a[i] = x1[i] + a[i];
            free(x1), free(x2);
        }
        float *s = a;
        a = b, b = s;
    }
    snake_fwd(&c->act_out, b, rows);
    conv_fwd(&c->conv_out, b, rows, a);
    for (int i = 0; i < rows; i++) pcm[i] = a[i] > 1.0f ? 1.0f : (a[i] < -1.0f ? -1.0f : a[i]);
    c->frames += frames;
    free(a), free(b), free(q1), free(q2), free(t);
    return 0;
}

void ora_codec_free(ora_codec *c) {
    if (!c) return;
    free(c->codebook);
    for (int l = 0; l < TF_LAYERS; l++) free(c->keys[l]), free(c->values[l]);
    free(c->pre.hist);
    for (int i = 0; i < 2; i++) free(c->up[i].w), free(c->up[i].b), free(c->up[i].hist), free(c->next[i].hist);
    free(c->conv0.hist);
    for (int b = 0; b < 4; b++) {
        Block *k = &c->blocks[b];
        free(k->act.alpha), free(k->act.inv_beta), free(k->up.w), free(k->up.b), free(k->up.hist);
        for (int r = 0; r < 3; r++) {
            Res *u = &k->res[r];
            free(u->a1.alpha), free(u->a1.inv_beta), free(u->a2.alpha), free(u->a2.inv_beta);
            free(u->c1.hist), free(u->c2.hist);
        }
    }
    free(c->act_out.alpha), free(c->act_out.inv_beta), free(c->conv_out.hist);
    free(c);
}
