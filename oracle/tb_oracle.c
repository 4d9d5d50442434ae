/*
 * tb_oracle.c -- CPU restatement of TinyBrain's quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and timed CPU baseline for
 * libtinybrain_cuda.  Never linked into, loaded by or called from the product.
 *
 * Each function names the Swift source it restates (paths relative to the
 * vivekptnk/tinybrain project root).  Arithmetic is fp32 in the reference's
 * order wherever the reference is scalar Swift; the only place the reference
 * delegates to a closed library is the fp32 GEMM (Accelerate cblas_sgemm,
 * Tensor.swift:850-858), whose summation order is unspecified.  That boundary
 * is "parity unpinned": mode 0 restates it as a sequential-k fp32 sum over the
 * fully dequantized weight (what the reference materialises), mode 1 as an
 * fp64 sum (the "truth" the GPU path is compared against).
 *
 * Compile without -ffast-math: the quantizers depend on IEEE division and
 * round-half-away-from-zero (roundf), exactly as Swift's `/` and `round`.
 */
#include "tb_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void orc_set_threads(int32_t n) {
    g_threads = n;
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}

int32_t orc_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* Float.leastNonzeroMagnitude */
#define ORC_FLT_TRUE_MIN 1.40129846e-45f

/* ------------------------------------------------------------------------ */
/* Quantization                                                              */
/* ------------------------------------------------------------------------ */

/* QuantizedTensor.swift:379-424 (quantizePerChannel): one scale per output
 * column n of the [K (in), N (out)] row-major weight; scale = absMax/127 (1 for
 * an all-zero column); q = clamp(round(w/scale), -127, 127). */
void orc_quantize_int8_per_channel(const float *W, int64_t K, int64_t N,
                                   int8_t *Q, float *scales) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        float absmax = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            float v = fabsf(W[k * N + n]);
            if (v > absmax) absmax = v;
        }
        scales[n] = (absmax < ORC_FLT_TRUE_MIN) ? 1.0f : absmax / 127.0f;
    }
#pragma omp parallel for schedule(static)
    for (int64_t k = 0; k < K; ++k) {
        for (int64_t n = 0; n < N; ++n) {
            float q = roundf(W[k * N + n] / scales[n]);
            q = fmaxf(-127.0f, fminf(127.0f, q));
            Q[k * N + n] = (int8_t)q;
        }
    }
}

/* QuantizedTensor.swift:502-560 (quantizeINT4): flat groups of group_size
 * elements; absMax = max(|min|, |max|); scale = absMax/7 (1 if zero);
 * q = clamp(round(x/scale), -7, 7); even flat index -> high nibble, odd -> low
 * nibble; zero point 0.  Packed length is ceil(count/2). */
void orc_quantize_int4_group(const float *x, int64_t count, int64_t gs,
                             uint8_t *packed, float *scales, int8_t *zp) {
    int64_t ngroups = (count + gs - 1) / gs;
    /* A group may share its first/last byte with a neighbour when gs is odd;
     * run groups in order within a thread's block and split blocks on even
     * element boundaries so no byte is written by two threads. */
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < ngroups; ++g) {
        int64_t start = g * gs, end = start + gs < count ? start + gs : count;
        float mn = x[start], mx = x[start];
        for (int64_t i = start + 1; i < end; ++i) {
            if (x[i] < mn) mn = x[i];
            if (x[i] > mx) mx = x[i];
        }
        float a = fabsf(mn), b = fabsf(mx);
        float absmax = a > b ? a : b;
        float s = (absmax < ORC_FLT_TRUE_MIN) ? 1.0f : absmax / 7.0f;
        scales[g] = s;
        if (zp) zp[g] = 0;
        if (gs % 2 == 0) {
            for (int64_t i = start; i < end; ++i) {
                float q = roundf(x[i] / s);
                int8_t c = (int8_t)fmaxf(-7.0f, fminf(7.0f, q));
                if ((i & 1) == 0)
                    packed[i >> 1] = (uint8_t)((c & 0x0F) << 4);
                else
                    packed[i >> 1] |= (uint8_t)(c & 0x0F);
            }
        }
    }
    if (gs % 2 != 0) { /* odd group size: sequential pack (groups share bytes) */
        for (int64_t i = 0; i < count; ++i) {
            float s = scales[i / gs];
            float q = roundf(x[i] / s);
            int8_t c = (int8_t)fmaxf(-7.0f, fminf(7.0f, q));
            if ((i & 1) == 0)
                packed[i >> 1] = (uint8_t)((c & 0x0F) << 4);
            else
                packed[i >> 1] |= (uint8_t)(c & 0x0F);
        }
    }
}

/* QuantizedTensor.swift:241-255: w = (q - zp[n]) * scale[n], column scale. */
void orc_dequantize_int8_per_channel(const int8_t *Q, const float *scales,
                                     const int8_t *zp, int64_t K, int64_t N,
                                     float *W) {
#pragma omp parallel for schedule(static)
    for (int64_t k = 0; k < K; ++k)
        for (int64_t n = 0; n < N; ++n)
            W[k * N + n] = ((float)Q[k * N + n] - (float)(zp ? zp[n] : 0)) * scales[n];
}

static inline int8_t orc_nibble(const uint8_t *packed, int64_t i) {
    /* QuantizedTensor.swift:195-212: high nibble for even i, sign-extend > 7 */
    uint8_t raw = (i & 1) == 0 ? (uint8_t)((packed[i >> 1] >> 4) & 0x0F)
                               : (uint8_t)(packed[i >> 1] & 0x0F);
    return raw > 7 ? (int8_t)(raw - 16) : (int8_t)raw;
}

/* QuantizedTensor.swift:186-216: w = (nibble - zp[g]) * scale[g], g = i/gs. */
void orc_dequantize_int4_group(const uint8_t *packed, const float *scales,
                               const int8_t *zp, int64_t count, int64_t gs,
                               float *W) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i) {
        int64_t g = i / gs;
        W[i] = ((float)orc_nibble(packed, i) - (float)(zp ? zp[g] : 0)) * scales[g];
    }
}

/* ------------------------------------------------------------------------ */
/* Quantized matmul                                                          */
/* ------------------------------------------------------------------------ */

static inline float orc_wval(const orc_qtensor *w, int64_t k, int64_t n) {
    int64_t i = k * w->N + n;
    if (w->precision == 8) {
        const int8_t *q = (const int8_t *)w->data;
        return ((float)q[i] - (float)(w->zero_points ? w->zero_points[n] : 0)) * w->scales[n];
    }
    int64_t g = i / w->group_size;
    return ((float)orc_nibble((const uint8_t *)w->data, i) -
            (float)(w->zero_points ? w->zero_points[g] : 0)) * w->scales[g];
}

/* QuantizedTensor.swift:627-643 CPU branch: dequantize() then matmulCPU
 * (Tensor.swift:839-861, cblas_sgemm RowMajor NoTrans/NoTrans, alpha 1 beta 0). */
void orc_qmatmul(const float *x, int64_t M, const orc_qtensor *w, float *y,
                 int mode) {
    const int64_t K = w->K, N = w->N;
    if (mode == 0) {
        float *Wf = (float *)malloc(sizeof(float) * (size_t)(K * N));
        if (w->precision == 8)
            orc_dequantize_int8_per_channel((const int8_t *)w->data, w->scales,
                                            w->zero_points, K, N, Wf);
        else
            orc_dequantize_int4_group((const uint8_t *)w->data, w->scales,
                                      w->zero_points, K * N, w->group_size, Wf);
        for (int64_t m = 0; m < M; ++m) {
            const float *xr = x + m * K;
            float *yr = y + m * N;
#pragma omp parallel for schedule(static)
            for (int64_t nb = 0; nb < N; nb += 256) {
                int64_t ne = nb + 256 < N ? nb + 256 : N;
                float acc[256];
                for (int64_t n = nb; n < ne; ++n) acc[n - nb] = 0.0f;
                for (int64_t k = 0; k < K; ++k) {
                    const float xv = xr[k];
                    const float *wr = Wf + k * N;
                    for (int64_t n = nb; n < ne; ++n) acc[n - nb] += xv * wr[n];
                }
                for (int64_t n = nb; n < ne; ++n) yr[n] = acc[n - nb];
            }
        }
        free(Wf);
        return;
    }
    /* mode 1: fp64 accumulation of x[k] * fp32(dequant(w[k][n])) */
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * K;
        float *yr = y + m * N;
#pragma omp parallel for schedule(static)
        for (int64_t nb = 0; nb < N; nb += 256) {
            int64_t ne = nb + 256 < N ? nb + 256 : N;
            double acc[256];
            for (int64_t n = nb; n < ne; ++n) acc[n - nb] = 0.0;
            if (w->precision == 8) {
                const int8_t *q = (const int8_t *)w->data;
                for (int64_t k = 0; k < K; ++k) {
                    const double xv = (double)xr[k];
                    const int8_t *qr = q + k * N;
                    for (int64_t n = nb; n < ne; ++n) {
                        float wv = ((float)qr[n] - (float)(w->zero_points ? w->zero_points[n] : 0)) *
                                   w->scales[n];
                        acc[n - nb] += xv * (double)wv;
                    }
                }
            } else {
                for (int64_t k = 0; k < K; ++k) {
                    const double xv = (double)xr[k];
                    for (int64_t n = nb; n < ne; ++n)
                        acc[n - nb] += xv * (double)orc_wval(w, k, n);
                }
            }
            for (int64_t n = nb; n < ne; ++n) yr[n] = (float)acc[n - nb];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Elementwise ops                                                           */
/* ------------------------------------------------------------------------ */

/* Tensor.swift:1538-1558 (rmsNormCPU): sequential fp32 sum of squares,
 * invRMS = 1 / sqrt(ss/H + eps), y = x * invRMS * w. */
void orc_rmsnorm(const float *x, const float *w, int64_t H, float eps, float *y) {
    float ss = 0.0f;
    for (int64_t i = 0; i < H; ++i) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)H + eps);
    for (int64_t i = 0; i < H; ++i) y[i] = x[i] * inv * w[i];
}

/* Tensor.swift:1135-1142 (siluCPU) */
float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* Tensor.swift:1107-1121 (geluCPU): tanh approximation. */
float orc_gelu(float x) {
    const float s = sqrtf(2.0f / 3.14159265358979323846f);
    float x3 = x * x * x;
    float inner = s * (x + 0.044715f * x3);
    return 0.5f * x * (1.0f + tanhf(inner));
}

/* Tensor.swift:1281-1295 (softmaxCPU): exp(x - max) / (sum + 1e-7). */
void orc_softmax(const float *x, int64_t n, float *y) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; ++i)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        y[i] = expf(x[i] - mx);
        sum += y[i];
    }
    for (int64_t i = 0; i < n; ++i) y[i] = y[i] / (sum + 1e-7f);
}

/* ModelRunner.swift:470-494 (applyRoPE): adjacent pairs (i, i+1), theta =
 * 10000^(-i/rDims) in fp32, angle = Float(position) * theta. */
void orc_rope(float *v, int64_t head_dim, int64_t num_heads, int64_t position,
              int64_t rotary_dims) {
    for (int64_t h = 0; h < num_heads; ++h) {
        float *p = v + h * head_dim;
        for (int64_t i = 0; i < rotary_dims; i += 2) {
            float freq = (float)i / (float)rotary_dims;
            float theta = powf(10000.0f, -freq);
            float angle = (float)position * theta;
            float c = cosf(angle), s = sinf(angle);
            float x0 = p[i], x1 = p[i + 1];
            p[i] = x0 * c - x1 * s;
            p[i + 1] = x0 * s + x1 * c;
        }
    }
}

/* ModelRunner.swift:519-579, one query head: scores are fp32 sequential dots
 * times 1/sqrt(d); softmax without epsilon; the context is the fp32
 * sequential p-weighted sum of V rows.  sc: L floats of scratch. */
static void attn_head(const float *qh, const float *K, const float *V, int64_t L, int64_t kvdim, int64_t kvh,
                      int64_t d, float scale, float *sc, float *ch, float *probs) {
    for (int64_t j = 0; j < L; ++j) {
        float dot = 0.0f;
        const float *kr = K + j * kvdim + kvh * d;
        for (int64_t t = 0; t < d; ++t) dot += qh[t] * kr[t];
        sc[j] = dot * scale;
    }
    float mx = L > 0 ? sc[0] : 0.0f;
    for (int64_t j = 1; j < L; ++j)
        if (sc[j] > mx) mx = sc[j];
    float sum = 0.0f;
    for (int64_t j = 0; j < L; ++j) {
        sc[j] = expf(sc[j] - mx);
        sum += sc[j];
    }
    for (int64_t j = 0; j < L; ++j) sc[j] = sc[j] / sum;
    if (probs) memcpy(probs, sc, sizeof(float) * (size_t)L);
    for (int64_t t = 0; t < d; ++t) ch[t] = 0.0f;
    for (int64_t j = 0; j < L; ++j) {
        const float w = sc[j];
        const float *vr = V + j * kvdim + kvh * d;
        for (int64_t t = 0; t < d; ++t) ch[t] += w * vr[t];
    }
}

/* ModelRunner.swift:519-579: per head, kvHead = head / (H/Hkv).  Heads are
 * independent, so they run in parallel for long contexts (same results). */
void orc_attention(const float *q, const float *K, const float *V, int64_t L,
                   int64_t H, int64_t Hkv, int64_t d, float *ctx, float *probs) {
    const float scale = 1.0f / sqrtf((float)d);
    const int64_t rep = H / Hkv, kvdim = Hkv * d;
#pragma omp parallel if (L * H >= 65536)
    {
        float *sc = (float *)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
#pragma omp for schedule(static)
        for (int64_t h = 0; h < H; ++h)
            attn_head(q + h * d, K, V, L, kvdim, h / rep, d, scale, sc, ctx + h * d, probs ? probs + h * L : NULL);
        free(sc);
    }
}

/* Sampler.swift:126-138 (greedy): first index with the strict maximum. */
int64_t orc_greedy(const float *logits, int64_t V) {
    int64_t best = 0;
    float bv = -INFINITY;
    for (int64_t i = 0; i < V; ++i)
        if (logits[i] > bv) {
            bv = logits[i];
            best = i;
        }
    return best;
}

/* ------------------------------------------------------------------------ */
/* Model and runner                                                          */
/* ------------------------------------------------------------------------ */

typedef struct {
    int has;
    orc_qtensor w;
    const float *bias;
} orc_proj;

typedef struct {
    orc_proj p[ORC_NPROJ];
    const float *in_norm, *post_norm;
} orc_layer;

struct orc_model {
    orc_config cfg;
    const float *emb;
    const float *final_norm;
    orc_proj out;
    orc_layer *layers;
};

orc_model *orc_model_create(const orc_config *cfg) {
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->cfg = *cfg;
    if (m->cfg.rms_eps == 0.0f) m->cfg.rms_eps = 1e-5f;
    m->layers = (orc_layer *)calloc((size_t)cfg->num_layers, sizeof(orc_layer));
    return m;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    free(m->layers);
    free(m);
}

void orc_model_set_embedding(orc_model *m, const float *emb) { m->emb = emb; }
void orc_model_set_final_norm(orc_model *m, const float *w) { m->final_norm = w; }
void orc_model_set_output(orc_model *m, const orc_qtensor *w, const float *bias) {
    m->out.has = 1;
    m->out.w = *w;
    m->out.bias = bias;
}
void orc_model_set_layer_norms(orc_model *m, int64_t layer, const float *in_norm,
                               const float *post_norm) {
    m->layers[layer].in_norm = in_norm;
    m->layers[layer].post_norm = post_norm;
}
void orc_model_set_proj(orc_model *m, int64_t layer, int32_t which,
                        const orc_qtensor *w, const float *bias) {
    orc_proj *p = &m->layers[layer].p[which];
    p->has = w != NULL;
    if (w) p->w = *w;
    p->bias = bias;
}

/* KVCache.swift:108-325 with PageAllocator.swift:35-152: per layer a pool of
 * maxPages pages of pageSize rows, a LIFO free list, a logical-page map, and
 * FIFO eviction of the lowest logical page once length reaches maxTokens. */
typedef struct {
    float *kpool, *vpool;     /* [max_pages][page][kvdim] */
    int64_t *free_stack;      /* LIFO */
    int64_t nfree;
    int64_t *map;             /* logical page -> pool index, -1 = absent */
    int64_t map_cap;
    int64_t length;
} orc_kvlayer;

struct orc_runner {
    const orc_model *m;
    int mode;
    int64_t pos;
    int64_t page, max_pages, kvdim;
    orc_kvlayer *kv;
    /* scratch */
    float *h, *x, *q, *k, *v, *ctx, *tmp, *ff1, *ff2, *K, *V;
    int64_t kv_gather_cap;
    /* InferenceObserver hooks (InferenceObserver.swift:40-84), NULL = off */
    float *obs_norms;        /* [num_layers] layer-entry ||h||_2 */
    float *obs_attn;         /* [num_layers][attn_stride] = [H][L] per layer */
    int64_t obs_attn_stride;
    float *obs_final;        /* [H] final hidden state (post-norm, pre-projection) */
};

void orc_runner_set_observer(orc_runner *r, float *norms, float *attn, int64_t attn_stride, float *final_hidden) {
    r->obs_norms = norms;
    r->obs_attn = attn;
    r->obs_attn_stride = attn_stride;
    r->obs_final = final_hidden;
}

static void kv_layer_reset(orc_runner *r, orc_kvlayer *L) {
    L->nfree = r->max_pages;
    for (int64_t i = 0; i < r->max_pages; ++i) L->free_stack[i] = r->max_pages - 1 - i;
    for (int64_t i = 0; i < L->map_cap; ++i) L->map[i] = -1;
    L->length = 0;
}

orc_runner *orc_runner_create(const orc_model *m, int32_t mode, int32_t nthreads) {
    if (nthreads > 0) orc_set_threads(nthreads);
    orc_runner *r = (orc_runner *)calloc(1, sizeof(orc_runner));
    const orc_config *c = &m->cfg;
    r->m = m;
    r->mode = mode;
    r->page = 16;
    r->max_pages = (c->max_seq_len + r->page - 1) / r->page;
    r->kvdim = (c->hidden / c->num_heads) * c->num_kv_heads;
    r->kv = (orc_kvlayer *)calloc((size_t)c->num_layers, sizeof(orc_kvlayer));
    for (int64_t l = 0; l < c->num_layers; ++l) {
        orc_kvlayer *L = &r->kv[l];
        size_t n = (size_t)(r->max_pages * r->page * r->kvdim);
        L->kpool = (float *)calloc(n, sizeof(float));
        L->vpool = (float *)calloc(n, sizeof(float));
        L->free_stack = (int64_t *)malloc(sizeof(int64_t) * (size_t)r->max_pages);
        L->map_cap = r->max_pages + 1;
        L->map = (int64_t *)malloc(sizeof(int64_t) * (size_t)L->map_cap);
        kv_layer_reset(r, L);
    }
    int64_t H = c->hidden, I = c->intermediate;
    int64_t big = H > I ? H : I;
    if (c->vocab > big) big = c->vocab;
    r->h = (float *)calloc((size_t)H, sizeof(float));
    r->x = (float *)calloc((size_t)big, sizeof(float));
    r->q = (float *)calloc((size_t)H, sizeof(float));
    r->k = (float *)calloc((size_t)r->kvdim, sizeof(float));
    r->v = (float *)calloc((size_t)r->kvdim, sizeof(float));
    r->ctx = (float *)calloc((size_t)H, sizeof(float));
    r->tmp = (float *)calloc((size_t)big, sizeof(float));
    r->ff1 = (float *)calloc((size_t)big, sizeof(float));
    r->ff2 = (float *)calloc((size_t)big, sizeof(float));
    return r;
}

void orc_runner_free(orc_runner *r) {
    if (!r) return;
    for (int64_t l = 0; l < r->m->cfg.num_layers; ++l) {
        free(r->kv[l].kpool);
        free(r->kv[l].vpool);
        free(r->kv[l].free_stack);
        free(r->kv[l].map);
    }
    free(r->kv);
    free(r->h); free(r->x); free(r->q); free(r->k); free(r->v); free(r->ctx);
    free(r->tmp); free(r->ff1); free(r->ff2); free(r->K); free(r->V);
    free(r);
}

/* ModelRunner.swift:213-217 + KVCache.swift:313-325 */
void orc_runner_reset(orc_runner *r) {
    for (int64_t l = 0; l < r->m->cfg.num_layers; ++l) kv_layer_reset(r, &r->kv[l]);
    r->pos = 0;
}

int64_t orc_runner_position(const orc_runner *r) { return r->pos; }

/* KVCache.swift:138-143: max over layers */
int64_t orc_runner_kv_length(const orc_runner *r) {
    int64_t mx = 0;
    for (int64_t l = 0; l < r->m->cfg.num_layers; ++l)
        if (r->kv[l].length > mx) mx = r->kv[l].length;
    return mx;
}

int64_t orc_runner_max_pages(const orc_runner *r) { return r->max_pages; }

/* KVCache.swift:352-356: status of logical pages 0..maxPages-1 */
void orc_runner_page_status(const orc_runner *r, int64_t layer, uint8_t *status) {
    const orc_kvlayer *L = &r->kv[layer];
    for (int64_t i = 0; i < r->max_pages; ++i)
        status[i] = (i < L->map_cap && L->map[i] >= 0) ? 1 : 0;
}

/* KVCache.swift:293-308 */
static void kv_evict_oldest(orc_runner *r, orc_kvlayer *L) {
    for (int64_t i = 0; i < L->map_cap; ++i) {
        if (L->map[i] >= 0) {
            L->free_stack[L->nfree++] = L->map[i];
            L->map[i] = -1;
            return;
        }
    }
}

/* KVCache.swift:157-224 */
static void kv_append(orc_runner *r, int64_t layer, const float *k, const float *v,
                      int64_t pos) {
    orc_kvlayer *L = &r->kv[layer];
    const int64_t maxTokens = r->m->cfg.max_seq_len;
    while (L->length >= maxTokens) {
        kv_evict_oldest(r, L);
        L->length = L->length - r->page > 0 ? L->length - r->page : 0;
    }
    int64_t pid = pos / r->page, off = pos % r->page;
    if (pid >= L->map_cap) {
        int64_t ncap = pid * 2 + 1;
        L->map = (int64_t *)realloc(L->map, sizeof(int64_t) * (size_t)ncap);
        for (int64_t i = L->map_cap; i < ncap; ++i) L->map[i] = -1;
        L->map_cap = ncap;
    }
    if (L->map[pid] < 0) {
        if (L->nfree == 0) kv_evict_oldest(r, L);
        if (L->nfree == 0) abort(); /* the reference calls fatalError */
        int64_t idx = L->free_stack[--L->nfree];
        memset(L->kpool + idx * r->page * r->kvdim, 0, sizeof(float) * (size_t)(r->page * r->kvdim));
        memset(L->vpool + idx * r->page * r->kvdim, 0, sizeof(float) * (size_t)(r->page * r->kvdim));
        L->map[pid] = idx;
    }
    int64_t base = (L->map[pid] * r->page + off) * r->kvdim;
    memcpy(L->kpool + base, k, sizeof(float) * (size_t)r->kvdim);
    memcpy(L->vpool + base, v, sizeof(float) * (size_t)r->kvdim);
    if (pos + 1 > L->length) L->length = pos + 1;
    if (L->length > maxTokens) L->length = maxTokens;
}

/* KVCache.swift:232-288: rows of absent pages read as zeros */
static void kv_gather(orc_runner *r, int64_t layer, int64_t L_, float *K, float *V) {
    orc_kvlayer *L = &r->kv[layer];
    for (int64_t p = 0; p < L_; ++p) {
        int64_t pid = p / r->page, off = p % r->page;
        if (pid < L->map_cap && L->map[pid] >= 0) {
            int64_t base = (L->map[pid] * r->page + off) * r->kvdim;
            memcpy(K + p * r->kvdim, L->kpool + base, sizeof(float) * (size_t)r->kvdim);
            memcpy(V + p * r->kvdim, L->vpool + base, sizeof(float) * (size_t)r->kvdim);
        } else {
            memset(K + p * r->kvdim, 0, sizeof(float) * (size_t)r->kvdim);
            memset(V + p * r->kvdim, 0, sizeof(float) * (size_t)r->kvdim);
        }
    }
}

/* ModelWeights.swift:48-68 (LinearLayerWeights.apply): x*W then + bias. */
static void apply_proj(const orc_runner *r, const orc_proj *p, const float *x, float *y) {
    orc_qmatmul(x, 1, &p->w, y, r->mode);
    if (p->bias)
        for (int64_t n = 0; n < p->w.N; ++n) y[n] += p->bias[n];
}

/* ModelRunner.swift:168-208 (step), 392-459 (applyLayer, LLaMA and toy
 * branches), 496-592 (attention). */
void orc_runner_step(orc_runner *r, int64_t token, float *logits) {
    const orc_model *m = r->m;
    const orc_config *c = &m->cfg;
    const int64_t H = c->hidden, d = c->hidden / c->num_heads;
    const int64_t L_ = r->pos + 1;
    if (L_ > r->kv_gather_cap) {
        r->kv_gather_cap = L_ * 2;
        free(r->K);
        free(r->V);
        r->K = (float *)malloc(sizeof(float) * (size_t)(r->kv_gather_cap * r->kvdim));
        r->V = (float *)malloc(sizeof(float) * (size_t)(r->kv_gather_cap * r->kvdim));
    }
    memcpy(r->h, m->emb + token * H, sizeof(float) * (size_t)H);
    for (int64_t l = 0; l < c->num_layers; ++l) {
        const orc_layer *ly = &m->layers[l];
        if (r->obs_norms) { /* ModelRunner.swift:395-399: sqrt(reduce(0) { $0 + $1*$1 }) */
            float ss = 0.0f;
            for (int64_t i = 0; i < H; ++i) ss = ss + r->h[i] * r->h[i];
            r->obs_norms[l] = sqrtf(ss);
        }
        const float *xin = r->h;
        if (ly->in_norm) {
            orc_rmsnorm(r->h, ly->in_norm, H, c->rms_eps, r->x);
            xin = r->x;
        }
        apply_proj(r, &ly->p[ORC_Q], xin, r->q);
        apply_proj(r, &ly->p[ORC_K], xin, r->k);
        apply_proj(r, &ly->p[ORC_V], xin, r->v);
        orc_rope(r->q, d, c->num_heads, r->pos, d);
        orc_rope(r->k, d, c->num_kv_heads, r->pos, d);
        kv_append(r, l, r->k, r->v, r->pos);
        kv_gather(r, l, L_, r->K, r->V);
        /* ModelRunner.swift:582-586: weights flattened numHeads x seqLen */
        orc_attention(r->q, r->K, r->V, L_, c->num_heads, c->num_kv_heads, d, r->ctx,
                      r->obs_attn ? r->obs_attn + l * r->obs_attn_stride : NULL);
        apply_proj(r, &ly->p[ORC_O], r->ctx, r->tmp);
        for (int64_t i = 0; i < H; ++i) r->h[i] = r->h[i] + r->tmp[i]; /* residual1 */
        const float *x2 = r->h;
        if (ly->post_norm) {
            orc_rmsnorm(r->h, ly->post_norm, H, c->rms_eps, r->x);
            x2 = r->x;
        }
        if (ly->p[ORC_GATE].has) {
            const int64_t I = ly->p[ORC_GATE].w.N;
            apply_proj(r, &ly->p[ORC_GATE], x2, r->ff1);
            apply_proj(r, &ly->p[ORC_UP], x2, r->ff2);
            for (int64_t i = 0; i < I; ++i) r->ff1[i] = orc_silu(r->ff1[i]) * r->ff2[i];
        } else {
            const int64_t I = ly->p[ORC_UP].w.N;
            apply_proj(r, &ly->p[ORC_UP], x2, r->ff1);
            for (int64_t i = 0; i < I; ++i) r->ff1[i] = orc_gelu(r->ff1[i]);
        }
        apply_proj(r, &ly->p[ORC_DOWN], r->ff1, r->tmp);
        for (int64_t i = 0; i < H; ++i) r->h[i] = r->h[i] + r->tmp[i];
    }
    const float *hf = r->h;
    if (m->final_norm) {
        orc_rmsnorm(r->h, m->final_norm, H, c->rms_eps, r->x);
        hf = r->x;
    }
    if (r->obs_final) memcpy(r->obs_final, hf, sizeof(float) * (size_t)H); /* ModelRunner.swift:195 */
    apply_proj(r, &m->out, hf, logits);
    r->pos += 1;
}

/* Mode 1 matmul of M rows at once (chunked prefill): per row exactly the
 * arithmetic of orc_qmatmul mode 1 (fp64 sum over ascending k of x[k] *
 * fp32(dequant w[k][n])), with each dequantized weight reused across rows. */
#define ORC_NB 64
static void qmatmul_rows_f64(const float *x, int64_t M, const orc_qtensor *w, float *y) {
    const int64_t K = w->K, N = w->N;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t nb = 0; nb < N; nb += ORC_NB) {
        const int64_t ne = nb + ORC_NB < N ? nb + ORC_NB : N, nn = ne - nb;
        double *acc = (double *)calloc((size_t)(M * ORC_NB), sizeof(double));
        float wv[ORC_NB];
        for (int64_t k = 0; k < K; ++k) {
            if (w->precision == 8) {
                const int8_t *qr = (const int8_t *)w->data + k * N;
                for (int64_t j = 0; j < nn; ++j) {
                    const int64_t n = nb + j;
                    wv[j] = ((float)qr[n] - (float)(w->zero_points ? w->zero_points[n] : 0)) * w->scales[n];
                }
            } else {
                for (int64_t j = 0; j < nn; ++j) wv[j] = orc_wval(w, k, nb + j);
            }
            for (int64_t m = 0; m < M; ++m) {
                const double xv = (double)x[m * K + k];
                double *a = acc + m * ORC_NB;
                for (int64_t j = 0; j < nn; ++j) a[j] += xv * (double)wv[j];
            }
        }
        for (int64_t m = 0; m < M; ++m)
            for (int64_t j = 0; j < nn; ++j) y[m * N + nb + j] = (float)acc[m * ORC_NB + j];
        free(acc);
    }
}

static void apply_proj_rows(const orc_runner *r, const orc_proj *p, const float *x, int64_t M, float *y) {
    qmatmul_rows_f64(x, M, &p->w, y);
    if (p->bias)
        for (int64_t m = 0; m < M; ++m)
            for (int64_t n = 0; n < p->w.N; ++n) y[m * p->w.N + n] += p->bias[n];
}

/* Prompt processing for test fixtures: the same results, bit for bit, as
 * calling orc_runner_step for each token and discarding the logits (the
 * reference discards prompt-step logits, ModelRunner.swift:240-244), computed
 * layer by layer over chunks of up to 64 tokens.  Token t of a chunk attends
 * to positions 0..pos+t; its K/V rows are appended before any of the chunk's
 * attention runs, which reads only rows up to its own position.  Runs step by
 * step where the chunk would evict pages, in mode 0, or with an observer. */
void orc_runner_prefill(orc_runner *r, const int64_t *tokens, int64_t n) {
    const orc_model *m = r->m;
    const orc_config *c = &m->cfg;
    if (n <= 0) return;
    if (r->mode != 1 || r->obs_norms || r->obs_attn || r->obs_final || r->pos + n > c->max_seq_len) {
        float *lg = (float *)malloc(sizeof(float) * (size_t)c->vocab);
        for (int64_t i = 0; i < n; ++i) orc_runner_step(r, tokens[i], lg);
        free(lg);
        return;
    }
    const int64_t H = c->hidden, d = c->hidden / c->num_heads, kvd = r->kvdim;
    int64_t I = 0;
    for (int64_t l = 0; l < c->num_layers; ++l) {
        const orc_layer *ly = &m->layers[l];
        const int64_t w = ly->p[ORC_GATE].has ? ly->p[ORC_GATE].w.N : ly->p[ORC_UP].w.N;
        if (w > I) I = w;
    }
    const int64_t T = 64;
    float *h = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *x = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *q = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *k = (float *)malloc(sizeof(float) * (size_t)(T * kvd));
    float *v = (float *)malloc(sizeof(float) * (size_t)(T * kvd));
    float *cx = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(T * H));
    float *f1 = (float *)malloc(sizeof(float) * (size_t)(T * I));
    float *f2 = (float *)malloc(sizeof(float) * (size_t)(T * I));
    const int64_t Lmax = r->pos + n;
    float *K = (float *)malloc(sizeof(float) * (size_t)(Lmax * kvd));
    float *V = (float *)malloc(sizeof(float) * (size_t)(Lmax * kvd));
    const float scale = 1.0f / sqrtf((float)d);
    const int64_t rep = c->num_heads / c->num_kv_heads;
    for (int64_t c0 = 0; c0 < n; c0 += T) {
        const int64_t Tc = n - c0 < T ? n - c0 : T;
        for (int64_t t = 0; t < Tc; ++t) memcpy(h + t * H, m->emb + tokens[c0 + t] * H, sizeof(float) * (size_t)H);
        for (int64_t l = 0; l < c->num_layers; ++l) {
            const orc_layer *ly = &m->layers[l];
            const float *xin = h;
            if (ly->in_norm) {
                for (int64_t t = 0; t < Tc; ++t) orc_rmsnorm(h + t * H, ly->in_norm, H, c->rms_eps, x + t * H);
                xin = x;
            }
            apply_proj_rows(r, &ly->p[ORC_Q], xin, Tc, q);
            apply_proj_rows(r, &ly->p[ORC_K], xin, Tc, k);
            apply_proj_rows(r, &ly->p[ORC_V], xin, Tc, v);
            for (int64_t t = 0; t < Tc; ++t) {
                orc_rope(q + t * H, d, c->num_heads, r->pos + t, d);
                orc_rope(k + t * kvd, d, c->num_kv_heads, r->pos + t, d);
                kv_append(r, l, k + t * kvd, v + t * kvd, r->pos + t);
            }
            kv_gather(r, l, r->pos + Tc, K, V);
#pragma omp parallel
            {
                float *sc = (float *)malloc(sizeof(float) * (size_t)(r->pos + Tc));
#pragma omp for schedule(dynamic, 1) collapse(2)
                for (int64_t t = 0; t < Tc; ++t)
                    for (int64_t hh = 0; hh < c->num_heads; ++hh)
                        attn_head(q + t * H + hh * d, K, V, r->pos + t + 1, kvd, hh / rep, d, scale, sc,
                                  cx + t * H + hh * d, NULL);
                free(sc);
            }
            apply_proj_rows(r, &ly->p[ORC_O], cx, Tc, tmp);
            for (int64_t i = 0; i < Tc * H; ++i) h[i] = h[i] + tmp[i];
            const float *x2 = h;
            if (ly->post_norm) {
                for (int64_t t = 0; t < Tc; ++t) orc_rmsnorm(h + t * H, ly->post_norm, H, c->rms_eps, x + t * H);
                x2 = x;
            }
            int64_t Il;
            if (ly->p[ORC_GATE].has) {
                Il = ly->p[ORC_GATE].w.N;
                apply_proj_rows(r, &ly->p[ORC_GATE], x2, Tc, f1);
                apply_proj_rows(r, &ly->p[ORC_UP], x2, Tc, f2);
                for (int64_t i = 0; i < Tc * Il; ++i) f1[i] = orc_silu(f1[i]) * f2[i];
            } else {
                Il = ly->p[ORC_UP].w.N;
                apply_proj_rows(r, &ly->p[ORC_UP], x2, Tc, f1);
                for (int64_t i = 0; i < Tc * Il; ++i) f1[i] = orc_gelu(f1[i]);
            }
            apply_proj_rows(r, &ly->p[ORC_DOWN], f1, Tc, tmp);
            for (int64_t i = 0; i < Tc * H; ++i) h[i] = h[i] + tmp[i];
        }
        r->pos += Tc;
    }
    free(h); free(x); free(q); free(k); free(v); free(cx); free(tmp); free(f1); free(f2); free(K); free(V);
}

/* Benchmark support (the CPU baseline's bounded samples): puts the runner at
 * position L with a KV cache of L synthetic rows per layer (uniform values in
 * [-1, 1) from an LCG, appended through the cache's own paging rules), so
 * that the next step does the work of a decode step at context L+1 without
 * a CPU prefill of L prompt tokens.  The step's numbers are not meaningful;
 * its cost is. */
void orc_runner_fill_context(orc_runner *r, int64_t L, uint64_t seed) {
    orc_runner_reset(r);
    const int64_t kvd = r->kvdim;
    float *k = (float *)malloc(sizeof(float) * (size_t)kvd);
    float *v = (float *)malloc(sizeof(float) * (size_t)kvd);
    uint64_t s = seed ? seed : 1;
    for (int64_t l = 0; l < r->m->cfg.num_layers; ++l)
        for (int64_t pos = 0; pos < L; ++pos) {
            for (int64_t i = 0; i < kvd; ++i) {
                s = s * 6364136223846793005ULL + 1442695040888963407ULL;
                k[i] = (float)(int32_t)(s >> 32) * 4.656612873077393e-10f;
                s = s * 6364136223846793005ULL + 1442695040888963407ULL;
                v[i] = (float)(int32_t)(s >> 32) * 4.656612873077393e-10f;
            }
            kv_append(r, l, k, v, pos);
        }
    r->pos = L;
    free(k);
    free(v);
}

/* ModelWeights.swift:18-29 SeededGenerator (seed 0 -> 0xdeadbeef; state =
 * 6364136223846793005 * state + 1) and Tensor.swift:1623-1644 Tensor.random:
 * Box-Muller pairs in fp32, u = Float.random(in: 0..<1) taken as the low 24
 * bits of the 32-bit truncation of next() times 2^-24 (Swift's standard
 * library, which is not in the reference tree), u1 clamped to the least
 * nonzero magnitude.  Parallel over pairs with an LCG jump per chunk. */
#define ORC_LCG_A 6364136223846793005ULL
static uint64_t orc_lcg_jump(uint64_t s, uint64_t n) {
    uint64_t A = 1, Cc = 0, a = ORC_LCG_A, cc = 1;
    while (n) {
        if (n & 1) {
            A = A * a;
            Cc = Cc * a + cc;
        }
        cc = (a + 1) * cc;
        a = a * a;
        n >>= 1;
    }
    return A * s + Cc;
}

uint64_t orc_rng_seed(uint64_t seed) { return seed != 0 ? seed : 0xdeadbeefULL; }

void orc_rng_fill_normal(uint64_t *state, float mean, float stdv, int64_t n, float *out) {
    const int64_t pairs = (n + 1) / 2;
    const uint64_t s0 = *state;
    const int64_t chunk = 1 << 16;
#pragma omp parallel for schedule(static)
    for (int64_t pb = 0; pb < pairs; pb += chunk) {
        const int64_t pe = pb + chunk < pairs ? pb + chunk : pairs;
        uint64_t s = orc_lcg_jump(s0, (uint64_t)(2 * pb));
        const float two_pi = 2.0f * 3.14159265358979323846f;
        for (int64_t pi = pb; pi < pe; ++pi) {
            s = ORC_LCG_A * s + 1;
            float u1 = (float)((uint32_t)s & 0xFFFFFFu) * 5.9604644775390625e-08f;
            s = ORC_LCG_A * s + 1;
            const float u2 = (float)((uint32_t)s & 0xFFFFFFu) * 5.9604644775390625e-08f;
            if (u1 < 1.40129846e-45f) u1 = 1.40129846e-45f;
            const float rr = sqrtf(-2.0f * logf(u1));
            const float th = two_pi * u2;
            const int64_t i = 2 * pi;
            out[i] = mean + stdv * rr * cosf(th);
            if (i + 1 < n) out[i + 1] = mean + stdv * rr * sinf(th);
        }
    }
    *state = orc_lcg_jump(s0, (uint64_t)(2 * pairs));
}

/* Sampler.swift:369-381: LCG (Numerical Recipes constants). */
uint64_t orc_lcg_next(uint64_t *state) {
    *state = *state * 6364136223846793005ULL + 1442695040888963407ULL;
    return *state;
}

/* Order of Swift's `sorted { $0.element > $1.element }` on (index, value)
 * pairs: descending value; the reference's sort is not stable, so equal
 * values keep ascending index here (a documented choice). */
typedef struct { float v; int64_t i; } orc_kv;
static int orc_kv_desc(const void *a, const void *b) {
    const orc_kv *x = (const orc_kv *)a, *y = (const orc_kv *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return x->i < y->i ? -1 : (x->i > y->i ? 1 : 0);
}

int64_t orc_sample_detailed(const float *logits, int64_t V, const orc_sampler *cfg, const int64_t *history,
                            int64_t n_history, uint64_t *rng, float *prob, float *entropy) {
    float *x = (float *)malloc(sizeof(float) * (size_t)V);
    float *p = (float *)malloc(sizeof(float) * (size_t)V);
    orc_kv *srt = (orc_kv *)malloc(sizeof(orc_kv) * (size_t)V);
    memcpy(x, logits, sizeof(float) * (size_t)V);
    /* 1. repetition penalty, sign-aware, once per history entry (Sampler.swift:409-421) */
    if (cfg->repetition_penalty != 1.0f && n_history > 0) {
        const float pen = cfg->repetition_penalty;
        for (int64_t h = 0; h < n_history; ++h) {
            const int64_t t = history[h];
            if (t >= 0 && t < V) x[t] = x[t] > 0 ? x[t] / pen : x[t] * pen;
        }
    }
    /* 2. top-k, else top-p (Sampler.swift:428-448) */
    if (cfg->top_k > 0) {
        for (int64_t i = 0; i < V; ++i) { srt[i].v = x[i]; srt[i].i = i; }
        qsort(srt, (size_t)V, sizeof(orc_kv), orc_kv_desc);
        char *keep = (char *)calloc((size_t)V, 1);
        for (int64_t i = 0; i < cfg->top_k && i < V; ++i) keep[srt[i].i] = 1;
        for (int64_t i = 0; i < V; ++i)
            if (!keep[i]) x[i] = -INFINITY;
        free(keep);
    } else if (cfg->has_top_p) {
        orc_softmax(x, V, p);
        for (int64_t i = 0; i < V; ++i) { srt[i].v = p[i]; srt[i].i = i; }
        qsort(srt, (size_t)V, sizeof(orc_kv), orc_kv_desc);
        float cum = 0.0f;
        int64_t cutoff = V;
        for (int64_t i = 0; i < V; ++i) {
            cum += srt[i].v;
            if (cum >= cfg->top_p) { cutoff = i + 1; break; }
        }
        char *keep = (char *)calloc((size_t)V, 1);
        for (int64_t i = 0; i < cutoff; ++i) keep[srt[i].i] = 1;
        for (int64_t i = 0; i < V; ++i)
            if (!keep[i]) x[i] = -INFINITY;
        free(keep);
    }
    /* 3. temperature (Sampler.swift:451-458): below 0.01 the logits stay unscaled */
    const float temp = cfg->temperature > 0 ? cfg->temperature : 0.0f;
    if (!(temp < 0.01f))
        for (int64_t i = 0; i < V; ++i) x[i] = x[i] / temp;
    /* 4. final distribution and entropy (Sampler.swift:461-466) */
    orc_softmax(x, V, p);
    float ent = 0.0f;
    for (int64_t i = 0; i < V; ++i)
        if (p[i] > 0) ent -= p[i] * logf(p[i]);
    /* 5. CDF draw (Sampler.swift:340-359) */
    const float threshold = (float)orc_lcg_next(rng) / (float)UINT64_MAX;
    float cum = 0.0f;
    int64_t tok = V - 1;
    for (int64_t i = 0; i < V; ++i) {
        cum += p[i];
        if (threshold <= cum) { tok = i; break; }
    }
    if (prob) *prob = p[tok];
    if (entropy) *entropy = ent;
    free(x);
    free(p);
    free(srt);
    return tok;
}

/* ModelRunner.swift:227-298 with Sampler.sampleDetailed (history = prompt +
 * generated tokens). */
int64_t orc_generate_sampled(orc_runner *r, const int64_t *prompt, int64_t n_prompt, int64_t max_tokens,
                             const orc_sampler *cfg, uint64_t *rng, int64_t *out_tokens, float *out_prob,
                             float *out_entropy) {
    const int64_t V = r->m->cfg.vocab;
    float *logits = (float *)malloc(sizeof(float) * (size_t)V);
    int64_t *hist = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_prompt + max_tokens + 1));
    int64_t nh = 0, cur = 0;
    for (int64_t i = 0; i < n_prompt; ++i) {
        int64_t t = prompt[i] < 0 ? 0 : (prompt[i] > V - 1 ? V - 1 : prompt[i]);
        hist[nh++] = t;
        if (i + 1 < n_prompt)
            orc_runner_step(r, t, logits);
        else
            cur = t;
    }
    for (int64_t g = 0; g < max_tokens; ++g) {
        orc_runner_step(r, cur, logits);
        float pr = 0.0f, en = 0.0f;
        const int64_t tok = orc_sample_detailed(logits, V, cfg, hist, nh, rng, &pr, &en);
        out_tokens[g] = tok;
        if (out_prob) out_prob[g] = pr;
        if (out_entropy) out_entropy[g] = en;
        hist[nh++] = tok;
        cur = tok;
    }
    free(logits);
    free(hist);
    return max_tokens;
}

/* PerplexityHarness.swift:141-193 (computePerplexity): teacher forcing over
 * tokens[0..n-2]; per step log P(tokens[i+1]) = logit - (log(sum exp(logit -
 * max)) + max) with the max in fp32 and the sum in fp64; returns
 * Float(exp(-mean)). */
float orc_perplexity(orc_runner *r, const int64_t *tokens, int64_t n, double *sum_logprob) {
    const int64_t V = r->m->cfg.vocab;
    float *logits = (float *)malloc(sizeof(float) * (size_t)V);
    double sum = 0.0;
    for (int64_t i = 0; i + 1 < n; ++i) {
        orc_runner_step(r, tokens[i], logits);
        float mx = logits[0];
        for (int64_t j = 1; j < V; ++j)
            if (logits[j] > mx) mx = logits[j];
        double se = 0.0;
        for (int64_t j = 0; j < V; ++j) se += exp((double)logits[j] - (double)mx);
        sum += (double)logits[tokens[i + 1]] - (log(se) + (double)mx);
    }
    free(logits);
    if (sum_logprob) *sum_logprob = sum;
    return n > 1 ? (float)exp(-sum / (double)(n - 1)) : 0.0f;
}

/* ModelRunner.swift:227-298 with greedy sampling (Sampler.swift:126-138). */
int64_t orc_generate_greedy(orc_runner *r, const int64_t *prompt, int64_t n_prompt,
                            int64_t max_tokens, int64_t *out_tokens, float *out_gap) {
    const int64_t V = r->m->cfg.vocab;
    float *logits = (float *)malloc(sizeof(float) * (size_t)V);
    int64_t cur = 0;
    int64_t *pre = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_prompt > 0 ? n_prompt : 1));
    for (int64_t i = 0; i < n_prompt; ++i) {
        int64_t t = prompt[i] < 0 ? 0 : (prompt[i] > V - 1 ? V - 1 : prompt[i]);
        if (i + 1 < n_prompt)
            pre[i] = t;
        else
            cur = t;
    }
    orc_runner_prefill(r, pre, n_prompt - 1);
    free(pre);
    for (int64_t g = 0; g < max_tokens; ++g) {
        orc_runner_step(r, cur, logits);
        int64_t best = orc_greedy(logits, V);
        if (out_gap) {
            float second = -INFINITY;
            for (int64_t i = 0; i < V; ++i)
                if (i != best && logits[i] > second) second = logits[i];
            out_gap[g] = logits[best] - second;
        }
        out_tokens[g] = best;
        cur = best;
    }
    free(logits);
    return max_tokens;
}
