/*
 * oracle.c — CPU restatement of Aaedn's token loop. TEST INFRASTRUCTURE ONLY
 * (see oracle.h): the checker for the CUDA path, never the thing measured or
 * shipped. Built twice by oracle/Makefile: a strict build (no fast-math, no
 * FMA contraction) for parity, and a build with the reference's own
 * CMakeLists.txt:5 flags (-O3 -mavx2 -mfma -ffast-math) for the timed CPU
 * baseline.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void or_set_threads(int n) { g_threads = n; }
int or_get_threads(void)
{
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* fp16                                                                       */
/* ------------------------------------------------------------------------ */
float or_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t exp = (uint32_t)(h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    float v;
    if (exp == 0)
        v = ldexpf((float)man, -24); /* zero / subnormal: man * 2^-24 exactly */
    else if (exp == 31)
        v = man ? NAN : INFINITY;
    else
        v = ldexpf((float)(man | 0x400u), (int)exp - 25);
    return sign ? -v : v;
}

/* double -> binary16, round to nearest even (numpy's float16(python float)
 * conversion, which tools/convert_model.py:49 relies on). */
uint16_t or_f64_to_f16(double d)
{
    uint16_t sign = signbit(d) ? 0x8000u : 0u;
    if (isnan(d))
        return 0x7E00u;
    double a = fabs(d);
    if (a >= 65520.0) /* halfway between 65504 and 2^16 rounds to even -> inf */
        return sign | 0x7C00u;
    if (a < ldexp(1.0, -14))
    {
        /* subnormal range: units of 2^-24, round half even */
        double r = nearbyint(a * ldexp(1.0, 24));
        return sign | (uint16_t)r; /* r == 1024 is the smallest normal, encoded the same */
    }
    int e;
    double m = frexp(a, &e); /* a = m * 2^e, m in [0.5, 1) */
    int E = e - 1;           /* a = (2m) * 2^E, 2m in [1, 2) */
    double r = nearbyint(m * 2.0 * 1024.0);
    if (r >= 2048.0)
    {
        r = 1024.0;
        E += 1;
    }
    if (E > 15)
        return sign | 0x7C00u;
    return sign | (uint16_t)(((E + 15) << 10) | ((uint32_t)r - 1024u));
}

/* ------------------------------------------------------------------------ */
/* Quantizer: tools/convert_model.py:24-55                                   */
/* ------------------------------------------------------------------------ */
void or_quantize_q4(const float* x, size_t n, uint8_t* data, uint16_t* scales)
{
    const size_t BS = 32; /* convert_model.py:12 */
    size_t n_blocks = (n + BS - 1) / BS;
    memset(data, 0, (n + 1) / 2); /* pack_nibbles_unsigned zero-initialises, :25 */
    /* blocks own disjoint bytes (32 codes = 16 bytes): the loop runs over
     * them in parallel with the same results as the sequential order */
    long long NB = (long long)n_blocks;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long long bb = 0; bb < NB; ++bb)
    {
        size_t b = (size_t)bb;
        size_t start = b * BS, end = start + BS < n ? start + BS : n;
        /* :47 max_val = float(np.max(np.abs(block))) -- max taken in fp32 */
        float mx = 0.0f;
        for (size_t i = start; i < end; ++i)
        {
            float a = fabsf(x[i]);
            if (a > mx)
                mx = a;
        }
        double max_val = (double)mx;
        /* :48 scale = max_val / 7.0 (a Python float, i.e. fp64) */
        double scale = max_val > 0.0 ? max_val / 7.0 : 1.0;
        /* :49 np.float16(scale): fp64 -> fp16 directly, round half even */
        scales[b] = or_f64_to_f16(scale);
        if (max_val > 0.0)
        {
            /* :51 block / scale: fp32 array over a weak Python float -> the
             * division runs in fp32 (NEP 50); np.rint is round-half-even. */
            float sf = (float)scale;
            for (size_t i = start; i < end; ++i)
            {
                float qf = nearbyintf(x[i] / sf);
                int q;
                if (!(qf > 0.0f)) /* clip(.., 0, 15), :52 */
                    q = 0;
                else if (qf > 15.0f)
                    q = 15;
                else
                    q = (int)qf;
                /* :24-33 low nibble = even element, high nibble = odd */
                if ((i & 1) == 0)
                    data[i / 2] = (uint8_t)(data[i / 2] | (q & 0x0F));
                else
                    data[i / 2] = (uint8_t)(data[i / 2] | ((q & 0x0F) << 4));
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Dequant: src/dequant.cpp:7-28                                             */
/* ------------------------------------------------------------------------ */
static void dequant_impl(const uint8_t* data, const uint16_t* scales, float* out, size_t n, int f16)
{
    if (!data || !scales || scales[0] == 0) /* dequant.cpp:9-14 */
    {
        for (size_t i = 0; i < n; ++i)
            out[i] = 0.0f;
        return;
    }
    for (size_t blk = 0; blk < n; blk += 32) /* dequant.cpp:16-27 */
    {
        size_t rem = (blk + 32 <= n) ? 32 : (n - blk);
        float scale = f16 ? or_f16_to_f32(scales[blk / 32]) : (float)scales[blk / 32];
        for (size_t i = 0; i < rem; ++i)
        {
            uint8_t byte = data[(blk + i) / 2];
            uint8_t val = (i % 2 == 0) ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
            out[blk + i] = (float)val * scale;
        }
    }
}

void or_dequant_4bit(const uint8_t* data, const uint16_t* scales, float* out, size_t n)
{
    dequant_impl(data, scales, out, n, 0);
}

void or_dequant_4bit_f16(const uint8_t* data, const uint16_t* scales, float* out, size_t n)
{
    dequant_impl(data, scales, out, n, 1);
}

/* ------------------------------------------------------------------------ */
/* Canonical matmuls (D1, D2)                                                */
/* ------------------------------------------------------------------------ */
static inline float scale_of(uint16_t s, int kind)
{
    return kind == 0 ? or_f16_to_f32(s) : (float)s;
}

void or_q4_matmul(const float* in, const uint8_t* w, const uint16_t* s, float* out, size_t M, size_t N,
                  size_t K, size_t lda, size_t ldb, size_t ldc, int scale_kind)
{
    long long NN = (long long)N;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long long nn = 0; nn < NN; ++nn)
    {
        size_t n = (size_t)nn;
        const uint8_t* row = w + n * (ldb / 2);
        const uint16_t* rs = s + n * (ldb / 32);
        for (size_t m = 0; m < M; ++m)
        {
            const float* x = in + m * lda;
            float sum = 0.0f;
            for (size_t k = 0; k < K; ++k)
            {
                uint8_t byte = row[k / 2];
                uint8_t c = (k & 1) ? (uint8_t)((byte >> 4) & 0x0F) : (uint8_t)(byte & 0x0F);
                float wv = (float)c * scale_of(rs[k / 32], scale_kind); /* ffn.cpp:42 */
                sum += x[k] * wv;                                        /* ffn.cpp:43 */
            }
            out[m * ldc + n] = sum;
        }
    }
}

void or_f32_matmul(const float* in, const float* w, float* out, size_t M, size_t N, size_t K, size_t lda,
                   size_t ldw, size_t ldc)
{
    long long NN = (long long)N;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long long nn = 0; nn < NN; ++nn)
    {
        size_t n = (size_t)nn;
        for (size_t m = 0; m < M; ++m)
        {
            float sum = 0.0f;
            for (size_t k = 0; k < K; ++k)
                sum += in[m * lda + k] * w[n * ldw + k]; /* transformer.cpp:236 */
            out[m * ldc + n] = sum;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* RMSNorm: src/rmsnorm.cpp:8-51 (same 8-lane partial-sum order)            */
/* ------------------------------------------------------------------------ */
void or_rmsnorm(const float* in, float* out, const float* w, size_t n, float eps)
{
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    for (; i + 7 < n; i += 8) /* :13-18 */
        for (int j = 0; j < 8; ++j)
            lane[j] += in[i + j] * in[i + j];
    /* :20-24 low+high halves, then two horizontal adds */
    float a0 = lane[0] + lane[4], a1 = lane[1] + lane[5], a2 = lane[2] + lane[6], a3 = lane[3] + lane[7];
    float sum = (a0 + a1) + (a2 + a3);
    for (; i < n; ++i) /* :29-32 */
        sum += in[i] * in[i];
    float rms = 1.0f / sqrtf(sum / (float)n + eps); /* :34 */
    for (i = 0; i < n; ++i)                         /* :37-50 */
        out[i] = in[i] * rms * w[i];
}

/* ------------------------------------------------------------------------ */
/* RoPE                                                                      */
/* ------------------------------------------------------------------------ */
void or_rope_tables_ref(float* cos_t, float* sin_t, size_t max_seq, size_t head_dim)
{
    size_t half = head_dim / 2; /* rope.cpp:14-31 */
    float base_freq = 10000.0f;
    for (size_t pos = 0; pos < max_seq; ++pos)
        for (size_t i = 0; i < half; ++i)
        {
            float freq = base_freq / powf(2.0f, (float)i / (float)half);
            float angle = (float)pos * freq;
            cos_t[pos * half + i] = cosf(angle);
            sin_t[pos * half + i] = sinf(angle);
        }
}

void or_rope_tables(float* cos_t, float* sin_t, size_t max_seq, size_t head_dim, double theta)
{
    size_t half = head_dim / 2; /* D3 */
    for (size_t pos = 0; pos < max_seq; ++pos)
        for (size_t i = 0; i < half; ++i)
        {
            double inv_freq = pow(theta, -2.0 * (double)i / (double)head_dim);
            double angle = (double)pos * inv_freq;
            cos_t[pos * half + i] = (float)cos(angle);
            sin_t[pos * half + i] = (float)sin(angle);
        }
}

void or_rope_apply(float* q, float* k, size_t seq_len, size_t head_dim, const float* cos_t, const float* sin_t)
{
    if (!cos_t || !sin_t) /* rope.cpp:38-39 */
        return;
    size_t half = head_dim / 2;
    for (size_t pos = 0; pos < seq_len; ++pos) /* rope.cpp:43-62 */
        for (size_t i = 0; i < half; ++i)
        {
            float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
            float q0 = q[pos * head_dim + i], q1 = q[pos * head_dim + i + half];
            q[pos * head_dim + i] = c * q0 - s * q1;
            q[pos * head_dim + i + half] = s * q0 + c * q1;
            float k0 = k[pos * head_dim + i], k1 = k[pos * head_dim + i + half];
            k[pos * head_dim + i] = c * k0 - s * k1;
            k[pos * head_dim + i + half] = s * k0 + c * k1;
        }
}

/* ------------------------------------------------------------------------ */
/* Attention: src/attention.cpp:10-84 (head index added, D4)                */
/* ------------------------------------------------------------------------ */
static void attention_head(const float* qh, const float* k_cache, const float* v_cache, size_t row_stride,
                           size_t head_off, const uint32_t* segments, size_t num_segments, float* oh,
                           size_t head_dim, float scale, float* scores)
{
    for (size_t i = 0; i < head_dim; ++i)
        oh[i] = 0.0f;
    size_t idx = 0;
    for (size_t seg = 0; seg < num_segments; ++seg) /* :30-44 */
    {
        uint32_t start = segments[2 * seg], len = segments[2 * seg + 1];
        for (uint32_t t = 0; t < len; ++t)
        {
            const float* kr = k_cache + (size_t)(start + t) * row_stride + head_off;
            float dot = 0.0f;
            for (size_t i = 0; i < head_dim; ++i)
                dot += qh[i] * kr[i];
            scores[idx++] = dot * scale;
        }
    }
    if (idx == 0)
        return;
    float mx = scores[0]; /* :46-51 */
    for (size_t i = 1; i < idx; ++i)
        if (scores[i] > mx)
            mx = scores[i];
    float sum = 0.0f; /* :53-59 */
    for (size_t i = 0; i < idx; ++i)
    {
        float e = expf(scores[i] - mx);
        scores[i] = e;
        sum += e;
    }
    float inv = 1.0f / sum; /* :61-65 */
    for (size_t i = 0; i < idx; ++i)
        scores[i] *= inv;
    idx = 0; /* :67-82 */
    for (size_t seg = 0; seg < num_segments; ++seg)
    {
        uint32_t start = segments[2 * seg], len = segments[2 * seg + 1];
        for (uint32_t t = 0; t < len; ++t)
        {
            float wgt = scores[idx++];
            const float* vr = v_cache + (size_t)(start + t) * row_stride + head_off;
            for (size_t i = 0; i < head_dim; ++i)
                oh[i] += wgt * vr[i];
        }
    }
}

void or_attention(const float* q, const float* k_cache, const float* v_cache, const uint32_t* segments,
                  size_t num_segments, float* out, size_t n_heads, size_t head_dim, float scale)
{
    if (!q || !k_cache || !v_cache || !segments) /* :13-18 */
    {
        for (size_t i = 0; i < n_heads * head_dim; ++i)
            out[i] = 0.0f;
        return;
    }
    size_t total = 0;
    for (size_t s = 0; s < num_segments; ++s)
        total += segments[2 * s + 1];
    float* scores = (float*)malloc((total ? total : 1) * sizeof(float));
    for (size_t h = 0; h < n_heads; ++h)
        attention_head(q + h * head_dim, k_cache, v_cache, n_heads * head_dim, h * head_dim, segments,
                       num_segments, out + h * head_dim, head_dim, scale, scores);
    free(scores);
}

/* ------------------------------------------------------------------------ */
/* ffn_swiglu with the reference's own semantics: src/ffn.cpp:18-77          */
/* ------------------------------------------------------------------------ */
void or_ffn_swiglu_refsem(const float* in, float* out, size_t batch, size_t hidden, size_t ffn,
                          const uint8_t* gate, const uint8_t* up, const uint8_t* down, const uint16_t* gs,
                          const uint16_t* us, const uint16_t* ds)
{
    float* g = (float*)malloc(ffn * sizeof(float));
    float* u = (float*)malloc(ffn * sizeof(float));
    for (size_t b = 0; b < batch; ++b)
    {
        const float* x = in + b * hidden;
        for (size_t j = 0; j < ffn; ++j) /* :36-46 */
        {
            float sum = 0.0f;
            for (size_t i = 0; i < hidden; ++i)
            {
                uint8_t val = (gate[j * hidden / 2 + i / 2] >> ((i % 2) * 4)) & 0x0F;
                float w = (float)val * (float)gs[j / 32];
                sum += x[i] * w;
            }
            g[j] = sum;
        }
        for (size_t j = 0; j < ffn; ++j) /* :48-58 */
        {
            float sum = 0.0f;
            for (size_t i = 0; i < hidden; ++i)
            {
                uint8_t val = (up[j * hidden / 2 + i / 2] >> ((i % 2) * 4)) & 0x0F;
                float w = (float)val * (float)us[j / 32];
                sum += x[i] * w;
            }
            u[j] = sum;
        }
        for (size_t j = 0; j < ffn; ++j) /* :60-63 */
            g[j] = g[j] * (g[j] / (1.0f + expf(-g[j])));
        for (size_t i = 0; i < hidden; ++i) /* :65-75 */
        {
            float sum = 0.0f;
            for (size_t j = 0; j < ffn; ++j)
            {
                uint8_t val = (down[i * ffn / 2 + j / 2] >> ((j % 2) * 4)) & 0x0F;
                float w = (float)val * (float)ds[i / 32];
                sum += g[j] * u[j] * w;
            }
            out[b * hidden + i] = sum;
        }
    }
    free(g);
    free(u);
}

/* ------------------------------------------------------------------------ */
/* .abn v2 acceptance: src/quant.cpp:31-119                                  */
/* ------------------------------------------------------------------------ */
uint32_t or_fnv1a32(const uint8_t* p, size_t n, uint32_t h)
{
    for (size_t i = 0; i < n; ++i) /* quant.cpp:12-20 */
    {
        h ^= p[i];
        h *= 0x01000193u;
    }
    return h;
}

static uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }

int or_abn_v2_accepts(const uint8_t* f, size_t size)
{
    if (size < 64) /* header read fails, quant.cpp:52-60 */
        return 0;
    if (memcmp(f, "AAEDNMDL", 8) != 0 || rd32(f + 8) != 2u) /* :62 */
        return 0;
    uint64_t payload = (uint64_t)rd32(f + 12) | (uint64_t)rd32(f + 16) << 32;
    uint32_t checksum = rd32(f + 20);
    uint32_t hidden = rd32(f + 40);
    size_t dsz = ((size_t)hidden * hidden) / 2;              /* :68 */
    size_t ssz = ((size_t)hidden * hidden / 32) * 2;         /* :69 */
    if ((uint64_t)(dsz + ssz) != payload)                    /* :72 */
        return 0;
    if (size < 64 + dsz + ssz) /* short read, :87-103 */
        return 0;
    uint32_t h = or_fnv1a32(f + 64, dsz, 0x811C9DC5u); /* :105-108 */
    h = or_fnv1a32(f + 64 + dsz, ssz, h);
    return h == checksum;
}

/* ------------------------------------------------------------------------ */
/* Model oracle: src/transformer.cpp:128-243 with D1..D8                     */
/* ------------------------------------------------------------------------ */
struct or_model
{
    or_config c;
    or_weights w;
    uint32_t pos;
    float *k_cache, *v_cache; /* [L][max_seq][n_kv][hd] */
    float *cos_t, *sin_t;     /* [max_seq][hd/2] */
    float *hidden, *normed, *q, *k, *v, *attn, *tmp, *gate, *up, *scores;
};

or_model* or_model_create(const or_config* cfg, const or_weights* w)
{
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    if (!m)
        return NULL;
    m->c = *cfg;
    m->w = *w;
    const or_config* c = cfg;
    size_t kvsz = (size_t)c->n_layers * c->max_seq * c->n_kv_heads * c->head_dim;
    m->k_cache = (float*)calloc(kvsz, sizeof(float));
    m->v_cache = (float*)calloc(kvsz, sizeof(float));
    m->cos_t = (float*)malloc((size_t)c->max_seq * (c->head_dim / 2) * sizeof(float));
    m->sin_t = (float*)malloc((size_t)c->max_seq * (c->head_dim / 2) * sizeof(float));
    size_t qd = (size_t)c->n_heads * c->head_dim, kd = (size_t)c->n_kv_heads * c->head_dim;
    m->hidden = (float*)malloc(c->dim * sizeof(float));
    m->normed = (float*)malloc(c->dim * sizeof(float));
    m->q = (float*)malloc(qd * sizeof(float));
    m->k = (float*)malloc(kd * sizeof(float));
    m->v = (float*)malloc(kd * sizeof(float));
    m->attn = (float*)malloc(qd * sizeof(float));
    m->tmp = (float*)malloc(c->dim * sizeof(float));
    m->gate = (float*)malloc(c->ffn_dim * sizeof(float));
    m->up = (float*)malloc(c->ffn_dim * sizeof(float));
    m->scores = (float*)malloc((size_t)c->n_heads * c->max_seq * sizeof(float));
    if (!m->k_cache || !m->v_cache || !m->cos_t || !m->sin_t || !m->scores)
    {
        or_model_destroy(m);
        return NULL;
    }
    or_rope_tables(m->cos_t, m->sin_t, c->max_seq, c->head_dim, c->rope_theta);
    m->pos = 0;
    return m;
}

void or_model_destroy(or_model* m)
{
    if (!m)
        return;
    free(m->k_cache);
    free(m->v_cache);
    free(m->cos_t);
    free(m->sin_t);
    free(m->hidden);
    free(m->normed);
    free(m->q);
    free(m->k);
    free(m->v);
    free(m->attn);
    free(m->tmp);
    free(m->gate);
    free(m->up);
    free(m->scores);
    free(m);
}

void or_model_reset(or_model* m) { m->pos = 0; }
uint32_t or_model_pos(const or_model* m) { return m->pos; }

static void matvec_q4(const or_q4* w, const float* x, float* y, size_t N, size_t K)
{
    or_q4_matmul(x, w->data, w->scales, y, 1, N, K, K, K, N, 0);
}

/* rotate-half on every head of a [heads][hd] vector at position pos (D3,
 * pairing as rope.cpp:50-60) */
static void rope_heads(float* v, size_t heads, size_t hd, const float* cos_row, const float* sin_row)
{
    size_t half = hd / 2;
    for (size_t h = 0; h < heads; ++h)
    {
        float* x = v + h * hd;
        for (size_t i = 0; i < half; ++i)
        {
            float c = cos_row[i], s = sin_row[i];
            float x0 = x[i], x1 = x[i + half];
            x[i] = c * x0 - s * x1;
            x[i + half] = s * x0 + c * x1;
        }
    }
}

int or_model_step(or_model* m, uint32_t token, float* logits, float* hidden_out)
{
    const or_config* c = &m->c;
    const or_weights* w = &m->w;
    if (token >= c->vocab || m->pos >= c->max_seq) /* transformer.cpp:137-142 */
        return -1;
    const size_t D = c->dim, hd = c->head_dim, H = c->n_heads, KV = c->n_kv_heads;
    const size_t qd = H * hd, kd = KV * hd, F = c->ffn_dim;
    const uint32_t pos = m->pos;
    memcpy(m->hidden, w->embedding + (size_t)token * D, D * sizeof(float)); /* :144-146 */
    const float scale = 1.0f / sqrtf((float)hd);                             /* :198 */
    const size_t half = hd / 2;
    for (uint32_t l = 0; l < c->n_layers; ++l) /* :148-228 */
    {
        or_rmsnorm(m->hidden, m->normed, w->attn_norm[l], D, c->eps); /* :150-153 */
        matvec_q4(&w->wq[l], m->normed, m->q, qd, D);                 /* :155-178 (D2) */
        matvec_q4(&w->wk[l], m->normed, m->k, kd, D);
        matvec_q4(&w->wv[l], m->normed, m->v, kd, D);
        rope_heads(m->q, H, hd, m->cos_t + (size_t)pos * half, m->sin_t + (size_t)pos * half); /* D3 */
        rope_heads(m->k, KV, hd, m->cos_t + (size_t)pos * half, m->sin_t + (size_t)pos * half);
        size_t lbase = (size_t)l * c->max_seq * kd; /* D5: append at pos */
        memcpy(m->k_cache + lbase + (size_t)pos * kd, m->k, kd * sizeof(float));
        memcpy(m->v_cache + lbase + (size_t)pos * kd, m->v, kd * sizeof(float));
        uint32_t seg[2] = {0, pos + 1};
        long long HH = (long long)H;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
        for (long long hh = 0; hh < HH; ++hh) /* D4: GQA head h reads kv head h/(H/KV) */
        {
            size_t h = (size_t)hh;
            size_t kvh = h / (H / KV);
            attention_head(m->q + h * hd, m->k_cache + lbase, m->v_cache + lbase, kd, kvh * hd, seg, 1,
                           m->attn + h * hd, hd, scale, m->scores + h * c->max_seq);
        }
        matvec_q4(&w->wo[l], m->attn, m->tmp, D, qd); /* :206-215 */
        for (size_t j = 0; j < D; ++j)
            m->hidden[j] = m->tmp[j] + m->hidden[j];
        or_rmsnorm(m->hidden, m->normed, w->ffn_norm[l], D, c->eps); /* :217-220 */
        matvec_q4(&w->wg[l], m->normed, m->gate, F, D);             /* :222-224 (D6) */
        matvec_q4(&w->wu[l], m->normed, m->up, F, D);
        for (size_t j = 0; j < F; ++j)
        {
            float g = m->gate[j];
            m->gate[j] = (g / (1.0f + expf(-g))) * m->up[j];
        }
        matvec_q4(&w->wd[l], m->gate, m->tmp, D, F);
        for (size_t j = 0; j < D; ++j) /* :226-227 */
            m->hidden[j] = m->tmp[j] + m->hidden[j];
        if (hidden_out)
            memcpy(hidden_out + (size_t)l * D, m->hidden, D * sizeof(float));
    }
    or_rmsnorm(m->hidden, m->normed, w->final_norm, D, c->eps);          /* :230 (D8) */
    or_f32_matmul(m->normed, w->lm_head, logits, 1, c->vocab, D, D, D, c->vocab); /* :232-238 */
    m->pos = pos + 1;                                                        /* :240 (D7) */
    return 0;
}

uint32_t or_argmax(const float* v, size_t n)
{
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (v[i] > v[best])
            best = i;
    return (uint32_t)best;
}

int or_model_generate(or_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_new, uint32_t* out_tokens,
                      float* last_logits)
{
    float* logits = (float*)malloc(m->c.vocab * sizeof(float));
    if (!logits || n_prompt == 0)
    {
        free(logits);
        return -1;
    }
    int rc = 0;
    for (size_t i = 0; i < n_prompt && rc == 0; ++i)
        rc = or_model_step(m, prompt[i], logits, NULL);
    for (size_t i = 0; i < n_new && rc == 0; ++i)
    {
        uint32_t t = or_argmax(logits, m->c.vocab);
        out_tokens[i] = t;
        if (i + 1 < n_new)
            rc = or_model_step(m, t, logits, NULL);
    }
    if (last_logits && rc == 0)
        memcpy(last_logits, logits, m->c.vocab * sizeof(float));
    free(logits);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* Seeded synthetic inputs                                                    */
/* ------------------------------------------------------------------------ */
/* The counter-based generator the library's synthetic models are built from
 * (its aaedn_synth_normal / aaedn_synth_tokens), restated here so that a test
 * or the CPU baseline builds the same weights and prompts without loading
 * the library: splitmix64 keyed by (seed, tensor id), one 64-bit draw per
 * element pair, Box-Muller in fp64. */
static uint64_t or_splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t or_stream_key(uint64_t seed, uint64_t id)
{
    return or_splitmix64(seed ^ or_splitmix64(id + 0x632BE59BD9B4E019ull));
}

void or_synth_normal(uint64_t seed, uint64_t id, float std_dev, float* out, size_t n)
{
    const uint64_t key = or_stream_key(seed, id);
    const double two_pi = 6.283185307179586476925286766559;
    long long pairs = (long long)((n + 1) / 2);
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long long pp = 0; pp < pairs; ++pp)
    {
        size_t i = (size_t)pp * 2;
        uint64_t h = or_splitmix64(key + (uint64_t)pp * 0x9E3779B97F4A7C15ull);
        double u1 = ((double)(h >> 40) + 1.0) * (1.0 / 16777216.0); /* (0, 1] */
        double u2 = (double)(h & 0xFFFFFFull) * (1.0 / 16777216.0);  /* [0, 1) */
        double r = sqrt(-2.0 * log(u1));
        double t = two_pi * u2;
        out[i] = (float)(std_dev * r * cos(t));
        if (i + 1 < n)
            out[i + 1] = (float)(std_dev * r * sin(t));
    }
}

void or_synth_tokens(uint64_t seed, uint64_t id, uint32_t vocab, uint32_t* out, size_t n)
{
    const uint64_t key = or_stream_key(seed, id ^ 0x746F6B656E73ull);
    for (size_t i = 0; i < n; ++i)
        out[i] = (uint32_t)(or_splitmix64(key + i * 0x9E3779B97F4A7C15ull) % vocab);
}

/* Timing aid of the CPU baseline: move the sequence to position pos with
 * every cached K/V row below it filled from a fixed pattern, so a decode step
 * at pos does the work of one at that position (the attention reads pos + 1
 * rows) without the pos prompt steps before it. The logits that follow are
 * not those of any prompt. Returns -1 when pos is outside the cache. */
int or_model_seek(or_model* m, uint32_t pos)
{
    const or_config* c = &m->c;
    if (pos >= c->max_seq)
        return -1;
    const size_t kd = (size_t)c->n_kv_heads * c->head_dim;
    long long L = (long long)c->n_layers;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long long l = 0; l < L; ++l)
    {
        size_t base = (size_t)l * c->max_seq * kd;
        for (size_t i = 0; i < (size_t)pos * kd; ++i)
        {
            uint64_t h = or_splitmix64((uint64_t)l * 0x100000000ull + i);
            m->k_cache[base + i] = (float)((double)(h >> 40) * (1.0 / 16777216.0) - 0.5);
            m->v_cache[base + i] = (float)((double)(h & 0xFFFFFFull) * (1.0 / 16777216.0) - 0.5);
        }
    }
    m->pos = pos;
    return 0;
}
