/*
 * CPU oracle: plain-C restatement of the reference CPU algorithms on the
 * mini_llama hot path.  TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Build with -ffp-contract=off: every fp32 operation below is one IEEE rounding
 * in the same order as the reference C++ (which is compiled in ISO C++17 mode,
 * where GCC does not contract), so results are bit-identical to the reference.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "synth.h"

/* ---- fp16 conversion: src/quant.cpp:17-52 (round half up on bit 12) ---- */
uint16_t orc_f32_to_f16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof(bits));
    uint32_t sign = (bits >> 16) & 0x8000u;
    int32_t exponent = (int32_t)((bits >> 23) & 0xffu) - 127 + 15;
    uint32_t mantissa = bits & 0x7fffffu;
    if (exponent <= 0) {
        if (exponent < -10) return (uint16_t)sign;
        mantissa |= 0x800000u;
        uint32_t shifted = mantissa >> (1 - exponent);
        if (shifted & 0x1000u) shifted += 0x2000u;
        return (uint16_t)(sign | (shifted >> 13));
    }
    if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
    if (mantissa & 0x1000u) {
        mantissa += 0x2000u;
        if (mantissa & 0x800000u) {
            mantissa = 0;
            exponent += 1;
            if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
        }
    }
    return (uint16_t)(sign | ((uint32_t)exponent << 10) | (mantissa >> 13));
}

/* ---- src/quant.cpp:54-82 ---- */
float orc_f16_to_f32(uint16_t value) {
    uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
    uint32_t exponent = (value >> 10) & 0x1fu;
    uint32_t mantissa = value & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int32_t e = 1;
            while ((mantissa & 0x400u) == 0) {
                mantissa <<= 1;
                e -= 1;
            }
            mantissa &= 0x3ffu;
            bits = sign | ((uint32_t)(e - 15 + 127) << 23) | (mantissa << 13);
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent - 15 + 127) << 23) | (mantissa << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

size_t orc_block_bytes(int qtype) {
    switch (qtype) {
        case ORC_Q80: return sizeof(orc_block_q80);
        case ORC_Q40: return sizeof(orc_block_q40);
        case ORC_Q41: return sizeof(orc_block_q41);
        default: return 0;
    }
}

/* ---- Q8_0: src/quant.cpp:104-152 ---- */
static void quantize_q80_block(const float* x, int len, orc_block_q80* b) {
    memset(b, 0, sizeof(*b));
    float max_abs = 0.0f;
    for (int i = 0; i < len; ++i) max_abs = fmaxf(max_abs, fabsf(x[i]));
    if (max_abs > 0.0f) {
        float d = max_abs / 127.0f;
        b->d = orc_f32_to_f16(d);
        float stored = orc_f16_to_f32(b->d);
        float inv = (stored == 0.0f) ? 0.0f : 1.0f / stored;
        for (int i = 0; i < len; ++i) {
            int q = (int)roundf(x[i] * inv);
            if (q > 127) q = 127;
            else if (q < -127) q = -127;
            b->qs[i] = (int8_t)q;
        }
    }
}

/* ---- Q4_0: src/quant.cpp:182-240 (d = max|x|/7, q = round(x/d + 8)) ---- */
static void quantize_q40_block(const float* x, int len, orc_block_q40* b) {
    memset(b, 0, sizeof(*b));
    float max_abs = 0.0f;
    for (int i = 0; i < len; ++i) max_abs = fmaxf(max_abs, fabsf(x[i]));
    if (max_abs > 0.0f) {
        float d = max_abs / 7.0f;
        b->d = orc_f32_to_f16(d);
        float stored = orc_f16_to_f32(b->d);
        float inv = (stored == 0.0f) ? 0.0f : 1.0f / stored;
        for (int i = 0; i < 16; ++i) {
            float x0 = (i < len) ? x[i] * inv : 0.0f;
            float x1 = (i + 16 < len) ? x[i + 16] * inv : 0.0f;
            int q0 = (int)roundf(x0 + 8.0f);
            int q1 = (int)roundf(x1 + 8.0f);
            if (q0 < 0) q0 = 0;
            if (q0 > 15) q0 = 15;
            if (q1 < 0) q1 = 0;
            if (q1 > 15) q1 = 15;
            b->qs[i] = (uint8_t)((q1 << 4) | q0);
        }
    }
}

/* ---- Q4_1: the only Q4_1 quantizer of the reference is the GPU test's
 * QuantizeQ41ForTest, test/gpu_core_test.cpp:156-198 (d = range/15, m = min,
 * q = round((x - m)/d), division not reciprocal). ---- */
static void quantize_q41_block(const float* x, int len, orc_block_q41* b) {
    memset(b, 0, sizeof(*b));
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < len; ++i) {
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
    }
    float range = mx - mn;
    b->d = orc_f32_to_f16(range > 0.0f ? range / 15.0f : 0.0f);
    b->m = orc_f32_to_f16(isfinite(mn) ? mn : 0.0f);
    float d = orc_f16_to_f32(b->d);
    float m = orc_f16_to_f32(b->m);
    for (int i = 0; i < 16; ++i) {
        int q0 = (i < len && d != 0.0f) ? (int)roundf((x[i] - m) / d) : 0;
        int q1 = (i + 16 < len && d != 0.0f) ? (int)roundf((x[i + 16] - m) / d) : 0;
        q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
        q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
        b->qs[i] = (uint8_t)(q0 | (q1 << 4));
    }
}

void orc_quantize(int qtype, const float* x, int rows, int cols, void* out) {
    int nb = (cols + 31) / 32;
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; b < nb; ++b) {
            int begin = b * 32;
            int len = cols - begin < 32 ? cols - begin : 32;
            const float* src = x + (size_t)r * cols + begin;
            size_t idx = (size_t)r * nb + b;
            if (qtype == ORC_Q80) quantize_q80_block(src, len, (orc_block_q80*)out + idx);
            else if (qtype == ORC_Q40) quantize_q40_block(src, len, (orc_block_q40*)out + idx);
            else if (qtype == ORC_Q41) quantize_q41_block(src, len, (orc_block_q41*)out + idx);
        }
    }
}

/* ---- dequant of one element: src/quant.cpp:383-407 ---- */
static inline float deq(int qtype, const void* blk, int i) {
    if (qtype == ORC_Q80) {
        const orc_block_q80* b = (const orc_block_q80*)blk;
        float d = orc_f16_to_f32(b->d);
        return d * (float)b->qs[i];
    }
    if (qtype == ORC_Q40) {
        const orc_block_q40* b = (const orc_block_q40*)blk;
        float d = orc_f16_to_f32(b->d);
        int q = i < 16 ? (int)(b->qs[i] & 0x0f) - 8 : (int)(b->qs[i - 16] >> 4) - 8;
        return d * (float)q;
    }
    const orc_block_q41* b = (const orc_block_q41*)blk;
    float d = orc_f16_to_f32(b->d);
    float m = orc_f16_to_f32(b->m);
    int q = i < 16 ? (int)(b->qs[i] & 0x0f) : (int)(b->qs[i - 16] >> 4);
    return d * (float)q + m;
}

/* ---- src/quant.cpp:153-317 ---- */
void orc_dequantize(int qtype, const void* blocks, int rows, int cols, float* out) {
    int nb = (cols + 31) / 32;
    size_t bb = orc_block_bytes(qtype);
    for (int r = 0; r < rows; ++r)
        for (int k = 0; k < cols; ++k) {
            const char* blk = (const char*)blocks + ((size_t)r * nb + k / 32) * bb;
            out[(size_t)r * cols + k] = deq(qtype, blk, k % 32);
        }
}

/* ---- linear: src/quant.cpp:322-382 ---- */
typedef struct {
    int qtype, M, K, N, begin, end;
    const float* x;
    const void* w;
    float* y;
} linear_job;

static void linear_range(const linear_job* j) {
    int nb = (j->K + 31) / 32;
    size_t bb = orc_block_bytes(j->qtype);
    for (int flat = j->begin; flat < j->end; ++flat) {
        int row = flat / j->N;
        int n = flat % j->N;
        const float* xr = j->x + (size_t)row * j->K;
        const char* wr = (const char*)j->w + (size_t)n * nb * bb;
        float sum = 0.0f;
        for (int b = 0; b < nb; ++b) {
            int k0 = b * 32;
            int k1 = k0 + 32 < j->K ? k0 + 32 : j->K;
            const char* blk = wr + (size_t)b * bb;
            for (int k = k0; k < k1; ++k) {
                float w = deq(j->qtype, blk, k - k0);
                sum += w * xr[k];
            }
        }
        j->y[(size_t)row * j->N + n] = sum;
    }
}

static void* linear_thread(void* arg) {
    linear_range((const linear_job*)arg);
    return NULL;
}

void orc_linear(int qtype, const float* x, int M, int K, const void* w, int N, float* y,
                int threads) {
    int total = M * N;
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    if (threads == 1 || total < threads * 16) {
        linear_job j = {qtype, M, K, N, 0, total, x, w, y};
        linear_range(&j);
        return;
    }
    pthread_t tid[64];
    linear_job jobs[64];
    int chunk = total / threads, rem = total % threads, start = 0;
    for (int t = 0; t < threads; ++t) {
        int cnt = chunk + (t < rem ? 1 : 0);
        linear_job j = {qtype, M, K, N, start, start + cnt, x, w, y};
        jobs[t] = j;
        start += cnt;
        pthread_create(&tid[t], NULL, linear_thread, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
}

/* ---- src/ops.cpp:49-69 ---- */
void orc_rmsnorm(const float* x, const float* w, int n, float eps, float* y) {
    float ss = 0.0f;
    for (int i = 0; i < n; ++i) ss += x[i] * x[i];
    ss = ss / (float)n;
    float scale = 1.0f / sqrtf(ss + eps);
    for (int i = 0; i < n; ++i) y[i] = x[i] * scale * w[i];
}

/* ---- rope tables: src/context.cpp:16-25 ---- */
void orc_rope_tables(int max_seq_len, int head_dim, float theta, float* cos_t, float* sin_t) {
    int half = head_dim / 2;
    for (int pos = 0; pos < max_seq_len; ++pos)
        for (int i = 0; i < half; ++i) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
            cos_t[(size_t)pos * half + i] = cosf((float)pos * freq);
            sin_t[(size_t)pos * half + i] = sinf((float)pos * freq);
        }
}

/* ---- src/ops.cpp:123-168 ---- */
void orc_rope_apply(float* x, int rows, int head_dim, int pos, const float* cos_t,
                    const float* sin_t, int neox) {
    int half = head_dim / 2;
    size_t off = (size_t)pos * half;
    for (int r = 0; r < rows; ++r) {
        float* row = x + (size_t)r * head_dim;
        for (int i = 0; i < half; ++i) {
            int a = neox ? i : 2 * i;
            int b = neox ? i + half : 2 * i + 1;
            float c = cos_t[off + i], s = sin_t[off + i];
            float x0 = row[a], x1 = row[b];
            row[a] = x0 * c - x1 * s;
            row[b] = x0 * s + x1 * c;
        }
    }
}

void orc_rope_direct(float* x, int rows, int head_dim, int pos, float theta, int neox) {
    int half = head_dim / 2;
    for (int r = 0; r < rows; ++r) {
        float* row = x + (size_t)r * head_dim;
        for (int i = 0; i < half; ++i) {
            int a = neox ? i : 2 * i;
            int b = neox ? i + half : 2 * i + 1;
            float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
            float c = cosf((float)pos * freq), s = sinf((float)pos * freq);
            float x0 = row[a], x1 = row[b];
            row[a] = x0 * c - x1 * s;
            row[b] = x0 * s + x1 * c;
        }
    }
}

/* ---- GQA decode attention: src/forward.cpp:483-563 ---- */
void orc_attention(const float* q, const float* kcache, const float* vcache, int layer, int pos,
                   int max_seq_len, int n_heads, int n_kv_heads, int head_dim, float* out,
                   float* scores) {
    float scale = 1.0f / sqrtf((float)head_dim);
    int group = n_heads / n_kv_heads;
    size_t pos_stride = (size_t)n_kv_heads * head_dim;
    size_t layer_base = (size_t)layer * max_seq_len * pos_stride;
    for (int h = 0; h < n_heads; ++h) {
        int kvh = h / group;
        const float* qh = q + (size_t)h * head_dim;
        for (int p = 0; p <= pos; ++p) {
            const float* k = kcache + layer_base + (size_t)p * pos_stride + (size_t)kvh * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; ++d) dot += qh[d] * k[d];
            scores[p] = dot * scale;
        }
        float mx = scores[0];
        for (int p = 1; p <= pos; ++p) mx = scores[p] > mx ? scores[p] : mx;
        float sum = 0.0f;
        for (int p = 0; p <= pos; ++p) {
            scores[p] = expf(scores[p] - mx);
            sum += scores[p];
        }
        for (int p = 0; p <= pos; ++p) scores[p] /= sum;
        for (int d = 0; d < head_dim; ++d) {
            float val = 0.0f;
            for (int p = 0; p <= pos; ++p) {
                const float* v =
                    vcache + layer_base + (size_t)p * pos_stride + (size_t)kvh * head_dim;
                val += scores[p] * v[d];
            }
            out[(size_t)h * head_dim + d] = val;
        }
    }
}

/* ---- src/ops.cpp:72-120, :199-212 ---- */
void orc_softmax(const float* x, int n, float* y) {
    float mx = x[0];
    for (int i = 1; i < n; ++i)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        y[i] = expf(x[i] - mx);
        sum += y[i];
    }
    for (int i = 0; i < n; ++i) y[i] /= sum;
}

void orc_silu(const float* x, int n, float* y) {
    for (int i = 0; i < n; ++i) y[i] = x[i] / (1.0f + expf(-x[i]));
}

void orc_swiglu(const float* gate, const float* up, int n, float* y) {
    for (int i = 0; i < n; ++i) {
        float v = gate[i];
        float sig = 1.0f / (1.0f + expf(-v));
        y[i] = v * sig * up[i];
    }
}

int orc_argmax(const float* x, int n) {
    int idx = 0;
    float mx = x[0];
    for (int i = 0; i < n; ++i)
        if (x[i] > mx) {
            idx = i;
            mx = x[i];
        }
    return idx;
}

/* ---- synthetic inputs (threaded fill) ---- */
typedef struct {
    float* out;
    size_t begin, end;
    uint64_t key;
    double sigma;
} fill_job;

static void* fill_thread(void* arg) {
    fill_job* j = (fill_job*)arg;
    for (size_t i = j->begin; i < j->end; ++i) j->out[i] = synth_normal(j->key, i, j->sigma);
    return NULL;
}

void orc_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream, double sigma,
                      int threads) {
    uint64_t key = synth_key(seed, stream);
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    if (threads == 1 || n < (size_t)1 << 16) {
        fill_job j = {out, 0, n, key, sigma};
        fill_thread(&j);
        return;
    }
    pthread_t tid[64];
    fill_job jobs[64];
    size_t chunk = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        size_t b = (size_t)t * chunk, e = b + chunk < n ? b + chunk : n;
        if (b > n) b = n;
        fill_job j = {out, b, e, key, sigma};
        jobs[t] = j;
        pthread_create(&tid[t], NULL, fill_thread, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
}

void orc_synth_tokens(int* out, int n, uint64_t seed, int vocab) {
    uint64_t key = synth_key(seed, SYNTH_STREAM_PROMPT);
    for (int i = 0; i < n; ++i) out[i] = (int)synth_index(key, (uint64_t)i, (uint32_t)vocab);
}

/* ---- synthetic transformer: forward of src/forward.cpp:592-666 ---- */
typedef struct {
    float* attn_norm;
    float* ffn_norm;
    void* wq;
    void* wk;
    void* wv;
    void* wo;
    void* gate;
    void* up;
    void* down;
    float* bq;
    float* bk;
    float* bv;
} orc_layer;

struct orc_model {
    orc_config c;
    int threads;
    float* embedding;
    float* final_norm;
    void* lm_head;
    orc_layer* layers;
    float* kcache;
    float* vcache;
    float* cos_t;
    float* sin_t;
    float *x, *h, *q, *k, *v, *att, *proj, *gate, *up, *ff, *scores;
};

static size_t qbytes(int qtype, int rows, int cols) {
    return (size_t)rows * ((cols + 31) / 32) * orc_block_bytes(qtype);
}

static void* make_linear(const orc_config* c, uint64_t seed, uint64_t stream, int rows, int cols,
                         float* scratch, int threads) {
    orc_synth_normal(scratch, (size_t)rows * cols, seed, stream, 0.02, threads);
    void* q = malloc(qbytes(c->qtype, rows, cols));
    orc_quantize(c->qtype, scratch, rows, cols, q);
    return q;
}

static float* make_vec(int n, float fill) {
    float* v = (float*)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < n; ++i) v[i] = fill;
    return v;
}

orc_model* orc_model_create_synth(const orc_config* cfg, uint64_t seed, int threads) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    m->threads = threads;
    const orc_config* c = &m->c;
    int D = c->dim, F = c->hidden_dim, V = c->vocab_size;
    int QD = c->n_heads * c->head_dim, KD = c->n_kv_heads * c->head_dim;
    size_t biggest = (size_t)F * D;
    if ((size_t)V * D > biggest) biggest = (size_t)V * D;
    if ((size_t)QD * D > biggest) biggest = (size_t)QD * D;
    float* scratch = (float*)malloc(sizeof(float) * biggest);

    m->embedding = (float*)malloc(sizeof(float) * (size_t)V * D);
    orc_synth_normal(m->embedding, (size_t)V * D, seed, SYNTH_STREAM_EMBEDDING, 0.02, threads);
    m->final_norm = make_vec(D, 1.0f);
    m->layers = (orc_layer*)calloc((size_t)c->n_layers, sizeof(orc_layer));
    for (int l = 0; l < c->n_layers; ++l) {
        orc_layer* L = &m->layers[l];
        L->attn_norm = make_vec(D, 1.0f);
        L->ffn_norm = make_vec(D, 1.0f);
        L->wq = make_linear(c, seed, synth_stream_layer(l, SYNTH_KIND_WQ), QD, D, scratch, threads);
        L->wk = make_linear(c, seed, synth_stream_layer(l, SYNTH_KIND_WK), KD, D, scratch, threads);
        L->wv = make_linear(c, seed, synth_stream_layer(l, SYNTH_KIND_WV), KD, D, scratch, threads);
        L->wo = make_linear(c, seed, synth_stream_layer(l, SYNTH_KIND_WO), D, QD, scratch, threads);
        L->gate = make_linear(c, seed, synth_stream_layer(l, SYNTH_KIND_GATE), F, D, scratch,
                              threads);
        L->up = make_linear(c, seed, synth_stream_layer(l, SYNTH_KIND_UP), F, D, scratch, threads);
        L->down = make_linear(c, seed, synth_stream_layer(l, SYNTH_KIND_DOWN), D, F, scratch,
                              threads);
        if (c->qkv_bias) {
            L->bq = (float*)malloc(sizeof(float) * QD);
            L->bk = (float*)malloc(sizeof(float) * KD);
            L->bv = (float*)malloc(sizeof(float) * KD);
            orc_synth_normal(L->bq, QD, seed, synth_stream_layer(l, SYNTH_KIND_BQ), 0.02, 1);
            orc_synth_normal(L->bk, KD, seed, synth_stream_layer(l, SYNTH_KIND_BK), 0.02, 1);
            orc_synth_normal(L->bv, KD, seed, synth_stream_layer(l, SYNTH_KIND_BV), 0.02, 1);
        }
    }
    if (c->tied_embedding) {
        m->lm_head = malloc(qbytes(c->qtype, V, D));
        orc_quantize(c->qtype, m->embedding, V, D, m->lm_head);
    } else {
        m->lm_head = make_linear(c, seed, SYNTH_STREAM_LM_HEAD, V, D, scratch, threads);
    }
    free(scratch);

    size_t cache = (size_t)c->n_layers * c->max_seq_len * KD;
    m->kcache = (float*)calloc(cache, sizeof(float));
    m->vcache = (float*)calloc(cache, sizeof(float));
    int half = c->head_dim / 2;
    m->cos_t = (float*)malloc(sizeof(float) * (size_t)c->max_seq_len * half);
    m->sin_t = (float*)malloc(sizeof(float) * (size_t)c->max_seq_len * half);
    orc_rope_tables(c->max_seq_len, c->head_dim, c->rope_theta, m->cos_t, m->sin_t);
    m->x = make_vec(D, 0.f);
    m->h = make_vec(D, 0.f);
    m->q = make_vec(QD, 0.f);
    m->k = make_vec(KD, 0.f);
    m->v = make_vec(KD, 0.f);
    m->att = make_vec(QD, 0.f);
    m->proj = make_vec(D, 0.f);
    m->gate = make_vec(F, 0.f);
    m->up = make_vec(F, 0.f);
    m->ff = make_vec(F, 0.f);
    m->scores = make_vec(c->max_seq_len, 0.f);
    return m;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    for (int l = 0; l < m->c.n_layers; ++l) {
        orc_layer* L = &m->layers[l];
        free(L->attn_norm);
        free(L->ffn_norm);
        free(L->wq);
        free(L->wk);
        free(L->wv);
        free(L->wo);
        free(L->gate);
        free(L->up);
        free(L->down);
        free(L->bq);
        free(L->bk);
        free(L->bv);
    }
    free(m->layers);
    free(m->embedding);
    free(m->final_norm);
    free(m->lm_head);
    free(m->kcache);
    free(m->vcache);
    free(m->cos_t);
    free(m->sin_t);
    free(m->x);
    free(m->h);
    free(m->q);
    free(m->k);
    free(m->v);
    free(m->att);
    free(m->proj);
    free(m->gate);
    free(m->up);
    free(m->ff);
    free(m->scores);
    free(m);
}

const void* orc_model_tensor(const orc_model* m, int layer, int kind, size_t* bytes) {
    const orc_config* c = &m->c;
    int D = c->dim, F = c->hidden_dim, V = c->vocab_size;
    int QD = c->n_heads * c->head_dim, KD = c->n_kv_heads * c->head_dim;
    const orc_layer* L = (layer >= 0 && layer < c->n_layers) ? &m->layers[layer] : NULL;
    size_t b = 0;
    const void* p = NULL;
    switch (kind) {
        case ORC_T_EMBEDDING: p = m->embedding; b = sizeof(float) * (size_t)V * D; break;
        case ORC_T_FINAL_NORM: p = m->final_norm; b = sizeof(float) * D; break;
        case ORC_T_LM_HEAD: p = m->lm_head; b = qbytes(c->qtype, V, D); break;
        default:
            if (!L) break;
            switch (kind) {
                case ORC_T_ATTN_NORM: p = L->attn_norm; b = sizeof(float) * D; break;
                case ORC_T_FFN_NORM: p = L->ffn_norm; b = sizeof(float) * D; break;
                case ORC_T_WQ: p = L->wq; b = qbytes(c->qtype, QD, D); break;
                case ORC_T_WK: p = L->wk; b = qbytes(c->qtype, KD, D); break;
                case ORC_T_WV: p = L->wv; b = qbytes(c->qtype, KD, D); break;
                case ORC_T_WO: p = L->wo; b = qbytes(c->qtype, D, QD); break;
                case ORC_T_GATE: p = L->gate; b = qbytes(c->qtype, F, D); break;
                case ORC_T_UP: p = L->up; b = qbytes(c->qtype, F, D); break;
                case ORC_T_DOWN: p = L->down; b = qbytes(c->qtype, D, F); break;
                case ORC_T_BQ: p = L->bq; b = L->bq ? sizeof(float) * QD : 0; break;
                case ORC_T_BK: p = L->bk; b = L->bk ? sizeof(float) * KD : 0; break;
                case ORC_T_BV: p = L->bv; b = L->bv ? sizeof(float) * KD : 0; break;
                default: break;
            }
    }
    if (bytes) *bytes = b;
    return p;
}

void orc_model_reset(orc_model* m) {
    const orc_config* c = &m->c;
    size_t cache = (size_t)c->n_layers * c->max_seq_len * c->n_kv_heads * c->head_dim;
    memset(m->kcache, 0, cache * sizeof(float));
    memset(m->vcache, 0, cache * sizeof(float));
}

int orc_model_forward(orc_model* m, int token, int pos, float* logits) {
    const orc_config* c = &m->c;
    int D = c->dim, F = c->hidden_dim;
    int QD = c->n_heads * c->head_dim, KD = c->n_kv_heads * c->head_dim;
    if (token < 0 || token >= c->vocab_size || pos < 0 || pos >= c->max_seq_len) return -1;
    int qt = c->qtype, T = m->threads;
    memcpy(m->x, m->embedding + (size_t)token * D, sizeof(float) * D);
    size_t pos_stride = (size_t)KD;
    for (int l = 0; l < c->n_layers; ++l) {
        orc_layer* L = &m->layers[l];
        orc_rmsnorm(m->x, L->attn_norm, D, c->rms_norm_eps, m->h);
        orc_linear(qt, m->h, 1, D, L->wq, QD, m->q, T);
        orc_linear(qt, m->h, 1, D, L->wk, KD, m->k, T);
        orc_linear(qt, m->h, 1, D, L->wv, KD, m->v, T);
        if (L->bq) {
            for (int i = 0; i < QD; ++i) m->q[i] += L->bq[i];
            for (int i = 0; i < KD; ++i) m->k[i] += L->bk[i];
            for (int i = 0; i < KD; ++i) m->v[i] += L->bv[i];
        }
        orc_rope_apply(m->q, c->n_heads, c->head_dim, pos, m->cos_t, m->sin_t, c->rope_neox);
        orc_rope_apply(m->k, c->n_kv_heads, c->head_dim, pos, m->cos_t, m->sin_t, c->rope_neox);
        size_t slot = ((size_t)l * c->max_seq_len + pos) * pos_stride;
        memcpy(m->kcache + slot, m->k, sizeof(float) * KD);
        memcpy(m->vcache + slot, m->v, sizeof(float) * KD);
        orc_attention(m->q, m->kcache, m->vcache, l, pos, c->max_seq_len, c->n_heads,
                      c->n_kv_heads, c->head_dim, m->att, m->scores);
        orc_linear(qt, m->att, 1, QD, L->wo, D, m->proj, T);
        for (int i = 0; i < D; ++i) m->x[i] = m->x[i] + m->proj[i];
        orc_rmsnorm(m->x, L->ffn_norm, D, c->rms_norm_eps, m->h);
        orc_linear(qt, m->h, 1, D, L->gate, F, m->gate, T);
        orc_linear(qt, m->h, 1, D, L->up, F, m->up, T);
        orc_swiglu(m->gate, m->up, F, m->ff);
        orc_linear(qt, m->ff, 1, F, L->down, D, m->proj, T);
        for (int i = 0; i < D; ++i) m->x[i] = m->x[i] + m->proj[i];
    }
    orc_rmsnorm(m->x, m->final_norm, D, c->rms_norm_eps, m->h);
    orc_linear(qt, m->h, 1, D, m->lm_head, c->vocab_size, logits, T);
    return 0;
}
