/*
 * ekv_oracle.c -- CPU restatement of the reference path. TEST INFRASTRUCTURE ONLY.
 *
 * Used as the parity checker by tests/, by __graft_entry__.smoke(), and as the timed CPU
 * baseline by bench.py. The product library never links or calls this file.
 * Every function names the reference lines it restates; ekv_oracle.h has the overview.
 */
#include "ekv_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

const char *ekvo_version(void) { return "ekv-oracle 1"; }

/* ------------------------------------------------------------------------------------------
 * Number formats
 * ------------------------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* gguf-py quants.py:204-213: NaN is forced quiet by setting bit 6 of the upper half, then
 * round-to-nearest-even on the dropped 16 bits. */
uint16_t ekvo_f32_to_bf16(float x) {
    uint32_t n = f2u(x);
    if ((n & 0x7fffffffu) > 0x7f800000u) n = (n & 0xffff0000u) | (64u << 16);
    uint64_t r = ((uint64_t)n + (0x7fffu + ((n >> 16) & 1u))) >> 16;
    return (uint16_t)r;
}

float ekvo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

void ekvo_f32_to_bf16_n(const float *x, uint16_t *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = ekvo_f32_to_bf16(x[i]);
}

void ekvo_bf16_to_f32_n(const uint16_t *x, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = ekvo_bf16_to_f32(x[i]);
}

/* IEEE binary16 with round-to-nearest-even, the conversion numpy's astype(np.float16) makes
 * (gguf-py quants.py:390 stores the Q8_0 scale that way). */
uint16_t ekvo_f32_to_f16(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {
        if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                   /* below 2^-14: subnormal */
        if (ax < 0x33000000u) return (uint16_t)sign;          /* below 2^-25: zero      */
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;                      /* 14..24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t r = ax - 0x38000000u;
    r = (r + 0xfffu + ((r >> 13) & 1u)) >> 13;
    return (uint16_t)(sign | r);
}

float ekvo_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    const uint32_t m = (uint32_t)h & 0x3ffu;
    if (e == 0) {
        if (m == 0) return u2f(sign);
        /* subnormal: m * 2^-24, exact in f32 */
        const float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* gguf-py quants.py:378-393 (bit-exact with quantize_row_q8_0_ref in ggml-quants.c):
 *   d  = max|x| / 127            (float32 division)
 *   id = d ? 1/d : 0             (float32 division)
 *   q  = roundf(x * id)          (np_roundf quants.py:43-47 rounds half away from zero)
 *   block = { fp16(d), int8 q[32] }  (d rounded to nearest even)
 * The quantised values use the float32 d, not its fp16 rounding. */
void ekvo_quantize_q8_0(const float *x, int64_t n, uint8_t *out) {
    const int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const float *xb = x + b * 32;
        uint8_t *ob = out + b * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = ekvo_f32_to_f16(d);
        memcpy(ob, &dh, 2);
        for (int j = 0; j < 32; ++j) {
            const float r = roundf(xb[j] * id);
            ob[2 + j] = (uint8_t)(int8_t)r;
        }
    }
}

/* gguf-py quants.py:395-401: x = qs * float(d) */
void ekvo_dequantize_q8_0(const uint8_t *blocks, int64_t n, float *out) {
    const int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *ib = blocks + b * 34;
        uint16_t dh;
        memcpy(&dh, ib, 2);
        const float d = ekvo_f16_to_f32(dh);
        for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)ib[2 + j] * d;
    }
}

/* ------------------------------------------------------------------------------------------
 * Masks
 * ------------------------------------------------------------------------------------------ */

/* LingBot-VA flex masks over per-token metadata (models/lingbot_va.cpp:9273-9348): the packed
 * words decoded back to the reference's seq_ids (-1 = padding), frame_ids and noise_ids. */
static void flex_decode(int32_t w, int64_t *seq, int64_t *frame, int64_t *noise) {
    const uint32_t u = (uint32_t)w;
    *seq = (int64_t)(u >> 24) - 1;
    *noise = (int64_t)((u >> 23) & 1u);
    *frame = (int64_t)(u & 0x7FFFFFu);
}

/* flex_self_allowed, models/lingbot_va.cpp:9336-9344 */
static int flex_self_allowed(int32_t qw, int32_t kw, int64_t window_size) {
    int64_t qs, qf, qn, ks, kf, kn;
    flex_decode(qw, &qs, &qf, &qn);
    flex_decode(kw, &ks, &kf, &kn);
    if (qs < 0 || qs != ks) return 0;
    const int clean2clean = qn == 1 && kn == 1 && kf <= qf;
    const int noise2clean = qn == 0 && kn == 1 && kf < qf;
    const int noise2noise = qn == 0 && kn == 0 && kf == qf;
    const int64_t df = qf > kf ? qf - kf : kf - qf;
    return (clean2clean || noise2clean || noise2noise) && df <= window_size;
}

/* flex_cross_allowed, models/lingbot_va.cpp:9346-9348 (the key word carries its text_seq_id) */
static int flex_cross_allowed(int32_t qw, int32_t kw) {
    int64_t qs, qf, qn, ks, kf, kn;
    flex_decode(qw, &qs, &qf, &qn);
    flex_decode(kw, &ks, &kf, &kn);
    return qs >= 0 && qs == ks;
}

static int flex_ok(const ekvo_mask *m, const ekvo_seq *s, int32_t q, int32_t k) {
    if (!(m->flags & (EKVO_MASK_FLEX_SELF | EKVO_MASK_FLEX_CROSS))) return 1;
    if (!s->flex_meta) return 0;
    const int32_t qw = s->flex_meta[m->flex_q0 + q], kw = s->flex_meta[m->flex_k0 + k];
    if ((m->flags & EKVO_MASK_FLEX_SELF) && !flex_self_allowed(qw, kw, m->flex_window)) return 0;
    if ((m->flags & EKVO_MASK_FLEX_CROSS) && !flex_cross_allowed(qw, kw)) return 0;
    return 1;
}

int ekvo_allowed(const ekvo_mask *m, const ekvo_seq *s, int32_t q, int32_t k) {
    if (k < 0) return 0;
    if (k < s->n_prefix + s->n_suffix && !flex_ok(m, s, q, k)) return 0;
    if (k < s->n_prefix) {
        /* padding: models/smolvla.cpp:707-716 sets -inf on keys with prefix_valid == 0 */
        if (k >= s->prefix_valid) return 0;
        /* GR00T cross masks, models/groot_n1.cpp:708-718:
         * text mask = valid && !image, image mask = valid && image */
        const int in_span = k >= s->span_begin && k < s->span_end;
        if ((m->flags & EKVO_MASK_SPAN_ONLY) && !in_span) return 0;
        if ((m->flags & EKVO_MASK_SPAN_EXCLUDE) && in_span) return 0;
        if (m->flags & EKVO_MASK_BLOCK_CAUSAL) {
            /* Bidirectional inside a chunk, causal across chunks, `window_chunks` chunks
             * visible (the query's own included); padded slots of a chunk are invalid. */
            const int32_t kc = k / m->chunk_stride;
            const int32_t within = k - kc * m->chunk_stride;
            if (within >= m->chunk_tokens) return 0;
            const int32_t qc = m->q_chunk0 + q / m->chunk_tokens;
            if (kc > qc || qc - kc >= m->window_chunks) return 0;
        }
        return 1;
    }
    const int32_t sk = k - s->n_prefix;
    if (sk >= s->n_suffix) return 0;
    /* models/smolvla.cpp:718-720: causal inside the action chunk */
    if ((m->flags & EKVO_MASK_SUFFIX_CAUSAL) && sk > q) return 0;
    /* models/hy_vla.cpp:2355-2367: suffix row 0 sees only suffix key 0 */
    if ((m->flags & EKVO_MASK_SUFFIX_PREFIX_LM) && q == 0 && sk != 0) return 0;
    /* pi0.5: everything else visible (mask all zeros, models/pi05.cpp:880-882) */
    return 1;
}

/* ------------------------------------------------------------------------------------------
 * Attention, ggml op semantics (models/pi05.cpp:414-421):
 *   kq   = mul_mat(K, Q)            F32 dot products over head_dim
 *   attn = soft_max_ext(kq, mask, scale, 0): softmax(kq*scale + mask) per query row,
 *          exponentials in float, their sum in double (ggml_float), then scaled by 1/sum
 *   kqv  = mul_mat(V, attn)         F32 accumulation over keys
 * Rows with no visible key give 0 (models/lingbot_va.cpp:9503-9506).
 * ------------------------------------------------------------------------------------------ */

typedef struct {
    const ekvo_attn_args *a;
    atomic_int next;
} attn_job;

static void attn_row_f32(const ekvo_attn_args *a, int32_t b, int32_t t, float *w) {
    const int32_t D = a->D, Hq = a->Hq, Hkv = a->Hkv, L = a->Lk_max;
    const int32_t group = Hq / Hkv;
    const ekvo_seq *s = &a->seqs[b];
    const int32_t nk = s->n_prefix + s->n_suffix;
    for (int32_t h = 0; h < Hq; ++h) {
        const int32_t g = h / group;
        const float *qr = a->q + (((int64_t)b * a->Tq + t) * Hq + h) * D;
        float *o = a->out + (((int64_t)b * a->Tq + t) * Hq + h) * D;
        float mx = -INFINITY;
        for (int32_t k = 0; k < nk && k < L; ++k) {
            w[k] = -INFINITY;
            if (!ekvo_allowed(&a->mask, s, t, k)) continue;
            const float *kr = a->k + (((int64_t)b * L + k) * Hkv + g) * D;
            float dot = 0.0f;
            for (int32_t d = 0; d < D; ++d) dot += kr[d] * qr[d];
            float x = dot * a->scale;
            if (a->dense_mask) x += a->dense_mask[((int64_t)b * a->Tq + t) * L + k];
            w[k] = x;
            if (x > mx) mx = x;
        }
        for (int32_t d = 0; d < D; ++d) o[d] = 0.0f;
        if (mx == -INFINITY) continue;
        double sum = 0.0;
        for (int32_t k = 0; k < nk && k < L; ++k) {
            const float e = (w[k] == -INFINITY) ? 0.0f : expf(w[k] - mx);
            w[k] = e;
            sum += (double)e;
        }
        const float inv = (float)(1.0 / sum);
        for (int32_t k = 0; k < nk && k < L; ++k) {
            if (w[k] == 0.0f) continue;
            const float p = w[k] * inv;
            const float *vr = a->v + (((int64_t)b * L + k) * Hkv + g) * D;
            for (int32_t d = 0; d < D; ++d) o[d] += p * vr[d];
        }
    }
}

/* One query row (b, t, h) into o[D], as attn_row_f32 computes it. */
static void attn_one_row_f32(const ekvo_attn_args *a, int32_t b, int32_t t, int32_t h, float *w, float *o) {
    const int32_t D = a->D, Hq = a->Hq, Hkv = a->Hkv, L = a->Lk_max;
    const int32_t g = h / (Hq / Hkv);
    const ekvo_seq *s = &a->seqs[b];
    const int32_t nk = s->n_prefix + s->n_suffix;
    const float *qr = a->q + (((int64_t)b * a->Tq + t) * Hq + h) * D;
    float mx = -INFINITY;
    for (int32_t k = 0; k < nk && k < L; ++k) {
        w[k] = -INFINITY;
        if (!ekvo_allowed(&a->mask, s, t, k)) continue;
        const float *kr = a->k + (((int64_t)b * L + k) * Hkv + g) * D;
        float dot = 0.0f;
        for (int32_t d = 0; d < D; ++d) dot += kr[d] * qr[d];
        float x = dot * a->scale;
        if (a->dense_mask) x += a->dense_mask[((int64_t)b * a->Tq + t) * L + k];
        w[k] = x;
        if (x > mx) mx = x;
    }
    for (int32_t d = 0; d < D; ++d) o[d] = 0.0f;
    if (mx == -INFINITY) return;
    double sum = 0.0;
    for (int32_t k = 0; k < nk && k < L; ++k) {
        const float e = (w[k] == -INFINITY) ? 0.0f : expf(w[k] - mx);
        w[k] = e;
        sum += (double)e;
    }
    const float inv = (float)(1.0 / sum);
    for (int32_t k = 0; k < nk && k < L; ++k) {
        if (w[k] == 0.0f) continue;
        const float p = w[k] * inv;
        const float *vr = a->v + (((int64_t)b * L + k) * Hkv + g) * D;
        for (int32_t d = 0; d < D; ++d) o[d] += p * vr[d];
    }
}

typedef struct {
    const ekvo_attn_args *a;
    int32_t n_rows;
    const int32_t *rows;
    float *out;
    atomic_int next;
} rows_job;

static void *rows_worker(void *arg) {
    rows_job *j = (rows_job *)arg;
    float *w = (float *)malloc(sizeof(float) * (size_t)(j->a->Lk_max > 0 ? j->a->Lk_max : 1));
    for (;;) {
        const int i = atomic_fetch_add(&j->next, 1);
        if (i >= j->n_rows) break;
        attn_one_row_f32(j->a, j->rows[3 * i], j->rows[3 * i + 1], j->rows[3 * i + 2], w, j->out + (int64_t)i * j->a->D);
    }
    free(w);
    return NULL;
}

static void *attn_worker(void *arg) {
    attn_job *j = (attn_job *)arg;
    const ekvo_attn_args *a = j->a;
    float *w = (float *)malloc(sizeof(float) * (size_t)(a->Lk_max > 0 ? a->Lk_max : 1));
    for (;;) {
        const int item = atomic_fetch_add(&j->next, 1);
        if (item >= a->B * a->Tq) break;
        attn_row_f32(a, item / a->Tq, item % a->Tq, w);
    }
    free(w);
    return NULL;
}

static int check_args(const ekvo_attn_args *a) {
    if (!a || !a->q || !a->k || !a->v || !a->seqs || !a->out) return -1;
    if (a->B <= 0 || a->Tq <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->D <= 0 || a->Lk_max < 0) return -1;
    if (a->Hq % a->Hkv) return -1;
    if ((a->mask.flags & EKVO_MASK_BLOCK_CAUSAL) &&
        (a->mask.chunk_tokens <= 0 || a->mask.chunk_stride < a->mask.chunk_tokens ||
         a->mask.window_chunks <= 0))
        return -1;
    return 0;
}

int ekvo_attention_f32(const ekvo_attn_args *a, int n_threads) {
    if (check_args(a)) return -1;
    attn_job job;
    job.a = a;
    atomic_init(&job.next, 0);
    if (n_threads <= 1) {
        attn_worker(&job);
        return 0;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, attn_worker, &job);
    for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
    free(th);
    return 0;
}

int ekvo_attention_rows(const ekvo_attn_args *a, int32_t n_rows, const int32_t *rows, float *out, int n_threads) {
    if (check_args(a) || n_rows < 0 || (n_rows && (!rows || !out))) return -1;
    for (int32_t i = 0; i < n_rows; ++i)
        if (rows[3 * i] < 0 || rows[3 * i] >= a->B || rows[3 * i + 1] < 0 || rows[3 * i + 1] >= a->Tq ||
            rows[3 * i + 2] < 0 || rows[3 * i + 2] >= a->Hq)
            return -1;
    rows_job job;
    job.a = a;
    job.n_rows = n_rows;
    job.rows = rows;
    job.out = out;
    atomic_init(&job.next, 0);
    if (n_threads <= 1) {
        rows_worker(&job);
        return 0;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, rows_worker, &job);
    for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
    free(th);
    return 0;
}

int ekvo_attention_f64(const ekvo_attn_args *a, double *out) {
    if (check_args(a) || !out) return -1;
    const int32_t D = a->D, Hq = a->Hq, Hkv = a->Hkv, L = a->Lk_max;
    const int32_t group = Hq / Hkv;
    double *w = (double *)malloc(sizeof(double) * (size_t)(L > 0 ? L : 1));
    for (int32_t b = 0; b < a->B; ++b) {
        const ekvo_seq *s = &a->seqs[b];
        const int32_t nk = s->n_prefix + s->n_suffix;
        for (int32_t t = 0; t < a->Tq; ++t) {
            for (int32_t h = 0; h < Hq; ++h) {
                const int32_t g = h / group;
                const float *qr = a->q + (((int64_t)b * a->Tq + t) * Hq + h) * D;
                double *o = out + (((int64_t)b * a->Tq + t) * Hq + h) * D;
                double mx = -INFINITY;
                int any = 0;
                for (int32_t k = 0; k < nk && k < L; ++k) {
                    w[k] = -INFINITY;
                    if (!ekvo_allowed(&a->mask, s, t, k)) continue;
                    const float *kr = a->k + (((int64_t)b * L + k) * Hkv + g) * D;
                    double dot = 0.0;
                    for (int32_t d = 0; d < D; ++d) dot += (double)kr[d] * (double)qr[d];
                    double x = dot * (double)a->scale;
                    if (a->dense_mask) x += (double)a->dense_mask[((int64_t)b * a->Tq + t) * L + k];
                    w[k] = x;
                    if (x > mx) mx = x;
                    any = 1;
                }
                for (int32_t d = 0; d < D; ++d) o[d] = 0.0;
                if (!any || mx == -INFINITY) continue;
                double sum = 0.0;
                for (int32_t k = 0; k < nk && k < L; ++k) {
                    w[k] = (w[k] == -INFINITY) ? 0.0 : exp(w[k] - mx);
                    sum += w[k];
                }
                for (int32_t k = 0; k < nk && k < L; ++k) {
                    if (w[k] == 0.0) continue;
                    const double p = w[k] / sum;
                    const float *vr = a->v + (((int64_t)b * L + k) * Hkv + g) * D;
                    for (int32_t d = 0; d < D; ++d) o[d] += p * (double)vr[d];
                }
            }
        }
    }
    free(w);
    return 0;
}

/* ------------------------------------------------------------------------------------------
 * Timed CPU baseline: the reference's per-call work on the host (models/pi05.cpp:406-421):
 * the prefix K/V rows of the layer are turned into f32 (dequantised when Q8_0), the suffix
 * is concatenated, and every (token, head) row runs K*Q, masked softmax, V*attn in f32.
 * Parallel over (call, request) items on a shared counter.
 * ------------------------------------------------------------------------------------------ */

typedef struct {
    const ekvo_cache_args *a;
    atomic_int next;
} cache_job;

static void *cache_worker(void *arg) {
    cache_job *j = (cache_job *)arg;
    const ekvo_cache_args *a = j->a;
    const int32_t D = a->D, Hq = a->Hq, Hkv = a->Hkv, Tq = a->Tq;
    const int32_t Lmax = a->max_prefix + a->n_suffix;
    const int32_t group = Hq / Hkv;
    float *kf = (float *)malloc(sizeof(float) * (size_t)Lmax * Hkv * D);
    float *vf = (float *)malloc(sizeof(float) * (size_t)Lmax * Hkv * D);
    float *w = (float *)malloc(sizeof(float) * (size_t)Lmax);
    float *qf = (float *)malloc(sizeof(float) * (size_t)D);
    /* Each worker writes a private output; only the last call's rows (one item per request)
     * go to the caller's buffer, so no two threads write the same row. */
    float *own = (float *)malloc(sizeof(float) * (size_t)Tq * Hq * D);
    const int64_t row_elems = (int64_t)Hkv * D;
    const int64_t row_bytes = a->kv_is_q8 ? row_elems / 32 * 34 : row_elems * 2;
    for (;;) {
        const int item = atomic_fetch_add(&j->next, 1);
        if (item >= a->n_calls * a->B) break;
        const int32_t c = item / a->B, b = item % a->B;
        const int32_t l = c % a->n_layers;
        const int32_t np = a->n_prefix[b], nv = a->prefix_valid[b];
        const int64_t pbase = ((int64_t)l * a->B + b) * a->max_prefix;
        for (int32_t t = 0; t < np; ++t) {
            const uint8_t *kr = a->prefix_k + (pbase + t) * row_bytes;
            const uint8_t *vr = a->prefix_v + (pbase + t) * row_bytes;
            if (a->kv_is_q8) {
                ekvo_dequantize_q8_0(kr, row_elems, kf + (int64_t)t * row_elems);
                ekvo_dequantize_q8_0(vr, row_elems, vf + (int64_t)t * row_elems);
            } else {
                ekvo_bf16_to_f32_n((const uint16_t *)kr, kf + (int64_t)t * row_elems, row_elems);
                ekvo_bf16_to_f32_n((const uint16_t *)vr, vf + (int64_t)t * row_elems, row_elems);
            }
        }
        const int64_t sbase = ((int64_t)l * a->B + b) * a->n_suffix * row_elems;
        ekvo_bf16_to_f32_n(a->suffix_k + sbase, kf + (int64_t)np * row_elems, (int64_t)a->n_suffix * row_elems);
        ekvo_bf16_to_f32_n(a->suffix_v + sbase, vf + (int64_t)np * row_elems, (int64_t)a->n_suffix * row_elems);
        const int32_t nk = np + a->n_suffix;
        for (int32_t t = 0; t < Tq; ++t) {
            for (int32_t h = 0; h < Hq; ++h) {
                const int32_t g = h / group;
                const uint16_t *qb = a->q + ((((int64_t)c * a->B + b) * Tq + t) * Hq + h) * D;
                ekvo_bf16_to_f32_n(qb, qf, D);
                float *o = (c == a->n_calls - 1 ? a->out + (int64_t)b * Tq * Hq * D : own) +
                           ((int64_t)t * Hq + h) * D;
                float mx = -INFINITY;
                for (int32_t k = 0; k < nk; ++k) {
                    if (k < np && k >= nv) { w[k] = -INFINITY; continue; }
                    const float *kr = kf + ((int64_t)k * Hkv + g) * D;
                    float dot = 0.0f;
                    for (int32_t d = 0; d < D; ++d) dot += kr[d] * qf[d];
                    w[k] = dot * a->scale;
                    if (w[k] > mx) mx = w[k];
                }
                double sum = 0.0;
                for (int32_t k = 0; k < nk; ++k) {
                    const float e = w[k] == -INFINITY ? 0.0f : expf(w[k] - mx);
                    w[k] = e;
                    sum += (double)e;
                }
                const float inv = (float)(1.0 / sum);
                for (int32_t d = 0; d < D; ++d) o[d] = 0.0f;
                for (int32_t k = 0; k < nk; ++k) {
                    if (w[k] == 0.0f) continue;
                    const float p = w[k] * inv;
                    const float *vr = vf + ((int64_t)k * Hkv + g) * D;
                    for (int32_t d = 0; d < D; ++d) o[d] += p * vr[d];
                }
            }
        }
    }
    free(kf);
    free(vf);
    free(w);
    free(qf);
    free(own);
    return NULL;
}

int ekvo_cache_attention_run(const ekvo_cache_args *a, int n_threads) {
    if (!a || a->B <= 0 || a->Hq % a->Hkv || a->n_layers <= 0 || a->n_calls <= 0) return -1;
    if (a->kv_is_q8 && (a->Hkv * a->D) % 32) return -1;
    cache_job job;
    job.a = a;
    atomic_init(&job.next, 0);
    if (n_threads <= 1) {
        cache_worker(&job);
        return 0;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, cache_worker, &job);
    for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
    free(th);
    return 0;
}
