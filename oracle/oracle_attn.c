/*
 * oracle_attn.c -- CPU restatement of diffuse-rs canvas attention and the
 * element-wise ops around it. TEST INFRASTRUCTURE ONLY (parity checker and
 * timed CPU baseline); the product never links it.
 *
 * Built with -ffp-contract=off so that scalar expressions round exactly as the
 * Rust reference does (rustc never contracts a*b+c into an FMA); the AVX2 row
 * uses explicit FMA intrinsics where the reference does.
 * exp/tanh/pow/sin/cos are glibc's expf/tanhf/powf/sinf/cosf, which is what
 * Rust's f32::exp / tanh / powf / sin_cos call on Linux.
 */
#include "oracle_attn.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ACC_STACK 256 /* attention.rs:138 */

/* visible(): src/model/attention.rs:35-57. */
int or_visible(int64_t qpos, int64_t kpos, int64_t qseq, int64_t kseq,
               int64_t window, int64_t prefix) {
    if (qseq != kseq) return 0;
    if (window >= 0) {
        int64_t d = qpos > kpos ? qpos - kpos : kpos - qpos; /* usize::abs_diff */
        if (d >= window) return 0;
    }
    if (prefix >= 0 && qpos < prefix) return kpos <= qpos;
    return 1;
}

/* Rows::seq_at (attention.rs:73-76): empty seq means id 0. */
static inline int64_t seq_at(const or_rows* r, int64_t i) {
    return (r->seq && i < r->n_seq) ? r->seq[i] : 0;
}

/* Per-row causal prefix (attention.rs:151): per-row array if non-empty,
 * else the shape's scalar. */
static inline int64_t prefix_at(const or_rows* qr, const or_shape* s, int64_t i) {
    return (qr->prefix && qr->n_prefix > 0) ? qr->prefix[i] : s->causal_prefix;
}

/* Build-side extension: attention-logit soft-cap, applied after scaling. */
static inline float apply_softcap(float score, float cap) {
    return cap > 0.0f ? cap * tanhf(score / cap) : score;
}

/* attention_row_scalar: src/model/attention.rs:142-186. */
static void row_scalar(float* out, const float* q, const float* k, const float* v,
                       const or_shape* s, const or_rows* qr, const or_rows* kr,
                       int64_t head, int64_t i) {
    const int64_t hd = s->head_dim;
    const float scale = s->scale;
    const int64_t qo = i * s->n_head * hd + head * hd;
    const int64_t kv_stride = s->n_head_kv * hd;
    const int64_t kv_off = (head / (s->n_head / s->n_head_kv)) * hd; /* :149 */
    const int64_t qpos = qr->pos[i], qseq = seq_at(qr, i);
    const int64_t prefix = prefix_at(qr, s, i);

    float acc_stack[ACC_STACK];
    float* acc = hd <= ACC_STACK ? acc_stack : (float*)malloc(sizeof(float) * hd);
    for (int64_t d = 0; d < hd; ++d) acc[d] = 0.0f;
    float max = -INFINITY, sum = 0.0f;
    for (int64_t j = 0; j < s->nk; ++j) {
        if (!or_visible(qpos, kr->pos[j], qseq, seq_at(kr, j), s->sliding_window, prefix))
            continue;
        const int64_t ko = j * kv_stride + kv_off;
        float dot = -0.0f; /* Rust's f32 Sum folds from -0.0 */
        for (int64_t d = 0; d < hd; ++d) dot += q[qo + d] * k[ko + d];
        float score = apply_softcap(dot * scale, s->softcap);

        float new_max = fmaxf(max, score);
        float correction = expf(max - new_max);
        float w = expf(score - new_max);
        sum = sum * correction + w;
        for (int64_t d = 0; d < hd; ++d) acc[d] = acc[d] * correction + w * v[ko + d];
        max = new_max;
    }
    float inv = 1.0f / sum;
    for (int64_t d = 0; d < hd; ++d) out[qo + d] = acc[d] * inv;
    if (acc != acc_stack) free(acc);
}

/* hsum_avx2: src/model/ops.rs:353-362, same lane order. */
__attribute__((target("avx2,fma"))) static inline float hsum_avx2(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 s = _mm_add_ps(lo, hi);
    __m128 s2 = _mm_add_ps(s, _mm_shuffle_ps(s, s, 0xB1));  /* 0b10_11_00_01 */
    __m128 s3 = _mm_add_ps(s2, _mm_shuffle_ps(s2, s2, 0x4E)); /* 0b01_00_11_10 */
    return _mm_cvtss_f32(s3);
}

/* attention_row_avx2: src/model/attention.rs:267-345 (x86 production path). */
__attribute__((target("avx2,fma"))) static void row_avx2(
    float* out, const float* q, const float* k, const float* v, const or_shape* s,
    const or_rows* qr, const or_rows* kr, int64_t head, int64_t i) {
    const int64_t hd = s->head_dim;
    const float scale = s->scale;
    const int64_t qo = i * s->n_head * hd + head * hd;
    const int64_t kv_stride = s->n_head_kv * hd;
    const int64_t kv_off = (head / (s->n_head / s->n_head_kv)) * hd;
    const int64_t qpos = qr->pos[i], qseq = seq_at(qr, i);
    const int64_t prefix = prefix_at(qr, s, i);

    float acc_stack[ACC_STACK];
    float* acc = hd <= ACC_STACK ? acc_stack : (float*)malloc(sizeof(float) * hd);
    for (int64_t d = 0; d < hd; ++d) acc[d] = 0.0f;
    float max = -INFINITY, sum = 0.0f;
    for (int64_t j = 0; j < s->nk; ++j) {
        if (!or_visible(qpos, kr->pos[j], qseq, seq_at(kr, j), s->sliding_window, prefix))
            continue;
        const int64_t ko = j * kv_stride + kv_off;
        __m256 dot_vec = _mm256_setzero_ps();
        int64_t d = 0;
        for (; d + 8 <= hd; d += 8) {
            __m256 qv = _mm256_loadu_ps(q + qo + d);
            __m256 kv = _mm256_loadu_ps(k + ko + d);
            dot_vec = _mm256_fmadd_ps(qv, kv, dot_vec);
        }
        float dot = hsum_avx2(dot_vec);
        for (; d < hd; ++d) dot += q[qo + d] * k[ko + d];
        float score = apply_softcap(dot * scale, s->softcap);

        float new_max = fmaxf(max, score);
        float correction = expf(max - new_max);
        float w = expf(score - new_max);
        sum = sum * correction + w;

        __m256 cv = _mm256_set1_ps(correction);
        __m256 wv = _mm256_set1_ps(w);
        d = 0;
        for (; d + 8 <= hd; d += 8) {
            __m256 av = _mm256_loadu_ps(acc + d);
            __m256 vv = _mm256_loadu_ps(v + ko + d);
            _mm256_storeu_ps(acc + d, _mm256_fmadd_ps(wv, vv, _mm256_mul_ps(av, cv)));
        }
        for (; d < hd; ++d) acc[d] = acc[d] * correction + w * v[ko + d];
        max = new_max;
    }
    __m256 inv = _mm256_set1_ps(1.0f / sum);
    int64_t d = 0;
    for (; d + 8 <= hd; d += 8)
        _mm256_storeu_ps(out + qo + d, _mm256_mul_ps(_mm256_loadu_ps(acc + d), inv));
    for (; d < hd; ++d) out[qo + d] = acc[d] / sum;
    if (acc != acc_stack) free(acc);
}

int or_have_avx2(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
}

int or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int run_tasks(float* out, const float* q, const float* k, const float* v,
                     const or_shape* s, const or_rows* qr, const or_rows* kr,
                     const int64_t* tasks, int64_t n_tasks, int kind, int threads) {
    if (kind == OR_ROW_AVX2 && !or_have_avx2()) return -1;
    if (s->n_head_kv <= 0 || s->n_head % s->n_head_kv != 0) return -2;
    int nt = threads > 0 ? threads : or_max_threads();
    (void)nt;
    /* rayon's into_par_iter over (head, query) tasks (attention.rs:116). */
#pragma omp parallel for schedule(dynamic, 16) num_threads(nt)
    for (int64_t t = 0; t < n_tasks; ++t) {
        int64_t task = tasks ? tasks[t] : t;
        int64_t head = task / s->nq, i = task % s->nq;
        if (kind == OR_ROW_AVX2)
            row_avx2(out, q, k, v, s, qr, kr, head, i);
        else
            row_scalar(out, q, k, v, s, qr, kr, head, i);
    }
    return 0;
}

int or_attention(float* out, const float* q, const float* k, const float* v,
                 const or_shape* s, const or_rows* qr, const or_rows* kr,
                 int kind, int threads) {
    return run_tasks(out, q, k, v, s, qr, kr, NULL, s->n_head * s->nq, kind, threads);
}

int or_attention_tasks(float* out, const float* q, const float* k, const float* v,
                       const or_shape* s, const or_rows* qr, const or_rows* kr,
                       const int64_t* tasks, int64_t n_tasks, int kind, int threads) {
    return run_tasks(out, q, k, v, s, qr, kr, tasks, n_tasks, kind, threads);
}

/* rms_norm_inplace: src/model/ops.rs:107-114 (sum of squares in f64 of the
 * f32 products, scale = 1 / (sqrt(ss/n + eps) as f32)). */
void or_rms_norm_inplace(float* x, const float* w, int64_t n, float eps) {
    double ss = 0.0;
    for (int64_t i = 0; i < n; ++i) ss += (double)(x[i] * x[i]);
    float scale = 1.0f / (float)sqrt(ss / (double)n + (double)eps);
    for (int64_t i = 0; i < n; ++i) x[i] = x[i] * scale * w[i];
}

/* rms_norm_noscale: src/model/ops.rs:117-124. */
void or_rms_norm_noscale(float* x, int64_t n, float eps) {
    double ss = 0.0;
    for (int64_t i = 0; i < n; ++i) ss += (double)(x[i] * x[i]);
    float scale = 1.0f / (float)sqrt(ss / (double)n + (double)eps);
    for (int64_t i = 0; i < n; ++i) x[i] *= scale;
}

/* norm_heads: src/model/ops.rs:385-389. */
void or_norm_heads(float* x, int64_t len, const float* w, int64_t hd, float eps) {
    for (int64_t off = 0; off < len; off += hd) {
        int64_t n = len - off < hd ? len - off : hd;
        or_rms_norm_inplace(x + off, w, n, eps);
    }
}

/* build_rope_cache_ff: src/model/ops.rs:398-416. */
void or_build_rope_cache(float* out, int64_t max_seq_len, int64_t rope_dim,
                         float theta, const float* ff) {
    int64_t half = rope_dim / 2;
    for (int64_t t = 0; t < max_seq_len; ++t) {
        for (int64_t i = 0; i < half; ++i) {
            float freq = 1.0f / powf(theta, 2.0f * (float)i / (float)rope_dim);
            if (ff) freq /= ff[i];
            float a = (float)t * freq;
            out[2 * (t * half + i) + 0] = sinf(a);
            out[2 * (t * half + i) + 1] = cosf(a);
        }
    }
}

/* rotate_rows: src/model/ops.rs:432-452 (NeoX half split). */
void or_rotate_rows(float* x, const float* rope, const int64_t* positions, int64_t n,
                    int64_t heads, int64_t hd, int64_t rot) {
    int64_t half = rot / 2;
    for (int64_t t = 0; t < n; ++t) {
        int64_t pos = positions[t];
        for (int64_t h = 0; h < heads; ++h) {
            int64_t off = t * heads * hd + h * hd;
            for (int64_t i = 0; i < half; ++i) {
                float sn = rope[2 * (pos * half + i) + 0];
                float cs = rope[2 * (pos * half + i) + 1];
                float a = x[off + i], b = x[off + half + i];
                x[off + i] = a * cs - b * sn;
                x[off + half + i] = a * sn + b * cs;
            }
        }
    }
}

/* StepCache::store: src/model/cache.rs:62-70. */
void or_cache_store(float* cache_k, float* cache_v, int64_t stride,
                    const int64_t* positions, int64_t n, const float* k, const float* v) {
    for (int64_t r = 0; r < n; ++r) {
        memcpy(cache_k + positions[r] * stride, k + r * stride, sizeof(float) * stride);
        memcpy(cache_v + positions[r] * stride, v + r * stride, sizeof(float) * stride);
    }
}

/* StepCache::gather: src/model/cache.rs:73-81. */
void or_cache_gather(const float* cache_k, const float* cache_v, int64_t stride,
                     const int64_t* positions, int64_t n, float* out_k, float* out_v) {
    for (int64_t r = 0; r < n; ++r) {
        memcpy(out_k + r * stride, cache_k + positions[r] * stride, sizeof(float) * stride);
        memcpy(out_v + r * stride, cache_v + positions[r] * stride, sizeof(float) * stride);
    }
}
