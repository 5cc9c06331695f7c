/*
 * oracle_sampler.c -- CPU restatement of the denoising step's per-candidate
 * statistics (src/model/sampler.rs). TEST INFRASTRUCTURE ONLY: the GPU
 * kernel's checker; the product never links it.
 *
 * Sequential f32 folds in the reference's order, built with
 * -ffp-contract=off; expf/logf/cosf/roundf are glibc's, what Rust's f32::exp,
 * ln, cos and round call on Linux.
 */
#include "oracle_attn.h"

#include <math.h>

/* compute_entropy: src/model/sampler.rs:7-20. */
float or_compute_entropy(const float* row, int64_t n) {
    float max = -INFINITY;
    for (int64_t i = 0; i < n; ++i) max = fmaxf(max, row[i]); /* f32::max fold */
    float sum_exp = 0.0f;
    for (int64_t i = 0; i < n; ++i) sum_exp += expf(row[i] - max);
    const float log_sum = logf(sum_exp);
    float acc = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        const float lp = (row[i] - max) - log_sum;
        const float p = expf(lp);
        if (p > 1e-10f) acc = acc - p * lp;
    }
    return acc;
}

/* log_sum_exp: src/model/sampler.rs:22-25. */
float or_log_sum_exp(const float* row, int64_t n) {
    float max = -INFINITY;
    for (int64_t i = 0; i < n; ++i) max = fmaxf(max, row[i]);
    float s = 0.0f;
    for (int64_t i = 0; i < n; ++i) s += expf(row[i] - max);
    return max + logf(s);
}

/* top2_logits: src/model/sampler.rs:75-87. */
void or_top2_logits(const float* row, int64_t n, float* top1, float* top2) {
    float t1 = -INFINITY, t2 = -INFINITY;
    for (int64_t i = 0; i < n; ++i) {
        const float l = row[i];
        if (l > t1) {
            t2 = t1;
            t1 = l;
        } else if (l > t2) {
            t2 = l;
        }
    }
    *top1 = t1;
    *top2 = t2;
}

/* pick_token at temperature 0: src/model/sampler.rs:754-764. */
int32_t or_pick_greedy(const float* row, int64_t n) {
    int64_t best = 0;
    float best_l = -INFINITY;
    for (int64_t j = 0; j < n; ++j)
        if (row[j] > best_l) {
            best = j;
            best_l = row[j];
        }
    return (int32_t)best;
}

/* collect_candidates (src/model/sampler.rs:720-749) for the greedy pick,
 * after suppress_mask_token / suppress_tokens (:90-113), which set the
 * suppressed logits of every row to -inf in place (rows_total rows). */
void or_candidate_stats(float* logits, int64_t rows_total, int64_t n_vocab,
                        const int32_t* rows, int64_t n_cand, int32_t mask_id,
                        const int32_t* suppress, int64_t n_suppress, int want_entropy,
                        int want_prob, int32_t* token, float* entropy, float* margin,
                        float* prob) {
    for (int64_t r = 0; r < rows_total; ++r) {
        float* row = logits + r * n_vocab;
        if (mask_id >= 0 && mask_id < n_vocab) row[mask_id] = -INFINITY;
        for (int64_t i = 0; i < n_suppress; ++i)
            if (suppress[i] >= 0 && suppress[i] < n_vocab) row[suppress[i]] = -INFINITY;
    }
    for (int64_t c = 0; c < n_cand; ++c) {
        const float* row = logits + (int64_t)rows[c] * n_vocab;
        float t1, t2;
        or_top2_logits(row, n_vocab, &t1, &t2);
        token[c] = or_pick_greedy(row, n_vocab);
        entropy[c] = want_entropy ? or_compute_entropy(row, n_vocab) : 0.0f;
        margin[c] = t1 - t2;
        prob[c] = want_prob ? expf(t1 - or_log_sum_exp(row, n_vocab)) : 0.0f;
    }
}

/* tokens_to_unmask: src/model/sampler.rs:115-132 (schedule 0 cosine,
 * 1 linear). */
int64_t or_tokens_to_unmask(int64_t step, int64_t total_steps, int64_t masked,
                            int32_t schedule) {
    int64_t steps_left = total_steps > step ? total_steps - step : 0;
    if (steps_left < 1) steps_left = 1;
    const float t0 = (float)step / (float)total_steps;
    const float t1 = (float)(step + 1) / (float)total_steps;
    float frac;
    if (schedule == 0) {
        float c0 = cosf(t0 * (float)M_PI_2);
        if (c0 < 1e-6f) c0 = 1e-6f; /* .max(1e-6) */
        const float c1 = cosf(t1 * (float)M_PI_2);
        frac = (c0 - c1) / c0;
    } else {
        frac = 1.0f / (float)steps_left;
    }
    const float nf = roundf(frac * (float)masked);
    int64_t n = (nf != nf || nf <= 0.0f) ? 0 : (int64_t)nf; /* `as usize` */
    if (n < (masked > 0 ? 1 : 0)) n = masked > 0 ? 1 : 0;
    return n < masked ? n : masked;
}
