/*
 * oracle_attn.h -- CPU restatement of diffuse-rs canvas attention.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * path and the timed CPU baseline in bench.py. Nothing in the product
 * (diffuse-rs_b200/) links, loads or calls it.
 *
 * Parity pins: the reference's own known-answer and relational tests
 * (src/model/tests.rs:70-237, :634-640, :55-68) restated as pytest cases over
 * the committed fixtures in tests/golden/. The Rust reference itself cannot be
 * built in this container (no cargo/rustc), so no reference binary output is
 * available; see the repository design notes.
 *
 * Conventions follow the reference exactly:
 *   q   [nq, n_head, hd]      row-major fp32
 *   k,v [nk, n_head_kv, hd]   row-major fp32
 *   out [nq, n_head * hd]     row-major fp32
 */
#ifndef ORACLE_ATTN_H
#define ORACLE_ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* AttnShape (src/model/attention.rs:10-27). Option<usize> is -1 for None.
 * softcap is a build-side extension with no reference semantics: 0 = off,
 * otherwise score <- softcap * tanh(score / softcap) after scaling. */
typedef struct {
    int64_t nq, nk, n_head, n_head_kv, head_dim;
    int64_t sliding_window; /* -1 = None */
    int64_t causal_prefix;  /* -1 = None */
    float scale;
    float softcap;          /* 0 = None (extension) */
} or_shape;

/* Rows (src/model/attention.rs:65-77). Empty slices are NULL / 0 length:
 * seq empty -> every row has id 0; prefix empty -> shape.causal_prefix. */
typedef struct {
    const int64_t* pos;
    const int64_t* seq;
    int64_t n_seq;
    const int64_t* prefix;
    int64_t n_prefix;
} or_rows;

enum { OR_ROW_SCALAR = 0, OR_ROW_AVX2 = 1 };

/* attention() (src/model/attention.rs:106-133): every (head, query) task,
 * threaded over `threads` OpenMP threads (<=0: all). kind selects the row
 * kernel: scalar (:142-186) or AVX2 (:267-345). Returns 0, or -1 when AVX2
 * was requested on a CPU without it. */
int or_attention(float* out, const float* q, const float* k, const float* v,
                 const or_shape* s, const or_rows* qr, const or_rows* kr,
                 int kind, int threads);

/* The same over a subset of tasks: task t = head * nq + query, as in
 * attention.rs:116-117. Used for bounded CPU-baseline samples and spot checks
 * of large configs. Only the rows named in `tasks` are written. */
int or_attention_tasks(float* out, const float* q, const float* k, const float* v,
                       const or_shape* s, const or_rows* qr, const or_rows* kr,
                       const int64_t* tasks, int64_t n_tasks, int kind, int threads);

/* visible() (src/model/attention.rs:35-57); window/prefix -1 = None. */
int or_visible(int64_t qpos, int64_t kpos, int64_t qseq, int64_t kseq,
               int64_t window, int64_t prefix);

/* rms_norm_inplace (src/model/ops.rs:107-114). */
void or_rms_norm_inplace(float* x, const float* w, int64_t n, float eps);
/* rms_norm_noscale (src/model/ops.rs:117-124). */
void or_rms_norm_noscale(float* x, int64_t n, float eps);
/* norm_heads (src/model/ops.rs:385-389): x has len elements, chunks of hd. */
void or_norm_heads(float* x, int64_t len, const float* w, int64_t hd, float eps);
/* build_rope_cache_ff (src/model/ops.rs:398-416). out holds
 * max_seq_len * (rope_dim/2) pairs (sin, cos); ff may be NULL. */
void or_build_rope_cache(float* out, int64_t max_seq_len, int64_t rope_dim,
                         float theta, const float* ff);
/* rotate_rows (src/model/ops.rs:432-452). */
void or_rotate_rows(float* x, const float* rope, const int64_t* positions, int64_t n,
                    int64_t heads, int64_t hd, int64_t rot);
/* StepCache::store / gather (src/model/cache.rs:62-81), one layer. */
void or_cache_store(float* cache_k, float* cache_v, int64_t stride,
                    const int64_t* positions, int64_t n, const float* k, const float* v);
void or_cache_gather(const float* cache_k, const float* cache_v, int64_t stride,
                     const int64_t* positions, int64_t n, float* out_k, float* out_v);

/* 1 when the running CPU has AVX2 and FMA. */
int or_have_avx2(void);
/* Number of OpenMP threads a call with threads<=0 uses. */
int or_max_threads(void);

/* Denoising-step statistics (oracle_sampler.c, src/model/sampler.rs). */
float or_compute_entropy(const float* row, int64_t n);
float or_log_sum_exp(const float* row, int64_t n);
void or_top2_logits(const float* row, int64_t n, float* top1, float* top2);
int32_t or_pick_greedy(const float* row, int64_t n);
void or_candidate_stats(float* logits, int64_t rows_total, int64_t n_vocab,
                        const int32_t* rows, int64_t n_cand, int32_t mask_id,
                        const int32_t* suppress, int64_t n_suppress, int want_entropy,
                        int want_prob, int32_t* token, float* entropy, float* margin,
                        float* prob);
int64_t or_tokens_to_unmask(int64_t step, int64_t total_steps, int64_t masked,
                            int32_t schedule);

/* Quantised weight formats and projections (oracle_quant.c, src/kernels.rs,
 * src/model/matmul.rs). qtype: GGML ids 1 F16, 2 Q4_0, 8 Q8_0, 12 Q4_K, 14 Q6_K. */
float or_f16_to_f32(uint16_t h);
int or_dequant_row(int32_t qtype, const uint8_t* row, int64_t cols, float* out);
int64_t or_row_bytes(int32_t qtype, int64_t cols);
void or_quantize_row_q8k(const float* x, int64_t n_blocks, float* d, int8_t* qs,
                         int16_t* bsums);
float or_vec_dot_q4k_q8k(const uint8_t* xb, const float* yd, const int8_t* yq,
                         const int16_t* ybs, int64_t n_blocks);
float or_vec_dot_q6k_q8k(const uint8_t* xb, const float* yd, const int8_t* yq,
                         int64_t n_blocks);
int or_linear_q8k(int32_t qtype, const uint8_t* w, int64_t rows, int64_t cols,
                  const float* act, int64_t n, float* out);

#ifdef __cplusplus
}
#endif
#endif
