/*
 * canvas_attn.h -- C ABI of the B200 canvas-attention library
 * (libcanvas_attn.so, built from diffuse-rs_b200/csrc/).
 *
 * Drop-in boundary for diffuse-rs's attention path. Each entry point names the
 * reference interface it replaces. Plain pointers and sizes only; no C++ or
 * torch types. All functions return CA_OK (0) or a negative ca_status and
 * never abort the process.
 *
 * Layouts are the reference's (src/model/attention.rs:101-106), row-major:
 *   Q   [tokens, n_head, head_dim]
 *   K,V [tokens, n_head_kv, head_dim]
 *   out [tokens, n_head * head_dim]
 * GQA maps query head h to kv head h / (n_head / n_head_kv)
 * (src/model/attention.rs:149).
 */
#ifndef CANVAS_ATTN_H
#define CANVAS_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    CA_OK = 0,
    CA_ERR_INVALID = -1,     /* bad shape, null pointer, inconsistent sizes */
    CA_ERR_UNSUPPORTED = -2, /* valid for the reference, not for this build (e.g. head_dim > 256) */
    CA_ERR_CUDA = -3,        /* a CUDA runtime/driver call failed */
    CA_ERR_TIMEOUT = -4,     /* a bounded device-side wait expired; outputs are undefined */
    CA_ERR_NOMEM = -5,       /* device or pinned allocation failed */
    CA_ERR_SCRATCH = -6      /* request larger than the fixed scratch of
                                ca_attention_block_dev_noalloc */
} ca_status;

/* Mirrors AttnShape (src/model/attention.rs:10-27). Option<usize> fields use
 * -1 for None. softcap is an extension with no reference counterpart:
 * 0 = off, else score <- softcap * tanh(score * scale / softcap). */
typedef struct {
    int64_t nq;
    int64_t nk;
    int64_t n_head;
    int64_t n_head_kv;
    int64_t head_dim;
    int64_t sliding_window; /* key visible iff |qpos - kpos| < window; -1 = None */
    int64_t causal_prefix;  /* query rows with qpos < prefix see kpos <= qpos; -1 = None */
    float scale;
    float softcap;
} ca_shape;

/* Mirrors Rows (src/model/attention.rs:65-77). pos has one entry per row.
 * seq / prefix may be NULL with length 0, which means the reference's empty
 * slice: every row in sequence 0 / the shape's scalar causal_prefix. */
typedef struct {
    const int64_t* pos;
    const int64_t* seq;
    size_t n_seq;
    const int64_t* prefix;
    size_t n_prefix;
} ca_rows;

/*
 * ca_attention_host_f32 -- replaces
 *   fn attention(out: &mut [f32], q: &[f32], k: &[f32], v: &[f32],
 *                s: AttnShape, qr: Rows, kr: Rows)
 *   (src/model/attention.rs:106), called at src/model/forward.rs:343.
 * Host fp32 buffers in and out, synchronous. Q/K/V are rounded to bf16 on
 * the GPU (fp32 accumulation, softmax weights in the precise two-term form;
 * head_dim is zero-padded to a multiple of 8 internally); masking is exactly
 * visible()
 * (src/model/attention.rs:35-57). A query row with no visible key gets NaN,
 * as the reference's acc * (1 / 0) does. Runs on the calling thread's
 * current CUDA device; calls are serialised per device by an internal lock,
 * and device buffers are kept (and grown) between calls.
 */
int ca_attention_host_f32(float* out, const float* q, const float* k, const float* v,
                          const ca_shape* s, const ca_rows* qr, const ca_rows* kr);

/* Device-resident arguments for ca_attention_dev (all pointers are device
 * pointers). Q/K/V are bf16. Sequences are either uniform
 * (cu_q == cu_k == NULL: batch sequences of sq queries and sk keys, stored
 * back to back) or varlen (cu_q/cu_k: int32 [batch + 1] row offsets, max_sq
 * bounds every sequence's query count). */
typedef struct {
    const void* q;  /* bf16 [total_q, n_head, head_dim]; token stride q_row_stride */
    const void* k;  /* bf16 [total_k, n_head_kv, head_dim]; stride kv_row_stride */
    const void* v;  /* bf16, same layout as k */
    void* out;      /* [total_q, n_head, head_dim]; stride out_row_stride */
    int32_t out_f32; /* 1: fp32 output, 0: bf16 output */
    int64_t q_row_stride;   /* elements between tokens; 0 = n_head * head_dim */
    int64_t kv_row_stride;  /* 0 = n_head_kv * head_dim */
    int64_t out_row_stride; /* 0 = n_head * head_dim */
    int32_t batch;
    int32_t sq;
    int32_t sk;
    const int32_t* cu_q;
    const int32_t* cu_k;
    int32_t max_sq;  /* varlen only: largest per-sequence query count */
    int64_t total_q; /* varlen only: rows in q/out (cu_q[batch]) */
    int64_t total_k; /* varlen only: rows in k/v (cu_k[batch]) */
    int32_t n_head;
    int32_t n_head_kv;
    int32_t head_dim;
    const int32_t* q_pos;    /* per global row; NULL = row index within its sequence */
    const int32_t* k_pos;
    const int32_t* q_seq;    /* per global row sequence id; NULL = all 0 */
    const int32_t* k_seq;
    const int32_t* q_prefix; /* per global query row; NULL = causal_prefix */
    int64_t sliding_window;  /* -1 = None */
    int64_t causal_prefix;   /* -1 = None */
    float scale;
    float softcap;           /* 0 = off (extension) */
    int32_t precise;         /* 1: softmax weights enter the PV product as two bf16
                                terms (hi + lo), ~2x the PV tensor work, error
                                ~256x smaller; 0: one bf16 term (fastest) */
    int32_t* status;         /* optional device int32: a bounded-wait expiry of this
                                call's kernels is stored here (CA_ERR_TIMEOUT) instead
                                of in the device-wide word that ca_device_status reads;
                                the caller zeroes and reads it. NULL = device-wide word */
    void* const* peer_out;   /* optional host array of n_peer_out device pointers into
                                other GPUs' buffers mapped into this process (e.g. by
                                ca_ipc_import): each receives exactly the rows written
                                to `out`, at the same element offsets and strides, as
                                the tiles finish (NVLink stores from the epilogue) */
    int32_t n_peer_out;      /* 0 .. CA_MAX_PEERS */
    const int32_t* seq_prefix; /* optional int32 [batch]: causal prefix of each sequence
                                  (Gemma's per-sequence canvas_start, forward.rs:153-160),
                                  negative = None; used when q_prefix is NULL and
                                  overrides causal_prefix */
    void* out_multicast;     /* optional NVLink multicast address (an NVLS multicast
                                  object, e.g. torch symmetric memory's multicast_ptr)
                                  bound to `out` on every rank of a head-sharded group,
                                  at the same offset as `out`: the epilogue writes each
                                  finished row once through it (multimem.st) and the
                                  switch delivers it to every rank's buffer, this one's
                                  included. Uniform batches only; peer_out must be
                                  empty. NULL = off */
} ca_dev_args;
#define CA_MAX_PEERS 7

/*
 * ca_attention_dev -- the device-resident form of attention()
 * (src/model/attention.rs:106-133): bf16 operands in HBM, fp32 accumulation,
 * asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream).
 * Batch is a grid dimension; varlen segments stand for the reference's
 * concatenated block-diagonal rows (src/model/forward.rs:113-160).
 * Allocates nothing. head_dim must be a multiple of 8 and <= 512.
 */
int ca_attention_dev(const ca_dev_args* a, void* stream);

/* Arguments of the fused attention block (pre-ops + cache + attention). */
typedef struct {
    const void* q;   /* bf16 [batch, n_active, n_head, head_dim], post-projection, pre-norm */
    const void* k;   /* bf16 [batch, n_active, n_head_kv, head_dim] */
    const void* v;   /* bf16 [batch, n_active, n_head_kv, head_dim] */
    int32_t batch;
    int32_t n_active;
    const int32_t* active_pos; /* int32 [batch, n_active] sequence positions */
    const float* q_norm_w;     /* fp32 [head_dim] or NULL (no q-norm) */
    const float* k_norm_w;     /* fp32 [head_dim] or NULL */
    int32_t v_norm;            /* 1: unweighted per-head RMSNorm of V (Gemma) */
    float rms_eps;
    const float* rope;         /* fp32 [rope_len, rope_dim/2, 2] (sin, cos) table */
    int32_t rope_len;
    int32_t rope_dim;          /* rotated dims per head (partial rotary), even */
    void* cache_k;             /* bf16 [batch, n_total, n_head_kv, head_dim] */
    void* cache_v;
    int32_t n_total;           /* positions per sequence; keys = all n_total positions */
    void* q_work;              /* bf16 [batch, n_active, n_head, head_dim] scratch (caller-owned);
                                  its contents are unspecified after the call (small head_dim-128
                                  calls rotate Q inside the attention kernel and leave it unwritten) */
    void* out;                 /* [batch, n_active, n_head, head_dim] */
    int32_t out_f32;
    int32_t n_head;
    int32_t n_head_kv;
    int32_t head_dim;
    int64_t sliding_window;
    int64_t causal_prefix;
    float scale;
    float softcap;
    int32_t precise;           /* as ca_dev_args.precise */
    int32_t* status;           /* as ca_dev_args.status */
    int64_t out_row_stride;    /* elements between tokens of out; 0 = n_head * head_dim
                                  (a head slice of a wider [tokens, heads, head_dim] buffer) */
    void* const* peer_out;     /* as ca_dev_args.peer_out (same offsets as out) */
    int32_t n_peer_out;
    /* Variable-length batches (the block-diagonal rows of forward_batch,
     * src/model/forward.rs:118-169): with cu_active set, sequence b's active
     * rows are rows cu_active[b] .. cu_active[b+1]-1 of q/k/v/active_pos/out
     * (n_active is ignored), and its cache is rows cu_total[b] ..
     * cu_total[b+1]-1 of cache_k/cache_v, position p at row cu_total[b] + p;
     * its keys are all of those positions. */
    const int32_t* cu_active;  /* int32 [batch + 1] or NULL (uniform) */
    const int32_t* cu_total;   /* int32 [batch + 1], required with cu_active */
    int32_t max_active;        /* varlen: largest per-sequence active count */
    int64_t total_active;      /* varlen: cu_active[batch] */
    int64_t total_cache;       /* varlen: cu_total[batch] */
    const int32_t* seq_prefix; /* as ca_dev_args.seq_prefix */
    void* out_multicast;       /* as ca_dev_args.out_multicast */
} ca_block_args;

/*
 * ca_attention_block_dev -- replaces the attention half of
 * Model::attention_block, src/model/forward.rs:296-343: per-head QK RMSNorm
 * (ops.rs:385-389, :107-114) -> optional V noscale norm (forward.rs:304-308)
 * -> NeoX RoPE at each row's position (ops.rs:420-452) -> StepCache::store of
 * post-RoPE K/V (cache.rs:62-70) -> attention over every cached position
 * (cache.rs:73-81 gather and forward.rs:312-317 concat become in-place reads:
 * after the store, cached ∪ active positions are exactly 0..n_total-1, so the
 * cache in position order is the key set). Active positions must be distinct
 * and every cached position must hold K/V stored by an earlier call.
 * Asynchronous on `stream`; allocates nothing.
 */
int ca_attention_block_dev(const ca_block_args* a, void* stream);

/*
 * ca_attention_block_dev_noalloc -- no counterpart in the reference. The
 * same fused block as ca_attention_block_dev for callers that cannot allocate
 * device memory themselves: hosts that link only this library and hold no
 * CUDA allocator, or programs whose framework owns every device allocation
 * and forbids extra cudaMalloc calls. The caller passes inputs, cache and
 * output as usual but leaves a->q_work NULL: the normed, rotated queries go to
 * a scratch array compiled into the library (static device memory of
 * CA_NOALLOC_SCRATCH_BYTES = 16 MiB on every GPU that loads the library,
 * held until process exit). A call whose queries pass through the scratch
 * (every call except head_dim-128 calls that rotate Q inside the attention
 * kernel) and needs more than that (batch * n_active * n_head * head_dim * 2
 * bytes > 16 MiB) returns CA_ERR_SCRATCH before anything is launched.
 * Nothing is allocated: no cudaMalloc, no cudaFree, no allocating library
 * call. Each call on a device looks up the scratch array's device address
 * (cudaGetSymbolAddress) with that device current until one lookup has
 * succeeded; make the first call before any stream capture. All calls share
 * the one array and it keeps the last call's values. Calls that run one after
 * another are unaffected, because each call writes all of the scratch it
 * reads before reading it. Calls whose GPU work overlaps (other streams,
 * other threads) race on the array and can return wrong outputs with no
 * error status: do not overlap them.
 */
int ca_attention_block_dev_noalloc(const ca_block_args* a, void* stream);
#define CA_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/*
 * Peer buffers for head-sharded layers (no counterpart in the reference,
 * whose CPU path has one address space). One process per GPU: a rank
 * exports its receive buffer, the others import it and pass the mapping in
 * peer_out, so the attention epilogue stores its head slice straight into
 * every rank's [tokens, n_head, head_dim] buffer over NVLink.
 * ca_ipc_export: handle (CA_IPC_HANDLE_BYTES bytes, opaque) and byte offset
 * of dev_ptr within its allocation. ca_ipc_import: maps that allocation of
 * another process on the current device and returns base + offset.
 * ca_ipc_close: unmaps a pointer ca_ipc_import returned. A receive buffer may
 * be rewritten by peers only after its owner has consumed it; the library
 * does not order one call's peer stores against another's reads (use a
 * barrier, e.g. a stream-ordered collective, between them).
 */
#define CA_IPC_HANDLE_BYTES 64
int ca_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset);
int ca_ipc_import(const void* handle, uint64_t offset, void** dev_ptr);
int ca_ipc_close(void* dev_ptr);

/* Arguments of ca_candidate_stats (device pointers unless noted). */
typedef struct {
    float* logits;            /* fp32 [rows, row_stride]: the step's logits */
    int64_t n_vocab;
    int64_t row_stride;       /* elements between rows; 0 = n_vocab */
    const int32_t* rows;      /* int32 [n_cand]: logit row of each candidate
                                 (its position minus the model's logit shift) */
    int32_t n_cand;
    int32_t mask_id;          /* mask token id, or < 0 for none */
    const int32_t* suppress;  /* int32 [n_suppress] token ids never committed, or NULL */
    int32_t n_suppress;
    int32_t want_entropy;     /* 0: entropy written as 0 (as the reference when unused) */
    int32_t want_prob;        /* 0: prob written as 0 */
    int32_t* token;           /* int32 [n_cand] out: greedy pick */
    float* entropy;           /* fp32 [n_cand] out (may be NULL when !want_entropy) */
    float* margin;            /* fp32 [n_cand] out: top1 - top2 (may be NULL) */
    float* prob;              /* fp32 [n_cand] out (may be NULL when !want_prob) */
} ca_cand_args;

/*
 * ca_candidate_stats -- replaces the per-candidate loop of
 * Denoiser::collect_candidates (src/model/sampler.rs:720-749) for the greedy
 * pick (pick_token, temperature 0, :754-764), after suppress_mask_token and
 * suppress_tokens (:90-113), on logits resident in HBM: one launch per
 * step, asynchronous on `stream`. For candidate i, over logit row rows[i]:
 * token = first index of the maximum (0 if every entry is -inf), margin =
 * top1 - top2 (top2_logits :75-87), entropy = compute_entropy (:7-20, the
 * p > 1e-10 rule included), prob = exp(top1 - log_sum_exp) (:22-25). As in
 * the reference, the mask token and the suppressed ids of the candidate rows
 * are set to -inf in `logits` itself. Sums are formed in a different order
 * than the reference's sequential f32 folds (results agree to ~1e-6
 * relative); token and margin are exact. Allocates nothing.
 */
int ca_candidate_stats(const ca_cand_args* a, void* stream);

/* tokens_to_unmask (src/model/sampler.rs:115-132), host, in the reference's
 * f32 arithmetic: how many of `masked` remaining tokens to commit at `step`
 * of `total_steps`. Returns the count, or CA_ERR_INVALID. */
#define CA_SCHEDULE_COSINE 0
#define CA_SCHEDULE_LINEAR 1
int64_t ca_tokens_to_unmask(int64_t step, int64_t total_steps, int64_t masked,
                            int32_t schedule);

/*
 * Projections around attention (src/model/forward.rs:275-294 QKV + bias,
 * :345-350 wo + residual) over the reference's quantised weights. The
 * weights are dequantised once (ca_dequantize, bit-identical in f32 to
 * dequantize_q4k_row / _q6k_row / _q4_0_row / _q8_0_row / f16_to_f32,
 * src/kernels.rs:46-217) and kept in HBM as bf16; each projection is then
 * one bf16 GEMM with fp32 accumulation (ca_linear). The reference instead
 * quantises the activations of Q4_K / Q6_K products to 8 bits per 256-value
 * block (src/model/matmul.rs:90-151); bf16 activations are closer to the
 * exact product than that.
 */
#define CA_QTYPE_F16 1
#define CA_QTYPE_Q4_0 2
#define CA_QTYPE_Q8_0 8
#define CA_QTYPE_Q4_K 12
#define CA_QTYPE_Q6_K 14

/*
 * ca_dequantize -- rows of GGUF blocks to bf16 (dst_f32 = 0) or fp32 on the
 * device, asynchronous on `stream`. src: `rows` rows of `cols` weights of
 * type qtype (device memory, rows packed back to back). Output row i (of
 * n_out) is source row row_ids[i] (device int32, e.g. token ids: the
 * embedding gather of embed_tokens, src/model/forward.rs:175-246), or row i
 * when row_ids is NULL, times `scale` (1 = none; Gemma's embed_scale).
 * dst: 16-byte aligned, row stride dst_stride elements (0 = cols, a
 * multiple of 8); Q4_K sources 8-byte aligned. cols must be a multiple of 256 (Q4_K, Q6_K), 32 (Q4_0,
 * Q8_0) or 8 (F16). A row id out of range skips that row and sets *status
 * (device int32, may be NULL) to 1.
 */
int ca_dequantize(int32_t qtype, const void* src, int64_t rows, int64_t cols,
                  const int32_t* row_ids, int64_t n_out, void* dst, int32_t dst_f32,
                  int64_t dst_stride, float scale, int32_t* status, void* stream);

/* Arguments of ca_linear (device pointers). */
typedef struct {
    const void* act;       /* bf16 [n, cols], row stride act_stride (0 = cols) */
    int64_t act_stride;
    const void* w;         /* bf16 [rows, cols] (e.g. from ca_dequantize) */
    const float* bias;     /* fp32 [rows] or NULL (add_bias, forward.rs:292-294) */
    const void* residual;  /* [n, rows] of out's type or NULL (residual_add,
                              forward.rs:350); may be the same buffer as out */
    void* out;             /* [n, rows]: bf16, or fp32 when out_f32 */
    int32_t out_f32;
    int64_t n;
    int64_t rows;
    int64_t cols;
} ca_linear_args;

/*
 * ca_linear -- replaces MatWeight::forward (src/model/matmul.rs:90-110,
 * out[t*rows + r] = act row t . weight row r) with the bias and residual
 * adds around it: out = act . W^T (+ bias) (+ residual), bf16 operands,
 * fp32 accumulation, one cuBLASLt GEMM with the bias and residual in its
 * epilogue (bf16 output with a bias: the product goes to an fp32 buffer and
 * one kernel adds bias and residual, so the output is rounded once),
 * asynchronous on `stream`. The first call on a device creates a cuBLASLt
 * handle and a 32 MiB workspace that the library keeps (and the fp32
 * buffer, grown on demand).
 */
int ca_linear(const ca_linear_args* a, void* stream);

/*
 * ca_build_rope_table -- replaces build_rope_cache_ff (src/model/ops.rs:398-416),
 * host side, run once at load like the reference. out: host fp32
 * [max_seq_len, rope_dim/2, 2] as (sin, cos); freq_factors may be NULL.
 */
int ca_build_rope_table(float* out, int64_t max_seq_len, int64_t rope_dim, float theta,
                        const float* freq_factors);

/* Reads and clears the device-wide error word of the current device after
 * synchronising `stream`: CA_OK, or CA_ERR_TIMEOUT if the bounded wait of a
 * kernel launched without a status word of its own (status == NULL) expired
 * since the last call. The word is shared by every stream and thread of the
 * process on that device; callers that need their own give each call a
 * status word. */
int ca_device_status(void* stream);

/*
 * ca_selftest_wait_timeout -- failure-detection self-test, no counterpart in
 * the reference (whose CPU path has no device waits). Launches one CTA on
 * `stream` that waits on an mbarrier nothing arrives on, through the same
 * bounded wait every pipeline wait of the attention kernel uses, giving up
 * after `limit_ns` nanoseconds (1 ns .. 1 s). The kernel returns normally;
 * a following ca_device_status(stream) returns CA_ERR_TIMEOUT once and then
 * CA_OK, and the CUDA context stays usable. Lets a host verify on its own
 * GPU that an expired wait is reported instead of hanging.
 */
int ca_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* The same self-test reporting to a caller-owned device int32 `status`
 * (the per-call word of ca_dev_args.status) instead of the device-wide word:
 * afterwards *status holds CA_ERR_TIMEOUT and ca_device_status is unaffected. */
int ca_selftest_wait_timeout_status(int64_t limit_ns, int32_t* status, void* stream);

/* Host-side fp32 -> bf16 rounding that ca_attention_host_f32 applies to
 * large calls before their host-to-device copies (no counterpart in the
 * reference, whose operands stay fp32): round to nearest even, every NaN to
 * 0x7FFF and overflow to infinity, the GPU's cvt.rn.bf16.f32, so the kernels
 * see the same operands as when they round on the device. Runs on a pool of
 * host threads; dst receives n bf16 bit patterns. Returns CA_ERR_INVALID for
 * null pointers with n > 0. */
int ca_round_bf16_host(const float* src, uint16_t* dst, uint64_t n);

/* Human-readable text of a ca_status. */
const char* ca_status_string(int status);

/* Library version, "canvas_attn <major>.<minor>.<patch> sm_100a". */
const char* ca_version(void);

#ifdef __cplusplus
}
#endif
#endif /* CANVAS_ATTN_H */
