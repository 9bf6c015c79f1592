/*
 * pm_sample.h -- C ABI of the B200 token-selection path (libpm_sample.so).
 *
 * Replaces the per-step token selection of PagedMoE's decode loop: the
 * logits processors, the log-softmax, the sampler and the draft acceptance
 * of a verify pass.  All pointers are device pointers unless stated; every
 * function takes a cudaStream_t (as void*) and returns a status code, never
 * aborts and allocates nothing.  The only process-wide state is per device:
 * each kernel's shared-memory attribute and occupancy, set up on the first
 * launch on that device, and the scratch array of pm_sample_rows_static.
 * Calls with separate workspaces may come from several host threads on
 * different streams.
 *
 * Reference interfaces replaced (paths within noahclark556/paged-moe):
 *   pm_sample_rows      sampler(logprobs) -> tokens, built by mlx-lm's
 *                       make_sampler (call sites pagedmoe/verify_decode.py:839,
 *                       :903, pagedmoe/lookup_decode.py:359, run.py:53) plus
 *                       the processor loop before it (verify_decode.py:828-835,
 *                       :889-899) fused into one pass over the logits.
 *   pm_apply_processors proc(tokens, logits) -> logits, built by mlx-lm's
 *                       make_logits_processors (verify_decode.py:830-831,
 *                       :895-896; lookup_decode.py:344-356), and the
 *                       where(mask, x, -inf) processors of
 *                       pagedmoe/think_budget.py:107-109 and rescue.py:240-245.
 *   pm_logprobs         logits - logsumexp(logits) (verify_decode.py:835, :899;
 *                       lookup_decode.py:358).
 *   pm_verify           the accept loop of a verify pass
 *                       (lookup_decode.py:363-369, verify_decode.py:903-921),
 *                       plus residual rejection sampling (no reference code).
 *   pm_shard_summarize / pm_shard_merge
 *                       vocab-sharded sampling (no reference code: the
 *                       reference runs on one device).
 */
#ifndef PM_SAMPLE_H
#define PM_SAMPLE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PM_API __attribute__((visibility("default")))
#else
#define PM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define PM_OK 0
#define PM_ERR_ARG (-1)          /* bad argument (null pointer, bad size, ...) */
#define PM_ERR_CUDA (-2)         /* a CUDA call failed; see pm_last_cuda_error */
#define PM_ERR_UNSUPPORTED (-3)  /* valid but outside this build's limits */
#define PM_ERR_WORKSPACE (-4)    /* workspace smaller than pm_*_workspace_bytes */

/* logits element types */
#define PM_DTYPE_F32 0
#define PM_DTYPE_BF16 1

/* noise sources */
#define PM_NOISE_PHILOX 0   /* Philox4x32-10 keyed by (seed, offset, row) */
#define PM_NOISE_INJECTED 1 /* caller-provided Gumbel values and uniforms */

/* pm_row_params.flags */
#define PM_F_GREEDY 0x1u    /* temperature == 0: argmax */
#define PM_F_TOP_P 0x2u     /* 0 < top_p < 1 */
#define PM_F_MIN_P 0x4u     /* min_p != 0 */
#define PM_F_REP 0x10u      /* repetition penalty on */
#define PM_F_PRES 0x20u     /* presence penalty on */
#define PM_F_FREQ 0x40u     /* frequency penalty on */
#define PM_F_UNBOUNDED 0x100u /* top_p or min_p on while top_k is off */
#define PM_F_FULL 0x200u    /* temperature > 0 and no filter: whole-vocabulary draw */

/* Per-row sampling and processor settings.  Scalars are the fp32 values the
 * reference's arithmetic sees: inv_temperature = fl32(1/temp),
 * top_p_comp = fl32(1 - top_p), log_min_p = fl32(log(min_p)), evaluated in
 * double first as Python does (mlx-lm make_sampler / make_logits_processors
 * keyword arguments; defaults resolved by pagedmoe/sampling.py:121-135). */
typedef struct pm_row_params {
    uint32_t flags;
    float inv_temperature;
    int32_t top_k;               /* <= 0: off */
    float top_p_comp;
    float log_min_p;
    int32_t min_tokens_to_keep;
    float repetition_penalty;
    int32_t repetition_context_size;
    float presence_penalty;
    int32_t presence_context_size;
    float frequency_penalty;
    int32_t frequency_context_size;
} pm_row_params;

/* Rows of logits plus the processors that act on them. */
typedef struct pm_rows {
    const void *logits;          /* [rows, row_stride] of dtype */
    int32_t dtype;               /* PM_DTYPE_* */
    int64_t rows;
    int64_t vocab;
    int64_t row_stride;          /* elements between rows (>= vocab) */
    const pm_row_params *params; /* [rows], or [1] when params_per_row == 0 */
    int32_t params_per_row;
    /* history the penalties read.  Without feed, row r uses
     * hist[r, 0:hist_len[r]].  With feed (a verify pass), row r belongs to
     * request b = r / feed_group at position i = r % feed_group and uses
     * hist[b, 0:hist_len[b]] followed by feed[b, 0:i+1], i.e. its history plus
     * [y] + drafts[:i] (reference verify_decode.py:889-898). */
    const int32_t *hist;         /* [hist_rows, hist_stride] or NULL */
    const int32_t *hist_len;     /* [hist_rows] or NULL (all hist_stride) */
    int64_t hist_stride;
    const int32_t *feed;         /* [rows / feed_group, feed_group] or NULL */
    int32_t feed_group;          /* rows per request when feed != NULL */
    /* logit bias shared by all rows (mlx-lm logit_bias) */
    const int32_t *bias_tokens;  /* [n_bias] distinct ids, ascending (an id out of order is not applied) */
    const float *bias_values;    /* [n_bias] */
    int32_t n_bias;
    /* allowed-token bitmask: bit v of word v/32 of row r; NULL = all allowed */
    const uint32_t *mask;        /* [rows, mask_stride] */
    int64_t mask_stride;         /* words, >= ceil(vocab / 32) */
    /* host-side bounds of the device params (they size the launch): the OR of
     * every row's flags, and the largest top_k of any row (0 if none). */
    uint32_t flags_any;
    int32_t top_k_max;
    /* forced token per row, -1 for none, or NULL: the row's logits become
     * where(arange == forced, logits, -inf) after the other processors (the
     * ThinkBudget processor, reference think_budget.py:107-109) */
    const int32_t *forced;
} pm_rows;

/* Noise of the draw. */
typedef struct pm_noise {
    int32_t mode;                /* PM_NOISE_* */
    uint64_t seed;
    uint64_t offset;             /* advances per step */
    uint32_t row_base;           /* Philox row id of row 0 */
    const float *gumbel;         /* injected: [rows, gumbel_stride] Gumbel values */
    int64_t gumbel_stride;
    const double *uniform;       /* injected: [rows, 2] uniforms in [0,1) */
} pm_noise;

/* Outputs of pm_sample_rows (only tokens is required). */
typedef struct pm_sample_out {
    int32_t *tokens;             /* [rows] */
    float *lse;                  /* [rows] row log-sum-exp of the processed logits, or NULL */
    float *token_logprob;        /* [rows] logprob of the chosen token, or NULL */
    int32_t *surv_ids;           /* [rows, surv_cap] survivors in rank order, or NULL */
    float *surv_probs;           /* [rows, surv_cap] their probabilities at temperature */
    int32_t *n_surv;             /* [rows] */
    int32_t surv_cap;
} pm_sample_out;

/* Workspace bytes pm_sample_rows needs for these rows.  Nothing in the
 * workspace needs to start at zero. */
PM_API size_t pm_sample_workspace_bytes(const pm_rows *rows);

/* One fused pass: processors, row log-sum-exp, top-k / top-p / min-p,
 * temperature and the draw, for every row.  Replaces mlx-lm's
 * make_sampler(...)(logprobs) after make_logits_processors(...) processors
 * (reference verify_decode.py:828-839). */
PM_API int pm_sample_rows(const pm_rows *rows, const pm_noise *noise, const pm_sample_out *out,
                   void *workspace, size_t workspace_bytes, void *stream);

/* Processed logits [rows, vocab] fp32 (logit bias, penalties, mask), the
 * callables of make_logits_processors (verify_decode.py:830-831). */
PM_API size_t pm_processors_workspace_bytes(const pm_rows *rows);
PM_API int pm_apply_processors(const pm_rows *rows, float *out, int64_t out_stride, void *workspace,
                        size_t workspace_bytes, void *stream);

/* Processed logits minus their row log-sum-exp (verify_decode.py:835). */
PM_API int pm_logprobs(const pm_rows *rows, float *out, int64_t out_stride, float *lse_out, void *workspace,
                size_t workspace_bytes, void *stream);

/* Draft acceptance of a verify pass.  rows->rows = requests * (k + 1): row
 * i of request b holds the target logits that judge drafts[b, i] (i < k) or
 * give the bonus token (i = k); rows->feed must be [y] + drafts per request
 * (feed_group = k + 1) so each row's processors see history + [y] + drafts[:i]
 * (reference verify_decode.py:889-898). */
#define PM_VERIFY_MATCH 0     /* reference rule: sample every row, keep drafts while equal
                                 (lookup_decode.py:363-369, verify_decode.py:915-921) */
#define PM_VERIFY_RESIDUAL 1  /* speculative rejection sampling: accept draft i when
                                 u_i * q_i(d) < p_i(d), else draw from max(p_i - q_i, 0) */

typedef struct pm_verify_args {
    int32_t mode;                /* PM_VERIFY_* */
    const int32_t *drafts;       /* [requests, n_draft] */
    int32_t n_draft;             /* k >= 0 */
    const void *draft_logits;    /* residual: [requests * k, draft_row_stride] logits of q */
    int32_t draft_dtype;         /* PM_DTYPE_* */
    int64_t draft_row_stride;
    const double *u_accept;      /* injected: [requests, k] uniforms, else Philox */
    const double *u_residual;    /* injected: [requests] uniforms, else Philox */
    int32_t *tokens;             /* out [requests, k + 1]: accepted drafts, then the
                                    request's own token; -1 after it */
    int32_t *n_accepted;         /* out [requests] */
    int32_t *row_tokens;         /* optional out [requests * (k + 1)]: each row's sample */
} pm_verify_args;

PM_API size_t pm_verify_workspace_bytes(const pm_rows *rows, const pm_verify_args *v);
PM_API int pm_verify(const pm_rows *rows, const pm_noise *noise, const pm_verify_args *v, void *workspace,
                     size_t workspace_bytes, void *stream);

/* Vocabulary-sharded sampling (no reference code: the reference runs on one
 * device).  A tensor-parallel LM head leaves shard i with the contiguous ids
 * [i * shard_width, min((i + 1) * shard_width, vocab_total)) of every row;
 * every shard but the last must be a whole number of 1024-token tiles.  Each
 * shard calls pm_shard_summarize on its slice (rows->vocab = its width, the
 * mask its slice of words, bias ids shifted to the slice; history ids stay
 * global), the caller all-gathers the summaries in shard order (one NCCL
 * all-gather of pm_shard_summary_bytes per shard), and pm_shard_merge gives
 * every rank the row's tokens -- the same tokens, log-sum-exp and survivor
 * lists pm_sample_rows gives on the unsharded rows.  Rows whose unbounded
 * top-p / min-p keeps more than 256 tokens are flagged (status 1, token -1):
 * the caller finishes them with pm_sample_rows on their whole rows (the
 * Python layer all-gathers the flagged rows' slices for that). */
typedef struct pm_shard {
    int32_t shard_index;
    int32_t n_shards;
    int64_t vocab_total;
    int64_t shard_width;         /* ids per shard (the last may hold fewer) */
} pm_shard;

PM_API size_t pm_shard_summary_bytes(const pm_rows *rows, const pm_shard *shard);
PM_API int pm_shard_summarize(const pm_rows *rows, const pm_shard *shard, const pm_noise *noise, void *summary,
                              void *workspace, size_t workspace_bytes, void *stream);
/* rows: the sampler settings (params, flags_any, top_k_max, rows) with
 * vocab = vocab_total; logits are not read.  summaries: [n_shards] summaries
 * back to back.  workspace: at least 4 * rows bytes (row status). */
PM_API int pm_shard_merge(const pm_rows *rows, const pm_shard *shard, const pm_noise *noise, const void *summaries,
                          const pm_sample_out *out, void *workspace, size_t workspace_bytes, void *stream);

/* Batched n-gram drafts: replaces lookup_decode.draft_ngram
 * (pagedmoe/lookup_decode.py:184-221), which scans one request's context per
 * call in Python.  For every request, up to k tokens that followed the
 * latest earlier occurrence of the longest suffix (n_max down to n_min
 * tokens; reference defaults 8 and 3, config.py:1288-1289) -- the latest
 * occurrence with k tokens after it, else the one with the most.  hist:
 * [requests, hist_stride] device ids with optional lengths; drafts:
 * [requests, k] (-1 after draft_len); match_n: the n that matched (0: none),
 * may be NULL.  n_max <= 32. */
PM_API int pm_draft_ngram(const int32_t *hist, const int32_t *hist_len, int64_t hist_stride, int64_t requests,
                          int32_t k, int32_t n_min, int32_t n_max, int32_t *drafts, int32_t *draft_len,
                          int32_t *match_n, void *stream);

/* Device ThinkBudget (reference pagedmoe/think_budget.py:75-109): for every
 * row, the token the close text forces next, or -1.  gen: [rows, gen_stride]
 * ids generated after the prompt (gen_len per row); piece_len / piece_end:
 * [table_size] decoded length and sentence-end flag per id; chars: per-row
 * budget; close: [n_close] ids ending with end_id; start_id < 0 when the
 * template opens reasoning in the prompt (open_in_prompt) -- else reasoning
 * counts only after the model's own start_id; slack: tokens to wait for a
 * sentence end (reference SLACK_TOKENS = 48).  forced: [rows] out, usable as
 * pm_rows.forced. */
PM_API int pm_think_budget(const int32_t *gen, const int32_t *gen_len, int64_t gen_stride, int64_t rows,
                           const int32_t *piece_len, const uint8_t *piece_end, int64_t table_size,
                           const int32_t *chars, const int32_t *close, int32_t n_close, int32_t end_id,
                           int32_t start_id, int32_t slack, int32_t *forced, void *stream);

/* The LM head: logits = hidden @ weight^T on the tensor cores (bf16 in, fp32
 * accumulate), the producer of the logits that the reference's decode step
 * computes before its processors and sampler (pagedmoe/verify_decode.py:821,
 * :824 for a plain step, :887 for a verify pass).  hidden: [n_tokens,
 * hidden_stride] bf16 (the final-norm output); weight: [vocab,
 * weight_stride] bf16 (row v: token v's output embedding).  Both 16-byte
 * aligned with strides a multiple of 8 elements. */
typedef struct pm_lmhead {
    const void *hidden;
    int64_t n_tokens;
    int64_t hidden_size;
    int64_t hidden_stride;       /* elements between rows */
    const void *weight;
    int64_t weight_stride;       /* elements between rows */
} pm_lmhead;

/* The logits themselves: [n_tokens, logits_stride] fp32 (stride a multiple
 * of 4, 16-byte aligned). */
PM_API int pm_lmhead_logits(const pm_lmhead *h, int64_t vocab, float *logits, int64_t logits_stride,
                            void *stream);

/* LM head fused with pm_sample_rows: the GEMM's epilogue writes the tile
 * statistics and candidates of each row, so the logits never reach device
 * memory; the results are those of pm_sample_rows on the logits that
 * pm_lmhead_logits computes (tokens, log-sum-exp, survivors, bit for bit).
 * rows: rows == h->n_tokens and rows->logits unused; greedy rows and rows
 * with 0 < top_k <= 256 (temperature, top_p and min_p on top), with the
 * processors (logit bias, repetition / presence / frequency penalties over
 * rows->hist) and the allowed-token mask.  Verify feeds, forced tokens,
 * unbounded top-p / min-p and whole-vocabulary draws return
 * PM_ERR_UNSUPPORTED (use pm_lmhead_logits + pm_sample_rows).  Row status
 * bit 128: a logit was NaN or +inf.  The workspace needs no zeroing. */
PM_API size_t pm_lmhead_sample_workspace_bytes(const pm_lmhead *h, const pm_rows *rows);
PM_API int pm_lmhead_sample(const pm_lmhead *h, const pm_rows *rows, const pm_noise *noise,
                            const pm_sample_out *out, void *workspace, size_t workspace_bytes, void *stream);

/* pm_sample_rows on scratch owned by the library (no counterpart in the
 * reference, which runs on MLX's allocator): for callers that cannot hand
 * over a device workspace or must not allocate between decode steps.
 * The scratch is a fixed device array of PM_STATIC_SCRATCH_BYTES per device;
 * a call whose rows need more (pm_sample_workspace_bytes(rows) larger than
 * that) returns PM_ERR_WORKSPACE and does nothing: use pm_sample_rows with a
 * workspace of that size instead.  The first call on a device looks the
 * scratch address up, so make it before any stream capture.  Nothing in the
 * scratch needs to start at zero.  One scratch per device: calls on the same
 * device must not overlap (they race on it); keep them on one stream or
 * serialise them. */
#define PM_STATIC_SCRATCH_BYTES (32u << 20)
PM_API int pm_sample_rows_static(const pm_rows *rows, const pm_noise *noise, const pm_sample_out *out,
                                 void *stream);

/* Self-check of the hardware 2^a that the bracketed statistics rely on (no
 * counterpart in the reference): evaluates it on the current device for
 * every fp32 a in [-126, 1] and writes the largest relative error against
 * the fp64 2^a to *max_rel_err (host memory).  Synchronous; allocates and
 * frees a few bytes of device memory.  The library's error budget assumes
 * at most 2^-20. */
PM_API int pm_selfcheck_ex2(double *max_rel_err);

/* Last CUDA error seen by this thread (cudaError_t value), 0 if none. */
PM_API int pm_last_cuda_error(void);

/* Library version string. */
PM_API const char *pm_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PM_SAMPLE_H */
