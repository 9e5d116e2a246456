/*
 * whisper_attn_b200 -- the Whisper decoder's per-step attention for B200 (sm_100a), as a C ABI.
 *
 * One shared library (libwhisper_attn_b200.so) with plain pointers and sizes: no torch types. Every entry point
 * launches asynchronously on the given CUDA stream (a cudaStream_t passed as void*; NULL = the legacy default
 * stream), never synchronises, never allocates, and is safe to record into a CUDA graph. Each returns a status
 * (WT_OK = 0); on failure wt_last_error() gives the calling thread's message. Device code never traps: offsets
 * are clamped to [0, C] and slot-table entries to [0, N-1], as the reference's kernels do.
 *
 * Element types: WT_F16 or WT_BF16 for every activation / cache tensor of a call. Every pointer must be 16-byte
 * aligned (checked). Layouts are the reference plugin's (contiguous, row-major):
 *   qkv      [N, 3*H*D]      queries, keys, values of the new token, heads in order
 *   k/v cache [N, H, C, D]   one layer's self-attention cache (capacity C)
 *   offset   [N]  int64      cached positions of each row (the new token's slot)
 *   src      [N, C] int32    for each cache slot of a row, the row whose cache holds it
 *   cross q  [W, S, H*D]     a window's S queries (its K beams x tokens), windows in order
 *   cross k/v [W, H, T, D]   one layer's cross-attention keys/values (T encoder frames), once per window
 *   part     [W, H, P, S, D+2] float32  split partials: unnormalised output, running max (log2 units), sum
 *
 * Reference interface each entry point replaces: Wataru-Nakata/whisper-trt, src/whisper_trt/attn_plugin.py and
 * search.py / beam_kernels.py (file:line given per function).
 */
#ifndef WHISPER_ATTN_B200_H
#define WHISPER_ATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WT_ABI_VERSION 1

/* element types */
#define WT_F16 0
#define WT_BF16 1

/* status codes */
#define WT_OK 0
#define WT_ERR_ARG 1         /* a size or pointer is invalid (null, negative, inconsistent) */
#define WT_ERR_ALIGN 2       /* a pointer is not 16-byte aligned */
#define WT_ERR_DTYPE 3       /* unknown element type */
#define WT_ERR_UNSUPPORTED 4 /* a valid shape this build has no kernel for (e.g. head_dim not 64) */
#define WT_ERR_WORKSPACE 5   /* workspace missing or smaller than the matching *_workspace() size */
#define WT_ERR_CUDA 6        /* the CUDA launch failed */

/* launch flags (wt_set_launch_flags)
 * WT_LAUNCH_PDL: programmatic dependent launch. A kernel may start while the kernel launched just before it in the
 *   same stream drains, and reads its predecessor-independent inputs before waiting for it: the self-attention
 *   step its offsets, slot table and cache (slots below the offsets), the cross-attention its cross keys/values.
 *   Those inputs must therefore not be written by the kernel launched immediately before (in a decoder step they
 *   come from earlier steps and the encoder; the queries, which the preceding GEMM produces, are always read after
 *   the wait). Every kernel waits for its predecessor before writing anything. */
#define WT_LAUNCH_PDL 1

int wt_abi_version(void);
const char *wt_status_string(int status);
/* The message of the calling thread's last failing call ("" if none). */
const char *wt_last_error(void);
/* Process-wide launch flags (WT_LAUNCH_*); returns the previous value. Default: 0. */
int wt_set_launch_flags(int flags);

/* Bounded waits. Every wait inside a kernel (an mbarrier that a TMA copy or the tensor cores complete, a request
 * one warp hands another) polls at most this many times, with back-off, then records an error code in the call's
 * device error word (the first 4 bytes of its workspace / error buffer) and gives up: the kernel returns, its
 * results are not valid, and the context stays usable. Process-wide, read at each launch; 0 restores the default
 * (2^22 polls: far beyond any wait that completes); returns the previous value. No counterpart in the reference
 * (whose kernels have no device-side waits). */
unsigned wt_set_wait_limit(unsigned polls);
/* Test hook for the bounded waits: when nonzero, launches of the fused cross-attention (wt_cross_attn) issue no
 * copy for the first ring stage of their first streaming warp, and launches of wt_logits32, wt_ln_linear and
 * wt_linear_residual leave out the row block of the first stage of their first CTA, so a wait on that stage must
 * run out (after wt_set_wait_limit's polls) and the call's error word is set; every other copy still lands and is
 * waited for before the kernel exits (nothing is left in flight). For tests of the failure path only: 0 (the
 * default) in use. Returns the previous value. No counterpart in the reference. */
int wt_set_test_withhold_stage(int on);

/* ---------------------------------------------------------------------------------------------------------
 * Self-attention of one new token per row over the row's cache slots < offset[r], each read from the row
 * src[r, j] names, plus the new token itself.
 * Replaces attn_plugin.py:488-501 self_attn_step_triton (kernel :309-350, config :482-485).
 *   y [N, 1, H*D] (element type of qkv) = softmax(q k^T / sqrt(D)) v over [gathered cache | new token].
 *   write_cache != 0: the new key/value are also written into the row's own slot offset[r] (if < C) of
 *   k_cache / v_cache (rows only read slots below their offset, so the result does not change).
 *   kv_splits: 0 = choose from the shape (wt_self_attn_step_splits); 1 = one CTA per (row, head); >1 = split
 *   every row's cache range into that many parts combined in-kernel, which needs `workspace` of
 *   wt_self_attn_step_workspace() bytes. kv_splits must be at least ceil(capacity / 1024).
 *   A workspace is laid out by the call's shape (rows, heads, head_dim, kv_splits): zero it before its first use
 *   with a shape; each call leaves its counters zeroed for the next call of the SAME shape (its partials stay as
 *   written, so another shape needs another -- or a re-zeroed -- workspace). Calls that may overlap on the GPU
 *   must not share a workspace.
 * ------------------------------------------------------------------------------------------------------- */
size_t wt_self_attn_step_workspace(int rows, int heads, int head_dim, int kv_splits);
int wt_self_attn_step_splits(int rows, int heads, int capacity, int head_dim);
int wt_self_attn_step(int dtype, const void *qkv, void *k_cache, void *v_cache, const int64_t *offset,
                      const int32_t *src, void *y, int rows, int heads, int capacity, int head_dim,
                      int write_cache, int kv_splits, void *workspace, size_t workspace_bytes, void *stream);
/* wt_self_attn_step_prefix: wt_self_attn_step (the same result, the same reference function, no key splits) for
 *   rows that come in groups of `group` consecutive rows (1-8: a window's beams or samples) sharing a prefix of
 *   their slot tables -- the prompt every row of a window reads from the window's first row, the beams' common
 *   ancestry. Row a + n of the group starting at row a shares keys [0, p) with row a, p the first position below
 *   min(offset[a + n], offset[a]) where their clamped slot-table entries differ (row a: its offset); when p >=
 *   min_shared, a first kernel attends those keys once for the whole group (tensor cores, the group's queries as
 *   one tile) and the step kernel after it attends the row's keys [p, offset) and the new token and merges the two.
 *   Rows that share less than min_shared keys are attended as by wt_self_attn_step. Needs `workspace` of
 *   wt_self_attn_step_prefix_workspace() bytes (no zeroing, any contents), not shared by calls that may overlap.
 *   head_dim 64, capacity <= 1024. No counterpart in the reference (an added entry point; the grouping is the
 *   caller's knowledge of its windows, which the reference's self_attn_step_triton does not receive). */
size_t wt_self_attn_step_prefix_workspace(int rows, int heads, int head_dim);
int wt_self_attn_step_prefix(int dtype, const void *qkv, void *k_cache, void *v_cache, const int64_t *offset,
                             const int32_t *src, void *y, int rows, int heads, int capacity, int head_dim,
                             int write_cache, int group, int min_shared, void *workspace, size_t workspace_bytes,
                             void *stream);

/* ---------------------------------------------------------------------------------------------------------
 * Self-attention of S = new_tokens new tokens per row (a prompt) over the row's cache slots < offset[r] (each read
 * from the row src[r, j] names) and, causally, the new tokens up to itself.
 * Replaces attn_plugin.py:462-479 self_attn_triton (kernel :275-307; op body :102-121).
 *   qkv [N, S, 3*H*D], caches [N, H, C, D] (read only: the caller stores the new keys/values), y [N, S, H*D].
 *   head_dim 64. No workspace; offset clamped to [0, C], slot-table rows to [0, N-1].
 * ------------------------------------------------------------------------------------------------------- */
int wt_self_attn(int dtype, const void *qkv, const void *k_cache, const void *v_cache, const int64_t *offset,
                 const int32_t *src, void *y, int rows, int new_tokens, int heads, int capacity, int head_dim,
                 void *stream);

/* ---------------------------------------------------------------------------------------------------------
 * Cross-attention, split over the T keys ("flash-decoding").
 * wt_cross_attn_split replaces attn_plugin.py:521-534 cross_attn_split_triton (kernel :378-409): slice i of
 *   chunk = ceil(T / splits) keys -> part[w, h, i, s, :] = (sum_j p_j v_j, m, sum_j p_j) with m the slice's
 *   maximum score in log2 units and p_j = exp2(score_j - m); a slice without keys gets m = -inf, 0, 0.
 * wt_cross_attn_combine replaces attn_plugin.py:537-546 cross_attn_combine_triton (kernel :411-435):
 *   y [W, S, H*D] = sum_i w_i acc_i / sum_i w_i l_i with w_i = exp2(m_i - max m).
 * wt_cross_attn replaces attn_plugin.py:504-518 cross_attn_triton (kernel :352-376): the same attention in one
 *   launch (split + combine, the last CTA of each (window, head) combines); needs `workspace` of
 *   wt_cross_attn_workspace() bytes, with the same per-shape rule as wt_self_attn_step's: zeroed before its
 *   first use with a shape, valid for further calls of that shape only, not shared by calls that may overlap.
 *   Its first 4 bytes are a device error word: non-zero after a kernel's bounded wait for its own TMA copies gave
 *   up (the output is then not valid); the kernel never hangs. With at most 8 queries per window (one CTA per
 *   (window, head), its key slices combined on chip) the workspace is that word alone (256 bytes); larger query
 *   groups take the stream-K kernel, whose size depends on the device's SM count.
 * ------------------------------------------------------------------------------------------------------- */
int wt_cross_attn_split(int dtype, const void *q, const void *k, const void *v, float *part, int windows,
                        int queries, int heads, int frames, int head_dim, int splits, void *stream);
/* wt_cross_attn_split_ws: wt_cross_attn_split (the same part, the same reference function) on the persistent
 *   stream-K TMA kernel of wt_cross_attn, its units the (window, head, slice) triples: it streams the keys at the
 *   fused kernel's rate where the per-slice kernel of wt_cross_attn_split takes one CTA per slice. Needs a workspace
 *   of wt_cross_attn_split_workspace() bytes (the per-shape rule of wt_cross_attn's); that size is 0 for shapes the
 *   stream-K kernel does not take (a 16-key block of some slice would hold no key, e.g. T < 16 * splits), which run
 *   the per-slice kernel and need no workspace. */
size_t wt_cross_attn_split_workspace(int windows, int queries, int heads, int frames, int head_dim, int splits);
int wt_cross_attn_split_ws(int dtype, const void *q, const void *k, const void *v, float *part, int windows,
                           int queries, int heads, int frames, int head_dim, int splits, void *workspace,
                           size_t workspace_bytes, void *stream);
int wt_cross_attn_combine(int dtype, const float *part, void *y, int windows, int queries, int heads,
                          int head_dim, int splits, void *stream);
size_t wt_cross_attn_workspace(int windows, int queries, int heads, int frames, int head_dim);
int wt_cross_attn(int dtype, const void *q, const void *k, const void *v, void *y, int windows, int queries,
                  int heads, int frames, int head_dim, void *workspace, size_t workspace_bytes, void *stream);
/* wt_cross_attn_noalloc: no counterpart in the reference. The same cross-attention as wt_cross_attn for callers
 *   that cannot allocate device memory while they run (a TensorRT-style plugin enqueue that must stay inside the
 *   memory its engine planned; an application whose device memory belongs to its own allocator or budget): it takes
 *   no workspace and allocates nothing. Its scratch is a fixed 8 MiB device array in this library (64 KiB of
 *   counters + partials), which every GPU that loads the library holds until the process exits. Shapes needing
 *   more (more than 16384 (window, head, query group) units, or partials above 8 MiB - 64 KiB -- e.g. more than
 *   ~24 queries per window at 32 windows) are rejected with WT_ERR_UNSUPPORTED. The first call on a device looks up
 *   the array's device address (cudaGetSymbolAddress); make that first call before any stream capture. Every call
 *   shares the array and clears its counters (cudaMemsetAsync on `stream`) before the kernel: calls that overlap
 *   on the GPU (other streams, other threads) race on it. */
int wt_cross_attn_noalloc(int dtype, const void *q, const void *k, const void *v, void *y, int windows,
                          int queries, int heads, int frames, int head_dim, void *stream);

/* ---------------------------------------------------------------------------------------------------------
 * KV-cache append and gather (bit-exact copies).
 * wt_cache_append: row r's new key/value (qkv[r, H*D:2*H*D], qkv[r, 2*H*D:]) into its own cache slot offset[r]
 *   when 0 <= offset[r] < C. The append of attn_plugin.py:327-330 (WRITE) alone, i.e. the cache scatter of
 *   search.py:249-250 for one layer and one token.
 * wt_gather_cache: out[r, h, j, :] = cache[src[r, j], h, j, :] for every slot j < C (src clamped to [0, N-1]).
 *   Replaces attn_plugin.py:92-99 gather_cache (the reference's materialised view of the slot table).
 * ------------------------------------------------------------------------------------------------------- */
int wt_cache_append(int dtype, const void *qkv, void *k_cache, void *v_cache, const int64_t *offset, int rows,
                    int heads, int capacity, int head_dim, void *stream);
int wt_gather_cache(int dtype, const void *cache, const int32_t *src, void *out, int rows, int heads,
                    int capacity, int head_dim, void *stream);

/* ---------------------------------------------------------------------------------------------------------
 * Slot-table bookkeeping (integers, bit-exact). N = windows * beams rows; row r belongs to window r / beams.
 * wt_beam_reorder: the new beams take their parents' slot tables, each marking the slot its parent wrote this
 *   step: for each window b with live[b] != 0 (live may be NULL = all) and beam k with parent p = parent[b, k]
 *   (0 <= p < beams): src[b*K+k] = src_old[b*K+p] and src[b*K+k, pos[b]] = b*K+p; with hist (may be NULL)
 *   hist[b*K+k] = hist_old[b*K+p] and, when token and t are given, hist[b*K+k, t[b]] = token[b*K+k];
 *   pos[b] += 1 when advance != 0; when offset (may be NULL) is given, offset[r] = pos[r / K] afterwards.
 *   search.py:258 + :401-409 + :263-264 (beam_kernels.py:241-248, :260-264).
 * wt_beam_update: beam_kernels.py:169-269 _update_kernel in beam mode (no sampled slots): from each window's
 *   best 2K candidates (top_s, top_i = beam*V + token, best first) CTranslate2's rules -- finished hypotheses
 *   registered, ended candidates replaced by the next non-ending secondary ones -- then the new beams' parents'
 *   histories and slot tables, scores, tokens; prompt windows (t < 0) get their next prompt token and mark their
 *   slot; windows not ending advance. State arrays as in the reference's Search (search.py:184-223).
 * wt_slot_reset: search.py:440-446 (_start): for each of n_slots slots s (0 <= s < windows; others ignored),
 *   rows s*K..s*K+K-1 read their own rows (src[r, :] = r) or, prefilled != 0, the slot's first row
 *   (src[r, :] = s*K).
 * Out-of-range parent / candidate indices are clamped to the window's beams, hypothesis slots beyond hyp_slots
 * are not written: a bad index never touches another window or memory outside the arrays.
 * ------------------------------------------------------------------------------------------------------- */
int wt_beam_reorder(int32_t *src, int64_t *hist, const int64_t *token, const int64_t *t, const int64_t *parent,
                    int64_t *pos, const uint8_t *live, int64_t *offset, int windows, int beams, int capacity,
                    int hist_len, int advance, void *stream);
int wt_beam_update(const float *top_s, const int64_t *top_i, int64_t *t, int64_t *pos, const int64_t *sot_pos,
                   const float *ns, float *no_speech, uint8_t *done, int64_t *hist, float *cum, int32_t *src,
                   int64_t *tokens, const int64_t *forced, int64_t *h_count, float *h_score, int64_t *h_len,
                   int64_t *h_tokens, const int64_t *last_t, int windows, int beams, int capacity, int hist_len,
                   int hyp_slots, int prompt_len, int vocab, int eot, void *stream);
int wt_slot_reset(int32_t *src, const int64_t *slots, int n_slots, int windows, int beams, int capacity,
                  int prefilled, void *stream);
/* wt_beam_update_mixed: wt_beam_update for a beam search with sampled slots (the reference's
 *   Search(sampling_slots=True)); replaces beam_kernels.py:169-269 _update_kernel with MIXED (its sampled branch
 *   :200-225). Windows with sampling[b] != 0 follow CTranslate2's GreedySearch rules on their rows' sampled tokens
 *   (samp_tok / samp_score [N], from wt_beam_sample): a row not yet done adds its token's log-probability to cum,
 *   appends the token to its history and length unless it is EOS, is done after EOS or at the last step; every row
 *   takes its token and marks its new slot; the window is done when all its rows are, else it advances. Other
 *   windows follow wt_beam_update. row_done [N] 0/1 bytes, length [N] int64. With sampling == NULL it is
 *   wt_beam_update (the other four may then be NULL). */
int wt_beam_update_mixed(const float *top_s, const int64_t *top_i, int64_t *t, int64_t *pos, const int64_t *sot_pos,
                         const float *ns, float *no_speech, uint8_t *done, int64_t *hist, float *cum, int32_t *src,
                         int64_t *tokens, const int64_t *forced, int64_t *h_count, float *h_score, int64_t *h_len,
                         int64_t *h_tokens, const int64_t *last_t, const uint8_t *sampling, const int64_t *samp_tok,
                         const float *samp_score, uint8_t *row_done, int64_t *length, int windows, int beams,
                         int capacity, int hist_len, int hyp_slots, int prompt_len, int vocab, int eot,
                         void *stream);
/* wt_beam_sample: each sampled row's next token, by Gumbel-max -- replaces beam_kernels.py:284-289 sample() (kernel
 *   :136-167) and the sampling of search.py:342-346 (_greedy), with search.py:104-129 uniform()'s counter-based
 *   random numbers. For every row r of a window b with sampling[b] != 0, done[b] == 0, t[b] >= 0 and
 *   row_done[r] == 0: u_v = uniform(seed[b], t[b], r % beams, v), g_v = scores[r, v] / temperature[b]
 *   - log(-log(max(u_v, 1e-20))); samp_tok[r] = the first v with the largest g_v, samp_score[r] = scores[r, that v]
 *   (scores [N, V]: the rows' log-probabilities, as wt_beam_scores_mixed writes them). Other rows are untouched. */
int wt_beam_sample(const float *scores, const int64_t *t, const uint8_t *done, const uint8_t *row_done,
                   const uint8_t *sampling, const float *temperature, const int64_t *seed, int64_t *samp_tok,
                   float *samp_score, int windows, int beams, int vocab, void *stream);

/* ---------------------------------------------------------------------------------------------------------
 * The vocabulary projection, fp32 accumulate and output: y [N, V] = x [N, d] . w [V, d]^T (x, w fp16 or bf16,
 * the same type), on the 5th-generation tensor cores (tcgen05).
 * Replaces attn_plugin.py:549-560 logits32_triton (kernel :438-455; op body :202-212).
 *   d a multiple of 8. `err`: a device int (zero it once): non-zero after a bounded wait of the kernel gave up.
 * ------------------------------------------------------------------------------------------------------- */
int wt_logits32(int dtype, const void *x, const void *w, float *y, int rows, int vocab, int d_model, int *err,
                void *stream);

/* ---------------------------------------------------------------------------------------------------------
 * The scoring half of a beam step, feeding wt_beam_update.
 * Replaces beam_kernels.py:351-361 scores() (kernel :36-135 _scores_kernel, beam mode) and the topk of
 * search.py:253 (PyTorch path: search.py:283-289 _choose, :313-338 _timestamp_rules, :369-371, :259-260):
 *   per row r of window b = r / beams: the logits [N, V] fp32 with the suppressed tokens (suppress [V], 0/1 bytes)
 *   and, at the window's first step (t[b] == 0), the begin-suppressed ones (begin [V]) set to the lowest float;
 *   with `timestamps`, CTranslate2's timestamp rules on the row's history hist [N, hist_len] (max_initial [1]);
 *   scores = log_softmax(masked) + cum[r] -> `scores` [N, V] (may be NULL: not written);
 *   ns [B] = exp(logit[no_speech] - logsumexp(logits)) of each window's first row;
 *   top_s / top_i [B, 2*beams]: the window's best 2K of its beams x V candidate scores, best first, equal scores
 *   in index order; top_i = beam * V + token. Up to 8 beams; beams * vocab < 2^31.
 *   Needs a workspace of wt_beam_scores_workspace() bytes, zeroed before first use (left zeroed by each call);
 *   calls that may overlap on the GPU must not share one.
 * ------------------------------------------------------------------------------------------------------- */
size_t wt_beam_scores_workspace(int windows, int beams);
int wt_beam_scores(const float *logits, const uint8_t *suppress, const uint8_t *begin, const int64_t *t,
                   const float *cum, const int64_t *hist, const int64_t *max_initial, float *scores, float *ns,
                   float *top_s, int64_t *top_i, int windows, int beams, int vocab, int hist_len, int timestamps,
                   int no_speech, int no_timestamps, int ts_begin, int eot, void *workspace, size_t workspace_bytes,
                   void *stream);
/* wt_beam_scores_mixed: wt_beam_scores for a search with sampled slots (beam_kernels.py:351-361 with MIXED,
 *   kernel :105-106): the rows of windows with sampling[b] != 0 score their log-probabilities alone (no cum);
 *   sampling [B] 0/1 bytes, or NULL (= wt_beam_scores). */
int wt_beam_scores_mixed(const float *logits, const uint8_t *suppress, const uint8_t *begin, const int64_t *t,
                         const float *cum, const uint8_t *sampling, const int64_t *hist, const int64_t *max_initial,
                         float *scores, float *ns, float *top_s, int64_t *top_i, int windows, int beams, int vocab,
                         int hist_len, int timestamps, int no_speech, int no_timestamps, int ts_begin, int eot,
                         void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------------------------------------------
 * The decoder step's linear layers with their LayerNorm, bias, GELU and residual fused around them, on the
 * 5th-generation tensor cores (tcgen05); x [rows, in], w [out, in] (nn.Linear layout), b [out], all of one 16-bit
 * type (fp16 or bf16); fp32 accumulation; in and out multiples of 8.
 * wt_layer_norm_bias replaces decoder_kernels.py:127-135 layer_norm_bias (kernel :100-115):
 *   y [rows, d] = LN(x) (fp32 statistics: mean, then the mean square of x - mean; rstd = 1/sqrt(var + eps);
 *   rounded), and x = x + bias in place (after it is read).
 * wt_ln_linear replaces decoder_kernels.py:138-146 ln_linear (kernel :42-75):
 *   y [rows, out] = LN(x) . w^T + b, rounded to the 16-bit type (LN(x) rounded first); gelu != 0: y =
 *   round(gelu(round(...))) with gelu(v) = v/2 (1 + erf(v / sqrt 2)) in fp32.
 * wt_linear_residual replaces decoder_kernels.py:149-157 linear_residual (kernel :77-97):
 *   y [rows, out] = round(round(x . w^T + b) + res); y may be res (the residual stream updated in place).
 *   Both GEMMs need a workspace of wt_dec_linear_workspace(rows, out, in, layer_norm) bytes (layer_norm: 1 for
 *   wt_ln_linear, 0 for wt_linear_residual; it depends on the device's SM count), zeroed before its first use and
 *   left with its counters zeroed by each call; its first 4 bytes are a device error word (non-zero after a bounded
 *   wait gave up). Calls that may overlap on the GPU must not share a workspace.
 * ------------------------------------------------------------------------------------------------------- */
size_t wt_dec_linear_workspace(int rows, int out_features, int in_features, int layer_norm);
int wt_layer_norm_bias(int dtype, void *x, const void *gamma, const void *beta, const void *bias, void *y, int rows,
                       int d, float eps, void *stream);
int wt_ln_linear(int dtype, const void *x, const void *gamma, const void *beta, const void *w, const void *b, void *y,
                 int rows, int out_features, int in_features, int gelu, float eps, void *workspace,
                 size_t workspace_bytes, void *stream);
int wt_linear_residual(int dtype, const void *x, const void *w, const void *b, const void *res, void *y, int rows,
                       int out_features, int in_features, void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* WHISPER_ATTN_B200_H */
