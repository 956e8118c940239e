/*
 * streaming_attention.h -- C ABI of the B200 (sm_100a) streaming Taylor-moment
 * + block-coreset causal attention library (libsa_b200.so).
 *
 * Every entry point takes raw pointers and sizes, enqueues its work on the
 * given CUDA stream (a cudaStream_t passed as void*, NULL = legacy default
 * stream) of the current device, and returns an int status (SA_OK == 0,
 * negative on error).  Nothing throws across this boundary.  After an error,
 * sa_last_error() returns a message for the calling thread.
 *
 * Tensor layouts (all contiguous, row-major, fp32 unless noted):
 *   q, k  [bh, n, d]      v, out  [bh, n, dv]
 *   bh = B*H sequences ("heads"); each is processed independently.
 *
 * Coreset draw tables (host-generated, copied to the device; see
 * streaming_attention_b200/draws.py).  nc = completed blocks per head =
 * (n - 1) / block_size, m = (block_size + 1) / 2 reps per completed block:
 *   dirs  [bh, nc, d]              fp32, unit projection direction per block
 *   coins [bh, nc, block_size/2]   fp32 uniform draws in [0,1) per pair
 *   perms [bh, nc, m]              int32 block-local indices (random
 *                                  compressor, and sorted_pair when
 *                                  block_size <= 2)
 *
 * Reference interfaces replaced (PositiveLoss/streaming-attention):
 *   sa_fast_attention      fast_article_causal_attention
 *                          (fast_article_attention.py:634-719) and its
 *                          per-sequence body (:522-631)
 *   sa_compress_blocks     _build_completed_block_reps (:364-434) +
 *                          _compress_one_completed_block (:312-361)
 *   sa_low_moments         low_degree_taylor_causal_sums (:262-285) and the
 *                          moment sketch (streaming_taylor_coreset_attention.py:229-296)
 *   sa_residual_combine    _block_coreset_residual_tail (:467-514),
 *                          _full_residual_tail (:437-464) and the final
 *                          num / clamp(den, eps) (:596-598)
 *   sa_feature_count       num_taylor_features (:137-148) /
 *                          SymmetricTaylorFeatureMap.total_features
 *                          (streaming_taylor_coreset_attention.py:180-182)
 */
#ifndef STREAMING_ATTENTION_H_
#define STREAMING_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define SA_OK 0
#define SA_ERR_INVALID_ARG (-1)   /* bad shape / size / pointer; ValueError */
#define SA_ERR_UNSUPPORTED (-2)   /* degree or dims beyond the kernels; NotImplementedError */
#define SA_ERR_CUDA (-3)          /* CUDA launch or runtime error; RuntimeError */
#define SA_ERR_TIMEOUT (-4)       /* a bounded device-side wait gave up */
#define SA_ERR_WORKSPACE (-5)     /* workspace smaller than sa_*_workspace_size */
#define SA_ERR_DEVICE_CHECK (-6)  /* a device-side index check failed (libsa_b200_checks.so only) */

/* compressor kinds (fast_article_attention.py:326, :332, :383) */
#define SA_COMPRESSOR_NONE 0
#define SA_COMPRESSOR_SORTED_PAIR 1
#define SA_COMPRESSOR_RANDOM 2

/* largest supported Taylor degree and feature count */
#define SA_MAX_DEGREE 3
#define SA_MAX_DIM 256
#define SA_MAX_VALUE_DIM 256

/* Library version, e.g. 100 for 0.1.0. */
int sa_version(void);

/* Message of the last error on this thread ("" if none). */
const char* sa_last_error(void);

/* Feature count sum_{l<=degree} C(dim+l-1, l). */
int sa_feature_count(int dim, int degree, int64_t* count);

/* Number of completed blocks that a later query reads: (n-1)/block_size
 * (fast_article_attention.py:403-407).  *reps_per_block = (block_size+1)/2,
 * or block_size for compressor none. */
int sa_block_counts(int64_t n, int block_size, int compressor, int64_t* completed_blocks,
                    int64_t* reps_per_block);

/* C1: compress every completed block of every head.
 * Outputs: rep_idx [bh, nc*m] int32 (global token index within the head, the
 * bit-exact selection), rep_k [bh, nc*m, d], rep_v [bh, nc*m, dv],
 * rep_w [bh, nc*m].  Any of rep_k / rep_v / rep_w may be NULL. */
int sa_compress_blocks(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                       int block_size, int compressor, const float* dirs, const float* coins,
                       const int32_t* perms, int32_t* rep_idx, float* rep_k, float* rep_v,
                       float* rep_w, void* stream);

/* Low-degree Taylor term of every query, with the moment state taken over the
 * completed blocks before the query's own block:
 *   low[i, :dv] = sum_{j < bstart(i)} P_t(scale q_i.k_j) v_j,
 *   low[i, dv]  = sum_{j < bstart(i)} P_t(scale q_i.k_j),
 * where bstart(i) = (i / block_size) * block_size.  low is [bh, n, dv+1].
 * When the tensor-core kernel applies (dv <= 64) it needs a caller workspace
 * of sa_low_moments_workspace_size bytes (256-byte aligned); otherwise the
 * workspace may be NULL. */
int sa_low_moments_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree, int block_size,
                                  size_t* bytes);
int sa_low_moments(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d,
                   int dv, int degree, int block_size, float scale, float* low, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Residual over the completed-block reps + exact current block, added to the
 * low term, then out = num / max(den, eps).  rep_k/rep_v/rep_w are the
 * outputs of sa_compress_blocks ([bh, nc*m, *]); for compressor none they are
 * ignored (every earlier key is a rep of weight 1).  For d <= 64 and
 * dv <= 128 the tensor-core kernel runs and needs a caller workspace of
 * sa_residual_combine_workspace_size bytes (256-byte aligned); otherwise the
 * workspace may be NULL. */
int sa_residual_combine_workspace_size(int64_t bh, int64_t n, int d, int dv, int block_size,
                                       int compressor, size_t* bytes);
int sa_residual_combine(const float* q, const float* k, const float* v, const float* rep_k,
                        const float* rep_v, const float* rep_w, const float* low, int64_t bh,
                        int64_t n, int d, int dv, int degree, int block_size, int compressor,
                        float scale, float eps, float* out, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Bytes of device workspace sa_fast_attention needs. */
int sa_fast_attention_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree,
                                     int block_size, int compressor, size_t* bytes);

/* The whole forward of fast_article_causal_attention for bh sequences.
 * rep_idx (nullable) receives the coreset selection [bh, nc*m].  workspace is
 * caller-owned device memory of at least sa_fast_attention_workspace_size
 * bytes, 256-byte aligned.  The call is ordered on `stream` like one kernel:
 * with a compressor and the tensor-core kernels, its moment scan runs on a
 * second stream of the device's highest priority (made, with two events, at
 * the first such call per host thread and caller stream -- at most 16 per
 * thread -- and kept until the process ends) that forks from and joins back
 * into `stream`; under graph capture, while stage events are set, or with
 * sa_set_moment_fork(0), everything runs on `stream` itself. */
int sa_fast_attention(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d,
                      int dv, int degree, int block_size, float scale, int compressor,
                      const float* dirs, const float* coins, const int32_t* perms, float eps,
                      float* out, int32_t* rep_idx, void* workspace, size_t workspace_bytes,
                      void* stream);

/* ---- run-time controls and status (no counterpart in the reference) -------
 * The reference runs eagerly on one device and has neither device-side waits
 * nor a status word; these entry points belong to this library's own runtime. */

/* The launch status word that sa_fast_attention, sa_low_moments,
 * sa_residual_combine, sa_article_segment_mean, sa_flash_causal_attention and
 * the shard calls keep in the first 4 bytes of their workspace: synchronises
 * `stream`, then returns SA_OK when no bounded device-side wait of the last
 * call on that workspace gave up, else SA_ERR_TIMEOUT (sa_last_error() names
 * the kernel's wait code), or SA_ERR_DEVICE_CHECK in a checks build. */
int sa_workspace_status(const void* workspace, void* stream);

/* Whether sa_fast_attention may fork its moment scan onto a second stream
 * (see sa_fast_attention), for the calling host thread: 1 (the default) lets
 * it, 0 runs every stage in order on the caller's stream.  Callers that
 * already overlap several forwards on streams of their own (this library's
 * host-tensor path does, for its chunks) gain nothing from the fork: a later
 * forward's moment scan, at the higher priority, then delays the earlier
 * forward's residual.  sa_moment_fork_enabled returns the current setting. */
int sa_set_moment_fork(int enable);
int sa_moment_fork_enabled(void);

/* 1 in libsa_b200_checks.so, the build with device-side index checks
 * (-DSA_DEVICE_CHECKS: a check that fails records its code, 900..999, in the
 * status word and the offending index 8 bytes after it, and skips the access;
 * sa_workspace_status then returns SA_ERR_DEVICE_CHECK), 0 in libsa_b200.so. */
int sa_device_checks_enabled(void);

/* How long one bounded device-side wait of the tensor-core kernels may take
 * before its CTA gives up, drains what it issued, records SA_ERR_TIMEOUT's
 * cause in the status word and leaves (the process-wide default, 0, means
 * 2 s).  Applies to launches made after the call, from any thread. */
int sa_set_wait_limit_ns(uint64_t limit_ns);

/* Measurement hook for the calling host thread: while `count` > 0,
 * sa_fast_attention records events[i] (cudaEvent_t handles, created by the
 * caller) on its stream at stage boundaries: 0 start, 1 after the k / v
 * operand splits, 2 after the compressor (and the split of its reps), 3 after
 * the moment scan, 4 after the residual (the end); the stages then run one
 * after another on that stream.  count = 0 turns it off. */
int sa_set_stage_events(void* const* events, int count);

/* ---- streaming (decode) state: ArticleStreamingAttention -------------------
 * The reference keeps, per attention stream, a Taylor moment sketch and a
 * merge-and-reduce coreset (streaming_taylor_coreset_attention.py:229-616).
 * Here that state lives in caller-owned device buffers: num [F, dv] and den [F]
 * (fp32, F = sa_feature_count(d, degree)), a pending block of raw keys /
 * values, and the level items (keys [m, d], values [m, dv], weights [m]).
 * The caller keeps the level structure and draws the compressor's random
 * numbers (as the streaming class in streaming_attention_b200/streaming.py does). */

/* Replaces TaylorMomentSketch.update (streaming_taylor_coreset_attention.py:262-279):
 * num[f, :] += (weight * phi_k(key)[f]) * value, den[f] += weight * phi_k(key)[f],
 * product then add, each rounded to fp32, as the reference does. */
int sa_stream_update(const float* key, const float* value, int d, int dv, int degree, float weight,
                     float* num_state, float* den_state, void* stream);

/* Replaces MergeReduceCoreset._compress (streaming_taylor_coreset_attention.py:414-470)
 * for one block of n >= 2 weighted items: sorted_pair (direction [d], coins
 * [n/2]; n <= 2 uses perm) or random (perm [ceil(n/2)] of the first draws of
 * randperm(n)).  Writes ceil(n/2) items; outputs must not overlap inputs. */
int sa_stream_compress(const float* keys, const float* values, const float* weights, int64_t n, int d,
                       int dv, int compressor, const float* direction, const float* coins,
                       const int32_t* perm, float* out_keys, float* out_values, float* out_weights,
                       void* stream);

/* Bytes of device workspace sa_stream_query needs. */
int sa_stream_query_workspace_size(int d, int dv, int degree, size_t* bytes);

/* Replaces ArticleStreamingAttention.query (streaming_taylor_coreset_attention.py:572-606):
 * out [dv] = (phi_q(scale q).[num, den] + sum over the pending block (weight 1)
 * and the level items of w (exp(x) - P_t(x)) [v, 1]) / max(den, eps), with
 * x = scale * (k . q).  dens (nullable) receives {den, low den, tail den}. */
int sa_stream_query(const float* query, int d, int dv, int degree, float scale, const float* num_state,
                    const float* den_state, const float* buf_keys, const float* buf_values, int64_t n_buf,
                    const float* lvl_keys, const float* lvl_values, const float* lvl_weights,
                    int64_t n_lvl, float eps, float* out, float* dens, void* workspace,
                    size_t workspace_bytes, void* stream);

/* ---- one shard of a long sequence split along N over GPUs ------------------
 * The reference has no multi-GPU path; these split one forward of
 * fast_article_causal_attention (fast_article_attention.py:634-719) over P
 * ranks that each hold a contiguous token range of every sequence (a whole
 * number of blocks).  Rank r: sa_shard_begin (local compression with the
 * global block ids, local moment scan, its moment state T_r), then the caller
 * all-gathers the states and reps, then sa_shard_end (exclusive prefix of the
 * earlier states, their contribution to the shard's queries, the residual
 * over the reps of every earlier block).  Needs the tensor-core kernels. */

/* Floats of one shard's moment state (the unit of the all-gather). */
int sa_shard_state_floats(int64_t bh, int d, int dv, int degree, int64_t* floats);

/* Bytes of workspace for both calls of a shard of n tokens whose residual reads
 * rep_rows reps per sequence (the reps of the blocks before the shard's last). */
int sa_shard_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree, int block_size,
                            int64_t rep_rows, size_t* bytes);

/* Local part.  dirs/coins/perms hold the draws of the shard's n_compress
 * blocks (global blocks c_off .. c_off+n_compress-1 of the sequence);
 * rep_k/rep_v/rep_w [bh, n_compress*m, *] receive the raw reps, rep_idx
 * (nullable) their global token indices; state_out receives T_r. */
int sa_shard_begin(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                   int degree, int block_size, float scale, int compressor, const float* dirs,
                   const float* coins, const int32_t* perms, int64_t n_compress, int64_t c_off,
                   float* state_out, float* rep_k, float* rep_v, float* rep_w, int32_t* rep_idx,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Global part, after the exchange.  states_before: the n_before states of the
 * earlier shards, contiguous in shard order; rep_k/rep_v/rep_w [bh, rep_rows,
 * *]: the reps of global blocks 0.. in order (for compressor none: every
 * earlier token, weight 1).  Same workspace as sa_shard_begin. */
int sa_shard_end(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                 int degree, int block_size, float scale, int compressor, float eps,
                 const float* states_before, int n_before, int64_t c_off, const float* rep_k,
                 const float* rep_v, const float* rep_w, int64_t rep_rows, float* out, void* workspace,
                 size_t workspace_bytes, void* stream);

/* Bytes of the library's built-in device scratch (per GPU). */
#define SA_STATIC_SCRATCH_BYTES (64u * 1024u * 1024u)

/* sa_fast_attention for callers that cannot allocate device memory.  It has
 * no counterpart in the reference; it exists for callers such as programs
 * whose device memory belongs entirely to another allocator, serving loops
 * that forbid cudaMalloc after start-up, or plain-C callers with no device
 * allocator.  Same arguments and result as sa_fast_attention, minus the
 * workspace: the scratch is a SA_STATIC_SCRATCH_BYTES array built into the
 * library, held by every GPU that loads it until the process exits.  Problems
 * whose sa_fast_attention_workspace_size exceeds it are rejected with
 * SA_ERR_INVALID_ARG.  The first call on each device loads the library's
 * device code there (make it before any stream capture); every call looks up
 * the array's address anew, so a device reset that moves it is harmless.  All
 * calls share the array: calls that overlap on the GPU race, so order them.
 * Allocates nothing. */
int sa_fast_attention_static_scratch(const float* q, const float* k, const float* v, int64_t bh,
                                     int64_t n, int d, int dv, int degree, int block_size,
                                     float scale, int compressor, const float* dirs,
                                     const float* coins, const int32_t* perms, float eps,
                                     float* out, int32_t* rep_idx, void* stream);

/* ---- the segment-mean variant (deterministic reps) -------------------------
 * Replaces triton_article_causal_attention (triton_article_attention.py:448-578)
 * and its kernel _article_direct_kernel (:266-370): the same low-degree
 * moments and exact current-block residual as sa_fast_attention, but each
 * completed block is represented by the means of its block_size/compress_stride
 * runs of compress_stride adjacent tokens, each of weight compress_stride, and
 * the exp of a score is taken of min(score, 80) (:331-333, :359).  degree 0, 1
 * or 2 (else SA_ERR_UNSUPPORTED); block_size % compress_stride != 0 is
 * SA_ERR_INVALID_ARG.  d <= 128 and dv <= 128.  key_dtype / value_dtype say
 * how the reference's reps were stored (the dtypes of its k and v, SA_REP_*):
 * the key and value means are rounded to them. */
#define SA_REP_FLOAT32 0
#define SA_REP_FLOAT16 1
#define SA_REP_BFLOAT16 2

/* Replaces build_segment_mean_coreset (triton_article_attention.py:190-245):
 * rep_k [bh, R, d], rep_v [bh, R, dv], R = (n-1)/block_size *
 * (block_size/compress_stride) (0 rows when n <= block_size). */
int sa_segment_mean_reps(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                         int block_size, int compress_stride, int key_dtype, int value_dtype,
                         float* rep_k, float* rep_v, void* stream);

/* Bytes of device workspace sa_article_segment_mean needs. */
int sa_article_segment_mean_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree,
                                           int block_size, int compress_stride, size_t* bytes);

/* The whole forward of the segment-mean variant for bh sequences. */
int sa_article_segment_mean(const float* q, const float* k, const float* v, int64_t bh, int64_t n,
                            int d, int dv, int degree, int block_size, int compress_stride,
                            float scale, int key_dtype, int value_dtype, float eps, float* out,
                            void* workspace,
                            size_t workspace_bytes, void* stream);

/* ---- exact causal softmax attention ----------------------------------------
 * Replaces triton_flash_causal_attention (triton_article_attention.py:580-637)
 * and its kernel _flash_causal_kernel (:372-435): out = softmax(scale q k^T,
 * causal) v with the running-maximum (online) softmax and
 * out = acc / max(l, 1e-20).  d <= 128, dv <= 256 (else SA_ERR_INVALID_ARG).
 * Tensor cores (3xTF32) for d <= 64 and dv <= 128 with a workspace of
 * sa_flash_causal_attention_workspace_size bytes (256-byte aligned); CUDA
 * cores otherwise (workspace size 0, may be NULL). */
int sa_flash_causal_attention_workspace_size(int64_t bh, int64_t n, int d, int dv, size_t* bytes);
int sa_flash_causal_attention(const float* q, const float* k, const float* v, int64_t bh, int64_t n,
                              int d, int dv, float scale, float* out, void* workspace,
                              size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* STREAMING_ATTENTION_H_ */
