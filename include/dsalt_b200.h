/*
 * dsalt_b200: B200 (sm_100a) kernels for the DSALT sparse-attention forward.
 *
 * C ABI: plain pointers, sizes and a CUDA stream (passed as void*). All pointers are
 * device pointers unless stated otherwise; nothing here allocates device memory —
 * callers pass output buffers and a workspace sized by the *_workspace_bytes queries.
 * Every entry point returns DSALT_OK (0) or an error code and leaves a message for
 * dsalt_last_error(). Kernels are launched asynchronously on `stream`.
 *
 * Each function cites the reference (LeonardoCofone/dsalt) interface it replaces.
 */
#ifndef DSALT_B200_H
#define DSALT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define DSALT_F32 0
#define DSALT_BF16 1
#define DSALT_F16 2

/* status codes */
#define DSALT_OK 0
#define DSALT_ERR_INVALID 1       /* bad shape, dtype, stride, alignment or pointer */
#define DSALT_ERR_UNSUPPORTED 2   /* valid request outside what the kernels implement */
#define DSALT_ERR_CUDA 3          /* a CUDA runtime/driver call failed */
#define DSALT_ERR_WORKSPACE 4     /* workspace smaller than the *_workspace_bytes query */
#define DSALT_ERR_DEVICE 5        /* a kernel gave up a bounded wait (see dsalt_device_status) */

/* selection modes */
#define DSALT_SELECT_GLOBAL 0       /* one landmark set per (head, sequence) */
#define DSALT_SELECT_BLOCK_CAUSAL 1 /* one landmark set per (head, block of queries) */

/* norm rounding of the selection signals */
#define DSALT_NORM_F32 0   /* fp32 norms (CUDA autocast runs `norm` in fp32) */
#define DSALT_NORM_INPUT 1 /* norms rounded to the input dtype (bf16/fp16 `norm` outside autocast) */

const char* dsalt_last_error(void);
int dsalt_version(void);

/* Reads (and clears, when `clear` != 0) the device status word that kernels set when a
 * bounded wait gives up. Synchronises `stream`. 0 = no error. The device addresses of this
 * word and of the no-allocation scratch array are looked up once per device and kept for
 * the life of the process: do not use the library across a cudaDeviceReset. */
int dsalt_device_status(int* status_out, int clear, void* stream);
/* Queues a copy of the device status word into host memory `status_host` (page-locked, so
 * that the copy is asynchronous) on `stream` and returns without synchronising; the value
 * is there once the stream has passed this point (e.g. an event recorded after the call
 * has completed). Lets a caller check every step without stalling the stream. */
int dsalt_device_status_async(int* status_host, void* stream);

/*
 * Window widths and selection signals, one pass over x and v.
 * Replaces DSALTAttention._window_sizes(x, floor=True)
 *   (dsalt/modules/dsalt_attention.py:270-284, win_gate at :223)
 * and the norms of hybrid_scores_per_head / _token_signals
 *   (dsalt/kernels/landmark_tokens_ker.py:47,52; results/causal_landmark_check.py:68-79).
 *
 * x        [T, d_model] (row stride x_stride elements), dtype x_dtype
 * gate_w   [d_model], gate_b [1]: win_gate weight/bias in gate_dtype; the logit is
 *          computed in gate_dtype (x converted to gate_dtype first, as autocast does)
 * v        [T, n_kv*head_dim] value projection x·W_Vᵀ (row stride v_stride), dtype v_dtype
 * w_out    [T] int32 widths, xnorm_out [T] fp32, vnorm_out [T, n_kv] fp32
 * logit_out [T] fp32 (nullable): the rounded win_gate logit
 * logit_in  [T] in gate_dtype (nullable): the win_gate logit as the caller computed it
 *          (e.g. torch's `win_gate(x)` under autocast, the reference's own op); the widths
 *          are then computed from it (gate_w / gate_b are still passed but no longer
 *          affect any output). Without it the logit is the float64-accumulated dot
 *          product rounded once to gate_dtype, which a library GEMV that accumulates in
 *          fp32 can round to the neighbouring value.
 */
int dsalt_token_signals(const void* x, int x_dtype, int64_t T, int d_model, int64_t x_stride,
                        const void* gate_w, const void* gate_b, int gate_dtype, int n_min, int n_max,
                        const void* v, int v_dtype, int64_t v_stride, int n_kv, int head_dim, int norm_mode,
                        int32_t* w_out, float* xnorm_out, float* vnorm_out, float* logit_out,
                        const void* logit_in, void* stream);

/*
 * Landmark selection.
 * DSALT_SELECT_GLOBAL replaces _compute_landmark_indices
 *   (dsalt/kernels/selectors.py:75-134) with hybrid_scores_per_head
 *   (dsalt/kernels/landmark_tokens_ker.py:19-61): statistics over all T packed tokens,
 *   top-k per (head, sequence) among tokens with seq_off >= w.
 * DSALT_SELECT_BLOCK_CAUSAL replaces the per-block _select of
 *   results/causal_landmark_check.py:82-113 (driven at :176-186): block b of each
 *   sequence draws from positions [0, b*block) with that prefix's statistics.
 *
 * xnorm [T], vnorm [T, n_kv], w [T] (int32), alpha [n_heads] (sigmoid(alpha_w), fp32)
 * cu_seqlens [n_seqs+1] int32 (device), max_seqlen: host upper bound of sequence lengths
 * lmk_out [n_heads, n_sets, k] int32: positions within the sequence, ascending, -1 padded.
 *   n_sets = n_seqs (global) or sum over sequences of ceil(L/block) (block-causal,
 *   numbered sequence after sequence).
 * zx_out [T], zv_out [T, n_kv] (nullable, global mode only): the standardized signals.
 * Tie rule: equal scores are taken lowest position first.
 */
size_t dsalt_select_workspace_bytes(int mode, int64_t T, int n_seqs, int max_seqlen, int n_heads, int n_kv,
                                    int k, int block);
int dsalt_select_landmarks(int mode, const float* xnorm, const float* vnorm, const int32_t* w,
                           const float* alpha, const int32_t* cu_seqlens, int n_seqs, int64_t T, int max_seqlen,
                           int n_heads, int n_kv, int k, int block, int32_t* lmk_out, float* zx_out,
                           float* zv_out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Sparse attention forward over A(i) = W(i) ∪ L(i).
 * Replaces dsalt_triton_attention / DSALTAttentionFunction.forward
 *   (dsalt/kernels/dsalt_triton_attn.py:259-311, :337-349) and _dsalt_fwd_kernel (:27-169),
 *   including _build_landmark_kv (dsalt/kernels/selectors.py:137-159) and
 *   _build_seq_block_map (selectors.py:37-67), which are done inside.
 *
 * q [T, n_heads, head_dim], k/v [T, n_kv, head_dim] (token strides q_stride, kv_stride in
 *   elements; heads contiguous), dtype DSALT_BF16 / DSALT_F16 (tensor cores; head_dim 64 or
 *   128) or DSALT_F32 (fp32 CUDA cores; head_dim 32, 64, 128 or 256). GQA: head h uses kv
 *   head h / (n_heads / n_kv).
 * w [T] int32 window widths (clamped to >= 1 inside).
 * lmk [n_heads, n_sets, k_lmk] int32 positions within the sequence, -1 = none. For the
 *   bf16/fp16 path every set must list its positions ascending with the -1 entries last
 *   (the format dsalt_select_landmarks writes); the fp32 path accepts any order.
 *   lmk_block = 0: one set per sequence; > 0: one set per lmk_block queries.
 * lmk_bias [n_heads, n_sets, k_lmk] fp32 (nullable): added to landmark logits.
 * out [T, n_heads, head_dim] in out_dtype; lse [T, n_heads] fp32 (nullable).
 */
size_t dsalt_attention_workspace_bytes(int64_t T, int n_seqs, int n_heads, int k_lmk, int lmk_block);
int dsalt_attention_fwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads, int n_kv,
                        int head_dim, int64_t q_stride, int64_t kv_stride, const int32_t* w, const int32_t* lmk,
                        const float* lmk_bias, int k_lmk, int lmk_block, const int32_t* cu_seqlens, int n_seqs,
                        int max_seqlen, void* out, int out_dtype, float* lse, void* workspace,
                        size_t workspace_bytes, void* stream);

/*
 * Backward of the sparse attention forward above.
 * Replaces dsalt_triton_backward / DSALTAttentionFunction.backward
 *   (dsalt/kernels/dsalt_triton_bwd.py:219-323, dsalt_triton_attn.py:313-327), i.e.
 *   _dsalt_bwd_preprocess (:18-49) and _dsalt_bwd_kernel (:52-216).
 *
 * q, k, v, w, lmk, lmk_bias, lmk_block, cu_seqlens as for the forward (lmk in the forward's
 *   ascending format); n_sets = lmk's second extent. out [T, n_heads, head_dim] is the
 *   forward's output in out_dtype and dout [T, n_heads, head_dim] its gradient in
 *   dout_dtype (both contiguous); lse [T, n_heads] fp32 the forward's log-sum-exp (natural
 *   log, -inf for rows with no key). Outputs (fp32, overwritten): dq [T, n_heads, head_dim],
 *   dk / dv [T, n_kv, head_dim] (summed over the heads of each kv group), d_bias
 *   [n_heads, n_sets, k_lmk] (nullable). head_dim 64 or 128; lmk_block a multiple of 64.
 *   S = q·kᵀ and dO·vᵀ on the tensor cores (mma.sync, fp32 accumulate) when q/k/v and dout
 *   share a 16-bit dtype, on CUDA cores otherwise; the gradient products on CUDA cores in
 *   fp32; dk, dv and d_bias accumulate with atomic adds, so their last bits vary from run to
 *   run.
 */
size_t dsalt_attention_bwd_workspace_bytes(int64_t T, int n_seqs);
int dsalt_attention_bwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads, int n_kv,
                        int head_dim, int64_t q_stride, int64_t kv_stride, const void* out, int out_dtype,
                        const void* dout, int dout_dtype, const float* lse, const int32_t* w, const int32_t* lmk,
                        const float* lmk_bias, int k_lmk, int lmk_block, int n_sets, const int32_t* cu_seqlens,
                        int n_seqs, float* dq, float* dk, float* dv, float* d_bias, void* workspace,
                        size_t workspace_bytes, void* stream);

/*
 * Training-time sparse attention with differentiable selectors (forward and backward).
 * Replaces dsalt_triton_train_attention / DSALTTrainAttentionFunction
 *   (dsalt/kernels/dsalt_triton_train.py:583-782): _train_fwd_kernel (:74-217),
 *   _train_bwd_preprocess, _train_bwd_kernel and _train_bwd_dkdv_kernel (:220-490).
 *
 * q [T, n_heads, head_dim], k/v [T, n_kv, head_dim] as for the forward above (any of bf16,
 *   fp16, fp32; head_dim 64 or 128). The forward runs bf16 / fp16 inputs with
 *   0 <= win_edge <= 4 on the tensor cores (P rounded to the input dtype for P·V, as the
 *   reference's tl.dot; 16-byte aligned rows), everything else on CUDA cores in fp32; the
 *   backward as dsalt_attention_bwd. w_cont [T] fp32: the
 *   continuous window widths w̃. lmk [n_heads, n_seqs, k_lmk] int32 positions (one set per
 *   sequence, any slot order, -1 = none) and lmk_logw [n_heads, n_seqs, k_lmk] fp32 their
 *   log-weights log σ(s/τ_lmk). Query i attends to the band 0 <= i - j <= w̃(i) with the soft
 *   edge log σ((w̃ - (i - j)) / tau_win) outside the core i - j <= w̃ - win_edge, and to the
 *   landmarks p < i - w̃, p <= i with logit + log-weight. Forward: out [T, n_heads, head_dim]
 *   in out_dtype, lse [T, n_heads] (natural log; nullable); workspace from
 *   dsalt_train_attention_fwd_workspace_bytes. Backward (workspace from
 *   dsalt_attention_bwd_workspace_bytes): from out, dout and lse, writes dq, dk, dv
 *   (fp32, as dsalt_attention_bwd), d_logw [n_heads, n_seqs, k_lmk] and d_w [T] (the
 *   gradient of w̃, summed over heads); dk, dv, d_logw and d_w accumulate with atomic adds.
 */
size_t dsalt_train_attention_fwd_workspace_bytes(int64_t T, int n_heads, int n_seqs, int k_lmk);
int dsalt_train_attention_fwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads,
                              int n_kv, int head_dim, int64_t q_stride, int64_t kv_stride, const float* w_cont,
                              const int32_t* lmk, const float* lmk_logw, int k_lmk, const int32_t* cu_seqlens,
                              int n_seqs, float tau_win, float win_edge, void* out, int out_dtype, float* lse,
                              void* workspace, size_t workspace_bytes, void* stream);
int dsalt_train_attention_bwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads, int n_kv,
                              int head_dim, int64_t q_stride, int64_t kv_stride, const void* out, int out_dtype,
                              const void* dout, int dout_dtype, const float* lse, const float* w_cont,
                              const int32_t* lmk, const float* lmk_logw, int k_lmk, const int32_t* cu_seqlens,
                              int n_seqs, float tau_win, float win_edge, float* dq, float* dk, float* dv,
                              float* d_logw, float* d_w, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Sequence-sharded forms (no counterpart in the reference, which runs on one GPU): one
 * rank's share of a single sequence of seq_len positions split across ranks.
 *
 * dsalt_select_block_range: the block-causal sets [set_lo, set_hi) of one sequence whose
 *   signals (xnorm, vnorm, w: every position of the sequence, e.g. all-gathered from the
 *   ranks) are given; only the prefix [0, set_hi * block) is read. Same sets as
 *   dsalt_select_landmarks(DSALT_SELECT_BLOCK_CAUSAL) for those blocks. lmk_out
 *   [n_heads, set_hi - set_lo, k].
 * dsalt_attention_fwd_sharded: queries = positions [q_pos0, q_pos0 + q_rows) (q, out,
 *   lse rows 0..q_rows-1); k/v (this GPU's memory: they are read by TMA tile loads; only
 *   lmk_k_src / lmk_v_src may point to other GPUs) rows = positions [kv_pos0, kv_pos0 + kv_rows), which must
 *   hold every window key of the local queries (kv_pos0 <= q_pos0 - max width + 1; keys
 *   below kv_pos0 read as zero); w [seq_len] widths by position; lmk [n_heads,
 *   n_local_sets, k_lmk] positions within the sequence (one set per lmk_block local
 *   queries, or one set when lmk_block = 0), ascending, -1 last. Landmark rows are read
 *   from lmk_k_src[r] / lmk_v_src[r] (device arrays of pointers; rank r holds positions
 *   [r * rows_per_src, (r+1) * rows_per_src) with the kv token stride), which may be other
 *   GPUs' memory mapped by dsalt_ipc_open (plain NVLink loads), gathered once per call into
 *   the workspace as 128-row tiles. q_pos0 and q_rows are multiples of 128 (and of
 *   lmk_block); bf16 / fp16 inputs; head_dim 64 or 128.
 * dsalt_ipc_export / dsalt_ipc_open / dsalt_ipc_close: CUDA IPC handles (64 bytes) of a
 *   device pointer inside an allocation, for the peer tables above.
 */
size_t dsalt_select_block_range_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block,
                                                int set_hi);
int dsalt_select_block_range(const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                             int64_t seq_len, int n_heads, int n_kv, int k, int block, int set_lo, int set_hi,
                             int32_t* lmk_out, void* workspace, size_t workspace_bytes, void* stream);
size_t dsalt_attention_sharded_workspace_bytes(int64_t q_rows, int n_heads, int k_lmk, int lmk_block, int head_dim);
/* dsalt_select_shard: the block-causal sets of rank `rank`'s blocks, with the selection's
 *   per-chunk work spread over the ranks (no counterpart in the reference; same sets as
 *   dsalt_select_landmarks(DSALT_SELECT_BLOCK_CAUSAL) on the whole sequence, i.e. as
 *   results/causal_landmark_check.py:82-113 per block). The sequence of seq_len positions
 *   splits into n_ranks contiguous shards of seq_len / n_ranks positions, a whole number
 *   of blocks each; rank r owns blocks (= chunks = sets) [r * cpr, (r + 1) * cpr).
 *   xnorm [seq_len], vnorm [seq_len, n_kv], w [seq_len]: whole-sequence arrays of which
 *   phases 1-3 read only the own shard; phase 4 reads earlier positions as well when some
 *   alpha lies outside [0, 1] (no dominance pruning then), so gather the signals first in
 *   that case. workspace (dsalt_select_shard_workspace_bytes, the same size on every
 *   rank); peer_workspaces: device array of the n_ranks ranks' workspace pointers (own
 *   entry included; peers mapped by dsalt_ipc_open). Call phases 1, 2, 3, 4 in order with
 *   a cross-GPU barrier (dsalt_peer_barrier) between consecutive phases: 1 chunk sums of
 *   the own blocks; 2 reads the others' sums, prefix statistics, dominance grids of the
 *   own blocks; 3 reads the earlier ranks' grid totals, survivors of the own blocks; 4
 *   reads the earlier ranks' survivors and writes lmk_out [n_heads, cpr, k]. A rank's
 *   workspace must not be reused before every rank has finished phase 4. n_kv <= 32. */
size_t dsalt_select_shard_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block);
int dsalt_select_shard(int phase, const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                       int64_t seq_len, int n_heads, int n_kv, int k, int block, int rank, int n_ranks,
                       void* workspace, size_t workspace_bytes, const void* const* peer_workspaces, int32_t* lmk_out,
                       void* stream);
int dsalt_attention_fwd_sharded(const void* q, const void* k, const void* v, int dtype, int64_t q_rows, int n_heads,
                                int n_kv, int head_dim, int64_t q_stride, int64_t kv_stride, int64_t q_pos0,
                                int64_t kv_pos0, int64_t kv_rows, int64_t seq_len, const int32_t* w,
                                const int32_t* lmk, const float* lmk_bias, int k_lmk, int lmk_block,
                                const void* const* lmk_k_src, const void* const* lmk_v_src, int64_t rows_per_src,
                                void* out, int out_dtype, float* lse, void* workspace, size_t workspace_bytes,
                                void* stream);
/* dsalt_peer_barrier: rank `rank` of n_ranks GPUs (one process each) stores `epoch` in its
 *   own flag (an int in its memory) and waits until every rank's flag (peer_flags: device
 *   array of the ranks' flag pointers, peers mapped by dsalt_ipc_open) has reached it;
 *   epochs must increase from call to call. epoch <= 0 takes the epoch from a device-side
 *   counter in own_flag[1] (incremented by the call; own_flag then points to two ints), so
 *   that a CUDA graph holding the call advances it on every replay. Memory written on this GPU before the call is
 *   visible to the peers' work queued after theirs. A wait longer than 2 s gives up and
 *   sets the device status word (no hang).
 * dsalt_peer_allgather: dst[j * bytes_per_rank ...] <- src[j][0 .. bytes_per_rank) for
 *   every rank j != rank (src: device array of the ranks' pointers; 16-byte multiples).
 * dsalt_peer_copy: bytes from src (this or a peer GPU's memory) to dst, on the stream. */
int dsalt_peer_barrier(int* own_flag, const int* const* peer_flags, int n_ranks, int rank, int epoch, void* stream);
int dsalt_peer_allgather(void* dst, const void* const* src, int n_ranks, int rank, int64_t bytes_per_rank,
                         void* stream);
int dsalt_peer_copy(void* dst, const void* src, int64_t bytes, void* stream);
int dsalt_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
int dsalt_ipc_open(const void* handle, int64_t offset, void** ptr_out);
int dsalt_ipc_close(void* ptr, int64_t offset);

/*
 * dsalt_attention_fwd without a workspace: no counterpart in the reference.
 * For callers that cannot allocate device memory: a host binding that holds only the
 * caller's q/k/v/out pointers and no device allocator of its own (a cgo, JNI or ctypes
 * binding with no framework behind it), or a serving loop whose memory pool is fully
 * reserved for its caches and may not grow between requests. The scratch that
 * dsalt_attention_fwd takes from `workspace` (two sequence tables of n_seqs+1 int32 and a
 * 32-byte plan per 128-query tile) comes here from a static device array of this library
 * (417 KB), one per device:
 *   - at most DSALT_NOALLOC_MAX_SEQS sequences and DSALT_NOALLOC_MAX_TOKENS tokens;
 *     larger requests fail with DSALT_ERR_UNSUPPORTED before any work is queued;
 *   - nothing in it needs to start at zero: each call rewrites the tables it reads;
 *   - every call on a device shares it, so calls that may overlap on one device (other
 *     streams, other host threads) race on it; the caller serialises them;
 *   - the first call on each device looks the array's address up (cudaGetSymbolAddress);
 *     make that first call before any stream capture begins.
 * Nothing is allocated (no cudaMalloc, no allocating library). Arguments, results and
 * error codes are otherwise those of dsalt_attention_fwd (the same kernels run).
 */
#define DSALT_NOALLOC_MAX_SEQS 4096
#define DSALT_NOALLOC_MAX_TOKENS 1048576
int dsalt_attention_fwd_noalloc(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads,
                                int n_kv, int head_dim, int64_t q_stride, int64_t kv_stride, const int32_t* w,
                                const int32_t* lmk, const float* lmk_bias, int k_lmk, int lmk_block,
                                const int32_t* cu_seqlens, int n_seqs, int max_seqlen, void* out, int out_dtype,
                                float* lse, void* stream);

/*
 * The whole inference core of DSALTAttention._packed after the projections and RoPE
 * (dsalt/modules/dsalt_attention.py:610-625): widths, signals, selection, attention.
 * Scratch for the intermediates comes from `workspace`
 * (dsalt_core_workspace_bytes); w_out / lmk_out (nullable) receive copies of the widths
 * and landmark sets; logit_in (nullable) is dsalt_token_signals' caller-computed logit.
 */
size_t dsalt_core_workspace_bytes(int mode, int64_t T, int n_seqs, int max_seqlen, int n_heads, int n_kv,
                                  int head_dim, int k, int block);
int dsalt_core_forward(int mode, const void* x, int x_dtype, int d_model, int64_t x_stride, const void* gate_w,
                       const void* gate_b, int gate_dtype, const void* logit_in, int n_min, int n_max,
                       const float* alpha, int norm_mode, const void* q, const void* k, const void* v, int qkv_dtype, int n_heads,
                       int n_kv, int head_dim, int64_t q_stride, int64_t kv_stride, int k_lmk, int block,
                       const int32_t* cu_seqlens, int n_seqs, int64_t T, int max_seqlen, void* out, int out_dtype,
                       int32_t* w_out, int32_t* lmk_out, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSALT_B200_H */
