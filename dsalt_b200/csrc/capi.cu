// C-ABI entry points (include/dsalt_b200.h): argument checks, workspace carving, and
// the fused core pipeline. No device memory is allocated here.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include <cuda.h>

#include "common.cuh"

namespace dsalt {

int launch_token_signals(const void* x, int x_dtype, int64_t T, int d_model, int64_t x_stride, const void* gate_w,
                         const void* gate_b, int gate_dtype, int n_min, int n_max, const void* v, int v_dtype,
                         int64_t v_stride, int n_kv, int head_dim, int norm_mode, int32_t* w_out, float* xnorm_out,
                         float* vnorm_out, float* logit_out, const void* logit_in, cudaStream_t stream);
size_t select_workspace_bytes(int mode, int64_t T, int n_seqs, int max_seqlen, int n_heads, int n_kv, int k,
                              int block);
int launch_select(int mode, const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                  const int32_t* cu, int n_seqs, int64_t T, int max_seqlen, int n_heads, int n_kv, int k, int block,
                  int32_t* lmk_out, float* zx_out, float* zv_out, void* workspace, size_t ws_bytes,
                  cudaStream_t stream, int set_lo = 0, int set_hi = -1);
size_t select_range_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block, int set_hi);
int launch_select_range(const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha, int64_t seq_len,
                        int n_heads, int n_kv, int k, int block, int set_lo, int set_hi, int32_t* lmk_out,
                        void* workspace, size_t ws_bytes, cudaStream_t stream);
int select_set_up_attributes();
size_t select_shard_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block);
int launch_select_shard(int phase, const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                        int64_t seq_len, int n_heads, int n_kv, int k, int block, int rank, int n_ranks, void* workspace,
                        size_t ws_bytes, const void* const* ws_peers, int32_t* lmk_out, cudaStream_t stream);
int launch_attn_f32(const float* q, const float* k, const float* v, int64_t T, int H, int Hkv, int D,
                    int64_t q_stride, int64_t kv_stride, const int32_t* w, const int32_t* lmk, const float* lmk_bias,
                    int k_lmk, int lmk_block, const int32_t* cu, int n_seqs, const int32_t* set_base, float scale,
                    void* out, int out_dtype, float* lse, cudaStream_t stream);
int launch_attn_tc(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int HD,
                   int64_t q_stride, int64_t kv_stride, const int32_t* w, const int32_t* lmk, const float* lmk_bias,
                   int k_lmk, int lmk_block, const int32_t* cu, int n_seqs, int32_t* set_base, int32_t* tile_base,
                   int4* plan, int64_t max_tiles, void* out, int out_dtype, float* lse, int* err,
                   cudaStream_t stream, const ShardArgs* shard = nullptr, const float* w_soft = nullptr,
                   float soft_edge = 0.f, float soft_tau = 1.f);
int launch_train_prep(const float* w_cont, int64_t T, const int32_t* lmk, const float* logw, int64_t n_sets,
                      int k_lmk, int32_t* w_int, int32_t* lmk_sorted, float* logw_sorted, cudaStream_t stream);
int launch_chunk_table(const int32_t* cu, int n_seqs, int C, int32_t* base, cudaStream_t stream);
size_t attention_bwd_workspace_bytes(int n_seqs);
int launch_attn_bwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int HD,
                    int64_t q_stride, int64_t kv_stride, const void* out, int out_dtype, const void* dout,
                    int dout_dtype, const float* lse, const int32_t* w, const int32_t* lmk, const float* lmk_bias,
                    int k_lmk, int lmk_block, const int32_t* cu, int n_seqs, float* dq, float* dk, float* dv,
                    float* d_bias, void* workspace, size_t ws_bytes, cudaStream_t stream,
                    const float* w_cont = nullptr, float tau = 1.f, float win_edge = 0.f, float* d_w = nullptr);
int launch_train_fwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int D,
                     int64_t q_stride, int64_t kv_stride, const float* w_cont, const int32_t* lmk, const float* logw,
                     int k_lmk, const int32_t* cu, int n_seqs, float tau, float win_edge, void* out, int out_dtype,
                     float* lse, cudaStream_t stream);
int launch_peer_barrier(int* own_flag, const int* const* flags, int n_ranks, int rank, int epoch, int* err,
                        cudaStream_t stream);
int launch_peer_allgather(void* dst, const void* const* src, int n_ranks, int rank, int64_t bytes_per_rank,
                          cudaStream_t stream);
int launch_peer_copy(void* dst, const void* src, int64_t bytes, cudaStream_t stream);

// ---------------------------------------------------------------- errors
static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return DSALT_OK;
  return fail(DSALT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// device status word (one per device, lives in this library's module)
__device__ int g_device_status;

int* device_status_ptr() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    ptrs[dev] = reinterpret_cast<int*>(p);
  }
  return ptrs[dev];
}

// Scratch of dsalt_attention_fwd_noalloc, laid out as dsalt_attention_fwd carves its
// workspace: the landmark-set and query-tile tables (n_seqs + 1 int32 each) and the
// per-tile plan (32 bytes per 128-query tile), sized for DSALT_NOALLOC_MAX_SEQS sequences
// and DSALT_NOALLOC_MAX_TOKENS tokens.
constexpr size_t NOALLOC_TABLE_BYTES = ((DSALT_NOALLOC_MAX_SEQS + 1) * sizeof(int32_t) + 255) & ~(size_t)255;
constexpr size_t NOALLOC_PLAN_BYTES = (size_t)(DSALT_NOALLOC_MAX_TOKENS / 128 + DSALT_NOALLOC_MAX_SEQS) * 32;
static __device__ __align__(256) int32_t
    g_noalloc_scratch[(2 * NOALLOC_TABLE_BYTES + NOALLOC_PLAN_BYTES) / sizeof(int32_t)];

static void* noalloc_scratch_ptr() {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

static bool valid_dtype(int dt) { return dt == DSALT_F32 || dt == DSALT_BF16 || dt == DSALT_F16; }
static inline size_t a256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace dsalt

using namespace dsalt;

extern "C" {

const char* dsalt_last_error(void) { return g_err; }

int dsalt_version(void) { return 1; }

int dsalt_device_status(int* status_out, int clear, void* stream) {
  if (!status_out) return fail(DSALT_ERR_INVALID, "device_status: null output");
  int* p = device_status_ptr();
  if (!p) return fail(DSALT_ERR_CUDA, "device_status: symbol address unavailable");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemcpyAsync(status_out, p, sizeof(int), cudaMemcpyDeviceToHost, s), "device_status read");
  if (rc) return rc;
  if (clear) {
    rc = check_cuda(cudaMemsetAsync(p, 0, sizeof(int), s), "device_status clear");
    if (rc) return rc;
  }
  return check_cuda(cudaStreamSynchronize(s), "device_status sync");
}

int dsalt_device_status_async(int* status_host, void* stream) {
  if (!status_host) return fail(DSALT_ERR_INVALID, "device_status_async: null output");
  int* p = device_status_ptr();
  if (!p) return fail(DSALT_ERR_CUDA, "device_status_async: symbol address unavailable");
  return check_cuda(cudaMemcpyAsync(status_host, p, sizeof(int), cudaMemcpyDeviceToHost,
                                    reinterpret_cast<cudaStream_t>(stream)),
                    "device_status_async copy");
}

int dsalt_token_signals(const void* x, int x_dtype, int64_t T, int d_model, int64_t x_stride, const void* gate_w,
                        const void* gate_b, int gate_dtype, int n_min, int n_max, const void* v, int v_dtype,
                        int64_t v_stride, int n_kv, int head_dim, int norm_mode, int32_t* w_out, float* xnorm_out,
                        float* vnorm_out, float* logit_out, const void* logit_in, void* stream) {
  return launch_token_signals(x, x_dtype, T, d_model, x_stride, gate_w, gate_b, gate_dtype, n_min, n_max, v, v_dtype,
                              v_stride, n_kv, head_dim, norm_mode, w_out, xnorm_out, vnorm_out, logit_out, logit_in,
                              reinterpret_cast<cudaStream_t>(stream));
}

size_t dsalt_select_workspace_bytes(int mode, int64_t T, int n_seqs, int max_seqlen, int n_heads, int n_kv, int k,
                                    int block) {
  return select_workspace_bytes(mode, T, n_seqs, max_seqlen, n_heads, n_kv, k, block);
}

int dsalt_select_landmarks(int mode, const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                           const int32_t* cu_seqlens, int n_seqs, int64_t T, int max_seqlen, int n_heads, int n_kv,
                           int k, int block, int32_t* lmk_out, float* zx_out, float* zv_out, void* workspace,
                           size_t workspace_bytes, void* stream) {
  return launch_select(mode, xnorm, vnorm, w, alpha, cu_seqlens, n_seqs, T, max_seqlen, n_heads, n_kv, k, block,
                       lmk_out, zx_out, zv_out, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

// landmark-set table | query-tile table | per-tile plan (tensor-core path)
static inline int64_t attention_max_tiles(int64_t T, int n_seqs) { return T / 128 + n_seqs; }

size_t dsalt_attention_workspace_bytes(int64_t T, int n_seqs, int n_heads, int k_lmk, int lmk_block) {
  (void)n_heads;
  (void)k_lmk;
  (void)lmk_block;
  if (n_seqs < 1 || T < 0) return 0;
  return 2 * a256(sizeof(int32_t) * (size_t)(n_seqs + 1)) + a256(32 * (size_t)attention_max_tiles(T, n_seqs));
}

int dsalt_attention_fwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads, int n_kv,
                        int head_dim, int64_t q_stride, int64_t kv_stride, const int32_t* w, const int32_t* lmk,
                        const float* lmk_bias, int k_lmk, int lmk_block, const int32_t* cu_seqlens, int n_seqs,
                        int max_seqlen, void* out, int out_dtype, float* lse, void* workspace, size_t workspace_bytes,
                        void* stream) {
  (void)max_seqlen;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (T < 0 || n_heads < 1 || n_kv < 1 || n_heads % n_kv || head_dim < 1 || n_seqs < 1 || k_lmk < 0 ||
      lmk_block < 0)
    return fail(DSALT_ERR_INVALID, "attention: bad sizes");
  if (!valid_dtype(dtype) || !valid_dtype(out_dtype)) return fail(DSALT_ERR_INVALID, "attention: dtype");
  if (q_stride < (int64_t)n_heads * head_dim || kv_stride < (int64_t)n_kv * head_dim)
    return fail(DSALT_ERR_INVALID, "attention: token stride smaller than heads x head_dim");
  if (T == 0) return DSALT_OK;
  if (!q || !k || !v || !w || !cu_seqlens || !out || (k_lmk > 0 && !lmk) || !workspace)
    return fail(DSALT_ERR_INVALID, "attention: null pointer");
  if (T > 0x7fffff00LL) return fail(DSALT_ERR_UNSUPPORTED, "attention: T too large");
  const size_t need = dsalt_attention_workspace_bytes(T, n_seqs, n_heads, k_lmk, lmk_block);
  if (workspace_bytes < need) return fail(DSALT_ERR_WORKSPACE, "attention: workspace %zu < %zu", workspace_bytes, need);
  int32_t* set_base = reinterpret_cast<int32_t*>(workspace);
  const size_t table_bytes = a256(sizeof(int32_t) * (size_t)(n_seqs + 1));
  int32_t* tile_base = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(workspace) + table_bytes);
  int4* plan = reinterpret_cast<int4*>(reinterpret_cast<char*>(workspace) + 2 * table_bytes);
  if (dtype == DSALT_F32) {
    int rc = DSALT_OK;
    if (lmk_block > 0 && (rc = launch_chunk_table(cu_seqlens, n_seqs, lmk_block, set_base, s))) return rc;
    return launch_attn_f32(reinterpret_cast<const float*>(q), reinterpret_cast<const float*>(k),
                           reinterpret_cast<const float*>(v), T, n_heads, n_kv, head_dim, q_stride, kv_stride, w, lmk,
                           lmk_bias, k_lmk, lmk_block, cu_seqlens, n_seqs, set_base,
                           (float)(1.0 / sqrt((double)head_dim)), out, out_dtype, lse, s);
  }
  return launch_attn_tc(q, k, v, dtype, T, n_heads, n_kv, head_dim, q_stride, kv_stride, w, lmk, lmk_bias, k_lmk,
                        lmk_block, cu_seqlens, n_seqs, set_base, tile_base, plan, attention_max_tiles(T, n_seqs), out,
                        out_dtype, lse, device_status_ptr(), s);
}

// attention workspace | integer widths [T] | sorted sets [H, S, k] | their log-weights
size_t dsalt_train_attention_fwd_workspace_bytes(int64_t T, int n_heads, int n_seqs, int k_lmk) {
  if (n_seqs < 1 || T < 0 || n_heads < 1 || k_lmk < 0) return 0;
  const size_t sets = (size_t)n_heads * n_seqs * k_lmk;
  return dsalt_attention_workspace_bytes(T, n_seqs, n_heads, k_lmk, 0) + a256(4 * (size_t)T) + 2 * a256(4 * sets);
}

int dsalt_train_attention_fwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads,
                              int n_kv, int head_dim, int64_t q_stride, int64_t kv_stride, const float* w_cont,
                              const int32_t* lmk, const float* lmk_logw, int k_lmk, const int32_t* cu_seqlens,
                              int n_seqs, float tau_win, float win_edge, void* out, int out_dtype, float* lse,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (T < 0 || n_heads < 1 || n_kv < 1 || n_heads % n_kv || n_seqs < 1 || k_lmk < 0 || !(tau_win > 0.f))
    return fail(DSALT_ERR_INVALID, "training attention: bad sizes");
  if (!valid_dtype(dtype) || !valid_dtype(out_dtype)) return fail(DSALT_ERR_INVALID, "training attention: dtype");
  if (q_stride < (int64_t)n_heads * head_dim || kv_stride < (int64_t)n_kv * head_dim)
    return fail(DSALT_ERR_INVALID, "training attention: token stride smaller than heads x head_dim");
  if (T == 0) return DSALT_OK;
  if (!q || !k || !v || !w_cont || !cu_seqlens || !out || (k_lmk > 0 && (!lmk || !lmk_logw)) || !workspace)
    return fail(DSALT_ERR_INVALID, "training attention: null pointer");
  if (T > 0x7fffff00LL) return fail(DSALT_ERR_UNSUPPORTED, "training attention: T too large");
  const size_t need = dsalt_train_attention_fwd_workspace_bytes(T, n_heads, n_seqs, k_lmk);
  if (workspace_bytes < need)
    return fail(DSALT_ERR_WORKSPACE, "training attention: workspace %zu < %zu", workspace_bytes, need);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // bf16 / fp16 with edge widths up to 4 (the reference's default is 4): the tensor-core
  // kernel's soft-edge mode; otherwise the CUDA-core kernel
  const bool tc = dtype != DSALT_F32 && (head_dim == 64 || head_dim == 128) && win_edge >= 0.f && win_edge <= 4.f &&
                  k_lmk <= 256 && !(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) &&
                  (q_stride * 2) % 16 == 0 && (kv_stride * 2) % 16 == 0;
  if (!tc)
    return launch_train_fwd(q, k, v, dtype, T, n_heads, n_kv, head_dim, q_stride, kv_stride, w_cont, lmk, lmk_logw,
                            k_lmk, cu_seqlens, n_seqs, tau_win, win_edge, out, out_dtype, lse, s);
  char* ws = reinterpret_cast<char*>(workspace);
  const size_t table_bytes = a256(sizeof(int32_t) * (size_t)(n_seqs + 1));
  int32_t* set_base = reinterpret_cast<int32_t*>(ws);
  int32_t* tile_base = reinterpret_cast<int32_t*>(ws + table_bytes);
  int4* plan = reinterpret_cast<int4*>(ws + 2 * table_bytes);
  char* tail = ws + dsalt_attention_workspace_bytes(T, n_seqs, n_heads, k_lmk, 0);
  const size_t sets = (size_t)n_heads * n_seqs * k_lmk;
  int32_t* w_int = reinterpret_cast<int32_t*>(tail);
  int32_t* lmk_sorted = reinterpret_cast<int32_t*>(tail + a256(4 * (size_t)T));
  float* logw_sorted = reinterpret_cast<float*>(tail + a256(4 * (size_t)T) + a256(4 * sets));
  int rc = launch_train_prep(w_cont, T, lmk, lmk_logw, (int64_t)n_heads * n_seqs, k_lmk, w_int, lmk_sorted,
                             logw_sorted, s);
  if (rc) return rc;
  return launch_attn_tc(q, k, v, dtype, T, n_heads, n_kv, head_dim, q_stride, kv_stride, w_int,
                        k_lmk > 0 ? lmk_sorted : nullptr, k_lmk > 0 ? logw_sorted : nullptr, k_lmk, 0, cu_seqlens,
                        n_seqs, set_base, tile_base, plan, attention_max_tiles(T, n_seqs), out, out_dtype, lse,
                        device_status_ptr(), s, nullptr, w_cont, win_edge, tau_win);
}

int dsalt_train_attention_bwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads, int n_kv,
                              int head_dim, int64_t q_stride, int64_t kv_stride, const void* out, int out_dtype,
                              const void* dout, int dout_dtype, const float* lse, const float* w_cont,
                              const int32_t* lmk, const float* lmk_logw, int k_lmk, const int32_t* cu_seqlens,
                              int n_seqs, float tau_win, float win_edge, float* dq, float* dk, float* dv,
                              float* d_logw, float* d_w, void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (T < 0 || n_heads < 1 || n_kv < 1 || n_heads % n_kv || head_dim < 1 || n_seqs < 1 || k_lmk < 0 ||
      !(tau_win > 0.f))
    return fail(DSALT_ERR_INVALID, "training attention backward: bad sizes");
  if (!valid_dtype(dtype) || !valid_dtype(out_dtype) || !valid_dtype(dout_dtype))
    return fail(DSALT_ERR_INVALID, "training attention backward: dtype");
  if (q_stride < (int64_t)n_heads * head_dim || kv_stride < (int64_t)n_kv * head_dim)
    return fail(DSALT_ERR_INVALID, "training attention backward: token stride smaller than heads x head_dim");
  if (T == 0) return DSALT_OK;
  if (!q || !k || !v || !out || !dout || !lse || !w_cont || !cu_seqlens || !dq || !dk || !dv || !d_w ||
      (k_lmk > 0 && (!lmk || !lmk_logw || !d_logw)) || !workspace)
    return fail(DSALT_ERR_INVALID, "training attention backward: null pointer");
  if (T > 0x7fffff00LL) return fail(DSALT_ERR_UNSUPPORTED, "training attention backward: T too large");
  int rc;
  if ((rc = check_cuda(cudaMemsetAsync(dk, 0, sizeof(float) * (size_t)T * n_kv * head_dim, s), "clear dk")) ||
      (rc = check_cuda(cudaMemsetAsync(dv, 0, sizeof(float) * (size_t)T * n_kv * head_dim, s), "clear dv")) ||
      (rc = check_cuda(cudaMemsetAsync(d_w, 0, sizeof(float) * (size_t)T, s), "clear d_w")))
    return rc;
  if (k_lmk > 0 && (rc = check_cuda(cudaMemsetAsync(d_logw, 0, sizeof(float) * (size_t)n_heads * n_seqs * k_lmk, s),
                                    "clear d_logw")))
    return rc;
  return launch_attn_bwd(q, k, v, dtype, T, n_heads, n_kv, head_dim, q_stride, kv_stride, out, out_dtype, dout,
                         dout_dtype, lse, nullptr, lmk, lmk_logw, k_lmk, 0, cu_seqlens, n_seqs, dq, dk, dv, d_logw,
                         workspace, workspace_bytes, s, w_cont, tau_win, win_edge, d_w);
}

size_t dsalt_attention_bwd_workspace_bytes(int64_t T, int n_seqs) {
  if (n_seqs < 1 || T < 0) return 0;
  return attention_bwd_workspace_bytes(n_seqs);
}

int dsalt_attention_bwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads, int n_kv,
                        int head_dim, int64_t q_stride, int64_t kv_stride, const void* out, int out_dtype,
                        const void* dout, int dout_dtype, const float* lse, const int32_t* w, const int32_t* lmk,
                        const float* lmk_bias, int k_lmk, int lmk_block, int n_sets, const int32_t* cu_seqlens,
                        int n_seqs, float* dq, float* dk, float* dv, float* d_bias, void* workspace,
                        size_t workspace_bytes, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (T < 0 || n_heads < 1 || n_kv < 1 || n_heads % n_kv || head_dim < 1 || n_seqs < 1 || k_lmk < 0 ||
      lmk_block < 0 || n_sets < 0)
    return fail(DSALT_ERR_INVALID, "attention backward: bad sizes");
  if (!valid_dtype(dtype) || !valid_dtype(out_dtype) || !valid_dtype(dout_dtype))
    return fail(DSALT_ERR_INVALID, "attention backward: dtype");
  if (q_stride < (int64_t)n_heads * head_dim || kv_stride < (int64_t)n_kv * head_dim)
    return fail(DSALT_ERR_INVALID, "attention backward: token stride smaller than heads x head_dim");
  if (T == 0) return DSALT_OK;
  if (!q || !k || !v || !out || !dout || !lse || !w || !cu_seqlens || !dq || !dk || !dv || (k_lmk > 0 && !lmk) ||
      !workspace)
    return fail(DSALT_ERR_INVALID, "attention backward: null pointer");
  if (T > 0x7fffff00LL) return fail(DSALT_ERR_UNSUPPORTED, "attention backward: T too large");
  // dk, dv and d_bias are sums over query tiles (atomic adds): cleared here, in stream order
  int rc;
  if ((rc = check_cuda(cudaMemsetAsync(dk, 0, sizeof(float) * (size_t)T * n_kv * head_dim, s), "clear dk")) ||
      (rc = check_cuda(cudaMemsetAsync(dv, 0, sizeof(float) * (size_t)T * n_kv * head_dim, s), "clear dv")))
    return rc;
  if (d_bias != nullptr && k_lmk > 0 &&
      (rc = check_cuda(cudaMemsetAsync(d_bias, 0, sizeof(float) * (size_t)n_heads * n_sets * k_lmk, s),
                       "clear d_bias")))
    return rc;
  return launch_attn_bwd(q, k, v, dtype, T, n_heads, n_kv, head_dim, q_stride, kv_stride, out, out_dtype, dout,
                         dout_dtype, lse, w, lmk, lmk_bias, k_lmk, lmk_block, cu_seqlens, n_seqs, dq, dk, dv, d_bias,
                         workspace, workspace_bytes, s);
}

size_t dsalt_select_block_range_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block,
                                                int set_hi) {
  return select_range_workspace_bytes(seq_len, n_heads, n_kv, k, block, set_hi);
}

int dsalt_select_block_range(const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                             int64_t seq_len, int n_heads, int n_kv, int k, int block, int set_lo, int set_hi,
                             int32_t* lmk_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (n_heads < 1 || n_kv < 1 || n_heads % n_kv || k < 0) return fail(DSALT_ERR_INVALID, "select range: bad sizes");
  if (!xnorm || !vnorm || !w || !alpha || !lmk_out) return fail(DSALT_ERR_INVALID, "select range: null pointer");
  if (seq_len > 0x7fffff00LL) return fail(DSALT_ERR_UNSUPPORTED, "select range: sequence too long");
  return launch_select_range(xnorm, vnorm, w, alpha, seq_len, n_heads, n_kv, k, block, set_lo, set_hi, lmk_out,
                             workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t dsalt_select_shard_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block) {
  return select_shard_workspace_bytes(seq_len, n_heads, n_kv, k, block);
}

int dsalt_select_shard(int phase, const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                       int64_t seq_len, int n_heads, int n_kv, int k, int block, int rank, int n_ranks,
                       void* workspace, size_t workspace_bytes, const void* const* peer_workspaces, int32_t* lmk_out,
                       void* stream) {
  return launch_select_shard(phase, xnorm, vnorm, w, alpha, seq_len, n_heads, n_kv, k, block, rank, n_ranks, workspace,
                             workspace_bytes, peer_workspaces, lmk_out, reinterpret_cast<cudaStream_t>(stream));
}

// plan | gathered landmark K tiles | V tiles
static size_t sharded_tile_bytes(int64_t q_rows, int n_heads, int k_lmk, int lmk_block, int head_dim) {
  const int64_t n_sets = lmk_block ? (q_rows + lmk_block - 1) / lmk_block : 1;
  const int64_t nlt = (k_lmk + 127) / 128;
  return a256((size_t)(n_sets * n_heads * nlt * 128) * head_dim * 2);
}

size_t dsalt_attention_sharded_workspace_bytes(int64_t q_rows, int n_heads, int k_lmk, int lmk_block, int head_dim) {
  if (q_rows < 0 || n_heads < 1 || k_lmk < 0 || lmk_block < 0 || head_dim < 1) return 0;
  return 256 + a256(32 * (size_t)(q_rows / 128 + 1)) + 2 * sharded_tile_bytes(q_rows, n_heads, k_lmk, lmk_block, head_dim);
}

int dsalt_attention_fwd_sharded(const void* q, const void* k, const void* v, int dtype, int64_t q_rows, int n_heads,
                                int n_kv, int head_dim, int64_t q_stride, int64_t kv_stride, int64_t q_pos0,
                                int64_t kv_pos0, int64_t kv_rows, int64_t seq_len, const int32_t* w,
                                const int32_t* lmk, const float* lmk_bias, int k_lmk, int lmk_block,
                                const void* const* lmk_k_src, const void* const* lmk_v_src, int64_t rows_per_src,
                                void* out, int out_dtype, float* lse, void* workspace, size_t workspace_bytes,
                                void* stream) {
  if (q_rows < 0 || n_heads < 1 || n_kv < 1 || n_heads % n_kv || head_dim < 1 || k_lmk < 0 || lmk_block < 0 ||
      kv_rows < 0 || rows_per_src < 1)
    return fail(DSALT_ERR_INVALID, "attention (sharded): bad sizes");
  if (dtype != DSALT_BF16 && dtype != DSALT_F16)
    return fail(DSALT_ERR_UNSUPPORTED, "attention (sharded): bf16 / fp16 inputs only");
  if (!valid_dtype(out_dtype)) return fail(DSALT_ERR_INVALID, "attention (sharded): dtype");
  if (q_rows == 0) return DSALT_OK;
  if (q_pos0 % 128 || q_rows % 128 || (lmk_block && q_pos0 % lmk_block))
    return fail(DSALT_ERR_UNSUPPORTED, "attention (sharded): shard must start and end on 128-query (and set) bounds");
  if (q_pos0 < 0 || kv_pos0 > q_pos0 || kv_pos0 + kv_rows < q_pos0 + q_rows || q_pos0 + q_rows > seq_len ||
      seq_len > 0x7fffff00LL)
    return fail(DSALT_ERR_INVALID, "attention (sharded): k/v rows must cover the shard's own positions");
  if (q_stride < (int64_t)n_heads * head_dim || kv_stride < (int64_t)n_kv * head_dim)
    return fail(DSALT_ERR_INVALID, "attention (sharded): token stride smaller than heads x head_dim");
  if (!q || !k || !v || !w || !out || (k_lmk > 0 && (!lmk || !lmk_k_src || !lmk_v_src)) || !workspace)
    return fail(DSALT_ERR_INVALID, "attention (sharded): null pointer");
  const size_t need = dsalt_attention_sharded_workspace_bytes(q_rows, n_heads, k_lmk, lmk_block, head_dim);
  if (workspace_bytes < need)
    return fail(DSALT_ERR_WORKSPACE, "attention (sharded): workspace %zu < %zu", workspace_bytes, need);
  char* ws = reinterpret_cast<char*>(workspace);
  const size_t plan_bytes = a256(32 * (size_t)(q_rows / 128 + 1));
  const size_t tile_bytes = sharded_tile_bytes(q_rows, n_heads, k_lmk, lmk_block, head_dim);
  ShardArgs sa{q_pos0, q_rows, kv_pos0, kv_rows, seq_len, rows_per_src, lmk_k_src, lmk_v_src,
               ws + 256 + plan_bytes, ws + 256 + plan_bytes + tile_bytes};
  int4* plan = reinterpret_cast<int4*>(ws + 256);
  int32_t* tables = reinterpret_cast<int32_t*>(workspace);
  return launch_attn_tc(q, k, v, dtype, q_rows, n_heads, n_kv, head_dim, q_stride, kv_stride, w, lmk, lmk_bias, k_lmk,
                        lmk_block, nullptr, 1, tables, tables + 32, plan, q_rows / 128, out, out_dtype, lse,
                        device_status_ptr(), reinterpret_cast<cudaStream_t>(stream), &sa);
}

int dsalt_peer_barrier(int* own_flag, const int* const* peer_flags, int n_ranks, int rank, int epoch, void* stream) {
  return launch_peer_barrier(own_flag, peer_flags, n_ranks, rank, epoch, device_status_ptr(),
                             reinterpret_cast<cudaStream_t>(stream));
}

int dsalt_peer_allgather(void* dst, const void* const* src, int n_ranks, int rank, int64_t bytes_per_rank,
                         void* stream) {
  return launch_peer_allgather(dst, src, n_ranks, rank, bytes_per_rank, reinterpret_cast<cudaStream_t>(stream));
}

int dsalt_peer_copy(void* dst, const void* src, int64_t bytes, void* stream) {
  return launch_peer_copy(dst, src, bytes, reinterpret_cast<cudaStream_t>(stream));
}

// device memory shared between the processes of one node (CUDA IPC, plain peer mappings)
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int dsalt_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return fail(DSALT_ERR_INVALID, "ipc export: null pointer");
  static GetAddressRangeFn range_fn = nullptr;
  if (!range_fn) {
    void* fp = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fp, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(DSALT_ERR_CUDA, "ipc export: cuMemGetAddressRange unavailable");
    range_fn = reinterpret_cast<GetAddressRangeFn>(fp);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS)
    return fail(DSALT_ERR_CUDA, "ipc export: pointer is not device memory");
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "ipc export");
  if (rc) return rc;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)((CUdeviceptr)ptr - base);
  return DSALT_OK;
}

int dsalt_ipc_open(const void* handle, int64_t offset, void** ptr_out) {
  if (!handle || !ptr_out) return fail(DSALT_ERR_INVALID, "ipc open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  int rc = check_cuda(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "ipc open");
  if (rc) return rc;
  *ptr_out = reinterpret_cast<char*>(base) + offset;
  return DSALT_OK;
}

int dsalt_ipc_close(void* ptr, int64_t offset) {
  if (!ptr) return fail(DSALT_ERR_INVALID, "ipc close: null pointer");
  return check_cuda(cudaIpcCloseMemHandle(reinterpret_cast<char*>(ptr) - offset), "ipc close");
}

// Callers without a device allocator (bindings that hold only the caller's pointers,
// serving loops whose pool may not grow) get the attention forward with its scratch in
// g_noalloc_scratch. Overlapping calls on one device share that array and race.
int dsalt_attention_fwd_noalloc(const void* q, const void* k, const void* v, int dtype, int64_t T, int n_heads,
                                int n_kv, int head_dim, int64_t q_stride, int64_t kv_stride, const int32_t* w,
                                const int32_t* lmk, const float* lmk_bias, int k_lmk, int lmk_block,
                                const int32_t* cu_seqlens, int n_seqs, int max_seqlen, void* out, int out_dtype,
                                float* lse, void* stream) {
  if (n_seqs > DSALT_NOALLOC_MAX_SEQS || T > DSALT_NOALLOC_MAX_TOKENS)
    return fail(DSALT_ERR_UNSUPPORTED,
                "attention (no-alloc): n_seqs %d / T %lld above the static scratch limit (%d sequences, %d tokens); "
                "use dsalt_attention_fwd with a workspace",
                n_seqs, (long long)T, DSALT_NOALLOC_MAX_SEQS, DSALT_NOALLOC_MAX_TOKENS);
  const size_t need = dsalt_attention_workspace_bytes(T, n_seqs, n_heads, k_lmk, lmk_block);
  if (need > sizeof(g_noalloc_scratch))
    return fail(DSALT_ERR_UNSUPPORTED, "attention (no-alloc): scratch %zu above %zu", need,
                sizeof(g_noalloc_scratch));
  void* scratch = noalloc_scratch_ptr();
  if (!scratch) return fail(DSALT_ERR_CUDA, "attention (no-alloc): scratch address unavailable");
  return dsalt_attention_fwd(q, k, v, dtype, T, n_heads, n_kv, head_dim, q_stride, kv_stride, w, lmk, lmk_bias, k_lmk,
                             lmk_block, cu_seqlens, n_seqs, max_seqlen, out, out_dtype, lse, scratch,
                             sizeof(g_noalloc_scratch), stream);
}

size_t dsalt_core_workspace_bytes(int mode, int64_t T, int n_seqs, int max_seqlen, int n_heads, int n_kv,
                                  int head_dim, int k, int block) {
  (void)head_dim;
  if (T < 0 || n_seqs < 1) return 0;
  const int64_t n_sets_max = mode == DSALT_SELECT_GLOBAL ? n_seqs : (block > 0 ? T / block + n_seqs : 0);
  size_t off = 0;
  off += a256(sizeof(int32_t) * (size_t)T);                           // widths
  off += a256(sizeof(float) * (size_t)T);                             // x norms
  off += a256(sizeof(float) * (size_t)T * n_kv);                      // value norms
  off += a256(sizeof(int32_t) * (size_t)n_heads * n_sets_max * k);    // landmark sets
  off += a256(dsalt_attention_workspace_bytes(T, n_seqs, n_heads, k, block));
  off += a256(select_workspace_bytes(mode, T, n_seqs, max_seqlen, n_heads, n_kv, k, block));
  return off;
}

int dsalt_core_forward(int mode, const void* x, int x_dtype, int d_model, int64_t x_stride, const void* gate_w,
                       const void* gate_b, int gate_dtype, const void* logit_in, int n_min, int n_max,
                       const float* alpha, int norm_mode, const void* q, const void* k, const void* v, int qkv_dtype, int n_heads, int n_kv,
                       int head_dim, int64_t q_stride, int64_t kv_stride, int k_lmk, int block,
                       const int32_t* cu_seqlens, int n_seqs, int64_t T, int max_seqlen, void* out, int out_dtype,
                       int32_t* w_out, int32_t* lmk_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (mode != DSALT_SELECT_GLOBAL && mode != DSALT_SELECT_BLOCK_CAUSAL) return fail(DSALT_ERR_INVALID, "core: mode");
  if (T < 0 || n_seqs < 1) return fail(DSALT_ERR_INVALID, "core: bad sizes");
  if (T == 0) return DSALT_OK;
  const size_t need = dsalt_core_workspace_bytes(mode, T, n_seqs, max_seqlen, n_heads, n_kv, head_dim, k_lmk, block);
  if (!workspace || workspace_bytes < need) return fail(DSALT_ERR_WORKSPACE, "core: workspace %zu < %zu", workspace_bytes, need);
  const int64_t n_sets_max = mode == DSALT_SELECT_GLOBAL ? n_seqs : T / block + n_seqs;
  char* ws = reinterpret_cast<char*>(workspace);
  size_t off = 0;
  int32_t* w = w_out ? w_out : reinterpret_cast<int32_t*>(ws + off);
  off += a256(sizeof(int32_t) * (size_t)T);
  float* xn = reinterpret_cast<float*>(ws + off);
  off += a256(sizeof(float) * (size_t)T);
  float* vn = reinterpret_cast<float*>(ws + off);
  off += a256(sizeof(float) * (size_t)T * n_kv);
  int32_t* lmk = lmk_out ? lmk_out : reinterpret_cast<int32_t*>(ws + off);
  off += a256(sizeof(int32_t) * (size_t)n_heads * n_sets_max * k_lmk);
  void* aws = ws + off;
  const size_t aws_bytes = a256(dsalt_attention_workspace_bytes(T, n_seqs, n_heads, k_lmk, block));
  off += aws_bytes;
  void* sws = ws + off;
  const size_t sws_bytes = workspace_bytes - off;
  int rc = dsalt_token_signals(x, x_dtype, T, d_model, x_stride, gate_w, gate_b, gate_dtype, n_min, n_max, v,
                               qkv_dtype, kv_stride, n_kv, head_dim, norm_mode, w, xn, vn, nullptr, logit_in, stream);
  if (rc) return rc;
  rc = dsalt_select_landmarks(mode, xn, vn, w, alpha, cu_seqlens, n_seqs, T, max_seqlen, n_heads, n_kv, k_lmk, block,
                              lmk, nullptr, nullptr, sws, sws_bytes, stream);
  if (rc) return rc;
  return dsalt_attention_fwd(q, k, v, qkv_dtype, T, n_heads, n_kv, head_dim, q_stride, kv_stride, w, lmk, nullptr,
                             k_lmk, mode == DSALT_SELECT_GLOBAL ? 0 : block, cu_seqlens, n_seqs, max_seqlen, out,
                             out_dtype, nullptr, aws, aws_bytes, stream);
}

}  // extern "C"
