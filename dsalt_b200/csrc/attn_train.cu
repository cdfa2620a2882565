// Training-time sparse attention with differentiable selectors, forward
// (reference: dsalt/kernels/dsalt_triton_train.py, _train_fwd_kernel :74-217).
//
// For query i of a sequence of length L (one landmark set per sequence) the keys are
//   the band j with 0 ≤ d = i − j ≤ w̃(i) (w̃ continuous), logit q·k·scale + b(d) with the
//     soft window edge b = 0 in the core d ≤ w̃ − win_edge and log σ((w̃ − d)/τ) outside it;
//   the landmarks p of the row's set with 0 ≤ p < L, p ≤ i and p < i − w̃, logit
//     q·k·scale + logw(slot) (the soft landmark weight, computed by the caller).
// Softmax statistics in fp32; rows with mass ≤ 1e-9 are zero; the log-sum-exp (natural
// log) is written for the backward. P is kept in fp32 for the P·V sum (the reference rounds
// it to the input dtype first, which moves its output by at most that rounding).
// CUDA cores: one warp per (query, head), lanes split the head dimension; q, k, v in any of
// bf16 / fp16 / fp32.
#include "common.cuh"

namespace dsalt {

template <int DPL>  // head_dim / 32 elements per lane
__global__ void __launch_bounds__(256) train_fwd_kernel(
    const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v, int dtype, int64_t T, int H,
    int Hkv, int64_t q_stride, int64_t kv_stride, const float* __restrict__ w_cont, const int32_t* __restrict__ lmk,
    const float* __restrict__ logw, int k_lmk, const int32_t* __restrict__ cu, int n_seqs, float scale, float tau,
    float win_edge, void* __restrict__ out, int out_dtype, float* __restrict__ lse) {
  constexpr int D = DPL * 32;
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= T * H) return;
  const int64_t t = item / H;
  const int h = (int)(item % H);
  const int hk = h / (H / Hkv);
  int lo_s = 0, hi_s = n_seqs;
  while (hi_s - lo_s > 1) {
    const int mid = (lo_s + hi_s) >> 1;
    if (cu[mid] <= t) lo_s = mid;
    else hi_s = mid;
  }
  const int s = lo_s;
  const int64_t start = cu[s];
  const int L = cu[s + 1] - cu[s];
  const int i = (int)(t - start);
  const float wc = w_cont[t];
  float qv[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) qv[d] = load_elem(q, t * q_stride + (int64_t)h * D + lane + 32 * d, dtype);
  float m = -INFINITY, l = 0.0f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) acc[d] = 0.0f;
  auto visit = [&](int64_t row, float bias) {
    float part = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; ++d)
      part = fmaf(qv[d], load_elem(k, row * kv_stride + (int64_t)hk * D + lane + 32 * d, dtype), part);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const float lg = part * scale + bias;
    const float mn = fmaxf(m, lg);
    const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
    const float p = expf(lg - mn);
    l = l * corr + p;
#pragma unroll
    for (int d = 0; d < DPL; ++d)
      acc[d] = acc[d] * corr + p * load_elem(v, row * kv_stride + (int64_t)hk * D + lane + 32 * d, dtype);
    m = mn;
  };
  // the band: d = i - j in [0, w̃], i.e. j from i - floor(w̃) (every d is an exact float)
  const int jlo = wc >= 0.0f ? max(0, i - (int)floorf(wc)) : i + 1;
  for (int j = jlo; j <= i; ++j) {
    const float d = (float)(i - j);
    if (!(d <= wc)) continue;
    float bias = 0.0f;
    if (!(d <= wc - win_edge)) {
      const float z = (wc - d) / tau;
      bias = -logf(1.0f + expf(-z));  // log σ(z)
    }
    visit(start + j, bias);
  }
  const int32_t* P = lmk + ((int64_t)h * n_seqs + s) * k_lmk;
  const float* W = logw + ((int64_t)h * n_seqs + s) * k_lmk;
  const float lim = (float)i - wc;
  for (int c = 0; c < k_lmk; ++c) {
    const int p = P[c];
    if (p >= 0 && p < L && p <= i && (float)p < lim) visit(start + p, W[c]);
  }
  const bool ok = l > 1e-9f;
  const float inv = ok ? 1.0f / l : 0.0f;
#pragma unroll
  for (int d = 0; d < DPL; ++d) {
    const float o = ok ? acc[d] * inv : 0.0f;
    const int64_t idx = t * (int64_t)H * D + (int64_t)h * D + lane + 32 * d;
    if (out_dtype == DSALT_F32) reinterpret_cast<float*>(out)[idx] = o;
    else if (out_dtype == DSALT_BF16) reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(o);
    else reinterpret_cast<__half*>(out)[idx] = __float2half_rn(o);
  }
  if (lse && lane == 0) lse[t * H + h] = ok ? m + logf(l) : -INFINITY;
}

int launch_train_fwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int D,
                     int64_t q_stride, int64_t kv_stride, const float* w_cont, const int32_t* lmk, const float* logw,
                     int k_lmk, const int32_t* cu, int n_seqs, float tau, float win_edge, void* out, int out_dtype,
                     float* lse, cudaStream_t stream) {
  const int64_t items = T * H;
  const unsigned blocks = (unsigned)((items + 7) / 8);
  const float scale = (float)(1.0 / sqrt((double)D));
  switch (D) {
#define DSALT_TRAIN_CASE(DD)                                                                                        \
  case DD:                                                                                                          \
    train_fwd_kernel<DD / 32><<<blocks, 256, 0, stream>>>(q, k, v, dtype, T, H, Hkv, q_stride, kv_stride, w_cont,  \
                                                          lmk, logw, k_lmk, cu, n_seqs, scale, tau, win_edge, out, \
                                                          out_dtype, lse);                                          \
    break;
    DSALT_TRAIN_CASE(64)
    DSALT_TRAIN_CASE(128)
#undef DSALT_TRAIN_CASE
    default:
      return fail(DSALT_ERR_UNSUPPORTED, "training attention: head_dim %d not in {64, 128}", D);
  }
  return check_cuda(cudaGetLastError(), "training attention launch");
}

}  // namespace dsalt
