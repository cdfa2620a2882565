// fp32 sparse attention forward on CUDA cores (fp32 inputs).
//
// Same semantics as the tensor-core kernel and as the reference's inference kernel
// (dsalt/kernels/dsalt_triton_attn.py:27-169): for query i of a sequence of length L the
// keys are the window j ∈ [max(0, i−w+1), i] and the landmarks p with 0 ≤ p < L, p ≤ i,
// p < i−w+1; softmax over their logits q·k·scale (+ bias on landmarks); rows whose softmax
// mass is ≤ 1e-9 are zero. Unlike the reference, which casts fp32 inputs to fp16
// (dsalt_triton_attn.py:266), everything stays in fp32 (expf, fp32 accumulation).
// One warp per (query, head); lanes split the head dimension.
#include "common.cuh"

namespace dsalt {

template <int DPL>  // head_dim / 32 elements per lane
__global__ void __launch_bounds__(256) attn_fwd_f32_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, int64_t T, int H, int Hkv,
    int64_t q_stride, int64_t kv_stride, const int32_t* __restrict__ w, const int32_t* __restrict__ lmk,
    const float* __restrict__ lmk_bias, int k_lmk, int lmk_block, const int32_t* __restrict__ cu, int n_seqs,
    const int32_t* __restrict__ set_base, float scale, void* __restrict__ out, int out_dtype, float* __restrict__ lse) {
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
  int wi = w[t];
  wi = wi < 1 ? 1 : wi;
  const int lo_raw = i - wi + 1;
  const int lo = lo_raw < 0 ? 0 : lo_raw;
  float qv[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) qv[d] = q[t * q_stride + (int64_t)h * D + lane + 32 * d];
  float m = -INFINITY, l = 0.0f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) acc[d] = 0.0f;
  auto visit = [&](int64_t row, float bias) {
    float part = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) part = fmaf(qv[d], k[row * kv_stride + (int64_t)hk * D + lane + 32 * d], part);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const float lg = part * scale + bias;
    const float mn = fmaxf(m, lg);
    const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
    const float p = expf(lg - mn);
    l = l * corr + p;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[d] = acc[d] * corr + p * v[row * kv_stride + (int64_t)hk * D + lane + 32 * d];
    m = mn;
  };
  for (int j = lo; j <= i; ++j) visit(start + j, 0.0f);
  const int set = lmk_block > 0 ? set_base[s] + i / lmk_block : s;
  const int n_sets = lmk_block > 0 ? set_base[n_seqs] : n_seqs;
  const int32_t* P = lmk + ((int64_t)h * n_sets + set) * k_lmk;
  for (int c = 0; c < k_lmk; ++c) {
    const int p = P[c];
    if (p >= 0 && p < L && p <= i && p < lo_raw)
      visit(start + p, lmk_bias ? lmk_bias[((int64_t)h * n_sets + set) * k_lmk + c] : 0.0f);
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

int launch_attn_f32(const float* q, const float* k, const float* v, int64_t T, int H, int Hkv, int D,
                    int64_t q_stride, int64_t kv_stride, const int32_t* w, const int32_t* lmk, const float* lmk_bias,
                    int k_lmk, int lmk_block, const int32_t* cu, int n_seqs, const int32_t* set_base, float scale,
                    void* out, int out_dtype, float* lse, cudaStream_t stream) {
  const int64_t items = T * H;
  const unsigned blocks = (unsigned)((items + 7) / 8);
  switch (D) {
#define DSALT_F32_CASE(DD)                                                                                     \
  case DD:                                                                                                     \
    attn_fwd_f32_kernel<DD / 32><<<blocks, 256, 0, stream>>>(q, k, v, T, H, Hkv, q_stride, kv_stride, w, lmk, \
                                                             lmk_bias, k_lmk, lmk_block, cu, n_seqs, set_base,  \
                                                             scale, out, out_dtype, lse);                      \
    break;
    DSALT_F32_CASE(32)
    DSALT_F32_CASE(64)
    DSALT_F32_CASE(128)
    DSALT_F32_CASE(256)
#undef DSALT_F32_CASE
    default:
      return fail(DSALT_ERR_UNSUPPORTED, "attention (fp32): head_dim %d not in {32, 64, 128, 256}", D);
  }
  return check_cuda(cudaGetLastError(), "attention fp32 launch");
}

}  // namespace dsalt
