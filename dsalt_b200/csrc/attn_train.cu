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
//
// CUDA cores, one warp per (query, head). Keys go 32 at a time, one per lane: each lane takes
// the full dot product of its key row with q (q in shared memory, read as broadcasts; the row
// in 16-byte loads), the warp reduces the chunk's max and sum once, and the (p, key) pairs are
// staged in shared memory for the P·V sum, where each lane owns head_dim/32 consecutive output
// dimensions. Warps are ordered head-major, so the 8 warps of a CTA are neighbouring queries
// of one head and read mostly the same band keys (L1 hits). q, k, v in bf16 / fp16 / fp32.
// This is the path for fp32 inputs and for edge widths above 4; bf16 / fp16 inputs otherwise
// run on the tensor-core attention kernel with its soft-edge mode (attn_tc.cu), fed by the
// prep kernels below.
#include "common.cuh"

namespace dsalt {
namespace train {

constexpr int WARPS = 8;

template <int DT>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  if constexpr (DT == DSALT_BF16) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));  // bf16 is the top half of f32
  } else {
    __half2 h;
    memcpy(&h, &u, 4);
    return __half22float2(h);
  }
}

// q · (the D elements at kr), q from shared memory.
template <int D, int DT>
__device__ __forceinline__ float dot_row(const void* kr, const float* qw, bool vec) {
  float s0 = 0.0f, s1 = 0.0f;
  if (vec) {
    if constexpr (DT == DSALT_F32) {
      const float4* p = reinterpret_cast<const float4*>(kr);
#pragma unroll
      for (int c = 0; c < D / 4; ++c) {
        const float4 u = __ldg(p + c);
        const float4 qa = *reinterpret_cast<const float4*>(qw + 4 * c);
        s0 = fmaf(qa.x, u.x, s0);
        s1 = fmaf(qa.y, u.y, s1);
        s0 = fmaf(qa.z, u.z, s0);
        s1 = fmaf(qa.w, u.w, s1);
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(kr);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 u = __ldg(p + c);
        const float4 qa = *reinterpret_cast<const float4*>(qw + 8 * c);
        const float4 qb = *reinterpret_cast<const float4*>(qw + 8 * c + 4);
        const float2 a = unpack2<DT>(u.x), b = unpack2<DT>(u.y), e = unpack2<DT>(u.z), f = unpack2<DT>(u.w);
        s0 = fmaf(qa.x, a.x, s0);
        s1 = fmaf(qa.y, a.y, s1);
        s0 = fmaf(qa.z, b.x, s0);
        s1 = fmaf(qa.w, b.y, s1);
        s0 = fmaf(qb.x, e.x, s0);
        s1 = fmaf(qb.y, e.y, s1);
        s0 = fmaf(qb.z, f.x, s0);
        s1 = fmaf(qb.w, f.y, s1);
      }
    }
  } else {
#pragma unroll 8
    for (int c = 0; c < D; ++c) s0 = fmaf(qw[c], load_elem(kr, c, DT), s0);
  }
  return s0 + s1;
}

// acc[0..DPL) += p · (the lane's DPL consecutive elements at vr + lane·DPL).
template <int DPL, int DT>
__device__ __forceinline__ void add_row(float (&acc)[DPL], float p, const void* vr, int lane, bool vec) {
  if (vec) {
    if constexpr (DT == DSALT_F32) {
      const float* r = reinterpret_cast<const float*>(vr) + lane * DPL;
      if constexpr (DPL == 2) {
        const float2 u = __ldg(reinterpret_cast<const float2*>(r));
        acc[0] = fmaf(p, u.x, acc[0]);
        acc[1] = fmaf(p, u.y, acc[1]);
      } else {
        const float4 u = __ldg(reinterpret_cast<const float4*>(r));
        acc[0] = fmaf(p, u.x, acc[0]);
        acc[1] = fmaf(p, u.y, acc[1]);
        acc[2] = fmaf(p, u.z, acc[2]);
        acc[3] = fmaf(p, u.w, acc[3]);
      }
    } else {
      const uint16_t* r = reinterpret_cast<const uint16_t*>(vr) + lane * DPL;
      if constexpr (DPL == 2) {
        const float2 a = unpack2<DT>(__ldg(reinterpret_cast<const uint32_t*>(r)));
        acc[0] = fmaf(p, a.x, acc[0]);
        acc[1] = fmaf(p, a.y, acc[1]);
      } else {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(r));
        const float2 a = unpack2<DT>(u.x), b = unpack2<DT>(u.y);
        acc[0] = fmaf(p, a.x, acc[0]);
        acc[1] = fmaf(p, a.y, acc[1]);
        acc[2] = fmaf(p, b.x, acc[2]);
        acc[3] = fmaf(p, b.y, acc[3]);
      }
    }
  } else {
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[d] = fmaf(p, load_elem(vr, lane * DPL + d, DT), acc[d]);
  }
}

template <int DPL, int DT>  // DPL = head_dim / 32 output dimensions per lane
__global__ void __launch_bounds__(WARPS * 32, 4) train_fwd_kernel(
    const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v, int64_t T, int H, int Hkv,
    int64_t q_stride, int64_t kv_stride, bool vec, const float* __restrict__ w_cont, const int32_t* __restrict__ lmk,
    const float* __restrict__ logw, int k_lmk, const int32_t* __restrict__ cu, int n_seqs, float scale, float tau,
    float win_edge, void* __restrict__ out, int out_dtype, float* __restrict__ lse) {
  constexpr int D = DPL * 32;
  constexpr int ES = DT == DSALT_F32 ? 4 : 2;
  __shared__ __align__(16) float qs[WARPS][D];
  __shared__ __align__(16) float ps[WARPS][32];
  __shared__ __align__(16) int js[WARPS][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t item = (int64_t)blockIdx.x * WARPS + warp;
  if (item >= T * H) return;  // whole warps only; nothing below synchronises the block
  const int h = (int)(item / T);
  const int64_t t = item - (int64_t)h * T;
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
  float* qw = qs[warp];
#pragma unroll
  for (int d = 0; d < DPL; ++d) qw[lane + 32 * d] = load_elem(q, t * q_stride + (int64_t)h * D + lane + 32 * d, DT);
  __syncwarp();
  const char* kb = static_cast<const char*>(k) + (int64_t)hk * D * ES;
  const char* vb = static_cast<const char*>(v) + (int64_t)hk * D * ES;
  const int64_t row_bytes = kv_stride * ES;
  float m = -INFINITY, l = 0.0f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) acc[d] = 0.0f;
  // one chunk: this lane's key j (sequence position) if valid, with its bias
  auto chunk = [&](bool valid, int j, float bias) {
    float sc = -INFINITY;
    if (valid) sc = dot_row<D, DT>(kb + (start + j) * row_bytes, qw, vec) * scale + bias;
    float cm = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    if (cm == -INFINITY) return;  // warp-uniform: nothing valid in this chunk
    const float mn = fmaxf(m, cm);
    const float corr = expf(m - mn);  // 0 while m is still -inf
    const float p = expf(sc - mn);    // 0 for invalid lanes
    float psum = p;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * corr + psum;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[d] *= corr;
    m = mn;
    ps[warp][lane] = p;
    js[warp][lane] = j;
    __syncwarp();
#pragma unroll 2
    for (int e = 0; e < 32; e += 4) {
      const float4 p4 = *reinterpret_cast<const float4*>(&ps[warp][e]);
      const int4 j4 = *reinterpret_cast<const int4*>(&js[warp][e]);
      // p is warp-uniform here, so are the branches; a zero p (invalid key) is skipped
      if (p4.x != 0.0f) add_row<DPL, DT>(acc, p4.x, vb + (start + j4.x) * row_bytes, lane, vec);
      if (p4.y != 0.0f) add_row<DPL, DT>(acc, p4.y, vb + (start + j4.y) * row_bytes, lane, vec);
      if (p4.z != 0.0f) add_row<DPL, DT>(acc, p4.z, vb + (start + j4.z) * row_bytes, lane, vec);
      if (p4.w != 0.0f) add_row<DPL, DT>(acc, p4.w, vb + (start + j4.w) * row_bytes, lane, vec);
    }
    __syncwarp();
  };
  // the band: d = i - j in [0, w̃], i.e. j from i - floor(w̃) (every d is an exact float)
  const int jlo = wc >= 0.0f ? max(0, i - (int)floorf(wc)) : i + 1;
  for (int j0 = jlo; j0 <= i; j0 += 32) {
    const int j = j0 + lane;
    const float d = (float)(i - j);
    const bool valid = j <= i && d <= wc;
    float bias = 0.0f;
    if (valid && !(d <= wc - win_edge)) {
      const float z = (wc - d) / tau;
      bias = -logf(1.0f + expf(-z));  // log σ(z)
    }
    chunk(valid, j, bias);
  }
  const int32_t* P = lmk + ((int64_t)h * n_seqs + s) * k_lmk;
  const float* W = logw + ((int64_t)h * n_seqs + s) * k_lmk;
  const float lim = (float)i - wc;
  for (int c0 = 0; c0 < k_lmk; c0 += 32) {
    const int c = c0 + lane;
    int p = -1;
    float bias = 0.0f;
    if (c < k_lmk) {
      p = P[c];
      bias = W[c];
    }
    const bool valid = p >= 0 && p < L && p <= i && (float)p < lim;
    chunk(valid, p, bias);
  }
  const bool ok = l > 1e-9f;
  const float inv = ok ? 1.0f / l : 0.0f;
  const int64_t base = t * (int64_t)H * D + (int64_t)h * D + lane * DPL;
#pragma unroll
  for (int d = 0; d < DPL; ++d) {
    const float o = ok ? acc[d] * inv : 0.0f;
    if (out_dtype == DSALT_F32) reinterpret_cast<float*>(out)[base + d] = o;
    else if (out_dtype == DSALT_BF16) reinterpret_cast<__nv_bfloat16*>(out)[base + d] = __float2bfloat16_rn(o);
    else reinterpret_cast<__half*>(out)[base + d] = __float2half_rn(o);
  }
  if (lse && lane == 0) lse[t * H + h] = ok ? m + logf(l) : -INFINITY;
}

// Inputs of the tensor-core path: integer widths floor(w̃) + 1 (0 where w̃ < 0: no band), with
// which the tensor-core kernel's window [i - w + 1, i] is the band d ≤ w̃ and its landmark
// rule p < i - w + 1 is p < i - w̃ (exact arithmetic; the CUDA-core kernel compares in fp32,
// which differs only where fl(i - w̃) rounds up to an integer).
__global__ void soft_widths_kernel(const float* __restrict__ w_cont, int64_t T, int32_t* __restrict__ w_int) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < T) {
    const float wc = w_cont[t];
    w_int[t] = wc >= 0.0f ? (int32_t)floorf(fminf(wc, 2.0e9f)) + 1 : 0;
  }
}

// One block per landmark set: positions ascending as unsigned values (so -1 goes last), ties
// by slot, each log-weight moved with its position (the order the tensor-core kernel reads).
__global__ void __launch_bounds__(256) sort_sets_kernel(const int32_t* __restrict__ lmk,
                                                        const float* __restrict__ logw, int k_lmk,
                                                        int32_t* __restrict__ lmk_out, float* __restrict__ logw_out) {
  __shared__ uint32_t key[256];
  const int64_t base = (int64_t)blockIdx.x * k_lmk;
  const int c = threadIdx.x;
  if (c < k_lmk) key[c] = (uint32_t)lmk[base + c];
  __syncthreads();
  if (c < k_lmk) {
    const uint32_t kc = key[c];
    int rank = 0;
    for (int o = 0; o < k_lmk; ++o) rank += (key[o] < kc) || (key[o] == kc && o < c);
    lmk_out[base + rank] = (int32_t)kc;
    logw_out[base + rank] = logw[base + c];
  }
}

}  // namespace train

int launch_train_prep(const float* w_cont, int64_t T, const int32_t* lmk, const float* logw, int64_t n_sets,
                      int k_lmk, int32_t* w_int, int32_t* lmk_sorted, float* logw_sorted, cudaStream_t stream) {
  if (k_lmk > 256) return fail(DSALT_ERR_UNSUPPORTED, "training attention: k_lmk %d above 256", k_lmk);
  if (T > 0) train::soft_widths_kernel<<<(unsigned)((T + 255) / 256), 256, 0, stream>>>(w_cont, T, w_int);
  if (n_sets > 0 && k_lmk > 0)
    train::sort_sets_kernel<<<(unsigned)n_sets, 256, 0, stream>>>(lmk, logw, k_lmk, lmk_sorted, logw_sorted);
  return check_cuda(cudaGetLastError(), "training attention prep launch");
}

int launch_train_fwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int D,
                     int64_t q_stride, int64_t kv_stride, const float* w_cont, const int32_t* lmk, const float* logw,
                     int k_lmk, const int32_t* cu, int n_seqs, float tau, float win_edge, void* out, int out_dtype,
                     float* lse, cudaStream_t stream) {
  const int64_t items = T * H;
  if (items == 0) return DSALT_OK;
  const unsigned blocks = (unsigned)((items + train::WARPS - 1) / train::WARPS);
  const float scale = (float)(1.0 / sqrt((double)D));
  const int es = dtype == DSALT_F32 ? 4 : 2;
  // vector loads need every key / value row of the head on a 16-byte boundary
  const bool vec = ((uintptr_t)k % 16 == 0) && ((uintptr_t)v % 16 == 0) && ((kv_stride * es) % 16 == 0);
#define DSALT_TRAIN_LAUNCH(DPL, DT)                                                                                   \
  train::train_fwd_kernel<DPL, DT><<<blocks, train::WARPS * 32, 0, stream>>>(                                        \
      q, k, v, T, H, Hkv, q_stride, kv_stride, vec, w_cont, lmk, logw, k_lmk, cu, n_seqs, scale, tau, win_edge, out, \
      out_dtype, lse)
#define DSALT_TRAIN_DT(DPL)                                    \
  if (dtype == DSALT_BF16) DSALT_TRAIN_LAUNCH(DPL, DSALT_BF16); \
  else if (dtype == DSALT_F16) DSALT_TRAIN_LAUNCH(DPL, DSALT_F16); \
  else DSALT_TRAIN_LAUNCH(DPL, DSALT_F32);
  switch (D) {
    case 64:
      DSALT_TRAIN_DT(2)
      break;
    case 128:
      DSALT_TRAIN_DT(4)
      break;
    default:
      return fail(DSALT_ERR_UNSUPPORTED, "training attention: head_dim %d not in {64, 128}", D);
  }
#undef DSALT_TRAIN_DT
#undef DSALT_TRAIN_LAUNCH
  return check_cuda(cudaGetLastError(), "training attention launch");
}

}  // namespace dsalt
