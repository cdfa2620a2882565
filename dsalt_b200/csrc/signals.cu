// Per-token window width and selection signals in one pass over x and v.
//
// Follows dsalt/modules/dsalt_attention.py:270-284 (width: win_gate logit, sigmoid,
// affine map, floor, clamp) and dsalt/kernels/landmark_tokens_ker.py:47,52 (the norms
// ‖x_i‖ and ‖(x W_Vᵀ)_{i,g}‖ used by the landmark score).
//
// Arithmetic contract (shared with the CPU oracle):
//  * logit: Σ x_i·g_i + b accumulated in float64 (products of two <=24-bit values are
//    exact) and rounded once to the gate dtype;
//  * sigmoid: 1/(1+expf(-l)) in fp32 (the expression torch's CUDA sigmoid evaluates),
//    then every op of `n_min + σ·(n_max−n_min)` rounds to the gate dtype, floor, >= 1;
//  * norms: sum of squares in float64 rounded once to fp32, IEEE fp32 sqrt, optionally
//    rounded to the input dtype.
// One warp per token; 16-byte vector loads; HBM-bound (reads x and v once). The wide
// variant issues all of a token's loads up front (enough bytes in flight for HBM rate).
#include <algorithm>

#include "common.cuh"

namespace dsalt {

template <int DT> struct Vec;
template <> struct Vec<DSALT_BF16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const void* p, float* out) {
    unpack(__ldg(reinterpret_cast<const uint4*>(p)), out);
  }
  static __device__ __forceinline__ void unpack(uint4 u, float* out) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      out[2 * i] = f.x;
      out[2 * i + 1] = f.y;
    }
  }
};
template <> struct Vec<DSALT_F16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const void* p, float* out) {
    unpack(__ldg(reinterpret_cast<const uint4*>(p)), out);
  }
  static __device__ __forceinline__ void unpack(uint4 u, float* out) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      out[2 * i] = f.x;
      out[2 * i + 1] = f.y;
    }
  }
};
template <> struct Vec<DSALT_F32> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const void* p, float* out) {
    float4 u = __ldg(reinterpret_cast<const float4*>(p));
    out[0] = u.x;
    out[1] = u.y;
    out[2] = u.z;
    out[3] = u.w;
  }
};

template <int DT> __device__ __forceinline__ const char* elem_ptr(const void* base, int64_t off) {
  constexpr int ES = DT == DSALT_F32 ? 4 : 2;
  return reinterpret_cast<const char*>(base) + off * ES;
}

__device__ __forceinline__ int width_from_logit(float l, int gate_dt, int n_min, int n_max) {
  // torch: one / (one + exp(-x)) in fp32 opmath, result rounded to the tensor dtype
  float s = 1.0f / (1.0f + expf(-l));
  s = round_to(s, gate_dt);
  float m = round_to(__fmul_rn(s, (float)(n_max - n_min)), gate_dt);
  float c = round_to(__fadd_rn(m, (float)n_min), gate_dt);
  float f = floorf(c);
  int w = (f >= 2147483520.0f) ? 2147483520 : (int)f;  // c is finite and bounded by n_max
  return w < 1 ? 1 : w;
}

template <int XDT, int VDT>
__global__ void __launch_bounds__(256) token_signals_kernel(
    const void* __restrict__ x, int64_t T, int d_model, int64_t x_stride, const void* __restrict__ gate_w,
    const void* __restrict__ gate_b, int gate_dt, int n_min, int n_max, const void* __restrict__ v, int64_t v_stride,
    int n_kv, int head_dim, int norm_mode, int32_t* __restrict__ w_out, float* __restrict__ xnorm_out,
    float* __restrict__ vnorm_out, float* __restrict__ logit_out, const void* __restrict__ logit_in) {
  constexpr int XN = Vec<XDT>::N;
  constexpr int VN = Vec<VDT>::N;
  const int lane = threadIdx.x & 31;
  const int warps_per_block = blockDim.x >> 5;
  const int64_t warp0 = (int64_t)blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * warps_per_block;
  const int x_chunks = d_model / XN;
  const int v_chunks_per_group = head_dim / VN;
  const int v_chunks = n_kv * v_chunks_per_group;
  const double bias = (double)load_elem(gate_b, 0, gate_dt);

  for (int64_t t = warp0; t < T; t += nwarps) {
    const char* xr = elem_ptr<XDT>(x, t * x_stride);
    double dot = 0.0, sq = 0.0;
    for (int c = lane; c < x_chunks; c += 32) {
      float xv[XN];
      Vec<XDT>::load(xr + (size_t)c * 16, xv);
#pragma unroll
      for (int i = 0; i < XN; ++i) {
        const float g = load_elem(gate_w, (int64_t)c * XN + i, gate_dt);
        const float xg = round_to(xv[i], gate_dt);
        dot = __fma_rn((double)xg, (double)g, dot);
        sq = __fma_rn((double)xv[i], (double)xv[i], sq);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      dot += __shfl_xor_sync(0xffffffffu, dot, o);
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
    }
    if (lane == 0) {
      const float logit = logit_in ? load_elem(logit_in, t, gate_dt) : f64_to(dot + bias, gate_dt);
      w_out[t] = width_from_logit(logit, gate_dt, n_min, n_max);
      if (logit_out) logit_out[t] = logit;
      float xn = sqrtf(__double2float_rn(sq));
      if (norm_mode == DSALT_NORM_INPUT) xn = round_to(xn, XDT);
      xnorm_out[t] = xn;
    }
    // value norms: head_dim/VN consecutive chunks form one kv group
    const char* vr = elem_ptr<VDT>(v, t * v_stride);
    if (v_chunks_per_group <= 32) {
      for (int base = 0; base < v_chunks; base += 32) {
        const int c = base + lane;
        double s = 0.0;
        if (c < v_chunks) {
          float vv[VN];
          Vec<VDT>::load(vr + (size_t)c * 16, vv);
#pragma unroll
          for (int i = 0; i < VN; ++i) s = __fma_rn((double)vv[i], (double)vv[i], s);
        }
        for (int o = v_chunks_per_group >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (c < v_chunks && (c % v_chunks_per_group) == 0) {
          float vn = sqrtf(__double2float_rn(s));
          if (norm_mode == DSALT_NORM_INPUT) vn = round_to(vn, VDT);
          vnorm_out[t * n_kv + c / v_chunks_per_group] = vn;
        }
      }
    } else {
      for (int g = 0; g < n_kv; ++g) {
        double s = 0.0;
        for (int c = lane; c < v_chunks_per_group; c += 32) {
          float vv[VN];
          Vec<VDT>::load(vr + ((size_t)g * v_chunks_per_group + c) * 16, vv);
#pragma unroll
          for (int i = 0; i < VN; ++i) s = __fma_rn((double)vv[i], (double)vv[i], s);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
          float vn = sqrtf(__double2float_rn(s));
          if (norm_mode == DSALT_NORM_INPUT) vn = round_to(vn, VDT);
          vnorm_out[t * n_kv + g] = vn;
        }
      }
    }
  }
}

// Four 16-byte read-only loads issued as one block, so that they are all in flight before
// the first result is used
__device__ __forceinline__ void ldg16x4(const uint4* q0, const uint4* q1, const uint4* q2, const uint4* q3,
                                        uint4* r) {
  const size_t p0 = __cvta_generic_to_global(q0), p1 = __cvta_generic_to_global(q1);
  const size_t p2 = __cvta_generic_to_global(q2), p3 = __cvta_generic_to_global(q3);
  asm volatile(
      "ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%16];\n\t"
      "ld.global.nc.v4.u32 {%4, %5, %6, %7}, [%17];\n\t"
      "ld.global.nc.v4.u32 {%8, %9, %10, %11}, [%18];\n\t"
      "ld.global.nc.v4.u32 {%12, %13, %14, %15}, [%19];"
      : "=r"(r[0].x), "=r"(r[0].y), "=r"(r[0].z), "=r"(r[0].w), "=r"(r[1].x), "=r"(r[1].y), "=r"(r[1].z),
        "=r"(r[1].w), "=r"(r[2].x), "=r"(r[2].y), "=r"(r[2].z), "=r"(r[2].w), "=r"(r[3].x), "=r"(r[3].y),
        "=r"(r[3].z), "=r"(r[3].w)
      : "l"(p0), "l"(p1), "l"(p2), "l"(p3));
}

// The reductions of one token held as XCM / VCM 16-byte chunks per lane (chunk j of lane l
// = row bytes [16 (l + 32 j), 16 (l + 32 j) + 16)): the gate logit and width, ‖x‖ and the
// per-head ‖v‖, in fp64 with a fixed accumulation order.
template <int XDT, int VDT, int XCM, int VCM>
__device__ __forceinline__ void reduce_token(const uint4* xq, const uint4* vq, const double* gws, int lane, int xc,
                                             int vc, int vcpg, bool xg_is_x, int gate_dt, double bias, int n_min,
                                             int n_max, int norm_mode, int n_kv, int64_t t, int32_t* w_out,
                                             float* xnorm_out, float* vnorm_out, float* logit_out,
                                             const void* logit_in) {
  constexpr int XN = Vec<XDT>::N;
  constexpr int VN = Vec<VDT>::N;
  double dot = 0.0, sq = 0.0;
#pragma unroll
  for (int j = 0; j < XCM; ++j) {
    if (j < xc) {
      float xv[XN];
      Vec<XDT>::unpack(xq[j], xv);
      const double* gj = gws + j * XN * 32 + lane;
      if (logit_in) {
        // the caller's logit: only the norm's sum
#pragma unroll
        for (int i = 0; i < XN; ++i) {
          const double xd = (double)xv[i];
          sq = __fma_rn(xd, xd, sq);
        }
      } else if (xg_is_x) {
#pragma unroll
        for (int i = 0; i < XN; ++i) {
          const double xd = (double)xv[i];
          dot = __fma_rn(xd, gj[i * 32], dot);
          sq = __fma_rn(xd, xd, sq);
        }
      } else {
#pragma unroll
        for (int i = 0; i < XN; ++i) {
          const double xd = (double)xv[i];
          dot = __fma_rn((double)round_to(xv[i], gate_dt), gj[i * 32], dot);
          sq = __fma_rn(xd, xd, sq);
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    dot += __shfl_xor_sync(0xffffffffu, dot, o);
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  if (lane == 0) {
    const float logit = logit_in ? load_elem(logit_in, t, gate_dt) : f64_to(dot + bias, gate_dt);
    w_out[t] = width_from_logit(logit, gate_dt, n_min, n_max);
    if (logit_out) logit_out[t] = logit;
    float xn = sqrtf(__double2float_rn(sq));
    if (norm_mode == DSALT_NORM_INPUT) xn = round_to(xn, XDT);
    xnorm_out[t] = xn;
  }
#pragma unroll
  for (int j = 0; j < VCM; ++j) {
    if (j < vc) {
      float vv[VN];
      Vec<VDT>::unpack(vq[j], vv);
      double s = 0.0;
#pragma unroll
      for (int i = 0; i < VN; ++i) s = __fma_rn((double)vv[i], (double)vv[i], s);
      for (int o = vcpg >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const int c = lane + 32 * j;
      if ((c % vcpg) == 0) {
        float vn = sqrtf(__double2float_rn(s));
        if (norm_mode == DSALT_NORM_INPUT) vn = round_to(vn, VDT);
        vnorm_out[t * n_kv + c / vcpg] = vn;
      }
    }
  }
}

// Same arithmetic (and accumulation order) as token_signals_kernel, for 16-bit x and v
// whose rows split into at most XCM (x) / VCM (v) 16-byte chunks per lane: every load of
// a token is issued before any is used, so a warp keeps its whole token (up to 8 KB) in
// flight; the gate weights sit in shared memory as fp64 (fp32->fp64 conversions run at a
// quarter of the fp64 FMA rate, so each element is converted once).
template <int XDT, int VDT, int XCM, int VCM>
__global__ void __launch_bounds__(256) token_signals_wide_kernel(
    const void* __restrict__ x, int64_t T, int d_model, int64_t x_stride, const void* __restrict__ gate_w,
    const void* __restrict__ gate_b, int gate_dt, int n_min, int n_max, const void* __restrict__ v, int64_t v_stride,
    int n_kv, int head_dim, int norm_mode, int32_t* __restrict__ w_out, float* __restrict__ xnorm_out,
    float* __restrict__ vnorm_out, float* __restrict__ logit_out, const void* __restrict__ logit_in) {
  constexpr int XN = Vec<XDT>::N;
  constexpr int VN = Vec<VDT>::N;
  // gate weight of element i of chunk lane + 32 j at gws[(j * XN + i) * 32 + lane]: the lanes
  // of a warp read consecutive doubles (no bank conflicts)
  extern __shared__ double gws[];
  for (int e = threadIdx.x; e < d_model; e += blockDim.x) {
    const int c = e / XN, i = e - c * XN, l = c & 31, j = c >> 5;
    gws[(j * XN + i) * 32 + l] = (double)load_elem(gate_w, e, gate_dt);
  }
  __syncthreads();
  // x is converted to the gate dtype before the product; for a gate in fp32 or in x's own
  // dtype that conversion is the identity, and one fp32->fp64 conversion serves both sums
  const bool xg_is_x = gate_dt == DSALT_F32 || gate_dt == XDT;
  const int lane = threadIdx.x & 31;
  const int warps_per_block = blockDim.x >> 5;
  const int64_t warp0 = (int64_t)blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * warps_per_block;
  const int xc = d_model / XN / 32;                 // x chunks per lane (<= XCM)
  const int vcpg = head_dim / VN;                    // v chunks per kv group (<= 32, power of two)
  const int vc = n_kv * vcpg / 32;                   // v chunks per lane (<= VCM)
  const double bias = (double)load_elem(gate_b, 0, gate_dt);
  for (int64_t t = warp0; t < T; t += nwarps) {
    const uint4* xr = reinterpret_cast<const uint4*>(elem_ptr<XDT>(x, t * x_stride));
    const uint4* vr = reinterpret_cast<const uint4*>(elem_ptr<VDT>(v, t * v_stride));
    // chunks past the row's end re-read chunk 0 (an L1 hit) and are not used
    uint4 xq[XCM], vq[VCM];
#pragma unroll
    for (int j = 0; j < XCM; j += 4)
      ldg16x4(xr + lane + 32 * (j < xc ? j : 0), xr + lane + 32 * (j + 1 < xc ? j + 1 : 0),
              xr + lane + 32 * (j + 2 < xc ? j + 2 : 0), xr + lane + 32 * (j + 3 < xc ? j + 3 : 0), xq + j);
#pragma unroll
    for (int j = 0; j < VCM; j += 4)
      ldg16x4(vr + lane + 32 * (j < vc ? j : 0), vr + lane + 32 * (j + 1 < vc ? j + 1 : 0),
              vr + lane + 32 * (j + 2 < vc ? j + 2 : 0), vr + lane + 32 * (j + 3 < vc ? j + 3 : 0), vq + j);
    reduce_token<XDT, VDT, XCM, VCM>(xq, vq, gws, lane, xc, vc, vcpg, xg_is_x, gate_dt, bias, n_min, n_max, norm_mode,
                                     n_kv, t, w_out, xnorm_out, vnorm_out, logit_out, logit_in);
  }
}

// The same per-token reductions with the rows streamed through shared memory by 1-D bulk
// copies: each warp keeps `stages` tokens in flight (its x and v rows, xc·512 + vc·512
// bytes each) besides the one it reduces. Lane 0 of a warp issues its copies; the warp
// waits on the stage's barrier (bounded), reads the rows from shared memory (lane l reads
// chunks l + 32 j: no bank conflicts), refills the stage and then reduces. With the
// reductions removed this streams x and v at the HBM copy rate; with them the kernel is
// bound by the fp64 reductions (exact sums), not by memory.
// Shared memory: gate weights (fp64) | barriers [warp][stage] | rows [warp][stage].
template <int XDT, int VDT, int XCM, int VCM>
__global__ void __launch_bounds__(1024) token_signals_bulk_kernel(
    const void* __restrict__ x, int64_t T, int d_model, int64_t x_stride, const void* __restrict__ gate_w,
    const void* __restrict__ gate_b, int gate_dt, int n_min, int n_max, const void* __restrict__ v, int64_t v_stride,
    int n_kv, int head_dim, int norm_mode, int32_t* __restrict__ w_out, float* __restrict__ xnorm_out,
    float* __restrict__ vnorm_out, float* __restrict__ logit_out, const void* __restrict__ logit_in, int stages,
    int* __restrict__ err) {
  constexpr int XN = Vec<XDT>::N;
  constexpr int VN = Vec<VDT>::N;
  extern __shared__ __align__(128) unsigned char sig_smem[];
  double* gws = reinterpret_cast<double*>(sig_smem);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int xc = d_model / XN / 32, vcpg = head_dim / VN, vc = n_kv * vcpg / 32;
  const uint32_t xbytes = (uint32_t)xc * 512, vbytes = (uint32_t)vc * 512, sbytes = xbytes + vbytes;
  const size_t gws_bytes = ((size_t)d_model * 8 + 127) & ~(size_t)127;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sig_smem + gws_bytes) + warp * stages;
  unsigned char* rows = sig_smem + gws_bytes + (((size_t)wpb * stages * 8 + 127) & ~(size_t)127) +
                        (size_t)warp * stages * sbytes;
  for (int e = threadIdx.x; e < d_model; e += blockDim.x) {
    const int c = e / XN, i = e - c * XN, l = c & 31, j = c >> 5;
    gws[(j * XN + i) * 32 + l] = (double)load_elem(gate_w, e, gate_dt);
  }
  if (lane == 0)
    for (int st = 0; st < stages; ++st) mbar_init(bars + st, 1);
  fence_barrier_init();
  __syncthreads();
  const bool xg_is_x = gate_dt == DSALT_F32 || gate_dt == XDT;
  const double bias = (double)load_elem(gate_b, 0, gate_dt);
  const int64_t warp0 = (int64_t)blockIdx.x * wpb + warp, nwarps = (int64_t)gridDim.x * wpb;
  auto issue = [&](int64_t t, int st) {
    mbar_arrive_expect_tx(bars + st, sbytes);
    const uint32_t dst = smem_u32(rows + (size_t)st * sbytes);
    bulk_load(dst, elem_ptr<XDT>(x, t * x_stride), xbytes, bars + st);
    bulk_load(dst + xbytes, elem_ptr<VDT>(v, t * v_stride), vbytes, bars + st);
  };
  if (lane == 0)
    for (int st = 0; st < stages; ++st)
      if (warp0 + st * nwarps < T) issue(warp0 + st * nwarps, st);
  int k = 0;
  for (int64_t t = warp0; t < T; t += nwarps, ++k) {
    const int st = k % stages;
    if (!mbar_wait(bars + st, (uint32_t)(k / stages) & 1, err, 50)) {
      // give the warp's copies still in flight (tokens k .. k + stages - 1) a bounded
      // chance to land before the block exits
      for (int q = k + 1; q < k + stages; ++q)
        if (warp0 + q * nwarps < T) mbar_wait(bars + q % stages, (uint32_t)(q / stages) & 1, err, 51, 100000000ull);
      break;
    }
    const uint4* xs = reinterpret_cast<const uint4*>(rows + (size_t)st * sbytes);
    const uint4* vs = reinterpret_cast<const uint4*>(rows + (size_t)st * sbytes + xbytes);
    uint4 xq[XCM], vq[VCM];
#pragma unroll
    for (int j = 0; j < XCM; ++j) xq[j] = xs[lane + 32 * (j < xc ? j : 0)];
#pragma unroll
    for (int j = 0; j < VCM; ++j) vq[j] = vs[lane + 32 * (j < vc ? j : 0)];
    __syncwarp();
    // every lane has read the stage: refill it with the warp's token `stages` steps ahead
    // (the generic-proxy reads are ordered before the copy's async-proxy writes)
    if (lane == 0 && t + stages * nwarps < T) {
      fence_proxy_async_smem();
      issue(t + stages * nwarps, st);
    }
    reduce_token<XDT, VDT, XCM, VCM>(xq, vq, gws, lane, xc, vc, vcpg, xg_is_x, gate_dt, bias, n_min, n_max, norm_mode,
                                     n_kv, t, w_out, xnorm_out, vnorm_out, logit_out, logit_in);
  }
}

static bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

int launch_token_signals(const void* x, int x_dtype, int64_t T, int d_model, int64_t x_stride, const void* gate_w,
                         const void* gate_b, int gate_dtype, int n_min, int n_max, const void* v, int v_dtype,
                         int64_t v_stride, int n_kv, int head_dim, int norm_mode, int32_t* w_out, float* xnorm_out,
                         float* vnorm_out, float* logit_out, const void* logit_in, cudaStream_t stream) {
  if (T < 0 || d_model <= 0 || n_kv <= 0 || head_dim <= 0) return fail(DSALT_ERR_INVALID, "token_signals: bad sizes");
  if (T == 0) return DSALT_OK;
  if (!x || !gate_w || !gate_b || !v || !w_out || !xnorm_out || !vnorm_out)
    return fail(DSALT_ERR_INVALID, "token_signals: null pointer");
  for (int dt : {x_dtype, v_dtype, gate_dtype})
    if (dt != DSALT_F32 && dt != DSALT_BF16 && dt != DSALT_F16) return fail(DSALT_ERR_INVALID, "token_signals: dtype");
  if (norm_mode != DSALT_NORM_F32 && norm_mode != DSALT_NORM_INPUT)
    return fail(DSALT_ERR_INVALID, "token_signals: norm_mode");
  if (n_max < n_min) return fail(DSALT_ERR_INVALID, "token_signals: n_max < n_min");
  const int xes = x_dtype == DSALT_F32 ? 4 : 2, ves = v_dtype == DSALT_F32 ? 4 : 2;
  const int xvec = 16 / xes, vvec = 16 / ves;
  if (d_model % xvec || head_dim % vvec || !is_pow2(head_dim / vvec))
    return fail(DSALT_ERR_UNSUPPORTED, "token_signals: d_model must be a multiple of %d and head_dim/%d a power of two",
                xvec, vvec);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(v)) & 15 || (x_stride * xes) % 16 ||
      (v_stride * ves) % 16)
    return fail(DSALT_ERR_INVALID, "token_signals: x/v rows must be 16-byte aligned");
  if (x_stride < d_model || v_stride < (int64_t)n_kv * head_dim) return fail(DSALT_ERR_INVALID, "token_signals: stride");
  const int threads = 256;
  int64_t blocks = (T + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  // wide path: 16-bit x and v, rows in whole 512-byte warp chunks (at most 8 per lane)
  const int xc = d_model / xvec, vcpg = head_dim / vvec, vtot = n_kv * vcpg;
  if (xes == 2 && x_dtype == v_dtype && xc % 32 == 0 && xc / 32 <= 8 && vcpg <= 32 && vtot % 32 == 0 &&
      vtot / 32 <= 8 && d_model <= 6144) {
    const bool x4 = xc / 32 <= 4, v4 = vtot / 32 <= 4;
    // bulk-copy path: 32 warps per block, one block per SM, one token in flight per warp
    // besides the one it reduces, when the rows fit in 200 KB of shared memory
    {
      const size_t sbytes = (size_t)(xc + vtot) * 16;
      const size_t gws_bytes = ((size_t)d_model * 8 + 127) & ~(size_t)127;
      const int wpb = 32, stages = 1;
      const size_t smem_b = gws_bytes + (((size_t)wpb * stages * 8 + 127) & ~(size_t)127) + (size_t)wpb * stages * sbytes;
      if (smem_b <= 200 * 1024) {
        int dev = 0, nsm = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        const int64_t bblocks = std::min<int64_t>((T + wpb - 1) / wpb, nsm);
        int rc = DSALT_OK;
#define DSALT_SIG_BULK(DT, XC, VC)                                                                                   \
  do {                                                                                                                \
    auto kern = token_signals_bulk_kernel<DT, DT, XC, VC>;                                                            \
    if ((rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_b),      \
                         "token_signals smem attr")))                                                                 \
      return rc;                                                                                                      \
    kern<<<(unsigned)bblocks, wpb * 32, smem_b, stream>>>(x, T, d_model, x_stride, gate_w, gate_b, gate_dtype, n_min, \
                                                         n_max, v, v_stride, n_kv, head_dim, norm_mode, w_out,         \
                                                         xnorm_out, vnorm_out, logit_out, logit_in, stages, device_status_ptr()); \
  } while (0)
        if (x_dtype == DSALT_BF16) {
          if (x4 && v4) DSALT_SIG_BULK(DSALT_BF16, 4, 4);
          else if (x4) DSALT_SIG_BULK(DSALT_BF16, 4, 8);
          else if (v4) DSALT_SIG_BULK(DSALT_BF16, 8, 4);
          else DSALT_SIG_BULK(DSALT_BF16, 8, 8);
        } else {
          if (x4 && v4) DSALT_SIG_BULK(DSALT_F16, 4, 4);
          else if (x4) DSALT_SIG_BULK(DSALT_F16, 4, 8);
          else if (v4) DSALT_SIG_BULK(DSALT_F16, 8, 4);
          else DSALT_SIG_BULK(DSALT_F16, 8, 8);
        }
#undef DSALT_SIG_BULK
        return check_cuda(cudaGetLastError(), "token_signals launch");
      }
    }
    const size_t smem = (size_t)d_model * sizeof(double);
#define DSALT_SIG_WIDE(DT, XC, VC)                                                                                 \
  token_signals_wide_kernel<DT, DT, XC, VC><<<(unsigned)blocks, threads, smem, stream>>>(                          \
      x, T, d_model, x_stride, gate_w, gate_b, gate_dtype, n_min, n_max, v, v_stride, n_kv, head_dim, norm_mode, \
      w_out, xnorm_out, vnorm_out, logit_out, logit_in)
    if (x_dtype == DSALT_BF16) {
      if (x4 && v4) DSALT_SIG_WIDE(DSALT_BF16, 4, 4);
      else if (x4) DSALT_SIG_WIDE(DSALT_BF16, 4, 8);
      else if (v4) DSALT_SIG_WIDE(DSALT_BF16, 8, 4);
      else DSALT_SIG_WIDE(DSALT_BF16, 8, 8);
    } else {
      if (x4 && v4) DSALT_SIG_WIDE(DSALT_F16, 4, 4);
      else if (x4) DSALT_SIG_WIDE(DSALT_F16, 4, 8);
      else if (v4) DSALT_SIG_WIDE(DSALT_F16, 8, 4);
      else DSALT_SIG_WIDE(DSALT_F16, 8, 8);
    }
#undef DSALT_SIG_WIDE
    return check_cuda(cudaGetLastError(), "token_signals launch");
  }
#define DSALT_SIG_LAUNCH(XD, VD)                                                                                   \
  token_signals_kernel<XD, VD><<<(unsigned)blocks, threads, 0, stream>>>(                                          \
      x, T, d_model, x_stride, gate_w, gate_b, gate_dtype, n_min, n_max, v, v_stride, n_kv, head_dim, norm_mode, \
      w_out, xnorm_out, vnorm_out, logit_out, logit_in)
  if (x_dtype == DSALT_BF16 && v_dtype == DSALT_BF16) DSALT_SIG_LAUNCH(DSALT_BF16, DSALT_BF16);
  else if (x_dtype == DSALT_F16 && v_dtype == DSALT_F16) DSALT_SIG_LAUNCH(DSALT_F16, DSALT_F16);
  else if (x_dtype == DSALT_F32 && v_dtype == DSALT_F32) DSALT_SIG_LAUNCH(DSALT_F32, DSALT_F32);
  else if (x_dtype == DSALT_F32 && v_dtype == DSALT_BF16) DSALT_SIG_LAUNCH(DSALT_F32, DSALT_BF16);
  else if (x_dtype == DSALT_F32 && v_dtype == DSALT_F16) DSALT_SIG_LAUNCH(DSALT_F32, DSALT_F16);
  else return fail(DSALT_ERR_UNSUPPORTED, "token_signals: x/v dtype combination");
#undef DSALT_SIG_LAUNCH
  return check_cuda(cudaGetLastError(), "token_signals launch");
}

}  // namespace dsalt
