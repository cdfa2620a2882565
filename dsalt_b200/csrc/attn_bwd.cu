// Backward of the sparse attention forward (reference: dsalt/kernels/dsalt_triton_bwd.py).
//
// Gradients of out = softmax(logits over A(i)) · V with A(i) = the window
// [max(0, i−w(i)+1), i] and the landmarks p of the row's set with 0 ≤ p < L, p ≤ i and
// p < i−w(i)+1, logits q·k·scale (+ landmark bias). As the reference (:18-212): the forward's
// log-sum-exp is reused, P is recomputed, delta = Σ_d O·dO, dS = P ⊙ (dO·Vᵀ − delta) · scale,
// dQ = dS·K, dK += dSᵀ·Q, dV += Pᵀ·dO (atomic adds: a key belongs to many query tiles),
// d_bias[h, set, slot] += Σ_i P (dO·v − delta). Rows whose log-sum-exp is −inf contribute
// nothing. Grouped kv heads: head h uses kv head h / (H / H_kv) and its kv gradients add into
// that head.
//
// S = Q·Kᵀ and dP = dO·Vᵀ on the tensor cores (mma.sync, fp32 accumulate) for 16-bit inputs,
// on CUDA cores otherwise; everything else on CUDA cores in fp32. One CTA per (64-query tile,
// head), 128 threads; the key axis is walked in 32-key tiles: the window band of the tile,
// then the landmark slots of its set. Per key tile the Q/dO tile (resident), the K/V tile and
// the P/dS tile sit in shared memory with padded rows (stride HD + 8 floats, for
// conflict-free 8-byte fragment loads). The CUDA-core phases are bound by shared-memory
// wavefronts (one per 4-byte load instruction; 16-byte loads cost four and gain nothing), so
// every thread holds a 4 x 4 register block: 4 rows x 4 keys of P / dS, 4 rows x HD/8 dims of
// dQ, 4 keys x HD/16 dims of dK and dV (0.5 shared-memory operands per FMA).
#include "common.cuh"

namespace dsalt {

int launch_chunk_table(const int32_t* cu, int n_seqs, int C, int32_t* base, cudaStream_t stream);

namespace bwd {

constexpr int BM = 64;        // queries per CTA
constexpr int BN = 32;        // keys per tile
constexpr int THREADS = 128;

template <int HD>
struct Smem {
  static constexpr int LD = HD + 8;  // padded row stride (floats): ≡ 8 mod 32
  static constexpr int Q_OFF = 0, DO_OFF = BM * LD, K_OFF = 2 * BM * LD, V_OFF = K_OFF + BN * LD;
  static constexpr int P_OFF = V_OFF + BN * LD, DS_OFF = P_OFF + BM * (BN + 1);
  static constexpr int FLOATS = DS_OFF + BM * (BN + 1);
  static constexpr size_t BYTES = (size_t)FLOATS * 4 + BM * 20 + BN * 8;  // + per-row and per-key words
};

struct Params {
  const void* q;
  const void* k;
  const void* v;
  int dtype;
  int H, Hkv;
  int64_t q_stride, kv_stride;  // elements between consecutive tokens
  const void* out;
  int out_dtype;
  const void* dout;
  int dout_dtype;
  const float* lse;  // [T, H], natural log
  const int32_t* w;
  const int32_t* lmk;
  const float* lmk_bias;
  int k_lmk, lmk_block;
  const int32_t* cu;
  int n_seqs;
  const int32_t* tile_base;  // per sequence: first 64-query tile
  const int32_t* set_base;   // per sequence: first landmark set (block mode)
  float scale;
  float* dq;      // [T, H, HD]
  float* dk;      // [T, Hkv, HD]
  float* dv;      // [T, Hkv, HD]
  float* d_bias;  // [H, n_sets, k] or null
  // training mode (soft selectors): continuous widths w̃ [T], soft edge τ and core margin,
  // gradient of w̃ summed over heads [T]; lmk_bias / d_bias are the landmark log-weights
  const float* w_cont;
  float tau, win_edge;
  float* d_w;
};

// two consecutive fp32 tile values (16-bit input values, so exact) packed as a 16-bit pair
template <int MT>
__device__ __forceinline__ uint32_t pack2(const float* a) {
  const float2 v = *reinterpret_cast<const float2*>(a);
  uint32_t r;
  if constexpr (MT == DSALT_BF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    memcpy(&r, &h, 4);
  } else {
    const __half2 h = __floats2half2_rn(v.x, v.y);
    memcpy(&r, &h, 4);
  }
  return r;
}
// d += a · b, one m16n8k16 tile, fp32 accumulate (PTX ISA fragment layouts)
template <int MT>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  if constexpr (MT == DSALT_BF16) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
}

template <int HD, bool TRAIN, int MT>  // MT: 0 CUDA cores, DSALT_BF16 / DSALT_F16 tensor-core S and dP
__global__ void __launch_bounds__(THREADS) attn_bwd_kernel(const Params p) {
  using SM = Smem<HD>;
  constexpr int LD = SM::LD;
  extern __shared__ float sm[];
  float* sq = sm + SM::Q_OFF;
  float* sdo = sm + SM::DO_OFF;
  float* sk = sm + SM::K_OFF;
  float* sv = sm + SM::V_OFF;
  float* sp = sm + SM::P_OFF;   // [BM][BN + 1]
  float* sds = sm + SM::DS_OFF;  // [BM][BN + 1]
  int* row_lo = reinterpret_cast<int*>(sm + SM::FLOATS);  // per row: window start (raw, may be < 0)
  int* row_ok = row_lo + BM;                                // per row: valid and finite lse
  float* row_lse = reinterpret_cast<float*>(row_ok + BM);
  float* row_delta = row_lse + BM;
  float* row_wc = row_delta + BM;                           // per row: continuous width (training mode)
  int* key_pos = reinterpret_cast<int*>(row_wc + BM);       // per key of the tile: position or -1
  int* key_slot = key_pos + BN;                             // landmark slot (or -1 for window keys)

  const int tile = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  if (tile >= p.tile_base[p.n_seqs]) return;
  int lo_s = 0, hi_s = p.n_seqs;  // sequence of this tile
  while (hi_s - lo_s > 1) {
    const int mid = (lo_s + hi_s) >> 1;
    if (p.tile_base[mid] <= tile) lo_s = mid;
    else hi_s = mid;
  }
  const int s = lo_s;
  const int seq0 = p.cu[s], L = p.cu[s + 1] - seq0;
  const int m0 = (tile - p.tile_base[s]) * BM;
  const int hk = h / (p.H / p.Hkv);
  const int set = p.lmk_block > 0 ? p.set_base[s] + m0 / p.lmk_block : s;
  const int n_sets = p.lmk_block > 0 ? p.set_base[p.n_seqs] : p.n_seqs;

  // resident Q and dO tiles (fp32), per-row window start, lse and delta = Σ O·dO
  for (int e = tid; e < BM * HD; e += THREADS) {
    const int r = e / HD, d = e - r * HD;
    const int i = m0 + r;
    float qv = 0.f, dov = 0.f;
    if (i < L) {
      const int64_t t = seq0 + i;
      qv = load_elem(p.q, t * p.q_stride + (int64_t)h * HD + d, p.dtype);
      dov = load_elem(p.dout, (t * p.H + h) * HD + d, p.dout_dtype);
    }
    sq[r * LD + d] = qv;
    sdo[r * LD + d] = dov;
  }
  {
    const int r = tid >> 1, part = tid & 1;  // 2 threads per row
    const int i = m0 + r;
    float acc = 0.f;
    if (i < L) {
      const int64_t t = seq0 + i;
      for (int d = part; d < HD; d += 2)
        acc += load_elem(p.out, (t * p.H + h) * HD + d, p.out_dtype) * load_elem(p.dout, (t * p.H + h) * HD + d,
                                                                               p.dout_dtype);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (part == 0) {
      float l = -INFINITY, wc = 0.f;
      int lo = 0x3fffffff;
      if (i < L) {
        const int64_t t = seq0 + i;
        l = p.lse[t * p.H + h];
        if constexpr (TRAIN) {
          wc = p.w_cont[t];  // band d = i - j in [0, w̃]: j from i - floor(w̃)
          lo = wc >= 0.f ? i - (int)floorf(wc) : i + 1;
        } else {
          lo = i - max(p.w[t], 1) + 1;
        }
      }
      row_delta[r] = acc;
      row_lse[r] = l;
      row_lo[r] = lo;
      row_wc[r] = wc;
      row_ok[r] = (i < L) && (l > -INFINITY);
    }
  }
  __syncthreads();
  int wmin_lo = 0x3fffffff;
  for (int r = 0; r < BM; ++r)
    if (row_ok[r]) wmin_lo = min(wmin_lo, max(row_lo[r], 0));
  const int i_last = min(m0 + BM, L) - 1;
  const int n_wt = wmin_lo > i_last ? 0 : (i_last - (wmin_lo & ~(BN - 1))) / BN + 1;  // window tiles
  const int kw0 = wmin_lo & ~(BN - 1);
  const int n_lt = (p.k_lmk + BN - 1) / BN;
  const int32_t* P = p.lmk + ((int64_t)h * n_sets + set) * p.k_lmk;
  const float* Bset = p.lmk_bias ? p.lmk_bias + ((int64_t)h * n_sets + set) * p.k_lmk : nullptr;

  // this thread's share of dQ: rows (tid >> 3) + 16 u, dims (tid & 7) + 8 m at dq_acc[u * HD/8 + m]
  float dq_acc[HD / 2];
  float dw_acc[4] = {0.f, 0.f, 0.f, 0.f};  // training mode: this thread's part of dL/dw̃ of its rows
#pragma unroll
  for (int m = 0; m < HD / 2; ++m) dq_acc[m] = 0.f;

  for (int kt = 0; kt < n_wt + n_lt; ++kt) {
    const bool is_w = kt < n_wt;
    const int lt = kt - n_wt;
    if (tid < BN) {
      int pos = -1, slot = -1;
      if (is_w) {
        const int j = kw0 + kt * BN + tid;
        pos = (j >= 0 && j < L) ? j : -1;
      } else {
        slot = lt * BN + tid;
        const int pp = slot < p.k_lmk ? P[slot] : -1;
        pos = (pp >= 0 && pp < L) ? pp : -1;
        if (slot >= p.k_lmk) slot = -1;
      }
      key_pos[tid] = pos;
      key_slot[tid] = slot;
    }
    __syncthreads();
    for (int e = tid; e < BN * HD; e += THREADS) {
      const int c = e / HD, d = e - c * HD;
      const int pos = key_pos[c];
      float kv = 0.f, vv = 0.f;
      if (pos >= 0) {
        const int64_t off = (seq0 + pos) * p.kv_stride + (int64_t)hk * HD + d;
        kv = load_elem(p.k, off, p.dtype);
        vv = load_elem(p.v, off, p.dtype);
      }
      sk[c * LD + d] = kv;
      sv[c * LD + d] = vv;
    }
    __syncthreads();
    // P and dS of one (row, key) from its logit s = q·k and dp = dO·v; returns rec · d(edge
    // bias)/dw̃ for the width gradient (training mode)
    auto emit = [&](int r, int c, float sv_, float dpv) -> float {
      const int i = m0 + r;
      const int pos = key_pos[c];
      const float wc = row_wc[r];
      bool valid = row_ok[r] && pos >= 0;
      float logit = sv_ * p.scale;
      float dbdw = 0.f;  // training mode: d(edge bias)/dw̃ of this window key
      if (is_w) {
        if constexpr (TRAIN) {
          const float d = (float)(i - pos);
          valid = valid && pos <= i && d <= wc;
          if (valid && !(d <= wc - p.win_edge)) {
            const float z = (wc - d) / p.tau;
            logit += -logf(1.0f + expf(-z));  // log σ(z)
            dbdw = (1.0f - 1.0f / (1.0f + expf(-z))) / p.tau;
          }
        } else {
          valid = valid && pos >= row_lo[r] && pos <= i;
        }
      } else {
        if constexpr (TRAIN) valid = valid && pos <= i && (float)pos < (float)i - wc;
        else valid = valid && pos <= i && pos < row_lo[r];
        if (valid && Bset) logit += Bset[key_slot[c]];
      }
      const float pr = valid ? expf(logit - row_lse[r]) : 0.f;
      const float rec = pr * (dpv - row_delta[r]);
      sp[r * (BN + 1) + c] = pr;
      sds[r * (BN + 1) + c] = rec;  // scaled below where dS is used
      return rec * dbdw;
    };
    if constexpr (MT != 0) {
      // S = Q·Kᵀ and dP = dO·Vᵀ on the tensor cores (mma.sync m16n8k16, fp32 accumulate):
      // warp w -> rows 16 w .. 16 w + 15, all 32 keys (four n8 tiles). Operands are the
      // 16-bit input values, exact in the fp32 tiles; fragments by 8-byte loads (row stride
      // HD + 8: a half warp's 16 loads hit distinct bank pairs).
      const int w = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3, rw = 16 * w;
      float sacc[4][4], dpacc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[j][e] = dpacc[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < HD; kk += 16) {
        uint32_t qa[4], da[4];
        qa[0] = pack2<MT>(sq + (rw + g) * LD + kk + 2 * t4);
        qa[1] = pack2<MT>(sq + (rw + g + 8) * LD + kk + 2 * t4);
        qa[2] = pack2<MT>(sq + (rw + g) * LD + kk + 2 * t4 + 8);
        qa[3] = pack2<MT>(sq + (rw + g + 8) * LD + kk + 2 * t4 + 8);
        da[0] = pack2<MT>(sdo + (rw + g) * LD + kk + 2 * t4);
        da[1] = pack2<MT>(sdo + (rw + g + 8) * LD + kk + 2 * t4);
        da[2] = pack2<MT>(sdo + (rw + g) * LD + kk + 2 * t4 + 8);
        da[3] = pack2<MT>(sdo + (rw + g + 8) * LD + kk + 2 * t4 + 8);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t kb[2] = {pack2<MT>(sk + (8 * j + g) * LD + kk + 2 * t4),
                                  pack2<MT>(sk + (8 * j + g) * LD + kk + 2 * t4 + 8)};
          const uint32_t vb[2] = {pack2<MT>(sv + (8 * j + g) * LD + kk + 2 * t4),
                                  pack2<MT>(sv + (8 * j + g) * LD + kk + 2 * t4 + 8)};
          mma16816<MT>(sacc[j], qa, kb);
          mma16816<MT>(dpacc[j], da, vb);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = emit(rw + g + 8 * (e >> 1), 8 * j + 2 * t4 + (e & 1), sacc[j][e], dpacc[j][e]);
          if constexpr (TRAIN) dw_acc[e >> 1] += x;
        }
    } else {
      // CUDA cores: thread -> rows rA + 16 u and keys c0 + 8 j (4 x 4 entries; per head-dim
      // step 8 + 8 shared-memory operands for 32 FMAs)
      const int rA = tid >> 3, c0 = tid & 7;
      float sacc[4][4], dpacc[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < 4; ++j) sacc[u][j] = dpacc[u][j] = 0.f;
#pragma unroll 2
      for (int d = 0; d < HD; ++d) {
        float a[4], b[4], kv[4], vv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          a[u] = sq[(rA + 16 * u) * LD + d];
          b[u] = sdo[(rA + 16 * u) * LD + d];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          kv[j] = sk[(c0 + 8 * j) * LD + d];
          vv[j] = sv[(c0 + 8 * j) * LD + d];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sacc[u][j] = fmaf(a[u], kv[j], sacc[u][j]);
            dpacc[u][j] = fmaf(b[u], vv[j], dpacc[u][j]);
          }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x = emit(rA + 16 * u, c0 + 8 * j, sacc[u][j], dpacc[u][j]);
          if constexpr (TRAIN) dw_acc[u] += x;
        }
    }
    __syncthreads();
    // dQ += dS · K (dS = rec · scale): thread -> rows rA + 16 u and dims d0 + 8 m
    {
      const int rA = tid >> 3, d0 = tid & 7;
#pragma unroll 2
      for (int c = 0; c < BN; ++c) {
        float ds[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) ds[u] = sds[(rA + 16 * u) * (BN + 1) + c] * p.scale;
#pragma unroll
        for (int m = 0; m < HD / 8; ++m) {
          const float kv = sk[c * LD + d0 + 8 * m];
#pragma unroll
          for (int u = 0; u < 4; ++u) dq_acc[u * (HD / 8) + m] = fmaf(ds[u], kv, dq_acc[u * (HD / 8) + m]);
        }
      }
    }
    // dK_tile = dSᵀ · Q, dV_tile = Pᵀ · dO: thread -> keys kA + 8 u and dims d0 + 16 m
    {
      const int kA = tid >> 4, d0 = tid & 15;
      constexpr int ND = HD / 16;
      float dkacc[4][ND], dvacc[4][ND];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int m = 0; m < ND; ++m) dkacc[u][m] = dvacc[u][m] = 0.f;
#pragma unroll 2
      for (int r = 0; r < BM; ++r) {
        float ds[4], pr[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          ds[u] = sds[r * (BN + 1) + kA + 8 * u] * p.scale;
          pr[u] = sp[r * (BN + 1) + kA + 8 * u];
        }
#pragma unroll
        for (int m = 0; m < ND; ++m) {
          const float qv = sq[r * LD + d0 + 16 * m], dov = sdo[r * LD + d0 + 16 * m];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            dkacc[u][m] = fmaf(ds[u], qv, dkacc[u][m]);
            dvacc[u][m] = fmaf(pr[u], dov, dvacc[u][m]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int pos = key_pos[kA + 8 * u];
        if (pos >= 0) {
          float* gk = p.dk + ((seq0 + pos) * (int64_t)p.Hkv + hk) * HD;
          float* gv = p.dv + ((seq0 + pos) * (int64_t)p.Hkv + hk) * HD;
#pragma unroll
          for (int m = 0; m < ND; ++m) {
            if (dkacc[u][m] != 0.f) atomicAdd(gk + d0 + 16 * m, dkacc[u][m]);
            if (dvacc[u][m] != 0.f) atomicAdd(gv + d0 + 16 * m, dvacc[u][m]);
          }
        }
      }
    }
    // landmark bias gradient: Σ_i P (dO·v − delta) per slot
    if (!is_w && p.d_bias != nullptr && tid < BN) {
      float acc = 0.f;
      for (int r = 0; r < BM; ++r) acc += sds[r * (BN + 1) + tid];
      const int slot = key_slot[tid];
      if (slot >= 0 && acc != 0.f) atomicAdd(p.d_bias + ((int64_t)h * n_sets + set) * p.k_lmk + slot, acc);
    }
    __syncthreads();
  }
  if constexpr (TRAIN) {
    // dL/dw̃ per row: the threads sharing a row hold parts of it (tensor-core path: rows
    // 16 w + (lane >> 2) + 8 u over lanes 4k .. 4k+3; CUDA cores: rows (tid >> 3) + 16 u over
    // lanes 8k .. 8k+7)
#pragma unroll
    for (int u = 0; u < (MT != 0 ? 2 : 4); ++u) {
      float v = dw_acc[u];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if constexpr (MT == 0) v += __shfl_xor_sync(0xffffffffu, v, 4);
      const int r = MT != 0 ? 16 * (tid >> 5) + ((tid & 31) >> 2) + 8 * u : (tid >> 3) + 16 * u;
      if (MT != 0 && (tid & 3) != 0) continue;
      if ((MT != 0 || (tid & 7) == 0) && m0 + r < L && v != 0.f) atomicAdd(p.d_w + seq0 + m0 + r, v);
    }
  }
  // dQ of this thread's rows and dims
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int r = (tid >> 3) + 16 * u, d0 = tid & 7;
    const int i = m0 + r;
    if (i < L) {
      float* g = p.dq + ((seq0 + i) * (int64_t)p.H + h) * HD;
#pragma unroll
      for (int m = 0; m < HD / 8; ++m) g[d0 + 8 * m] = dq_acc[u * (HD / 8) + m];
    }
  }
}

}  // namespace bwd

// two per-sequence tables of n_seqs + 1 ints (64-query tiles, landmark sets), 256-byte aligned
size_t attention_bwd_workspace_bytes(int n_seqs) { return 2 * ((((size_t)n_seqs + 1) * 4 + 255) / 256 * 256); }

int launch_attn_bwd(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int HD,
                    int64_t q_stride, int64_t kv_stride, const void* out, int out_dtype, const void* dout,
                    int dout_dtype, const float* lse, const int32_t* w, const int32_t* lmk, const float* lmk_bias,
                    int k_lmk, int lmk_block, const int32_t* cu, int n_seqs, float* dq, float* dk, float* dv,
                    float* d_bias, void* workspace, size_t ws_bytes, cudaStream_t stream, const float* w_cont,
                    float tau, float win_edge, float* d_w) {
  using namespace bwd;
  const bool train = w_cont != nullptr;  // training mode: soft selectors (one set per sequence)
  if (train && (lmk_block != 0 || !d_w || (k_lmk > 0 && !lmk_bias)))
    return fail(DSALT_ERR_INVALID, "training attention backward: one set per sequence, log-weights and d_w needed");
  if (HD != 64 && HD != 128) return fail(DSALT_ERR_UNSUPPORTED, "attention backward: head_dim %d (64, 128)", HD);
  if (H < 1 || Hkv < 1 || H % Hkv) return fail(DSALT_ERR_INVALID, "attention backward: heads %d / kv heads %d", H, Hkv);
  if (lmk_block > 0 && lmk_block % BM)
    return fail(DSALT_ERR_UNSUPPORTED, "attention backward: lmk_block must be a multiple of %d", BM);
  if (ws_bytes < attention_bwd_workspace_bytes(n_seqs))
    return fail(DSALT_ERR_WORKSPACE, "attention backward: workspace %zu < %zu", ws_bytes,
                attention_bwd_workspace_bytes(n_seqs));
  if (T == 0 || n_seqs == 0) return DSALT_OK;
  int32_t* tile_base = reinterpret_cast<int32_t*>(workspace);
  int32_t* set_base = tile_base + ((n_seqs + 1 + 63) / 64) * 64;
  int rc;
  if ((rc = launch_chunk_table(cu, n_seqs, BM, tile_base, stream))) return rc;
  if (lmk_block > 0 && (rc = launch_chunk_table(cu, n_seqs, lmk_block, set_base, stream))) return rc;
  Params p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.dtype = dtype;
  p.H = H;
  p.Hkv = Hkv;
  p.q_stride = q_stride;
  p.kv_stride = kv_stride;
  p.out = out;
  p.out_dtype = out_dtype;
  p.dout = dout;
  p.dout_dtype = dout_dtype;
  p.lse = lse;
  p.w = w;
  p.lmk = lmk;
  p.lmk_bias = lmk_bias;
  p.k_lmk = k_lmk;
  p.lmk_block = lmk_block;
  p.cu = cu;
  p.n_seqs = n_seqs;
  p.tile_base = tile_base;
  p.set_base = set_base;
  p.scale = (float)(1.0 / sqrt((double)HD));
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.d_bias = d_bias;
  p.w_cont = w_cont;
  p.tau = tau;
  p.win_edge = win_edge;
  p.d_w = d_w;
  const int64_t max_tiles = T / BM + n_seqs;
  // tensor-core S and dP when q/k/v and dO are the same 16-bit type (their values are exact
  // as MMA operands); otherwise CUDA cores
  const int mt = (dtype == DSALT_BF16 || dtype == DSALT_F16) && dout_dtype == dtype ? dtype : 0;
  void (*kern)(const Params);
#define DSALT_BWD_PICK(HD_, TR_)                                                        \
  kern = mt == DSALT_BF16 ? attn_bwd_kernel<HD_, TR_, DSALT_BF16>                      \
                          : (mt == DSALT_F16 ? attn_bwd_kernel<HD_, TR_, DSALT_F16>    \
                                             : attn_bwd_kernel<HD_, TR_, 0>)
  if (HD == 64) {
    if (train) DSALT_BWD_PICK(64, true);
    else DSALT_BWD_PICK(64, false);
  } else {
    if (train) DSALT_BWD_PICK(128, true);
    else DSALT_BWD_PICK(128, false);
  }
#undef DSALT_BWD_PICK
  const size_t smem = HD == 64 ? Smem<64>::BYTES : Smem<128>::BYTES;
  if ((rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "attention backward smem attr")))
    return rc;
  kern<<<dim3((unsigned)max_tiles, (unsigned)H), THREADS, smem, stream>>>(p);
  return check_cuda(cudaGetLastError(), "attention backward launch");
}

}  // namespace dsalt
