// Landmark selection kernels.
//
// Whole-sequence mode follows dsalt/kernels/selectors.py:75-134 with the score of
// dsalt/kernels/landmark_tokens_ker.py:47-60: mean/std of ‖x‖ and of each kv group's
// value norm over all packed tokens, s = α·z_v + (1−α)·z_x, tokens inside their own
// window (seq_off < w) excluded, top-k per (head, sequence).
//
// Block-causal mode follows results/causal_landmark_check.py:82-113 (driven per block at
// :176-186): for block b of a sequence the candidates are positions [0, b·B) and the
// statistics are those of that prefix (float64 mean, unbiased std, clamp 1e-6; z cast to
// fp32); blocks with fewer than two prefix tokens select nothing.
//
// Exactness: sums are double-double (the correctly rounded float64 of the exact sum);
// every other op replays the reference's IEEE op chain; ties go to the lower position.
//
// Block-causal pruning (exact): a candidate j is never among the top-k of any block if at
// least k uncovered tokens i < j have strictly larger value norm AND strictly larger
// x-norm — the fp32 score is non-decreasing in both signals for α ∈ [0,1], and ties go to
// the lower position. Tokens are binned on a 32x32 grid of thresholds; per block-sized
// chunk a 2-D suffix histogram of earlier chunks gives a lower bound on that count, and
// only tokens whose bound is < k remain candidates (a few thousand of 131072 on random
// inputs). Heads whose α is outside [0,1] skip the pruning.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace dsalt {

constexpr int NBIN = 32;                 // bins per signal for the dominance grid
constexpr int NCELL = NBIN * NBIN;
static_assert(NBIN == 32, "the dominance grid scans assume one bin per lane");
constexpr int GCHUNK = 4096;             // positions per CTA in whole-sequence phase 1
constexpr int STAT_CHUNK = 512;          // tokens per partial sum in whole-sequence mode
constexpr int SEL_THREADS = 512;
constexpr int KEY_CAP = 8192;            // candidate keys cached in shared memory
constexpr int BSEL_THREADS = 256;        // block-causal select: small CTAs, several per SM
constexpr int BSEL_KEY_CAP = 1536;       // its key cache (the prefix-dominance filter keeps ~1K)
constexpr int MAX_K = 1024;

// thresholds (in units of the sequence's std above its mean) of the dominance grid:
// coarse below the mean, fine in the upper tail where the top-k lives.
__constant__ float c_bin_t[NBIN - 1];

// ---------------------------------------------------------------------------
// sequence tables
// ---------------------------------------------------------------------------
__device__ __forceinline__ int find_seq(const int32_t* base, int n_seqs, int idx) {
  int lo = 0, hi = n_seqs;  // base[0] = 0 <= idx < base[n_seqs]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (base[mid] <= idx) lo = mid;
    else hi = mid;
  }
  return lo;
}

// base[s] = Σ_{s'<s} ceil(L_s'/C); one CTA.
__global__ void chunk_table_kernel(const int32_t* __restrict__ cu, int n_seqs, int C, int32_t* __restrict__ base) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int s0 = 0; s0 < n_seqs; s0 += blockDim.x) {
    const int s = s0 + threadIdx.x;
    int v = 0;
    if (s < n_seqs) {
      int L = cu[s + 1] - cu[s];
      v = L > 0 ? (L + C - 1) / C : 0;
    }
    // block inclusive scan
    int x = v;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int t = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      warp_tot[lane] = t;
    }
    __syncthreads();
    const int excl = carry + (wid ? warp_tot[wid - 1] : 0) + x - v;
    if (s < n_seqs) base[s] = excl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) base[n_seqs] = carry;
}

int launch_chunk_table(const int32_t* cu, int n_seqs, int C, int32_t* base, cudaStream_t stream) {
  chunk_table_kernel<<<1, 1024, 0, stream>>>(cu, n_seqs, C, base);
  return check_cuda(cudaGetLastError(), "sequence table launch");
}

// ---------------------------------------------------------------------------
// per-chunk double-double sums of each signal and of its square
// signal 0 = ‖x‖, signal 1+g = value norm of kv group g
// ---------------------------------------------------------------------------
struct Partial {
  double s1h, s1l, s2h, s2l;
};

__device__ __forceinline__ DD block_dd_sum(DD v, DD* red) {
  v = dd_warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  DD r = DD{0.0, 0.0};
  if (wid == 0) {
    r = lane < nw ? red[lane] : DD{0.0, 0.0};
    r = dd_warp_sum(r);
  }
  return r;  // valid in thread 0
}

// one warp per (chunk, signal): the double-double reduction is the costly part (fp64
// bound), so it runs once per warp rather than across a whole block
__global__ void __launch_bounds__(256) chunk_sums_kernel(const float* __restrict__ xn, const float* __restrict__ vn,
                                                         int n_kv, const int32_t* __restrict__ cu, int n_seqs,
                                                         const int32_t* __restrict__ base, int C, int n_chunks,
                                                         Partial* __restrict__ part, int c_lo = 0) {
  const int nsig = 1 + n_kv;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= (int64_t)n_chunks * nsig) return;
  const int c = c_lo + (int)(wid / nsig), sig = (int)(wid % nsig);
  const int total = base[n_seqs];
  Partial out{0.0, 0.0, 0.0, 0.0};
  if (c < total) {
    const int s = find_seq(base, n_seqs, c);
    const int lc = c - base[s];
    const int a = cu[s] + lc * C;
    const int b = min(cu[s + 1], a + C);
    DD s1{0.0, 0.0}, s2{0.0, 0.0};
    for (int t = a + lane; t < b; t += 32) {
      const double v = (double)(sig == 0 ? xn[t] : vn[(int64_t)t * n_kv + sig - 1]);
      s1 = dd_add_d(s1, v);
      s2 = dd_add_d(s2, __dmul_rn(v, v));  // exact: the square of an fp32 value fits a double
    }
    s1 = dd_warp_sum(s1);
    s2 = dd_warp_sum(s2);
    out = Partial{s1.hi, s1.lo, s2.hi, s2.lo};
  }
  if (lane == 0) part[(int64_t)c * nsig + sig] = out;
}

// ---------------------------------------------------------------------------
// whole-sequence statistics: fp32 mean and unbiased std (clamp 1e-6) over all T tokens
//   mean = fl32(S1/n); var = (S2 − (S1/n)·S1)/(n−1); std = fl32(sqrt(var))
// ---------------------------------------------------------------------------
__global__ void global_stats_kernel(const Partial* __restrict__ part, int n_chunks, int nsig, int64_t T,
                                    float* __restrict__ gstats) {
  __shared__ DD red1[32], red2[32];
  const int sig = blockIdx.x;
  DD s1{0.0, 0.0}, s2{0.0, 0.0};
  for (int c = threadIdx.x; c < n_chunks; c += blockDim.x) {
    const Partial p = part[(int64_t)c * nsig + sig];
    s1 = dd_add(s1, DD{p.s1h, p.s1l});
    s2 = dd_add(s2, DD{p.s2h, p.s2l});
  }
  DD r1 = block_dd_sum(s1, red1);
  DD r2 = block_dd_sum(s2, red2);
  if (threadIdx.x == 0) {
    const double S1 = dd_round(r1), S2 = dd_round(r2);
    const double n = (double)T;
    const double m64 = __ddiv_rn(S1, n);
    float stdv;
    if (T > 1) {
      const double var = __ddiv_rn(__dsub_rn(S2, __dmul_rn(m64, S1)), __dsub_rn(n, 1.0));
      stdv = __double2float_rn(__dsqrt_rn(var > 0.0 ? var : 0.0));
      stdv = fmaxf(stdv, 1e-6f);
    } else {
      stdv = __int_as_float(0x7fc00000);  // torch.std of one element is NaN
    }
    gstats[2 * sig] = __double2float_rn(m64);
    gstats[2 * sig + 1] = stdv;
  }
}

// ---------------------------------------------------------------------------
// block-wide top-k over 64-bit keys (0 = not a candidate), MSB-first radix select
// ---------------------------------------------------------------------------
struct TopkSmem {
  unsigned int hist[256];
  uint64_t prefix, mask;
  int kk, done, cnt, all;
};

template <class Get>
__device__ void block_topk_select(Get get, int N, int k, TopkSmem& sm, uint64_t& prefix_out, uint64_t& mask_out) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    sm.prefix = 0;
    sm.mask = 0;
    sm.kk = k;
    sm.done = 0;
    sm.all = 0;
  }
  __syncthreads();
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) sm.hist[i] = 0;
    __syncthreads();
    const uint64_t prefix = sm.prefix, mask = sm.mask;
    for (int i = tid; i < N; i += blockDim.x) {
      const uint64_t key = get(i);
      if (key != 0 && (key & mask) == prefix) atomicAdd(&sm.hist[(key >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (tid < 32) {
      const int lane = tid;
      unsigned int s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += sm.hist[255 - 8 * lane - j];
      unsigned int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        unsigned int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned int total = __shfl_sync(0xffffffffu, incl, 31);
      const int kk = sm.kk;
      if (total <= (unsigned)kk) {
        // every remaining candidate is selected
        if (lane == 0) {
          sm.done = 1;
          if (shift == 56) sm.all = 1;
        }
      } else {
        const unsigned ball = __ballot_sync(0xffffffffu, incl >= (unsigned)kk);
        const int L = __ffs(ball) - 1;
        if (lane == L) {
          unsigned int cum = incl - s;
          int d = 0;
          unsigned int above = cum;
#pragma unroll 1
          for (int j = 0; j < 8; ++j) {
            const int bin = 255 - 8 * lane - j;
            const unsigned int h = sm.hist[bin];
            if (cum + h >= (unsigned)kk) {
              d = bin;
              above = cum;
              break;
            }
            cum += h;
          }
          const int nk = kk - (int)above;
          sm.kk = nk;
          sm.prefix = prefix | ((uint64_t)d << shift);
          sm.mask = mask | ((uint64_t)0xFF << shift);
          if (sm.hist[d] == (unsigned)nk) sm.done = 1;
        }
      }
    }
    __syncthreads();
    if (sm.done) break;
  }
  prefix_out = sm.prefix;
  mask_out = sm.mask;
}

__device__ __forceinline__ bool topk_selected(uint64_t key, uint64_t prefix, uint64_t mask) {
  return key != 0 && (key & mask) >= prefix;
}

// emits the selected positions ascending, -1 padded to k
template <class Get>
__device__ void block_topk_positions(Get get, int N, int k, TopkSmem& sm, int32_t* sel, int32_t* __restrict__ out) {
  uint64_t prefix, mask;
  block_topk_select(get, N, k, sm, prefix, mask);
  if (threadIdx.x == 0) sm.cnt = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const uint64_t key = get(i);
    if (topk_selected(key, prefix, mask)) {
      const int slot = atomicAdd(&sm.cnt, 1);
      if (slot < k) sel[slot] = key_pos(key);
    }
  }
  __syncthreads();
  const int cnt = min(sm.cnt, k);
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    if (j < cnt) {
      const int p = sel[j];
      int rank = 0;
      for (int m = 0; m < cnt; ++m) rank += sel[m] < p;
      out[rank] = p;
    } else {
      out[j] = -1;
    }
  }
  __syncthreads();
}

// emits the selected keys (unordered), 0 padded to k
template <class Get>
__device__ void block_topk_keys(Get get, int N, int k, TopkSmem& sm, uint64_t* __restrict__ out) {
  uint64_t prefix, mask;
  block_topk_select(get, N, k, sm, prefix, mask);
  if (threadIdx.x == 0) sm.cnt = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const uint64_t key = get(i);
    if (topk_selected(key, prefix, mask)) {
      const int slot = atomicAdd(&sm.cnt, 1);
      if (slot < k) out[slot] = key;
    }
  }
  __syncthreads();
  const int cnt = min(sm.cnt, k);
  for (int j = cnt + threadIdx.x; j < k; j += blockDim.x) out[j] = 0;
  __syncthreads();
}

// fp32 score of the whole-sequence mode (landmark_tokens_ker.py:47-60)
__device__ __forceinline__ float global_score(float xnv, float vnv, float mx, float sx, float mv, float sv, float a) {
  const float zx = __fdiv_rn(__fsub_rn(xnv, mx), sx);
  const float zv = __fdiv_rn(__fsub_rn(vnv, mv), sv);
  return __fadd_rn(__fmul_rn(a, zv), __fmul_rn(__fsub_rn(1.0f, a), zx));
}

// ---------------------------------------------------------------------------
// whole-sequence phase 1: per (chunk of GCHUNK positions, head) local top-k keys
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(SEL_THREADS) global_phase1_kernel(
    const float* __restrict__ xn, const float* __restrict__ vn, const int32_t* __restrict__ w,
    const float* __restrict__ alpha, const float* __restrict__ gstats, const int32_t* __restrict__ cu, int n_seqs,
    const int32_t* __restrict__ gbase, int n_heads, int n_kv, int k, uint64_t* __restrict__ cand, float* zx_out,
    float* zv_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem_raw);
  __shared__ TopkSmem sm;
  const int gc = blockIdx.x, h = blockIdx.y;
  const int total = gbase[n_seqs];
  uint64_t* out = cand + ((int64_t)h * gridDim.x + gc) * k;
  if (gc >= total) {
    for (int j = threadIdx.x; j < k; j += blockDim.x) out[j] = 0;
    return;
  }
  const int s = find_seq(gbase, n_seqs, gc);
  const int start = cu[s];
  const int p0 = (gc - gbase[s]) * GCHUNK;
  const int p1 = min(cu[s + 1] - start, p0 + GCHUNK);
  const int N = p1 - p0;
  const int rep = n_heads / n_kv, g = h / rep;
  const float mx = gstats[0], sx = gstats[1], mv = gstats[2 * (1 + g)], sv = gstats[2 * (1 + g) + 1];
  const float a = alpha[h];
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const int p = p0 + i;
    const int64_t t = start + p;
    const float xv = xn[t], vv = vn[t * n_kv + g];
    const float sc = global_score(xv, vv, mx, sx, mv, sv, a);
    keys[i] = (p < w[t]) ? 0ull : make_key(sc, p);
    if (h == 0 && zx_out) zx_out[t] = __fdiv_rn(__fsub_rn(xv, mx), sx);
    if (h % rep == 0 && zv_out) zv_out[t * n_kv + g] = __fdiv_rn(__fsub_rn(vv, mv), sv);
  }
  __syncthreads();
  block_topk_keys([&](int i) { return keys[i]; }, N, k, sm, out);
}

// whole-sequence phase 2: merge the phase-1 keys of a sequence
__global__ void __launch_bounds__(SEL_THREADS) global_phase2_kernel(const uint64_t* __restrict__ cand, int n_gchunks_alloc,
                                                                    const int32_t* __restrict__ gbase, int n_seqs,
                                                                    int k, int32_t* __restrict__ lmk_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem_raw);
  __shared__ TopkSmem sm;
  __shared__ int32_t sel[MAX_K];
  const int s = blockIdx.x, h = blockIdx.y;
  const int c0 = gbase[s], c1 = gbase[s + 1];
  const int N = (c1 - c0) * k;
  const uint64_t* src = cand + ((int64_t)h * n_gchunks_alloc + c0) * k;
  int32_t* out = lmk_out + ((int64_t)h * n_seqs + s) * k;
  if (N <= KEY_CAP) {
    for (int i = threadIdx.x; i < N; i += blockDim.x) keys[i] = src[i];
    __syncthreads();
    block_topk_positions([&](int i) { return keys[i]; }, N, k, sm, sel, out);
  } else {
    block_topk_positions([&](int i) { return src[i]; }, N, k, sm, sel, out);
  }
}

// fp32 of the correctly rounded float64 quotient (v - mean) / sd, as the reference's
// float64 z-score cast to float32 (causal_landmark_check.py:104-105). The quotient is taken
// as (v - mean) * (1/sd), within 2 float64 ulps of the correctly rounded one; unless that
// lies within 4 ulps of a float32 rounding boundary (the 29 dropped mantissa bits close to
// their midpoint), both round to the same float32. Otherwise, and for tiny quotients, the
// exact division decides.
__device__ __forceinline__ float z_score(float v, double mean, double sd, double rinv) {
  const double d = __dsub_rn((double)v, mean);
  const double q = __dmul_rn(d, rinv);
  const long long bits = __double_as_longlong(q);
  const long long dropped = bits & ((1ll << 29) - 1);
  const long long dist = dropped - (1ll << 28);
  if ((dist > 4 || dist < -4) && fabs(q) > 1e-30) return __double2float_rn(q);
  return __double2float_rn(__ddiv_rn(d, sd));
}

// ---------------------------------------------------------------------------
// block-causal: prefix statistics per block and dominance-grid thresholds
// stats[set][sig] = (mean, sd) float64 of positions [0, b·C) (_std_at,
// causal_landmark_check.py:88-92); edges from the whole sequence's statistics.
// ---------------------------------------------------------------------------
__global__ void block_stats_kernel(const Partial* __restrict__ part, const int32_t* __restrict__ cu, int n_seqs,
                                   const int32_t* __restrict__ base, int nsig, int C, double2* __restrict__ stats,
                                   float* __restrict__ edges) {
  __shared__ DD sc1[256], sc2[256];
  __shared__ DD carry1, carry2;
  const int s = blockIdx.x, sig = blockIdx.y;
  const int c0 = base[s], nc = base[s + 1] - c0;
  const int L = cu[s + 1] - cu[s];
  if (threadIdx.x == 0) {
    carry1 = DD{0.0, 0.0};
    carry2 = DD{0.0, 0.0};
  }
  __syncthreads();
  for (int t0 = 0; t0 < nc; t0 += 256) {
    const int b = t0 + threadIdx.x;
    DD v1{0.0, 0.0}, v2{0.0, 0.0};
    if (b < nc) {
      const Partial p = part[(int64_t)(c0 + b) * nsig + sig];
      v1 = DD{p.s1h, p.s1l};
      v2 = DD{p.s2h, p.s2l};
    }
    sc1[threadIdx.x] = v1;
    sc2[threadIdx.x] = v2;
    __syncthreads();
    // Hillis-Steele inclusive scan
    for (int off = 1; off < 256; off <<= 1) {
      DD a1 = sc1[threadIdx.x], a2 = sc2[threadIdx.x];
      if (threadIdx.x >= off) {
        a1 = dd_add(a1, sc1[threadIdx.x - off]);
        a2 = dd_add(a2, sc2[threadIdx.x - off]);
      }
      __syncthreads();
      sc1[threadIdx.x] = a1;
      sc2[threadIdx.x] = a2;
      __syncthreads();
    }
    if (b < nc) {
      // exclusive prefix = carry + inclusive(b-1)
      DD e1 = carry1, e2 = carry2;
      if (threadIdx.x > 0) {
        e1 = dd_add(e1, sc1[threadIdx.x - 1]);
        e2 = dd_add(e2, sc2[threadIdx.x - 1]);
      }
      const int n = b * C;
      double2 st = make_double2(__int_as_float(0x7fc00000), 0.0);
      if (n >= 2) {
        const double S1 = dd_round(e1), S2 = dd_round(e2);
        const double dn = (double)n;
        const double mean = __ddiv_rn(S1, dn);
        const double var = __ddiv_rn(__dsub_rn(S2, __dmul_rn(__dmul_rn(dn, mean), mean)), (double)max(n - 1, 1));
        double sd = __dsqrt_rn(var > 0.0 ? var : 0.0);
        sd = sd > 1e-6 ? sd : 1e-6;
        st = make_double2(mean, sd);
      }
      stats[(int64_t)(c0 + b) * nsig + sig] = st;
    }
    __syncthreads();
    if (threadIdx.x == 255) {
      carry1 = dd_add(carry1, sc1[255]);
      carry2 = dd_add(carry2, sc2[255]);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    // whole-sequence mean / std: only used to place the dominance-grid thresholds
    const double n = (double)max(L, 1);
    const double S1 = dd_round(carry1), S2 = dd_round(carry2);
    const double mean = S1 / n;
    double var = (S2 - n * mean * mean) / fmax(n - 1.0, 1.0);
    const double sd = sqrt(var > 0.0 ? var : 0.0);
    for (int j = 0; j < NBIN - 1; ++j) edges[((int64_t)s * nsig + sig) * (NBIN - 1) + j] = (float)(mean + sd * c_bin_t[j]);
  }
}

// number of the NBIN-1 ascending thresholds e[j] <= v (binary search)
__device__ __forceinline__ int bin_of(float v, const float* e) {
  int b = 0;
#pragma unroll
  for (int step = NBIN / 2; step > 0; step >>= 1)
    if (b + step - 1 < NBIN - 1 && e[b + step - 1] <= v) b += step;
  return b;
}

// per (chunk, kv group): 2-D suffix histogram G[a][b] = #uncovered tokens of the chunk
// with value bin >= a and x bin >= b
__global__ void __launch_bounds__(256) dominance_hist_kernel(
    const float* __restrict__ xn, const float* __restrict__ vn, const int32_t* __restrict__ w, int n_kv,
    const int32_t* __restrict__ cu, int n_seqs, const int32_t* __restrict__ base, int C,
    const float* __restrict__ edges, int32_t* __restrict__ G) {
  __shared__ int32_t hist[NCELL];
  __shared__ float ex[NBIN - 1], ev[NBIN - 1];
  const int c = blockIdx.x, g = blockIdx.y, nsig = 1 + n_kv;
  const int total = base[n_seqs];
  int32_t* out = G + ((int64_t)c * n_kv + g) * NCELL;
  if (c >= total) return;
  const int s = find_seq(base, n_seqs, c);
  for (int i = threadIdx.x; i < NCELL; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x < NBIN - 1) {
    ex[threadIdx.x] = edges[((int64_t)s * nsig + 0) * (NBIN - 1) + threadIdx.x];
    ev[threadIdx.x] = edges[((int64_t)s * nsig + 1 + g) * (NBIN - 1) + threadIdx.x];
  }
  __syncthreads();
  const int start = cu[s];
  const int p0 = (c - base[s]) * C;
  const int p1 = min(cu[s + 1] - start, p0 + C);
  // tokens of a chunk cluster in few cells: one shared-memory atomic per distinct cell
  // and warp
  for (int p0w = p0; p0w < p1; p0w += blockDim.x) {
    const int p = p0w + threadIdx.x;
    int cell = -1;
    if (p < p1) {
      const int64_t t = start + p;
      if (p >= w[t]) cell = bin_of(vn[t * n_kv + g], ev) * NBIN + bin_of(xn[t], ex);
    }
    const unsigned same = __match_any_sync(0xffffffffu, cell);
    if (cell >= 0 && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[cell], __popc(same));
  }
  __syncthreads();
  // 2-D suffix sums, one warp-wide scan per row then per column (lane = bin)
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int row = wid; row < NBIN; row += nw) {  // along x bins
    int v = hist[row * NBIN + lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += y;
    }
    hist[row * NBIN + lane] = v;
  }
  __syncthreads();
  for (int col = wid; col < NBIN; col += nw) {  // along value bins
    int v = hist[lane * NBIN + col];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += y;
    }
    hist[lane * NBIN + col] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NCELL; i += blockDim.x) out[i] = hist[i];
}

// The same grids for gpb kv groups of a chunk per 512-thread CTA (n_kv <= 32): the token
// loads, ‖x‖ bins and coverage tests are shared by the CTA's groups. Shared memory: gpb
// 32×32 grids + edges.
__global__ void __launch_bounds__(512) dominance_hist_all_kernel(
    const float* __restrict__ xn, const float* __restrict__ vn, const int32_t* __restrict__ w, int n_kv,
    const int32_t* __restrict__ cu, int n_seqs, const int32_t* __restrict__ base, int C,
    const float* __restrict__ edges, int32_t* __restrict__ G, int gpb, int c_lo = 0) {
  // grids with rows padded to NBIN+1 entries, so that column scans hit distinct banks
  constexpr int RS = NBIN + 1;
  extern __shared__ int32_t hs[];
  // this CTA: kv groups [g0, g0 + gpb) of chunk c_lo + blockIdx.x
  int32_t* hist = hs;                                            // [gpb][NBIN][RS]
  float* ev = reinterpret_cast<float*>(hs + gpb * NBIN * RS);    // [gpb][NBIN-1]
  __shared__ float ex[NBIN - 1];
  const int c = c_lo + blockIdx.x, nsig = 1 + n_kv, g0 = blockIdx.y * gpb;
  const int total = base[n_seqs];
  if (c >= total) return;
  const int s = find_seq(base, n_seqs, c);
  for (int i = threadIdx.x; i < gpb * NBIN * RS; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x < NBIN - 1) ex[threadIdx.x] = edges[((int64_t)s * nsig + 0) * (NBIN - 1) + threadIdx.x];
  for (int i = threadIdx.x; i < gpb * (NBIN - 1); i += blockDim.x)
    ev[i] = edges[((int64_t)s * nsig + 1 + g0) * (NBIN - 1) + i];  // groups are consecutive
  __syncthreads();
  const int start = cu[s];
  const int p0 = (c - base[s]) * C;
  const int p1 = min(cu[s + 1] - start, p0 + C);
  for (int p0w = p0; p0w < p1; p0w += blockDim.x) {
    const int p = p0w + threadIdx.x;
    const int64_t t = start + p;
    const bool live = p < p1 && p >= w[t];
    const int bx = live ? bin_of(xn[t], ex) : 0;
    for (int g = 0; g < gpb; ++g) {
      const int cell = live ? (g * NBIN + bin_of(vn[t * n_kv + g0 + g], ev + g * (NBIN - 1))) * RS + bx : -1;
      const unsigned same = __match_any_sync(0xffffffffu, cell);
      if (cell >= 0 && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[cell], __popc(same));
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int row = wid; row < gpb * NBIN; row += nw) {  // suffix along x bins, row = (g, value bin)
    int v = hist[row * RS + lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += y;
    }
    hist[row * RS + lane] = v;
  }
  __syncthreads();
  for (int col = wid; col < gpb * NBIN; col += nw) {  // suffix along value bins, col = (g, x bin)
    const int g = col / NBIN, b = col % NBIN;
    int v = hist[(g * NBIN + lane) * RS + b];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += y;
    }
    hist[(g * NBIN + lane) * RS + b] = v;
  }
  __syncthreads();
  int32_t* out = G + ((int64_t)c * n_kv + g0) * NCELL;
  for (int i = threadIdx.x; i < gpb * NCELL; i += blockDim.x) out[i] = hist[(i / NBIN) * RS + (i % NBIN)];
}

// exclusive prefix over the chunks of each sequence, in place: G[c] <- Σ_{c'<c} G[c'].
// Two passes over segments of SCAN_SEG chunks: segment totals, then each segment's scan
// started from the sum of the totals before it (more independent chains in flight).
constexpr int SCAN_SEG = 16;
constexpr int SEG_SCAN_MAX_SEQS = 16;  // segment totals are kept per sequence

// single pass (packed inputs with many sequences): one thread per (sequence, group, cell)
__global__ void dominance_scan_serial_kernel(int32_t* __restrict__ G, const int32_t* __restrict__ base, int n_kv) {
  const int s = blockIdx.x / n_kv, g = blockIdx.x % n_kv;
  const int cell = blockIdx.y * blockDim.x + threadIdx.x;
  if (cell >= NCELL) return;
  int run = 0;
  const int c_end = base[s + 1];
  const int64_t stride = (int64_t)n_kv * NCELL;
  for (int c0 = base[s]; c0 < c_end; c0 += 16) {
    int32_t* p = G + ((int64_t)c0 * n_kv + g) * NCELL + cell;
    int v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = c0 + j < c_end ? p[j * stride] : 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (c0 + j < c_end) p[j * stride] = run;
      run += v[j];
    }
  }
}

__global__ void dominance_segsum_kernel(const int32_t* __restrict__ G, const int32_t* __restrict__ base, int n_seqs,
                                        int n_kv, int max_segs, int32_t* __restrict__ segsum) {
  const int s = blockIdx.x / n_kv, g = blockIdx.x % n_kv;
  const int cell = threadIdx.x + blockIdx.z * blockDim.x;
  const int seg = blockIdx.y;
  const int c0 = base[s] + seg * SCAN_SEG, c_end = base[s + 1];
  if (cell >= NCELL) return;
  int v = 0;
  if (c0 < c_end) {
    const int64_t stride = (int64_t)n_kv * NCELL;
    const int32_t* p = G + ((int64_t)c0 * n_kv + g) * NCELL + cell;
#pragma unroll
    for (int j = 0; j < SCAN_SEG; ++j) v += c0 + j < c_end ? p[j * stride] : 0;
  }
  segsum[(((int64_t)s * n_kv + g) * max_segs + seg) * NCELL + cell] = v;
}

__global__ void dominance_scan_kernel(int32_t* __restrict__ G, const int32_t* __restrict__ base, int n_kv,
                                      int max_segs, const int32_t* __restrict__ segsum) {
  const int s = blockIdx.x / n_kv, g = blockIdx.x % n_kv;
  const int cell = threadIdx.x + blockIdx.z * blockDim.x;
  const int seg = blockIdx.y;
  if (cell >= NCELL) return;
  const int c0 = base[s] + seg * SCAN_SEG, c_end = base[s + 1];
  if (c0 >= c_end) return;
  int run = 0;
  const int32_t* ss = segsum + ((int64_t)s * n_kv + g) * max_segs * NCELL + cell;
  for (int q = 0; q < seg; ++q) run += ss[(int64_t)q * NCELL];
  const int64_t stride = (int64_t)n_kv * NCELL;
  int32_t* p = G + ((int64_t)c0 * n_kv + g) * NCELL + cell;
  int v[SCAN_SEG];
#pragma unroll
  for (int j = 0; j < SCAN_SEG; ++j) v[j] = c0 + j < c_end ? p[j * stride] : 0;
#pragma unroll
  for (int j = 0; j < SCAN_SEG; ++j) {
    if (c0 + j < c_end) p[j * stride] = run;
    run += v[j];
  }
}

// survivors: uncovered tokens dominated (strictly, in both signals) by fewer than k
// uncovered tokens of earlier chunks; written in position order per (chunk, group) as
// records {position, ‖x‖, value norm of the group, dominance cell}, the cell being the
// grid index whose prefix count bounds the token's dominators from below (-1: none can
// dominate it)
__global__ void survivor_kernel(const float* __restrict__ xn, const float* __restrict__ vn,
                                const int32_t* __restrict__ w, int n_kv, const int32_t* __restrict__ cu, int n_seqs,
                                const int32_t* __restrict__ base, int C, const float* __restrict__ edges,
                                const int32_t* __restrict__ D, int k, int32_t* __restrict__ surv_cnt,
                                int4* __restrict__ surv_rec) {
  __shared__ float ex[NBIN - 1], ev[NBIN - 1];
  __shared__ int32_t wsum[32];
  const int c = blockIdx.x, g = blockIdx.y, nsig = 1 + n_kv;
  const int total = base[n_seqs];
  if (c >= total) return;
  const int s = find_seq(base, n_seqs, c);
  if (threadIdx.x < NBIN - 1) {
    ex[threadIdx.x] = edges[((int64_t)s * nsig + 0) * (NBIN - 1) + threadIdx.x];
    ev[threadIdx.x] = edges[((int64_t)s * nsig + 1 + g) * (NBIN - 1) + threadIdx.x];
  }
  __syncthreads();
  const int start = cu[s];
  const int p0 = (c - base[s]) * C;
  const int p1 = min(cu[s + 1] - start, p0 + C);
  const int32_t* Dc = D + ((int64_t)c * n_kv + g) * NCELL;
  int4* outp = surv_rec + ((int64_t)c * n_kv + g) * C;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int carry = 0;
  for (int q0 = p0; q0 < p1; q0 += blockDim.x) {
    const int p = q0 + threadIdx.x;
    int keep = 0;
    int4 rec;
    if (p < p1) {
      const int64_t t = start + p;
      if (p >= w[t]) {
        const float xv = xn[t], vv = vn[t * n_kv + g];
        const int a = bin_of(vv, ev), b = bin_of(xv, ex);
        const int cell = (a == NBIN - 1 || b == NBIN - 1) ? -1 : (a + 1) * NBIN + (b + 1);
        const int dom = cell < 0 ? 0 : Dc[cell];
        keep = dom < k;
        rec = make_int4(p, __float_as_int(xv), __float_as_int(vv), cell);
      }
    }
    const unsigned ball = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) wsum[wid] = __popc(ball);
    __syncthreads();
    int before = carry;
    for (int j = 0; j < wid; ++j) before += wsum[j];
    before += __popc(ball & ((1u << lane) - 1));
    if (keep) outp[before] = rec;
    int tot = 0;
    for (int j = 0; j < nw; ++j) tot += wsum[j];
    carry += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) surv_cnt[(int64_t)c * n_kv + g] = carry;
}

// survivor_kernel for gpb kv groups of a chunk per 512-thread CTA (n_kv <= 32); the
// records of a (chunk, group) are compacted in no particular order (the selection does not
// depend on it)
__global__ void __launch_bounds__(512) survivor_all_kernel(
    const float* __restrict__ xn, const float* __restrict__ vn, const int32_t* __restrict__ w, int n_kv,
    const int32_t* __restrict__ cu, int n_seqs, const int32_t* __restrict__ base, int C,
    const float* __restrict__ edges, const int32_t* __restrict__ D, int k, int32_t* __restrict__ surv_cnt,
    int4* __restrict__ surv_rec, int gpb, int c_lo = 0) {
  extern __shared__ float es[];  // [gpb][NBIN-1]
  __shared__ float ex[NBIN - 1];
  __shared__ int32_t cnt[32];
  const int c = c_lo + blockIdx.x, nsig = 1 + n_kv, g0 = blockIdx.y * gpb;
  const int total = base[n_seqs];
  if (c >= total) return;
  const int s = find_seq(base, n_seqs, c);
  if (threadIdx.x < NBIN - 1) ex[threadIdx.x] = edges[((int64_t)s * nsig + 0) * (NBIN - 1) + threadIdx.x];
  for (int i = threadIdx.x; i < gpb * (NBIN - 1); i += blockDim.x)
    es[i] = edges[((int64_t)s * nsig + 1 + g0) * (NBIN - 1) + i];
  if (threadIdx.x < 32) cnt[threadIdx.x] = 0;
  __syncthreads();
  const int start = cu[s];
  const int p0 = (c - base[s]) * C;
  const int p1 = min(cu[s + 1] - start, p0 + C);
  const int lane = threadIdx.x & 31;
  for (int p0w = p0; p0w < p1; p0w += blockDim.x) {
    const int p = p0w + threadIdx.x;
    const int64_t t = start + p;
    const bool live = p < p1 && p >= w[t];
    const float xv = live ? xn[t] : 0.0f;
    const int bx = live ? bin_of(xv, ex) : 0;
    for (int gl = 0; gl < gpb; ++gl) {
      const int g = g0 + gl;
      bool keep = false;
      int4 rec;
      if (live) {
        const float vv = vn[t * n_kv + g];
        const int a = bin_of(vv, es + gl * (NBIN - 1));
        const int cell = (a == NBIN - 1 || bx == NBIN - 1) ? -1 : (a + 1) * NBIN + (bx + 1);
        const int dom = cell < 0 ? 0 : D[((int64_t)c * n_kv + g) * NCELL + cell];
        keep = dom < k;
        rec = make_int4(p, __float_as_int(xv), __float_as_int(vv), cell);
      }
      const unsigned ball = __ballot_sync(0xffffffffu, keep);
      int slot0 = 0;
      if (lane == 0 && ball) slot0 = atomicAdd(&cnt[gl], __popc(ball));
      slot0 = __shfl_sync(0xffffffffu, slot0, 0);
      if (keep) surv_rec[((int64_t)c * n_kv + g) * C + slot0 + __popc(ball & ((1u << lane) - 1))] = rec;
    }
  }
  __syncthreads();
  if (threadIdx.x < gpb) surv_cnt[(int64_t)c * n_kv + g0 + threadIdx.x] = cnt[threadIdx.x];
}

// Packs every kv group's survivor records in chunk order, so that a block's candidates (the
// survivors of its sequence's earlier chunks) form one contiguous run: poff[c][g] = records of
// group g in chunks [0, c) (all sequences in turn; entry n_chunks holds the total), then a
// copy of each (chunk, group) list to its offset. n_chunks < 0: every chunk of the tables.
__global__ void __launch_bounds__(1024) survivor_offsets_kernel(const int32_t* __restrict__ cnt, int n_kv,
                                                                 const int32_t* __restrict__ base, int n_seqs,
                                                                 int n_chunks, int32_t* __restrict__ poff) {
  __shared__ int32_t wsum[32];
  const int g = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int nc = n_chunks >= 0 ? n_chunks : base[n_seqs];
  int carry = 0;
  for (int c0 = 0; c0 < nc; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    const int v = c < nc ? cnt[(int64_t)c * n_kv + g] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[wid] = x;
    __syncthreads();
    int before = carry, tot = 0;
    for (int q = 0; q < nw; ++q) {
      if (q < wid) before += wsum[q];
      tot += wsum[q];
    }
    if (c < nc) poff[(int64_t)c * n_kv + g] = before + x - v;
    carry += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) poff[(int64_t)nc * n_kv + g] = carry;
}

__global__ void pack_survivors_kernel(const int32_t* __restrict__ cnt, const int4* __restrict__ recs,
                                      const int32_t* __restrict__ poff, int n_kv, int C,
                                      const int32_t* __restrict__ base, int n_seqs, int n_chunks,
                                      int4* __restrict__ packed, int64_t rec_stride) {
  const int c = blockIdx.x, g = blockIdx.y;
  const int nc = n_chunks >= 0 ? n_chunks : base[n_seqs];
  if (c >= nc) return;
  const int64_t cg = (int64_t)c * n_kv + g;
  const int n = cnt[cg];
  const int4* src = recs + cg * C;
  int4* dst = packed + (int64_t)g * rec_stride + poff[cg];
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}


// per (block set, head): exact scores of the surviving candidates of earlier chunks
__global__ void __launch_bounds__(BSEL_THREADS, 6) block_select_kernel(
    const float* __restrict__ xn, const float* __restrict__ vn, const int32_t* __restrict__ w,
    const float* __restrict__ alpha, const int32_t* __restrict__ cu, int n_seqs, const int32_t* __restrict__ base,
    int C, int n_heads, int n_kv, int k, const double2* __restrict__ stats, const int32_t* __restrict__ D,
    const int32_t* __restrict__ poff, const int4* __restrict__ packed, int64_t rec_stride, int32_t* __restrict__ lmk_out,
    int set_lo, int n_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem_raw);
  __shared__ TopkSmem sm;
  __shared__ int32_t sel[MAX_K];
  __shared__ int32_t dsm[NCELL];
  __shared__ int32_t ncand;
  // sets set_lo + blockIdx.x; output [H, n_out, k] (n_out = all sets, or the range's)
  const int c = set_lo + blockIdx.x, h = blockIdx.y;
  const int total = base[n_seqs];
  if (c >= total) return;
  int32_t* out = lmk_out + ((int64_t)h * (n_out > 0 ? n_out : total) + (c - set_lo)) * k;
  const int s = find_seq(base, n_seqs, c);
  const int b = c - base[s];
  const int n = b * C;
  if (n < 2) {
    for (int j = threadIdx.x; j < k; j += blockDim.x) out[j] = -1;
    return;
  }
  const int nsig = 1 + n_kv, rep = n_heads / n_kv, g = h / rep;
  const int start = cu[s];
  const double2 stx = stats[(int64_t)c * nsig + 0];
  const double2 stv = stats[(int64_t)c * nsig + 1 + g];
  const float a = alpha[h];
  const bool pruned = a >= 0.0f && a <= 1.0f;
  const double rx = __drcp_rn(stx.y), rv = __drcp_rn(stv.y);
  auto score_key = [&](int p) -> uint64_t {
    const int64_t t = start + p;
    if (p >= n || p < w[t]) return 0ull;
    const float zx = z_score(xn[t], stx.x, stx.y, rx);
    const float zv = z_score(vn[t * n_kv + g], stv.x, stv.y, rv);
    const float sc = __fadd_rn(__fmul_rn(a, zv), __fmul_rn(__fsub_rn(1.0f, a), zx));
    return make_key(sc, p);
  };
  if (!pruned) {
    // every uncovered position of the prefix is a candidate
    if (n <= BSEL_KEY_CAP) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) keys[i] = score_key(i);
      __syncthreads();
      block_topk_positions([&](int i) { return keys[i]; }, n, k, sm, sel, out);
    } else {
      block_topk_positions(score_key, n, k, sm, sel, out);
    }
    return;
  }
  // the survivor records of chunks c0 .. c0 + b - 1 of this sequence, packed per kv group
  // (pack_survivors_kernel): one contiguous run of NS records
  const int c0 = base[s];
  const int lane = threadIdx.x & 31;
  const int p_lo = poff[(int64_t)c0 * n_kv + g];
  const int NS = poff[(int64_t)(c0 + b) * n_kv + g] - p_lo;
  const int4* R = packed + (int64_t)g * rec_stride + p_lo;
  if (threadIdx.x == 0) ncand = 0;
  // dominators of every grid cell among all uncovered tokens of the block's prefix
  const int32_t* Dc = D + ((int64_t)c * n_kv + g) * NCELL;
  for (int i = threadIdx.x; i < NCELL; i += blockDim.x) dsm[i] = Dc[i];
  __syncthreads();
  // Candidates: survivors of the earlier chunks that are still dominated by fewer than k
  // tokens of the whole prefix (a token with >= k dominators is outranked by them for any
  // alpha in [0, 1]), compacted into shared memory.
  const float a1 = __fsub_rn(1.0f, a);
  auto rec_key = [&](int4 r) -> uint64_t {
    const float zx = z_score(__int_as_float(r.y), stx.x, stx.y, rx);
    const float zv = z_score(__int_as_float(r.z), stv.x, stv.y, rv);
    const float sc = __fadd_rn(__fmul_rn(a, zv), __fmul_rn(a1, zx));
    return make_key(sc, r.x);
  };
  auto rec_of = [&](int i) -> const int4* { return R + i; };
  constexpr int U = 4;  // records per thread in flight
  for (int i0 = threadIdx.x; i0 - (int)threadIdx.x < NS; i0 += U * blockDim.x) {
    int4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      r[u] = i < NS ? *rec_of(i) : make_int4(0, 0, 0, 0x7fffffff);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool live = r[u].w != 0x7fffffff && (r[u].w < 0 || dsm[r[u].w] < k);
      const uint64_t key = live ? rec_key(r[u]) : 0ull;
      const unsigned ball = __ballot_sync(0xffffffffu, key != 0);
      int slot0 = 0;
      if (lane == 0 && ball) slot0 = atomicAdd(&ncand, __popc(ball));
      slot0 = __shfl_sync(0xffffffffu, slot0, 0);
      const int slot = slot0 + __popc(ball & ((1u << lane) - 1));
      if (key != 0 && slot < BSEL_KEY_CAP) keys[slot] = key;
    }
  }
  __syncthreads();
  const int N = ncand;
  if (N <= BSEL_KEY_CAP) {
    block_topk_positions([&](int i) { return keys[i]; }, N, k, sm, sel, out);
  } else {
    // more candidates than the cache holds: evaluate them from the survivor lists
    auto cand_key = [&](int i) -> uint64_t {
      const int4 r = *rec_of(i);
      return (r.w < 0 || dsm[r.w] < k) ? rec_key(r) : 0ull;
    };
    block_topk_positions(cand_key, NS, k, sm, sel, out);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

struct SelectLayout {
  size_t base_off, part_off, gstats_off, gbase_off, cand_off, stats_off, edges_off, G_off, seg_off, cnt_off, pos_off,
      poff_off, pack_off, total;
  int max_chunks, max_gchunks, nsig, max_segs;
};

static SelectLayout select_layout(int mode, int64_t T, int n_seqs, int n_heads, int n_kv, int k, int block) {
  SelectLayout L{};
  const int C = mode == DSALT_SELECT_GLOBAL ? STAT_CHUNK : block;
  L.nsig = 1 + n_kv;
  L.max_chunks = (int)(T / C) + n_seqs + 1;
  L.max_gchunks = (int)(T / GCHUNK) + n_seqs + 1;
  size_t off = 0;
  L.base_off = off;
  off = align256(off + sizeof(int32_t) * (n_seqs + 1));
  L.gbase_off = off;
  off = align256(off + sizeof(int32_t) * (n_seqs + 1));
  L.part_off = off;
  off = align256(off + sizeof(Partial) * (size_t)L.max_chunks * L.nsig);
  if (mode == DSALT_SELECT_GLOBAL) {
    L.gstats_off = off;
    off = align256(off + sizeof(float) * 2 * L.nsig);
    L.cand_off = off;
    off = align256(off + sizeof(uint64_t) * (size_t)n_heads * L.max_gchunks * k);
  } else {
    L.stats_off = off;
    off = align256(off + sizeof(double2) * (size_t)L.max_chunks * L.nsig);
    L.edges_off = off;
    off = align256(off + sizeof(float) * (size_t)n_seqs * L.nsig * (NBIN - 1));
    L.G_off = off;
    off = align256(off + sizeof(int32_t) * (size_t)L.max_chunks * n_kv * NCELL);
    L.max_segs = n_seqs <= SEG_SCAN_MAX_SEQS ? (L.max_chunks + SCAN_SEG - 1) / SCAN_SEG : 0;
    L.seg_off = off;
    off = align256(off + sizeof(int32_t) * (size_t)n_seqs * n_kv * L.max_segs * NCELL);
    L.cnt_off = off;
    off = align256(off + sizeof(int32_t) * (size_t)L.max_chunks * n_kv);
    L.pos_off = off;
    off = align256(off + sizeof(int4) * (size_t)L.max_chunks * n_kv * C);
    L.poff_off = off;  // per (chunk, group): first packed survivor record (+ one end entry)
    off = align256(off + sizeof(int32_t) * (size_t)(L.max_chunks + 1) * n_kv);
    L.pack_off = off;  // per group: the survivor records of every chunk, in chunk order
    off = align256(off + sizeof(int4) * (size_t)L.max_chunks * n_kv * C);
  }
  L.total = off;
  return L;
}

static int launch_pack_survivors(const SelectLayout& L, char* ws, int n_kv, int C, const int32_t* cbase, int n_seqs,
                                 int n_chunks, cudaStream_t stream) {
  const int32_t* cnt = reinterpret_cast<const int32_t*>(ws + L.cnt_off);
  const int4* recs = reinterpret_cast<const int4*>(ws + L.pos_off);
  int32_t* poff = reinterpret_cast<int32_t*>(ws + L.poff_off);
  int4* packed = reinterpret_cast<int4*>(ws + L.pack_off);
  survivor_offsets_kernel<<<n_kv, 1024, 0, stream>>>(cnt, n_kv, cbase, n_seqs, n_chunks, poff);
  const int grid_c = n_chunks >= 0 ? n_chunks : L.max_chunks;
  if (grid_c > 0)
    pack_survivors_kernel<<<dim3(grid_c, n_kv), 64, 0, stream>>>(cnt, recs, poff, n_kv, C, cbase, n_seqs, n_chunks,
                                                                  packed, (int64_t)L.max_chunks * C);
  return check_cuda(cudaGetLastError(), "survivor packing launch");
}

size_t select_workspace_bytes(int mode, int64_t T, int n_seqs, int max_seqlen, int n_heads, int n_kv, int k,
                              int block) {
  (void)max_seqlen;
  if (T < 0 || n_seqs < 1 || n_heads < 1 || n_kv < 1 || k < 0) return 0;
  if (mode == DSALT_SELECT_BLOCK_CAUSAL && block <= 0) return 0;
  return select_layout(mode, T, n_seqs, n_heads, n_kv, k, block).total;
}

static int upload_bin_table() {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && done[dev]) return DSALT_OK;
  float t[NBIN - 1];
  const int nlow = NBIN / 4;  // 8 thresholds in [-1, 1.5], 23 in [1.6, 4.5]
  for (int i = 0; i < nlow; ++i) t[i] = -1.0f + 2.5f * i / (nlow - 1);
  const int nhigh = NBIN - 1 - nlow;
  for (int i = 0; i < nhigh; ++i) t[nlow + i] = 1.6f + 2.9f * i / (nhigh - 1);
  int rc = check_cuda(cudaMemcpyToSymbol(c_bin_t, t, sizeof(t)), "bin table upload");
  if (rc == DSALT_OK && dev < 64) done[dev] = true;
  return rc;
}

int select_set_up_attributes();

int launch_select(int mode, const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                  const int32_t* cu, int n_seqs, int64_t T, int max_seqlen, int n_heads, int n_kv, int k, int block,
                  int32_t* lmk_out, float* zx_out, float* zv_out, void* workspace, size_t ws_bytes,
                  cudaStream_t stream, int set_lo, int set_hi) {
  if (mode != DSALT_SELECT_GLOBAL && mode != DSALT_SELECT_BLOCK_CAUSAL) return fail(DSALT_ERR_INVALID, "select: mode");
  if (n_seqs < 1 || n_heads < 1 || n_kv < 1 || n_heads % n_kv || T < 0 || k < 0)
    return fail(DSALT_ERR_INVALID, "select: bad sizes");
  if (k > MAX_K) return fail(DSALT_ERR_UNSUPPORTED, "select: k=%d above %d", k, MAX_K);
  if (T > 0x7fffff00LL) return fail(DSALT_ERR_UNSUPPORTED, "select: T too large");
  if (mode == DSALT_SELECT_BLOCK_CAUSAL && (block < 32 || block > 1024 || block % 32))
    return fail(DSALT_ERR_UNSUPPORTED, "select: block must be a multiple of 32 in [32, 1024]");
  if (k == 0 || T == 0) return DSALT_OK;
  if (!xnorm || !vnorm || !w || !alpha || !cu || !lmk_out || !workspace)
    return fail(DSALT_ERR_INVALID, "select: null pointer");
  const SelectLayout L = select_layout(mode, T, n_seqs, n_heads, n_kv, k, block);
  {
    int arc = select_set_up_attributes();  // per-device function attributes; cheap to repeat
    if (arc) return arc;
  }
  if (ws_bytes < L.total) return fail(DSALT_ERR_WORKSPACE, "select: workspace %zu < %zu", ws_bytes, L.total);
  char* ws = reinterpret_cast<char*>(workspace);
  int32_t* cbase = reinterpret_cast<int32_t*>(ws + L.base_off);
  Partial* part = reinterpret_cast<Partial*>(ws + L.part_off);
  const int C = mode == DSALT_SELECT_GLOBAL ? STAT_CHUNK : block;
  const int nsig = L.nsig;
  chunk_table_kernel<<<1, 1024, 0, stream>>>(cu, n_seqs, C, cbase);
  chunk_sums_kernel<<<(unsigned)(((int64_t)L.max_chunks * nsig + 7) / 8), 256, 0, stream>>>(xnorm, vnorm, n_kv, cu,
                                                                                           n_seqs, cbase, C,
                                                                                           L.max_chunks, part);
  if (mode == DSALT_SELECT_GLOBAL) {
    float* gstats = reinterpret_cast<float*>(ws + L.gstats_off);
    int32_t* gbase = reinterpret_cast<int32_t*>(ws + L.gbase_off);
    uint64_t* cand = reinterpret_cast<uint64_t*>(ws + L.cand_off);
    global_stats_kernel<<<nsig, 256, 0, stream>>>(part, L.max_chunks, nsig, T, gstats);
    chunk_table_kernel<<<1, 1024, 0, stream>>>(cu, n_seqs, GCHUNK, gbase);
    const size_t sm1 = sizeof(uint64_t) * GCHUNK;
    global_phase1_kernel<<<dim3(L.max_gchunks, n_heads), SEL_THREADS, sm1, stream>>>(
        xnorm, vnorm, w, alpha, gstats, cu, n_seqs, gbase, n_heads, n_kv, k, cand, zx_out, zv_out);
    const size_t sm2 = sizeof(uint64_t) * KEY_CAP;
    global_phase2_kernel<<<dim3(n_seqs, n_heads), SEL_THREADS, sm2, stream>>>(cand, L.max_gchunks, gbase, n_seqs, k,
                                                                                lmk_out);
  } else {
    int rc = upload_bin_table();
    if (rc) return rc;
    double2* stats = reinterpret_cast<double2*>(ws + L.stats_off);
    float* edges = reinterpret_cast<float*>(ws + L.edges_off);
    int32_t* G = reinterpret_cast<int32_t*>(ws + L.G_off);
    int32_t* cnt = reinterpret_cast<int32_t*>(ws + L.cnt_off);
    int4* recs = reinterpret_cast<int4*>(ws + L.pos_off);
    block_stats_kernel<<<dim3(n_seqs, nsig), 256, 0, stream>>>(part, cu, n_seqs, cbase, nsig, C, stats, edges);
    // kv groups per CTA: 4 when they divide evenly (more CTAs in flight per SM)
    const int gpb = n_kv % 4 == 0 ? 4 : (n_kv % 2 == 0 ? 2 : 1);
    if (n_kv <= 32) {
      const size_t smh = (size_t)gpb * (NBIN * (NBIN + 1) * sizeof(int32_t) + (NBIN - 1) * sizeof(float));
      dominance_hist_all_kernel<<<dim3(L.max_chunks, n_kv / gpb), 512, smh, stream>>>(xnorm, vnorm, w, n_kv, cu,
                                                                                      n_seqs, cbase, C, edges, G, gpb);
    } else {
      dominance_hist_kernel<<<dim3(L.max_chunks, n_kv), 256, 0, stream>>>(xnorm, vnorm, w, n_kv, cu, n_seqs, cbase,
                                                                          C, edges, G);
    }
    if (L.max_segs > 0) {
      int32_t* segsum = reinterpret_cast<int32_t*>(ws + L.seg_off);
      const dim3 sgrid(n_seqs * n_kv, L.max_segs, NCELL / 256);
      dominance_segsum_kernel<<<sgrid, 256, 0, stream>>>(G, cbase, n_seqs, n_kv, L.max_segs, segsum);
      dominance_scan_kernel<<<sgrid, 256, 0, stream>>>(G, cbase, n_kv, L.max_segs, segsum);
    } else {
      dominance_scan_serial_kernel<<<dim3(n_seqs * n_kv, NCELL / 256), 256, 0, stream>>>(G, cbase, n_kv);
    }
    if (n_kv <= 32) {
      survivor_all_kernel<<<dim3(L.max_chunks, n_kv / gpb), 512, (size_t)gpb * (NBIN - 1) * sizeof(float), stream>>>(
          xnorm, vnorm, w, n_kv, cu, n_seqs, cbase, C, edges, G, k, cnt, recs, gpb);
    } else {
      survivor_kernel<<<dim3(L.max_chunks, n_kv), 256, 0, stream>>>(xnorm, vnorm, w, n_kv, cu, n_seqs, cbase, C,
                                                                    edges, G, k, cnt, recs);
    }
    int rc2 = launch_pack_survivors(L, ws, n_kv, C, cbase, n_seqs, -1, stream);
    if (rc2) return rc2;
    const size_t sm3 = sizeof(uint64_t) * BSEL_KEY_CAP;
    const bool range = set_hi >= 0;
    block_select_kernel<<<dim3(range ? set_hi - set_lo : L.max_chunks, n_heads), BSEL_THREADS, sm3, stream>>>(
        xnorm, vnorm, w, alpha, cu, n_seqs, cbase, C, n_heads, n_kv, k, stats, G,
        reinterpret_cast<const int32_t*>(ws + L.poff_off), reinterpret_cast<const int4*>(ws + L.pack_off),
        (int64_t)L.max_chunks * C, lmk_out, range ? set_lo : 0, range ? set_hi - set_lo : 0);
  }
  return check_cuda(cudaGetLastError(), "select launch");
}

__global__ void prefix_cu_kernel(int32_t* cu, int T) {
  if (threadIdx.x == 0) {
    cu[0] = 0;
    cu[1] = T;
  }
}

// Block-causal sets [set_lo, set_hi) of one sequence whose signals cover positions
// [0, seq_len): only the prefix [0, set_hi * block) is read (later tokens cannot be
// landmarks of these blocks). Workspace: the selection workspace of that prefix + 256 B.
size_t select_range_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block, int set_hi) {
  if (block <= 0 || set_hi < 0) return 0;
  const int64_t Tp = std::min<int64_t>(seq_len, (int64_t)set_hi * block);
  return 256 + select_workspace_bytes(DSALT_SELECT_BLOCK_CAUSAL, Tp, 1, (int)Tp, n_heads, n_kv, k, block);
}

int launch_select_range(const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha, int64_t seq_len,
                        int n_heads, int n_kv, int k, int block, int set_lo, int set_hi, int32_t* lmk_out,
                        void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (block < 32 || block > 1024 || block % 32) return fail(DSALT_ERR_UNSUPPORTED, "select range: block");
  if (seq_len < 0 || set_lo < 0 || set_hi < set_lo || (int64_t)set_hi * block > seq_len + block - 1)
    return fail(DSALT_ERR_INVALID, "select range: sets [%d, %d) outside a sequence of %lld", set_lo, set_hi,
                (long long)seq_len);
  if (set_hi == set_lo || k == 0) return DSALT_OK;
  const size_t need = select_range_workspace_bytes(seq_len, n_heads, n_kv, k, block, set_hi);
  if (!workspace || ws_bytes < need) return fail(DSALT_ERR_WORKSPACE, "select range: workspace %zu < %zu", ws_bytes, need);
  const int64_t Tp = std::min<int64_t>(seq_len, (int64_t)set_hi * block);
  int32_t* cu = reinterpret_cast<int32_t*>(workspace);
  prefix_cu_kernel<<<1, 32, 0, stream>>>(cu, (int)Tp);
  int rc = check_cuda(cudaGetLastError(), "select range setup");
  if (rc) return rc;
  return launch_select(DSALT_SELECT_BLOCK_CAUSAL, xnorm, vnorm, w, alpha, cu, 1, Tp, (int)Tp, n_heads, n_kv, k, block,
                       lmk_out, nullptr, nullptr, reinterpret_cast<char*>(workspace) + 256, ws_bytes - 256, stream,
                       set_lo, set_hi);
}

// ---------------------------------------------------------------------------
// Sequence-sharded block-causal selection: one sequence of seq_len positions split into
// n_ranks contiguous shards of whole blocks, rank r owning chunks (= blocks = landmark
// sets) [r·cpr, (r+1)·cpr). Each rank computes the per-chunk records (partial sums,
// dominance grids, survivors) of its own chunks only and reads what it needs of the other
// ranks' from their workspaces (same layout on every rank: a peer's region is its
// workspace pointer plus the same offset; plain loads, peers mapped by CUDA IPC). The
// phases are separated by the caller's cross-GPU barriers:
//   1  chunk sums of the own chunks
//   2  the other ranks' chunk sums; prefix statistics of every chunk and the dominance-grid
//      thresholds from the whole sequence's statistics (identical on every rank); the
//      dominance grids of the own chunks and their total
//   3  the own chunks' exclusive prefix of the grids, started from the totals of the
//      earlier ranks; survivors of the own chunks
//   4  the survivor records of the earlier ranks' chunks; the own sets' top-k
// Results equal dsalt_select_landmarks(DSALT_SELECT_BLOCK_CAUSAL) on the whole sequence.
// ---------------------------------------------------------------------------
struct ShardLayout {
  SelectLayout L;
  size_t cu_off, tot_off, total;
  int n_chunks;
};

static ShardLayout shard_layout(int64_t seq_len, int n_heads, int n_kv, int k, int block) {
  ShardLayout S{};
  S.L = select_layout(DSALT_SELECT_BLOCK_CAUSAL, seq_len, 1, n_heads, n_kv, k, block);
  size_t off = S.L.total;
  S.cu_off = off;
  off = align256(off + 2 * sizeof(int32_t));
  S.tot_off = off;
  off = align256(off + sizeof(int32_t) * (size_t)n_kv * NCELL);
  S.total = off;
  S.n_chunks = (int)((seq_len + block - 1) / block);
  return S;
}

// the other ranks' chunk sums, from their workspaces
__global__ void gather_partials_kernel(Partial* __restrict__ part, const char* const* __restrict__ ws_peers,
                                       size_t part_off, int nsig, int n_chunks, int cpr, int rank) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n_chunks * nsig) return;
  const int owner = (int)(i / nsig) / cpr;
  if (owner == rank) return;
  part[i] = reinterpret_cast<const Partial*>(ws_peers[owner] + part_off)[i];
}

// per (group, cell): sum of the grids of chunks [c_lo, c_hi)
__global__ void dominance_total_kernel(const int32_t* __restrict__ G, int c_lo, int c_hi, int n_kv,
                                       int32_t* __restrict__ tot) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_kv * NCELL) return;
  const int g = i / NCELL, cell = i % NCELL;
  const int64_t stride = (int64_t)n_kv * NCELL;
  const int32_t* p = G + ((int64_t)c_lo * n_kv + g) * NCELL + cell;
  int run = 0;
  for (int c = c_lo; c < c_hi; c += 16) {
    int v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = c + j < c_hi ? p[(int64_t)(c - c_lo + j) * stride] : 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) run += v[j];
  }
  tot[i] = run;
}

// exclusive prefix over chunks [c_lo, c_hi), started from the totals of ranks 0..rank-1
__global__ void dominance_scan_shard_kernel(int32_t* __restrict__ G, int c_lo, int c_hi, int n_kv,
                                            const char* const* __restrict__ ws_peers, size_t tot_off, int rank) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_kv * NCELL) return;
  const int g = i / NCELL, cell = i % NCELL;
  int run = 0;
  for (int r = 0; r < rank; ++r) run += reinterpret_cast<const int32_t*>(ws_peers[r] + tot_off)[i];
  const int64_t stride = (int64_t)n_kv * NCELL;
  int32_t* p = G + ((int64_t)c_lo * n_kv + g) * NCELL + cell;
  for (int c = c_lo; c < c_hi; c += 16) {
    int v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = c + j < c_hi ? p[(int64_t)(c - c_lo + j) * stride] : 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (c + j < c_hi) p[(int64_t)(c - c_lo + j) * stride] = run;
      run += v[j];
    }
  }
}

// survivor counts and records of chunks [0, c_hi) owned by other ranks, from their workspaces
__global__ void gather_survivors_kernel(int32_t* __restrict__ cnt, int4* __restrict__ recs,
                                        const char* const* __restrict__ ws_peers, size_t cnt_off, size_t rec_off,
                                        int n_kv, int C, int cpr) {
  const int c = blockIdx.x, g = blockIdx.y, owner = c / cpr;
  const int64_t cg = (int64_t)c * n_kv + g;
  const int n = reinterpret_cast<const int32_t*>(ws_peers[owner] + cnt_off)[cg];
  if (threadIdx.x == 0) cnt[cg] = n;
  const int4* src = reinterpret_cast<const int4*>(ws_peers[owner] + rec_off) + cg * C;
  int4* dst = recs + cg * C;
  for (int j = threadIdx.x; j < n && j < C; j += blockDim.x) dst[j] = src[j];
}

size_t select_shard_workspace_bytes(int64_t seq_len, int n_heads, int n_kv, int k, int block) {
  if (seq_len < 1 || n_heads < 1 || n_kv < 1 || k < 0 || block <= 0) return 0;
  return shard_layout(seq_len, n_heads, n_kv, k, block).total;
}

int launch_select_shard(int phase, const float* xnorm, const float* vnorm, const int32_t* w, const float* alpha,
                        int64_t seq_len, int n_heads, int n_kv, int k, int block, int rank, int n_ranks, void* workspace,
                        size_t ws_bytes, const void* const* ws_peers, int32_t* lmk_out, cudaStream_t stream) {
  if (phase < 1 || phase > 4) return fail(DSALT_ERR_INVALID, "select shard: phase %d not in 1..4", phase);
  if (n_ranks < 1 || rank < 0 || rank >= n_ranks || n_heads < 1 || n_kv < 1 || n_heads % n_kv || k < 0)
    return fail(DSALT_ERR_INVALID, "select shard: bad sizes");
  if (block < 32 || block > 1024 || block % 32) return fail(DSALT_ERR_UNSUPPORTED, "select shard: block");
  if (seq_len < 1 || seq_len > 0x7fffff00LL || seq_len % ((int64_t)block * n_ranks))
    return fail(DSALT_ERR_UNSUPPORTED, "select shard: seq_len must split into whole blocks per rank");
  if (k > MAX_K) return fail(DSALT_ERR_UNSUPPORTED, "select shard: k=%d above %d", k, MAX_K);
  if (n_kv > 32) return fail(DSALT_ERR_UNSUPPORTED, "select shard: more than 32 kv groups");
  if (!xnorm || !vnorm || !w || !alpha || !workspace || !ws_peers || (phase == 4 && !lmk_out))
    return fail(DSALT_ERR_INVALID, "select shard: null pointer");
  const ShardLayout S = shard_layout(seq_len, n_heads, n_kv, k, block);
  if (ws_bytes < S.total) return fail(DSALT_ERR_WORKSPACE, "select shard: workspace %zu < %zu", ws_bytes, S.total);
  if (k == 0) {
    if (phase == 4) return fail(DSALT_ERR_UNSUPPORTED, "select shard: k = 0");
    return DSALT_OK;
  }
  int rc = select_set_up_attributes();
  if (rc) return rc;
  if ((rc = upload_bin_table())) return rc;
  const SelectLayout& L = S.L;
  char* ws = reinterpret_cast<char*>(workspace);
  int32_t* cbase = reinterpret_cast<int32_t*>(ws + L.base_off);
  int32_t* cu = reinterpret_cast<int32_t*>(ws + S.cu_off);
  Partial* part = reinterpret_cast<Partial*>(ws + L.part_off);
  double2* stats = reinterpret_cast<double2*>(ws + L.stats_off);
  float* edges = reinterpret_cast<float*>(ws + L.edges_off);
  int32_t* G = reinterpret_cast<int32_t*>(ws + L.G_off);
  int32_t* cnt = reinterpret_cast<int32_t*>(ws + L.cnt_off);
  int4* recs = reinterpret_cast<int4*>(ws + L.pos_off);
  int32_t* tot = reinterpret_cast<int32_t*>(ws + S.tot_off);
  const char* const* peers = reinterpret_cast<const char* const*>(ws_peers);
  const int C = block, nsig = 1 + n_kv;
  const int cpr = S.n_chunks / n_ranks, c_lo = rank * cpr, c_hi = c_lo + cpr;
  const int gpb = n_kv % 4 == 0 ? 4 : (n_kv % 2 == 0 ? 2 : 1);
  if (phase == 1) {
    prefix_cu_kernel<<<1, 32, 0, stream>>>(cu, (int)seq_len);
    chunk_table_kernel<<<1, 1024, 0, stream>>>(cu, 1, C, cbase);
    chunk_sums_kernel<<<(unsigned)(((int64_t)cpr * nsig + 7) / 8), 256, 0, stream>>>(xnorm, vnorm, n_kv, cu, 1, cbase,
                                                                                   C, cpr, part, c_lo);
  } else if (phase == 2) {
    const int64_t np = (int64_t)S.n_chunks * nsig;
    if (n_ranks > 1)
      gather_partials_kernel<<<(unsigned)((np + 255) / 256), 256, 0, stream>>>(part, peers, L.part_off, nsig,
                                                                              S.n_chunks, cpr, rank);
    block_stats_kernel<<<dim3(1, nsig), 256, 0, stream>>>(part, cu, 1, cbase, nsig, C, stats, edges);
    const size_t smh = (size_t)gpb * (NBIN * (NBIN + 1) * sizeof(int32_t) + (NBIN - 1) * sizeof(float));
    dominance_hist_all_kernel<<<dim3(cpr, n_kv / gpb), 512, smh, stream>>>(xnorm, vnorm, w, n_kv, cu, 1, cbase, C,
                                                                           edges, G, gpb, c_lo);
    dominance_total_kernel<<<(unsigned)((n_kv * NCELL + 255) / 256), 256, 0, stream>>>(G, c_lo, c_hi, n_kv, tot);
  } else if (phase == 3) {
    dominance_scan_shard_kernel<<<(unsigned)((n_kv * NCELL + 255) / 256), 256, 0, stream>>>(G, c_lo, c_hi, n_kv,
                                                                                            peers, S.tot_off, rank);
    survivor_all_kernel<<<dim3(cpr, n_kv / gpb), 512, (size_t)gpb * (NBIN - 1) * sizeof(float), stream>>>(
        xnorm, vnorm, w, n_kv, cu, 1, cbase, C, edges, G, k, cnt, recs, gpb, c_lo);
  } else {
    if (c_lo > 0)
      gather_survivors_kernel<<<dim3(c_lo, n_kv), 64, 0, stream>>>(cnt, recs, peers, L.cnt_off, L.pos_off, n_kv, C,
                                                                   cpr);
    if ((rc = launch_pack_survivors(L, ws, n_kv, C, cbase, 1, c_hi, stream))) return rc;
    const size_t sm3 = sizeof(uint64_t) * BSEL_KEY_CAP;
    block_select_kernel<<<dim3(cpr, n_heads), BSEL_THREADS, sm3, stream>>>(
        xnorm, vnorm, w, alpha, cu, 1, cbase, C, n_heads, n_kv, k, stats, G,
        reinterpret_cast<const int32_t*>(ws + L.poff_off), reinterpret_cast<const int4*>(ws + L.pack_off),
        (int64_t)L.max_chunks * C, lmk_out, c_lo, cpr);
  }
  return check_cuda(cudaGetLastError(), "select shard launch");
}

int select_set_up_attributes() {
  int rc = check_cuda(cudaFuncSetAttribute(global_phase2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(sizeof(uint64_t) * KEY_CAP)),
                      "smem attr");
  if (rc) return rc;
  rc = check_cuda(cudaFuncSetAttribute(dominance_hist_all_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)(32 * (NBIN * (NBIN + 1) * sizeof(int32_t) + (NBIN - 1) * sizeof(float)))),
                  "smem attr");
  if (rc) return rc;
  return check_cuda(cudaFuncSetAttribute(block_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(sizeof(uint64_t) * BSEL_KEY_CAP)),
                    "smem attr");
}

}  // namespace dsalt
