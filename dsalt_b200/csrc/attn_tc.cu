// Sparse attention forward on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Semantics of the reference's inference kernel (dsalt/kernels/dsalt_triton_attn.py:27-169):
// query i of a sequence attends to its window j ∈ [max(0, i−w(i)+1), i] and to the
// landmarks p of its set with 0 ≤ p < L, p ≤ i and p < i−w(i)+1 (the de-duplicating
// rule of :132-135); logits q·k·D^-½ (+ optional landmark bias); online softmax with
// fp32 statistics, P rounded to the input dtype for the P·V product (as the reference's
// tl.dot(p.to(bf16), v)); rows with softmax mass ≤ 1e-9 are zero.
//
// Work item = (128-query tile, head); persistent CTAs, one per SM. Per item the key
// axis is a band of 128-key window tiles starting at max(0, m0 − max_w + 1) plus
// ceil(k/128) landmark tiles. Roles (256 threads):
//   warp 0  producer: TMA (no multicast) for the Q tile and the K/V window tiles into a
//           4-stage ring; landmark K/V rows gathered with cp.async into the same ring
//           (replaces _build_landmark_kv, dsalt/kernels/selectors.py:137-159);
//   warp 1  TMEM allocation and the single-thread MMA issuer:
//           S = Q·Kᵀ (SS form, M=128 N=128 K=16 steps) into TMEM S[2],
//           O_j = P_j·V_j (TS form: P read from TMEM, V from smem, N = head_dim) into O[2];
//   warps 4-7 softmax: row r ↔ TMEM lane r; masks, running max/sum in registers, P
//           written back to TMEM as packed 16-bit pairs, O_j accumulated in registers
//           with the max-rescale, epilogue to global memory.
// TMEM columns: S0 S1 (128 each) | P0 P1 (64 each) | O0 O1 (head_dim each) — 512 total.
// Every mbarrier wait is bounded (common.cuh) and reports to the device status word.
#include <cuda.h>

#include "common.cuh"

namespace dsalt {

int launch_chunk_table(const int32_t* cu, int n_seqs, int C, int32_t* base, cudaStream_t stream);

namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NST = 4;
constexpr int NTHREADS = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_P = 256, COL_O = 384;
constexpr int MAX_LMK = 256;

struct Params {
  const void* k;
  const void* v;
  int H, Hkv;
  int64_t kv_stride;
  const int32_t* w;
  const int32_t* lmk;
  const float* lmk_bias;
  int k_lmk, lmk_block;
  const int32_t* cu;
  int n_seqs;
  const int32_t* set_base;
  const int32_t* tile_base;
  float scale_log2;
  uint32_t idesc_qk, idesc_pv;
  void* out;
  int out_dtype;
  float* lse;
  int* err;
};

struct Item {
  int s, start, L, m0, h, hk, kstart, nwt, nlt, set, n_sets;
};

__device__ __forceinline__ int find_seq(const int32_t* base, int n, int idx) {
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (base[mid] <= idx) lo = mid;
    else hi = mid;
  }
  return lo;
}

// warp-collective: every lane returns the same description of work item `item`
__device__ __forceinline__ Item item_info(const Params& p, int item) {
  Item f;
  const int tile = item / p.H;
  f.h = item - tile * p.H;
  f.hk = f.h / (p.H / p.Hkv);
  f.s = find_seq(p.tile_base, p.n_seqs, tile);
  f.start = p.cu[f.s];
  f.L = p.cu[f.s + 1] - f.start;
  f.m0 = (tile - p.tile_base[f.s]) * BM;
  int wm = 1;
  for (int r = threadIdx.x & 31; r < BM; r += 32) {
    const int i = f.m0 + r;
    if (i < f.L) wm = max(wm, p.w[f.start + i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wm = max(wm, __shfl_xor_sync(0xffffffffu, wm, o));
  const int hi = min(f.m0 + BM - 1, f.L - 1);
  f.kstart = max(0, f.m0 - wm + 1);
  f.nwt = (hi - f.kstart + BN) / BN;
  f.nlt = (p.k_lmk + BN - 1) / BN;
  f.n_sets = p.lmk_block ? p.set_base[p.n_seqs] : p.n_seqs;
  f.set = p.lmk_block ? p.set_base[f.s] + f.m0 / p.lmk_block : f.s;
  return f;
}

template <int HD>
struct Smem {
  static constexpr int NA = HD / 64;                       // 128-byte swizzle atoms per row
  static constexpr uint32_t TILE_BYTES = BM * HD * 2;      // one 128 x HD 16-bit tile
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t K_OFF = Q_OFF + 2 * TILE_BYTES;
  static constexpr uint32_t V_OFF = K_OFF + NST * TILE_BYTES;
  static constexpr uint32_t BAR_OFF = V_OFF + NST * TILE_BYTES;
  static constexpr int NBAR = 2 + 2 + NST + NST + 2 + 2 + 2 + 2 + 2;
  static constexpr uint32_t MISC_OFF = BAR_OFF + NBAR * 8;
  static constexpr uint32_t LPOS_OFF = MISC_OFF + 16;
  static constexpr uint32_t LBIAS_OFF = LPOS_OFF + MAX_LMK * 4;
  static constexpr uint32_t BYTES = LBIAS_OFF + MAX_LMK * 4;
};

// byte offset of 16-byte chunk c of row r in a 128B-swizzled K-major tile of HD columns
template <int HD>
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  const int atom = c >> 3, cc = c & 7;
  return (uint32_t)(atom * BM * 128 + r * 128 + ((cc ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using SM = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SM::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 2;
  uint64_t* kv_full = bars + 4;
  uint64_t* kv_empty = bars + 4 + NST;
  uint64_t* s_full = bars + 4 + 2 * NST;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_full + 4;
  uint64_t* o_full = s_full + 6;
  uint64_t* o_empty = s_full + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + SM::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + SM::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.tile_base[p.n_seqs] * p.H;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
    }
    for (int i = 0; i < NST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    int g = 0, it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
      const Item f = item_info(p, item);
      const int qb = it & 1;
      if (!mbar_wait(&q_empty[qb], ((it >> 1) & 1) ^ 1, p.err, 11)) { *abort_flag = 1; break; }
      if (lane == 0) {
        mbar_arrive_expect_tx(&q_full[qb], SM::TILE_BYTES);
        for (int a = 0; a < SM::NA; ++a)
          tma_load_3d(sbase + SM::Q_OFF + qb * SM::TILE_BYTES + a * BM * 128, &tm_q, &q_full[qb], a * 64, f.h,
                      f.start + f.m0);
      }
      const int NK = f.nwt + f.nlt;
      bool ok = true;
      for (int j = 0; j < NK; ++j, ++g) {
        const int st = g % NST;
        const uint32_t r = (uint32_t)(g / NST);
        if (!mbar_wait(&kv_empty[st], (r & 1) ^ 1, p.err, 12) || *abort_flag) { *abort_flag = 1; ok = false; break; }
        const uint32_t kdst = sbase + SM::K_OFF + st * SM::TILE_BYTES;
        const uint32_t vdst = sbase + SM::V_OFF + st * SM::TILE_BYTES;
        if (j < f.nwt) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&kv_full[st], 2 * SM::TILE_BYTES);
            const int row = f.start + f.kstart + j * BN;
            for (int a = 0; a < SM::NA; ++a) {
              tma_load_3d(kdst + a * BM * 128, &tm_k, &kv_full[st], a * 64, f.hk, row);
              tma_load_3d(vdst + a * BM * 128, &tm_v, &kv_full[st], a * 64, f.hk, row);
            }
          }
        } else {
          const int lt = j - f.nwt;
          const int32_t* P = p.lmk + ((int64_t)f.h * f.n_sets + f.set) * p.k_lmk;
          for (int rr = lane; rr < BN; rr += 32) {
            const int idx = lt * BN + rr;
            const int pos = idx < p.k_lmk ? P[idx] : -1;
            const bool valid = pos >= 0 && pos < f.L;
            const int64_t off = valid ? ((int64_t)(f.start + pos) * p.kv_stride + (int64_t)f.hk * HD) * 2 : 0;
            const char* ks = reinterpret_cast<const char*>(p.k) + off;
            const char* vs = reinterpret_cast<const char*>(p.v) + off;
#pragma unroll
            for (int c = 0; c < HD / 8; ++c) {
              const uint32_t o = swz_off<HD>(rr, c);
              cp_async_16(kdst + o, ks + c * 16, valid ? 16u : 0u);
              cp_async_16(vdst + o, vs + c * 16, valid ? 16u : 0u);
            }
          }
          cp_async_wait_all();
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&kv_full[st]);
        }
      }
      if (!ok) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t tS = tbase + COL_S, tP = tbase + COL_P, tO = tbase + COL_O;
    int g = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
      const Item f = item_info(p, item);
      const int NK = f.nwt + f.nlt;
      const int qb = it & 1;
      if (!mbar_wait(&q_full[qb], (it >> 1) & 1, p.err, 21)) { *abort_flag = 1; break; }
      const uint32_t qaddr = sbase + SM::Q_OFF + qb * SM::TILE_BYTES;
      auto issue_S = [&](int j) -> bool {
        const int gg = g + j, st = gg % NST, sb = gg & 1;
        const uint32_t r = (uint32_t)(gg / NST), rs = (uint32_t)(gg >> 1);
        if (!mbar_wait(&kv_full[st], r & 1, p.err, 22)) return false;
        if (!mbar_wait(&s_empty[sb], (rs & 1) ^ 1, p.err, 23)) return false;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t kaddr = sbase + SM::K_OFF + st * SM::TILE_BYTES;
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t koff = (ks >> 2) * BM * 128 + (ks & 3) * 32;
            umma_ss(tS + sb * BN, sw128_desc(qaddr + koff, 16, 1024), sw128_desc(kaddr + koff, 16, 1024),
                    p.idesc_qk, ks > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[sb]);
          if (j == NK - 1) umma_commit(&q_empty[qb]);
        }
        __syncwarp();
        return true;
      };
      if (!issue_S(0)) { *abort_flag = 1; break; }
      for (int j = 0; j < NK; ++j) {
        if (j + 1 < NK && !issue_S(j + 1)) { *abort_flag = 1; ok = false; break; }
        const int gg = g + j, st = gg % NST, sb = gg & 1;
        const uint32_t rs = (uint32_t)(gg >> 1);
        if (!mbar_wait(&p_full[sb], rs & 1, p.err, 24) || !mbar_wait(&o_empty[sb], (rs & 1) ^ 1, p.err, 25)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t vaddr = sbase + SM::V_OFF + st * SM::TILE_BYTES;
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks)
            umma_ts(tO + sb * HD, tP + sb * 64 + ks * 8, sw128_desc(vaddr + ks * 2048, BM * 128, 1024), p.idesc_pv,
                    ks > 0 ? 1u : 0u);
          umma_commit(&o_full[sb]);
          umma_commit(&kv_empty[st]);
        }
        __syncwarp();
      }
      g += NK;
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax
    const int q4 = warp - 4;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tS = tbase + lane_off + COL_S, tP = tbase + lane_off + COL_P, tO = tbase + lane_off + COL_O;
    const float LOG2E = 1.4426950408889634f;
    int g = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const Item f = item_info(p, item);
      const int NK = f.nwt + f.nlt;
      const int i = f.m0 + r;
      const bool vrow = i < f.L;
      int wi = vrow ? p.w[f.start + i] : 1;
      wi = wi < 1 ? 1 : wi;
      const int lo_raw = i - wi + 1;
      const int lo = lo_raw < 0 ? 0 : lo_raw;
      // landmark positions / biases of this item's set, read through L1 (no cross-warp
      // barrier: every wait in this kernel stays bounded)
      const int32_t* Pset = p.lmk + ((int64_t)f.h * f.n_sets + f.set) * p.k_lmk;
      const float* Bset = p.lmk_bias ? p.lmk_bias + ((int64_t)f.h * f.n_sets + f.set) * p.k_lmk : nullptr;
      float m_run = -INFINITY, l = 0.0f, m_acc = -INFINITY, m_last = -INFINITY;
      float acc[HD];
#pragma unroll
      for (int d = 0; d < HD; ++d) acc[d] = 0.0f;

      auto consume_O = [&](int gg, float m_t) -> bool {
        const int sb = gg & 1;
        const uint32_t rs = (uint32_t)(gg >> 1);
        if (!mbar_wait(&o_full[sb], rs & 1, p.err, 31)) return false;
        tc_fence_after();
        const float fac = (m_acc == -INFINITY) ? 0.0f : ex2_approx(m_acc - m_t);
#pragma unroll
        for (int cc = 0; cc < HD / 32; ++cc) {
          uint32_t o[32];
          DSALT_TMEM_LD32(tO + sb * HD + cc * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[cc * 32 + e] = fmaf(acc[cc * 32 + e], fac, __uint_as_float(o[e]));
        }
        tc_fence_before();
        mbar_arrive(&o_empty[sb]);
        m_acc = m_t;
        return true;
      };

      for (int j = 0; j < NK; ++j) {
        const int gg = g + j, sb = gg & 1;
        const uint32_t rs = (uint32_t)(gg >> 1);
        if (!mbar_wait(&s_full[sb], rs & 1, p.err, 32)) { ok = false; break; }
        tc_fence_after();
        const bool is_w = j < f.nwt;
        const int kb = f.kstart + j * BN;
        const int a = lo - kb, b = i - kb;  // window: valid columns [a, b]
        const bool full = vrow && is_w && a <= 0 && b >= BN - 1;
        const int lt = j - f.nwt;
        auto logit = [&](uint32_t bits, int col) -> float {
          const float s = __uint_as_float(bits) * p.scale_log2;
          if (full) return s;
          if (!vrow) return -INFINITY;
          if (is_w) return (col >= a && col <= b) ? s : -INFINITY;
          const int c = lt * BN + col;
          if (c >= p.k_lmk) return -INFINITY;
          const int pos = __ldg(Pset + c);
          if (pos < 0 || pos >= f.L || pos > i || pos >= lo_raw) return -INFINITY;
          return Bset ? s + __ldg(Bset + c) * LOG2E : s;
        };
        // pass 1: row max over the valid columns
        float mt = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t sv[32];
          DSALT_TMEM_LD32(tS + sb * BN + cc * 32, sv);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) mt = fmaxf(mt, logit(sv[e], cc * 32 + e));
        }
        const float m_new = fmaxf(m_run, mt);
        // pass 2: probabilities, row sum, P -> TMEM (16-bit pairs)
        float rsum = 0.0f;
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t sv[32];
          DSALT_TMEM_LD32(tS + sb * BN + cc * 32, sv);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float x0 = logit(sv[e], cc * 32 + e), x1 = logit(sv[e + 1], cc * 32 + e + 1);
            const float p0 = (x0 == -INFINITY) ? 0.0f : ex2_approx(x0 - m_new);
            const float p1 = (x1 == -INFINITY) ? 0.0f : ex2_approx(x1 - m_new);
            rsum += p0 + p1;
            pk[e >> 1] = (p.idesc_qk >> 7 & 1) ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
          }
          DSALT_TMEM_ST16(tP + sb * 64 + cc * 16, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&s_empty[sb]);
        mbar_arrive(&p_full[sb]);
        const float corr = (m_run == -INFINITY) ? 0.0f : ex2_approx(m_run - m_new);
        l = fmaf(l, corr, rsum);
        const float m_prev_tile = m_last;
        m_last = m_new;
        m_run = m_new;
        if (j >= 1 && !consume_O(gg - 1, m_prev_tile)) { ok = false; break; }
      }
      if (!ok) { *abort_flag = 1; break; }
      if (!consume_O(g + NK - 1, m_last)) { *abort_flag = 1; break; }
      g += NK;
      // epilogue
      if (vrow) {
        const bool good = l > 1e-9f;
        const float inv = good ? 1.0f / l : 0.0f;
        const int64_t row = (int64_t)(f.start + i);
        if (p.out_dtype == DSALT_F32) {
          float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (row * p.H + f.h) * HD);
#pragma unroll
          for (int d = 0; d < HD; d += 4)
            o[d / 4] = make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
        } else {
          uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + (row * p.H + f.h) * HD);
          const bool bf = p.out_dtype == DSALT_BF16;
#pragma unroll
          for (int d = 0; d < HD; d += 8) {
            uint4 u;
            u.x = bf ? pack_bf16x2(acc[d] * inv, acc[d + 1] * inv) : pack_f16x2(acc[d] * inv, acc[d + 1] * inv);
            u.y = bf ? pack_bf16x2(acc[d + 2] * inv, acc[d + 3] * inv) : pack_f16x2(acc[d + 2] * inv, acc[d + 3] * inv);
            u.z = bf ? pack_bf16x2(acc[d + 4] * inv, acc[d + 5] * inv) : pack_f16x2(acc[d + 4] * inv, acc[d + 5] * inv);
            u.w = bf ? pack_bf16x2(acc[d + 6] * inv, acc[d + 7] * inv) : pack_f16x2(acc[d + 6] * inv, acc[d + 7] * inv);
            o[d / 8] = u;
          }
        }
        if (p.lse) p.lse[row * p.H + f.h] = good ? (m_last + log2f(l)) * 0.6931471805599453f : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

static int make_map(CUtensorMap* m, const void* base, int dtype, int HD, int heads, int64_t T, int64_t row_stride) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return fail(DSALT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)heads, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)row_stride * 2};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)BM};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, dtype == DSALT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSALT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DSALT_OK;
}

}  // namespace tc

int launch_attn_tc(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int HD,
                   int64_t q_stride, int64_t kv_stride, const int32_t* w, const int32_t* lmk, const float* lmk_bias,
                   int k_lmk, int lmk_block, const int32_t* cu, int n_seqs, int32_t* set_base, int32_t* tile_base,
                   void* out, int out_dtype, float* lse, int* err, cudaStream_t stream) {
  using namespace tc;
  if (HD != 64) return fail(DSALT_ERR_UNSUPPORTED, "attention (tensor cores): head_dim %d not supported (64)", HD);
  if (k_lmk > MAX_LMK) return fail(DSALT_ERR_UNSUPPORTED, "attention: k_lmk %d above %d", k_lmk, MAX_LMK);
  if (lmk_block % BM) return fail(DSALT_ERR_UNSUPPORTED, "attention: lmk_block must be a multiple of %d", BM);
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15 || (q_stride * 2) % 16 ||
      (kv_stride * 2) % 16)
    return fail(DSALT_ERR_INVALID, "attention: q/k/v/out must be 16-byte aligned with 16-byte row strides");
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, q, dtype, HD, H, T, q_stride))) return rc;
  if ((rc = make_map(&mk, k, dtype, HD, Hkv, T, kv_stride))) return rc;
  if ((rc = make_map(&mv, v, dtype, HD, Hkv, T, kv_stride))) return rc;
  if ((rc = launch_chunk_table(cu, n_seqs, BM, tile_base, stream))) return rc;
  if (lmk_block > 0 && (rc = launch_chunk_table(cu, n_seqs, lmk_block, set_base, stream))) return rc;
  Params p{};
  p.k = k;
  p.v = v;
  p.H = H;
  p.Hkv = Hkv;
  p.kv_stride = kv_stride;
  p.w = w;
  p.lmk = lmk;
  p.lmk_bias = lmk_bias;
  p.k_lmk = k_lmk;
  p.lmk_block = lmk_block;
  p.cu = cu;
  p.n_seqs = n_seqs;
  p.set_base = set_base;
  p.tile_base = tile_base;
  p.scale_log2 = (float)(1.0 / sqrt((double)HD) * 1.4426950408889634);
  const uint32_t ab = dtype == DSALT_BF16 ? 1u : 0u;
  p.idesc_qk = umma_idesc_f16(ab, 0, 0, BM, BN);
  p.idesc_pv = umma_idesc_f16(ab, 0, 1, BM, HD);
  p.out = out;
  p.out_dtype = out_dtype;
  p.lse = lse;
  p.err = err;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t max_items = (T / BM + n_seqs) * (int64_t)H;
  const int grid = (int)(max_items < nsm ? max_items : nsm);
  if (grid <= 0) return DSALT_OK;
  const size_t smem = Smem<64>::BYTES + 1024;
  if ((rc = check_cuda(cudaFuncSetAttribute(attn_fwd_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem),
                       "attention smem attr")))
    return rc;
  attn_fwd_tc_kernel<64><<<grid, NTHREADS, smem, stream>>>(mq, mk, mv, p);
  return check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace dsalt
