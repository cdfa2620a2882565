// Sparse attention forward on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Semantics of the reference's inference kernel (dsalt/kernels/dsalt_triton_attn.py:27-169):
// query i of a sequence attends to its window j ∈ [max(0, i−w(i)+1), i] and to the
// landmarks p of its set with 0 ≤ p < L, p ≤ i and p < i−w(i)+1 (the de-duplicating
// rule of :132-135); logits q·k·D^-½ (+ optional landmark bias); softmax statistics in
// fp32, P rounded to the input dtype for the P·V product (as the reference's
// tl.dot(p.to(bf16), v)); rows with softmax mass ≤ 1e-9 are zero.
//
// Work item = (128-query tile, head); persistent CTAs, one per SM. Per item the key
// axis is a band of 128-key window tiles ending at the tile's last row and reaching back
// to max(0, m0 − max_w + 1), plus ceil(k/128) landmark tiles; the order is the diagonal
// window tile, the landmark tiles, then the other window tiles leftwards. Each CTA runs
// two independent pipelines (A, B) on alternate items; a pipeline is
//   a producer warp   TMA (no multicast) of the Q tile and the K/V window tiles into a
//                     3-stage K ring and a 2-stage V ring; landmark K/V rows gathered by
//                     TMA four-row gathers into the same rings (replaces
//                     _build_landmark_kv, selectors.py:137-159); once the current item's
//                     loads are issued it publishes the next item's description slot and
//                     prefetches that item's landmark rows into L2;
//   an MMA warp       one thread issues S = Q·Kᵀ (SS form) into TMEM and O += P·V (TS
//                     form: P read from TMEM, V from smem) into a TMEM accumulator;
//   4 softmax warps   row r ↔ TMEM lane r: the S row is read once into registers,
//                     masked, exponentiated; P goes back to TMEM as 16-bit pairs; O is
//                     rescaled in TMEM only when the running max grows by more than 2^8.
// TMEM (512 columns): per pipeline S (128) | P (64) | O (head_dim).
// Warps: 0/1 producer/MMA of A, 2/3 producer/MMA of B, 4-7 softmax A, 8-11 softmax B
// (head_dim 64); at head_dim 128 pipeline A alone: warps 0/1, 4-7 (2/3 idle).
// Every mbarrier wait is bounded (common.cuh) and reports to the device status word.
#include <cuda.h>

#include "common.cuh"

namespace dsalt {

int launch_chunk_table(const int32_t* cu, int n_seqs, int C, int32_t* base, cudaStream_t stream);

namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
// pipelines per CTA: two at head_dim 64; one at head_dim 128, whose tiles (Q + 3 K + 2 V
// stages of 32 KB) fill the shared memory and whose TMEM (S 128 | P 64 | O 128) takes 320
// of the 512 columns
template <int HD>
struct Pipes {
  static constexpr int N = HD == 64 ? 2 : 1;
  static constexpr int THREADS = 128 + 128 * N;
};
constexpr int NPIPE_MAX = 2;
constexpr int NSK = 3;          // K stages per pipeline (released when S = Q·Kᵀ completes)
constexpr int NSV = 2;          // V stages per pipeline (released when O += P·V completes)
constexpr int NQB = 1;          // Q buffers per pipeline
constexpr int NIS = 2;          // item-description slots per pipeline
// Register split with setmaxnreg. The block launches with 168 registers per thread
// (384 x 168 = 64512); warpgroup 0 (producers, MMA issuers) gives back to 88 and the two
// softmax warpgroups take 208: 128 x 88 + 256 x 208 = 64512, and every scheduler (one
// warp of each warpgroup) holds 88 + 2 x 208 = 504 <= 512 registers per lane. Each
// setmaxnreg sits at the top of its role's branch so that the compiler allocates each
// role with its own budget.
#ifndef DSALT_REGS_CTRL
#define DSALT_REGS_CTRL 88
#define DSALT_REGS_SOFTMAX 208
#endif
constexpr uint32_t REGS_CTRL = DSALT_REGS_CTRL, REGS_SOFTMAX = DSALT_REGS_SOFTMAX;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t PIPE_COLS = 256;                 // S 128 | P 64 | O 64 (head_dim 64)
constexpr uint32_t COL_S = 0, COL_P = 128, COL_O = 192;
constexpr int MAX_LMK = 256;
constexpr float OVERFLOW_SUM = 32768.0f;  // a tile's row sum above 2^15 (or NaN/inf) redoes the tile

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
  const int4* plan;  // per query tile: {q row base, L, m0, set}, {kstart, nwt, kv row base, w base}
  // Sharded mode (shard_tiles > 0): the local query tiles cover positions q_pos0 + 128 t of
  // one sequence; the landmark rows of each (local set, head) were gathered beforehand
  // (lmk_gather_kernel) into tiles loaded by TMA like window tiles.
  int shard_tiles, n_sets_local;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  float inv_scale;   // sqrt(head_dim): landmark bias in raw-logit units
  // soft window edge (training forward, SOFT kernels): continuous widths w̃ (w then holds
  // floor(w̃) + 1), edge width (≤ 4) and temperature
  const float* w_soft;
  float soft_edge, soft_tau;
  uint32_t idesc_qk, idesc_pv;
  void* out;
  int out_dtype;
  int out_v8;  // out is 32-byte aligned: rows written with 32-byte stores
  float* lse;
  int* err;
};

// positions are within the sequence; buffer row of position i: qb + i (q, out),
// kvb + i (k, v windows and packed landmarks); width of position i: w[wb + i]
struct Item {
  int qb, kvb, wb, L, m0, h, hk, kstart, nwt, nlt, set, n_sets;
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

// Per query tile (one warp each): the sequence it lies in and the band of key tiles its
// window needs. Window tiles end at the tile's last row, so that the last one holds
// every row's diagonal key; the first may start before the sequence (those keys are
// masked). Replaces _build_seq_block_map (selectors.py:37-67).
// Sharded mode (shard_tiles > 0): tile t is positions q_pos0 + 128 t of one sequence of
// length seq_len, q/out row = position - q_pos0, k/v row = position - kv_pos0, widths
// indexed by position, landmark set = position / lmk_block - set_lo.
__global__ void tile_plan_kernel(const int32_t* __restrict__ cu, int n_seqs, const int32_t* __restrict__ tile_base,
                                 const int32_t* __restrict__ set_base, int lmk_block, const int32_t* __restrict__ w,
                                 int4* __restrict__ plan, int shard_tiles, int q_pos0, int kv_pos0, int seq_len,
                                 int set_lo) {
  const int tile = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  int qb, kvb, wb, L, m0, set;
  if (shard_tiles > 0) {
    if (tile >= shard_tiles) return;
    qb = -q_pos0;
    kvb = -kv_pos0;
    wb = 0;
    L = seq_len;
    m0 = q_pos0 + tile * BM;
    set = lmk_block ? m0 / lmk_block - set_lo : 0;
  } else {
    if (tile >= tile_base[n_seqs]) return;
    const int s = find_seq(tile_base, n_seqs, tile);
    qb = kvb = wb = cu[s];
    L = cu[s + 1] - qb;
    m0 = (tile - tile_base[s]) * BM;
    set = lmk_block ? set_base[s] + m0 / lmk_block : s;
  }
  int wm = 1;
  for (int r = lane; r < BM; r += 32)
    if (m0 + r < L) wm = max(wm, __ldg(w + wb + m0 + r));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wm = max(wm, __shfl_xor_sync(0xffffffffu, wm, o));
  const int hi = min(m0 + BM - 1, L - 1);
  const int kmin = max(0, m0 - wm + 1);
  const int nwt = (hi - kmin + BN) / BN;
  if (lane == 0) {
    plan[2 * tile] = make_int4(qb, L, m0, set);
    plan[2 * tile + 1] = make_int4(hi + 1 - nwt * BN, nwt, kvb, wb);
  }
}

__device__ __forceinline__ Item make_item(const Params& p, int item, int4 a, int4 b, int n_sets) {
  Item f;
  const int tile = item / p.H;
  f.h = item - tile * p.H;
  f.hk = f.h / (p.H / p.Hkv);
  f.qb = a.x;
  f.L = a.y;
  f.m0 = a.z;
  f.set = a.w;
  f.kstart = b.x;
  f.nwt = b.y;
  f.kvb = b.z;
  f.wb = b.w;
  f.nlt = (p.k_lmk + BN - 1) / BN;
  f.n_sets = n_sets;
  return f;
}

// Processing order of an item's key tiles: the diagonal window tile (every valid row gets a
// finite running max on the first tile), the landmark tiles, then the other window tiles
// leftwards. The landmark rows are gathered while the diagonal tile's softmax runs; the
// leftmost window tile is often nearly empty and would not cover the gather.
// Returns the window-tile index, or -1 - (landmark tile).
__device__ __forceinline__ int tile_at(const Item& f, int t) {
  if (f.nwt == 0) return -1 - t;
  if (t == 0) return f.nwt - 1;
  if (t <= f.nlt) return -t;
  return f.nwt - 1 - (t - f.nlt);
}

template <int HD>
struct Smem {
  static constexpr int NA = HD / 64;                       // 128-byte swizzle atoms per row
  static constexpr uint32_t TILE_BYTES = BM * HD * 2;      // one 128 x HD 16-bit tile
  static constexpr uint32_t PIPE_BYTES = (NQB + NSK + NSV) * TILE_BYTES;
  static constexpr uint32_t Q_OFF = 0;                     // + pipe * PIPE_BYTES
  static constexpr uint32_t K_OFF = NQB * TILE_BYTES;
  static constexpr uint32_t V_OFF = K_OFF + NSK * TILE_BYTES;
  // item slots: description, per-row window widths, landmark positions
  static constexpr uint32_t SLOT_BYTES = 64 + BM * 4 + MAX_LMK * 4;
  static constexpr int NP = Pipes<HD>::N;
  static constexpr uint32_t SLOT_OFF = NP * PIPE_BYTES;  // + (pipe * NIS + slot) * SLOT_BYTES
  static constexpr uint32_t BAR_OFF = SLOT_OFF + NP * NIS * SLOT_BYTES;
  // per pipeline: q_full[NQB] q_empty[NQB] k_full[NSK] k_empty[NSK] v_full[NSV] v_empty[NSV]
  // s_full s_empty p_full o_full o_empty item_full[NIS] item_empty[NIS]
  static constexpr int NBAR_PIPE = 2 * NQB + 2 * NSK + 2 * NSV + 5 + 2 * NIS;
  static constexpr uint32_t MISC_OFF = BAR_OFF + NP * NBAR_PIPE * 8;
  static constexpr uint32_t BYTES = MISC_OFF + 16;
};

// byte offset of 16-byte chunk c of row r in a 128B-swizzled K-major tile of HD columns
template <int HD>
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  const int atom = c >> 3, cc = c & 7;
  return (uint32_t)(atom * BM * 128 + r * 128 + ((cc ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(__cvta_generic_to_global(p)));
}

__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
constexpr float MASKED_MAX = -1.0e20f;  // a row maximum below this means "no valid column"

// packed fp32 pair ops (sm_100)
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 up2(uint64_t r) {
  float2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(r));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Masking of one 32-column chunk (columns c0 .. c0 + 31) for a row whose valid columns are
// [a, b]: bit e of chunk_bits says whether column c0 + e is valid, and mask_chunk sets the
// others to -inf (exp2 gives exactly 0). One bit test and one select per column; this
// replaced two exact threshold adds and a three-input min per column (0.893 -> 0.858 ms at
// L = 131072 on B200, identical output), the softmax being bound by its instruction stream.
__device__ __forceinline__ uint32_t chunk_bits(int a, int b, int c0) {
  const int l = max(a - c0, 0), h = min(b - c0, 31);
  return l > h ? 0u : (0xFFFFFFFFu >> (31 - h)) & (0xFFFFFFFFu << l);
}
__device__ __forceinline__ void mask_chunk(float* xc, uint32_t m) {
#pragma unroll
  for (int e = 0; e < 32; ++e) xc[e] = ((m >> e) & 1u) ? xc[e] : -INFINITY;
}

// 2^y for a pair of values on the FMA pipe (the MUFU unit that runs ex2.approx issues 16
// results per clock per SM, a quarter of the FMA pipe's rate, so a share of each chunk's
// exponentials is computed here). Cody-Waite style reduction y = j + f with j = rint(y),
// taken exactly by the 1.5*2^23 shift (|y| < 2^22), and |f| <= 1/2; 2^f by a degree-3
// polynomial fitted for minimal relative error on [-1/2, 1/2] by iteratively reweighted
// least squares (Lawson's algorithm): max relative error 7.5e-5 evaluated in fp32, well
// below the 2^-9 of the bf16 rounding P goes through. j is added to the exponent field.
// y is clamped to [-126, 64] first: below, the result is a value <= 2^-126 instead of
// ~0 (the masked columns: negligible against the row's maximum, ~1); above, it is >= 2^64,
// which the tile-sum overflow check sends to the slow path like an infinite ex2 result.
constexpr float EXP2_C0 = 0.9999280571937561f, EXP2_C1 = 0.6932609677314758f, EXP2_C2 = 0.24261093139648438f,
                EXP2_C3 = 0.05517149344086647f;
constexpr float RINT_SHIFT = 12582912.0f;  // 1.5 * 2^23
__device__ __forceinline__ void exp2_poly2(uint64_t y, float& r0, float& r1) {
  float2 v = up2(y);
  v.x = fminf(fmaxf(v.x, -126.0f), 64.0f);
  v.y = fminf(fmaxf(v.y, -126.0f), 64.0f);
  const uint64_t yc = pk2(v.x, v.y);
  const uint64_t t = add2(yc, pk2(RINT_SHIFT, RINT_SHIFT));       // 1.5*2^23 + rint(y)
  const uint64_t j = add2(t, pk2(-RINT_SHIFT, -RINT_SHIFT));      // rint(y)
  const uint64_t f = fma2(j, pk2(-1.0f, -1.0f), yc);              // y - rint(y), exact
  uint64_t q = fma2(pk2(EXP2_C3, EXP2_C3), f, pk2(EXP2_C2, EXP2_C2));
  q = fma2(q, f, pk2(EXP2_C1, EXP2_C1));
  q = fma2(q, f, pk2(EXP2_C0, EXP2_C0));
  const float2 qq = up2(q), tt = up2(t);
  // the low 9 bits of t's encoding hold rint(y) mod 512: shifted by 23 they add rint(y) to
  // the exponent of 2^f (in [2^-1/2, 2^1/2]; exponent >= 126 - 126 stays non-negative)
  r0 = __uint_as_float(__float_as_uint(qq.x) + (__float_as_uint(tt.x) << 23));
  r1 = __uint_as_float(__float_as_uint(qq.y) + (__float_as_uint(tt.y) << 23));
}

// Pairs of a 32-column chunk whose exponentials take the polynomial (bit i: columns 2i,
// 2i+1); the others use ex2.approx. Measured on B200 at L = 131072 the softmax is bound by
// latency, not by the MUFU rate, and the extra FMA-pipe instructions cost more than they
// save (six pairs: 0.958 ms against 0.896 ms for none), so no pair uses it by default.
#ifndef DSALT_POLY_PAIRS
#define DSALT_POLY_PAIRS 0u
#endif

// P = 2^(x*sl - mu) of one 32-column chunk: 16-bit pairs into pk, fp32 row sums into s0/s1
template <bool BF>
__device__ __forceinline__ void exp_chunk(const float* xc, uint64_t sl2, uint64_t nmu2, uint64_t& s0, uint64_t& s1,
                                          uint32_t* pk) {
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const uint64_t y = fma2(pk2(xc[e], xc[e + 1]), sl2, nmu2);
    float q0, q1;
    if ((DSALT_POLY_PAIRS >> (e >> 1)) & 1u) {
      exp2_poly2(y, q0, q1);
    } else {
      const float2 yy = up2(y);
      q0 = ex2_approx(yy.x);
      q1 = ex2_approx(yy.y);
    }
    if ((e >> 1) & 1) s1 = add2(s1, pk2(q0, q1));
    else s0 = add2(s0, pk2(q0, q1));
    pk[e >> 1] = BF ? pack_bf16x2(q0, q1) : pack_f16x2(q0, q1);
  }
}

// 32-byte store (sm_100); the address must be 32-byte aligned
__device__ __forceinline__ void st_global_v8(void* ptr, const uint32_t* r) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(__cvta_generic_to_global(ptr)),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

struct PipeBars {
  uint64_t *q_full, *q_empty, *k_full, *k_empty, *v_full, *v_empty, *s_full, *s_empty, *p_full, *o_full, *o_empty,
      *it_full, *it_empty;
};

// one item's description as the producer publishes it to the MMA and softmax warps
struct Slot {
  Item f;
  int pad[16 - sizeof(Item) / 4];
  int32_t wv[BM];    // per row: window width (0 for rows past the sequence end)
  int32_t pos[MAX_LMK];
};
static_assert(sizeof(Item) <= 64, "item description must fit the slot header");

// P is packed to the input type: BF = bf16, else fp16
__device__ __forceinline__ uint32_t pack_p(bool bf, float lo, float hi) {
  return bf ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

template <int HD, bool BF, bool SOFT>
__global__ void __launch_bounds__(Pipes<HD>::THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_lk,
                       const __grid_constant__ CUtensorMap tm_lv, const Params p) {
  using SM = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(sm);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + SM::MISC_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = (p.shard_tiles > 0 ? p.shard_tiles : p.tile_base[p.n_seqs]) * p.H;

  if (threadIdx.x == 0) {
    for (int pp = 0; pp < SM::NP; ++pp) {
      uint64_t* b = reinterpret_cast<uint64_t*>(sm + SM::BAR_OFF) + pp * SM::NBAR_PIPE;
      for (int i = 0; i < NQB; ++i) {
        mbar_init(b + i, 1);        // q_full
        mbar_init(b + NQB + i, 1);  // q_empty
      }
      for (int i = 0; i < 2 * NSK + 2 * NSV; ++i) mbar_init(b + 2 * NQB + i, 1);  // K/V full and empty
      uint64_t* t = b + 2 * NQB + 2 * NSK + 2 * NSV;
      mbar_init(t + 0, 1);    // s_full
      mbar_init(t + 1, 128);  // s_empty
      mbar_init(t + 2, 128);  // p_full
      mbar_init(t + 3, 1);    // o_full
      mbar_init(t + 4, 128);  // o_empty
      for (int i = 0; i < NIS; ++i) {
        mbar_init(t + 5 + i, 1);              // item_full: the producer publishes
        mbar_init(t + 5 + NIS + i, 128 + 1);  // item_empty: 128 softmax threads + the MMA issuer
      }
    }
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

  // pipeline of this warp and its barriers / buffers
  const int pipe = warp < 4 ? (warp >> 1) : ((warp - 4) >> 2);
  PipeBars B;
  {
    uint64_t* b = reinterpret_cast<uint64_t*>(sm + SM::BAR_OFF) + pipe * SM::NBAR_PIPE;
    B.q_full = b;
    B.q_empty = b + NQB;
    B.k_full = b + 2 * NQB;
    B.k_empty = B.k_full + NSK;
    B.v_full = B.k_empty + NSK;
    B.v_empty = B.v_full + NSV;
    uint64_t* t = b + 2 * NQB + 2 * NSK + 2 * NSV;
    B.s_full = t;
    B.s_empty = t + 1;
    B.p_full = t + 2;
    B.o_full = t + 3;
    B.o_empty = t + 4;
    B.it_full = t + 5;
    B.it_empty = t + 5 + NIS;
  }
  Slot* slots = reinterpret_cast<Slot*>(sm + SM::SLOT_OFF) + pipe * NIS;
  const uint32_t pbase = sbase + pipe * SM::PIPE_BYTES;
  const uint32_t tpipe = tbase + pipe * PIPE_COLS;
  // items of this pipeline: the CTA's items alternate between the two pipelines
  const int item0 = blockIdx.x + pipe * gridDim.x, istride = SM::NP * gridDim.x;

  if (warp < 4) {
    if constexpr (SM::NP == 2) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CTRL));
    if (pipe >= SM::NP) {
      // control warps of a pipeline this head_dim does not have: idle
    } else if ((warp & 1) == 0) {
      // ---------------------------------------------------------------- producer
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        tma_prefetch_desc(&tm_lk);
        tma_prefetch_desc(&tm_lv);
      }
      const uint16_t* kg = reinterpret_cast<const uint16_t*>(p.k);
      const uint16_t* vg = reinterpret_cast<const uint16_t*>(p.v);
      const int n_sets = p.shard_tiles > 0 ? p.n_sets_local : p.lmk_block ? __ldg(p.set_base + p.n_seqs) : p.n_seqs;
      // Publish item `item_n` (the it_n-th of this pipeline) into its slot: the description
      // from the tile plan (a, b), then the rows' window widths and the landmark positions
      // by cp.async; the slot is full when the copies have landed.
      auto publish = [&](int item_n, int it_n, int4 a, int4 b) -> bool {
        const Item fn = make_item(p, item_n, a, b, n_sets);
        const int sl = it_n % NIS;
        if (!mbar_wait(&B.it_empty[sl], ((it_n / NIS) & 1) ^ 1, p.err, 13)) return false;
        Slot& S = slots[sl];
        if (lane == 0) S.f = fn;
        const int32_t* P = p.lmk + ((int64_t)fn.h * fn.n_sets + fn.set) * p.k_lmk;
        for (int c = lane; c < p.k_lmk; c += 32) cp_async_4(smem_u32(&S.pos[c]), P + c, 4u);
        for (int r = lane; r < BM; r += 32) {
          const bool vrow = fn.m0 + r < fn.L;
          cp_async_4(smem_u32(&S.wv[r]), p.w + fn.wb + (vrow ? fn.m0 + r : 0), vrow ? 4u : 0u);
        }
        cp_async_mbar_arrive(&B.it_full[sl]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.it_full[sl]);
        // the item's landmark rows are gathered an item later: bring them into L2 now
        // (scattered 128-byte rows; the gather would otherwise wait on DRAM latency)
        if (fn.nlt > 0 && p.shard_tiles == 0) {
          for (int c = lane; c < p.k_lmk; c += 32) {
            const int pos = __ldg(P + c);
            if (pos >= 0) {
              const int64_t off = (int64_t)(fn.kvb + pos) * p.kv_stride + (int64_t)fn.hk * HD;
#pragma unroll
              for (int a = 0; a < SM::NA; ++a) {  // one 128-byte line per 64 columns
                prefetch_l2(kg + off + a * 64);
                prefetch_l2(vg + off + a * 64);
              }
            }
          }
        }
        return true;
      };
      int g = 0, it = 0;
      bool ok = true;
      if (item0 < n_items) {
        const int t0 = item0 / p.H;
        ok = publish(item0, 0, __ldg(p.plan + 2 * t0), __ldg(p.plan + 2 * t0 + 1));
      }
      for (int item = item0; item < n_items && ok; item += istride, ++it) {
        const int sl_i = it % NIS;
        const Slot& S = slots[sl_i];
        const Item f = S.f;
        // the next item's plan: loaded now, published once this item's tile loads are issued
        // (publishing after the first tile instead interrupted the loads: 0.857 vs 0.845 ms)
        const int item_n = item + istride;
        const bool has_next = item_n < n_items;
        int4 an = make_int4(0, 0, 0, 0), bn = an;
        if (has_next) {
          an = __ldg(p.plan + 2 * (item_n / p.H));
          bn = __ldg(p.plan + 2 * (item_n / p.H) + 1);
        }
        const int qb = it % NQB;
        if (!mbar_wait(&B.q_empty[qb], ((it / NQB) & 1) ^ 1, p.err, 11)) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&B.q_full[qb], SM::TILE_BYTES);
          for (int a = 0; a < SM::NA; ++a)
            tma_load_3d(pbase + SM::Q_OFF + qb * SM::TILE_BYTES + a * BM * 128, &tm_q, &B.q_full[qb], a * 64, f.h,
                        f.qb + f.m0);
        }
        const int NK = f.nwt + f.nlt;
        for (int t = 0; t < NK; ++t, ++g) {
          const int jt = tile_at(f, t);
          const int sk = g % NSK, sv = g % NSV;
          const uint32_t kdst = pbase + SM::K_OFF + sk * SM::TILE_BYTES;
          const uint32_t vdst = pbase + SM::V_OFF + sv * SM::TILE_BYTES;
          if (jt >= 0) {
            const int row = f.kvb + f.kstart + jt * BN;
            if (!mbar_wait(&B.k_empty[sk], ((uint32_t)(g / NSK) & 1) ^ 1, p.err, 12)) { ok = false; break; }
            if (lane == 0) {
              mbar_arrive_expect_tx(&B.k_full[sk], SM::TILE_BYTES);
              for (int a = 0; a < SM::NA; ++a) tma_load_3d(kdst + a * BM * 128, &tm_k, &B.k_full[sk], a * 64, f.hk, row);
            }
            if (!mbar_wait(&B.v_empty[sv], ((uint32_t)(g / NSV) & 1) ^ 1, p.err, 14)) { ok = false; break; }
            if (lane == 0) {
              mbar_arrive_expect_tx(&B.v_full[sv], SM::TILE_BYTES);
              for (int a = 0; a < SM::NA; ++a) tma_load_3d(vdst + a * BM * 128, &tm_v, &B.v_full[sv], a * 64, f.hk, row);
            }
          } else {
            const int lt = -jt - 1;
            if (p.shard_tiles > 0) {
              // pre-gathered landmark tiles of (set, head)
              const int row = ((f.set * p.H + f.h) * f.nlt + lt) * BN;
              if (!mbar_wait(&B.k_empty[sk], ((uint32_t)(g / NSK) & 1) ^ 1, p.err, 12)) { ok = false; break; }
              if (lane == 0) {
                mbar_arrive_expect_tx(&B.k_full[sk], SM::TILE_BYTES);
                for (int a = 0; a < SM::NA; ++a) tma_load_3d(kdst + a * BM * 128, &tm_lk, &B.k_full[sk], a * 64, 0, row);
              }
              if (!mbar_wait(&B.v_empty[sv], ((uint32_t)(g / NSV) & 1) ^ 1, p.err, 14)) { ok = false; break; }
              if (lane == 0) {
                mbar_arrive_expect_tx(&B.v_full[sv], SM::TILE_BYTES);
                for (int a = 0; a < SM::NA; ++a) tma_load_3d(vdst + a * BM * 128, &tm_lv, &B.v_full[sv], a * 64, 0, row);
              }
              continue;
            }
            // landmark rows (replaces _build_landmark_kv): TMA gathers of four rows each (2-D
            // maps over the K / V rows, one 64-column box per row, no multicast), lane l
            // fetching rows 4l..4l+3 of the tile, so the producer never waits for them. Slots
            // past the set's length, with position -1 or outside the sequence read the
            // sequence's first row instead: their columns are masked by the row's landmark
            // count and carry P = 0 (or <= 2^-126), so the values never count. The positions
            // come from this item's slot.
            if (!mbar_wait(&B.it_full[sl_i], (uint32_t)(it / NIS) & 1, p.err, 15)) { ok = false; break; }
            if (!mbar_wait(&B.k_empty[sk], ((uint32_t)(g / NSK) & 1) ^ 1, p.err, 12)) { ok = false; break; }
            if (!mbar_wait(&B.v_empty[sv], ((uint32_t)(g / NSV) & 1) ^ 1, p.err, 14)) { ok = false; break; }
            if (lane == 0) {
              mbar_arrive_expect_tx(&B.k_full[sk], SM::TILE_BYTES);
              mbar_arrive_expect_tx(&B.v_full[sv], SM::TILE_BYTES);
            }
            __syncwarp();
            int rows[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int idx = lt * BN + 4 * lane + j;
              const int pos = idx < p.k_lmk ? S.pos[idx] : -1;
              rows[j] = f.kvb + ((unsigned)pos < (unsigned)f.L ? pos : 0);
            }
#pragma unroll
            for (int a = 0; a < SM::NA; ++a) {
              const uint32_t off = a * BM * 128 + lane * 512;
              const int col = f.hk * HD + a * 64;
              tma_gather4(kdst + off, &tm_lk, &B.k_full[sk], col, rows[0], rows[1], rows[2], rows[3]);
              tma_gather4(vdst + off, &tm_lv, &B.v_full[sv], col, rows[0], rows[1], rows[2], rows[3]);
            }
          }
        }
        if (ok && has_next && !publish(item_n, it + 1, an, bn)) ok = false;
      }
    } else {
      // ---------------------------------------------------------------- MMA issuer
      int g = 0, it = 0;
      uint32_t ns = 0, npv = 0;
      bool ok = true;
      for (int item = item0; item < n_items && ok; item += istride, ++it) {
        const int sl_i = it % NIS;
        if (!mbar_wait(&B.it_full[sl_i], (it / NIS) & 1, p.err, 26)) break;
        const Item f = slots[sl_i].f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.it_empty[sl_i]);
        const int NK = f.nwt + f.nlt;
        const int qb = it % NQB;
        if (!mbar_wait(&B.q_full[qb], (it / NQB) & 1, p.err, 21)) break;
        const uint32_t qaddr = pbase + SM::Q_OFF + qb * SM::TILE_BYTES;
        auto issue_S = [&](int t) -> bool {
          const int gg = g + t, sk = gg % NSK;
          if (!mbar_wait(&B.k_full[sk], (uint32_t)(gg / NSK) & 1, p.err, 22)) return false;
          if (!mbar_wait(B.s_empty, (ns & 1) ^ 1, p.err, 23)) return false;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t kaddr = pbase + SM::K_OFF + sk * SM::TILE_BYTES;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
              const uint32_t koff = (ks >> 2) * BM * 128 + (ks & 3) * 32;
              umma_ss(tpipe + COL_S, sw128_desc(qaddr + koff, 16, 1024), sw128_desc(kaddr + koff, 16, 1024),
                      p.idesc_qk, ks > 0 ? 1u : 0u);
            }
            umma_commit(B.s_full);
            umma_commit(&B.k_empty[sk]);
            if (t == NK - 1) umma_commit(&B.q_empty[qb]);
          }
          __syncwarp();
          ++ns;
          return true;
        };
        if (!issue_S(0)) { ok = false; break; }
        for (int t = 0; t < NK; ++t) {
          const int gg = g + t, sv = gg % NSV;
          // the softmax releases S_t before P_t is ready: refill S first
          if (t + 1 < NK && !issue_S(t + 1)) { ok = false; break; }
          if (t == 0 && !mbar_wait(B.o_empty, (it & 1) ^ 1, p.err, 25)) { ok = false; break; }
          if (!mbar_wait(B.p_full, npv & 1, p.err, 24)) { ok = false; break; }
          if (!mbar_wait(&B.v_full[sv], (uint32_t)(gg / NSV) & 1, p.err, 27)) { ok = false; break; }
          tc_fence_after();
          if (elect_one()) {
            const uint32_t vaddr = pbase + SM::V_OFF + sv * SM::TILE_BYTES;
#pragma unroll
            for (int ks = 0; ks < BN / 16; ++ks)
              umma_ts(tpipe + COL_O, tpipe + COL_P + ks * 8, sw128_desc(vaddr + ks * 2048, BM * 128, 1024),
                      p.idesc_pv, (ks > 0 || t > 0) ? 1u : 0u);
            umma_commit(B.o_full);
            umma_commit(&B.v_empty[sv]);
          }
          __syncwarp();
          ++npv;
        }
        g += NK;
      }
    }
  } else {
    if constexpr (SM::NP == 2) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_SOFTMAX));
    // ------------------------------------------------------------------ softmax
    const int quad = warp & 3;        // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;   // query row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tpipe + lane_off + COL_S;
    const uint32_t tP = tpipe + lane_off + COL_P;
    const uint32_t tO = tpipe + lane_off + COL_O;
    const float sl = p.scale_log2;
    uint32_t u = 0;
    bool ok = true;
    int it = 0;
    for (int item = item0; item < n_items && ok; item += istride, ++it) {
      const int sl_i = it % NIS;
      if (!mbar_wait(&B.it_full[sl_i], (it / NIS) & 1, p.err, 36)) break;
      const Slot& S = slots[sl_i];
      const Item f = S.f;
      const int i = f.m0 + r;
      const bool vrow = i < f.L;
      // the row's window [lo, i] and its landmark count: sets are ascending with -1 last,
      // so as unsigned values non-decreasing, and the landmarks the row may use
      // (0 <= p < min(L, i-w+1)) are a prefix of the set
      int lo, lcnt;
      // soft edge (SOFT): the first ne band columns from lo_raw, i.e. d = i - j from floor(w̃)
      // down, get log σ((w̃ - d)/τ) in raw-logit units eb0..eb3
      int lo_raw, ne = 0;
      float eb0 = 0.0f, eb1 = 0.0f, eb2 = 0.0f, eb3 = 0.0f;
      {
        const int wi = SOFT ? S.wv[r] : max(S.wv[r], 1);  // SOFT: width 0 = no band (w̃ < 0)
        lo_raw = i - wi + 1;
        if constexpr (SOFT) {
          if (vrow && wi > 0) {
            const float wc = __ldg(p.w_soft + f.wb + i);
            const int dhi = wi - 1;  // floor(w̃)
            const int dlo = max(0, (int)floorf(wc - p.soft_edge) + 1);  // core: d <= w̃ - edge
            ne = min(dhi - dlo + 1, 4);
            auto eb = [&](int kk) {
              const float z = (wc - (float)(dhi - kk)) / p.soft_tau;
              return -logf(1.0f + expf(-z)) * p.inv_scale;
            };
            if (ne > 0) eb0 = eb(0);
            if (ne > 1) eb1 = eb(1);
            if (ne > 2) eb2 = eb(2);
            if (ne > 3) eb3 = eb(3);
          }
        }
        lo = vrow ? max(lo_raw, 0) : 0x3fffffff;
        const unsigned lim = vrow ? (unsigned)max(0, min(f.L, lo_raw)) : 0u;
        int a0 = 0, a1 = p.k_lmk;
        while (a0 < a1) {
          const int mid = (a0 + a1) >> 1;
          if ((unsigned)S.pos[mid] < lim) a0 = mid + 1;
          else a1 = mid;
        }
        lcnt = a0;
      }
      mbar_arrive(&B.it_empty[sl_i]);
      const int NK = f.nwt + f.nlt;
      const float* Bset = p.lmk_bias ? p.lmk_bias + ((int64_t)f.h * f.n_sets + f.set) * p.k_lmk : nullptr;
      float m_acc = -INFINITY, l = 0.0f;  // running max (log2 units, stale) and row sum
      for (int t = 0; t < NK; ++t) {
        if (!mbar_wait(B.s_full, u & 1, p.err, 32)) { ok = false; break; }
        tc_fence_after();
        // the whole S row in registers: one TMEM round trip, then the buffer is released
        float x[BN];
        {
          uint32_t* xr = reinterpret_cast<uint32_t*>(x);
          DSALT_TMEM_LD32(tS, xr);
          DSALT_TMEM_LD32(tS + 32, (xr + 32));
          DSALT_TMEM_LD32(tS + 64, (xr + 64));
          DSALT_TMEM_LD32(tS + 96, (xr + 96));
        }
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(B.s_empty);
        // valid columns of this row in the tile: [a, b] (window: lo..i; landmarks: the
        // first lcnt entries of the ascending set)
        const int jt = tile_at(f, t);
        const bool is_w = jt >= 0;
        const int lt = -jt - 1;
        const int kb = f.kstart + jt * BN;
        const int a = is_w ? (vrow ? lo - kb : BN) : 0;
        const int b = is_w ? (vrow ? i - kb : -1) : lcnt - 1 - lt * BN;
        if (!is_w && Bset != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int idx = lt * BN + q * 32 + lane;
            const float bq = idx < p.k_lmk ? __ldg(Bset + idx) * p.inv_scale : 0.0f;
#pragma unroll
            for (int e = 0; e < 32; ++e) x[q * 32 + e] += __shfl_sync(0xffffffffu, bq, e);
          }
        }
        if constexpr (SOFT) {
          if (is_w) {
            // columns ea .. ea + ne - 1 of this tile carry the soft edge; only the chunks that
            // hold one of some lane's edge columns are visited (warp-uniform)
            const int ea = lo_raw - kb;
            uint32_t touch_l = 0;
#pragma unroll
            for (int cc = 0; cc < BN / 32; ++cc)
              touch_l |= (uint32_t)(ne > 0 && ea <= cc * 32 + 31 && ea + ne - 1 >= cc * 32) << cc;
            const uint32_t touch = __reduce_or_sync(0xffffffffu, touch_l);
#pragma unroll
            for (int cc = 0; cc < BN / 32; ++cc) {
              if (!((touch >> cc) & 1)) continue;
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const int kk = cc * 32 + e - ea;
                const float bv = kk == 0 ? eb0 : (kk == 1 ? eb1 : (kk == 2 ? eb2 : eb3));
                x[cc * 32 + e] += (unsigned)kk < (unsigned)ne ? bv : 0.0f;
              }
            }
          }
        }
        uint64_t s0 = pk2(0.f, 0.f), s1 = s0;
        // chunk classes, warp-uniform: bit c of `none` = no lane keeps chunk c (skipped);
        // bit c of `all` = every lane keeps all of chunk c (no masking)
        uint32_t none_l = 0, all_l = 0;
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          none_l |= (uint32_t)(b < cc * 32 || a > cc * 32 + 31) << cc;
          all_l |= (uint32_t)(a <= cc * 32 && b >= cc * 32 + 31) << cc;
        }
        const uint32_t none = __reduce_and_sync(0xffffffffu, none_l), all = __reduce_and_sync(0xffffffffu, all_l);
        bool slow = t == 0, p_free = t == 0;
        if (!slow) {
          // Fast path (every tile after the first): exponentials against the running max,
          // chunk by chunk, P stored to TMEM per chunk once the previous P·V has released the
          // P buffer. Overflow check on the tile's row sum: while it stays below 2^15 no P
          // entry exceeds 2^15 (finite in fp16 and bf16); otherwise the tile is redone on the
          // slow path with the row's new maximum.
          const float mu = (m_acc == -INFINITY) ? 0.0f : m_acc;
          const uint64_t sl2 = pk2(sl, sl), nmu2 = pk2(-mu, -mu);
#pragma unroll
          for (int cc = 0; cc < BN / 32; ++cc) {
            uint32_t pk[16];
            if ((none >> cc) & 1) {
#pragma unroll
              for (int e = 0; e < 16; ++e) pk[e] = 0u;
            } else {
              float* xc = x + cc * 32;
              if (!((all >> cc) & 1)) mask_chunk(xc, chunk_bits(a, b, cc * 32));
              exp_chunk<BF>(xc, sl2, nmu2, s0, s1, pk);
            }
            if (!p_free) {
              // previous P·V done: the P buffer may be overwritten
              if (!mbar_wait(B.o_full, (u - 1) & 1, p.err, 33)) { ok = false; break; }
              tc_fence_after();
              p_free = true;
            }
            DSALT_TMEM_ST16(tP + cc * 16, pk);
          }
          if (!ok) break;
          const float2 ss = up2(add2(s0, s1));
          slow = __any_sync(0xffffffffu, !(ss.x + ss.y <= OVERFLOW_SUM));
        }
        if (slow) {
          // masked row max; O and the row sum are rescaled when it grows (a chunk masked on
          // the fast path is masked again: -inf stays -inf)
          float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
          for (int cc = 0; cc < BN / 32; ++cc) {
            if ((none >> cc) & 1) continue;
            float* xc = x + cc * 32;
            if (!((all >> cc) & 1)) mask_chunk(xc, chunk_bits(a, b, cc * 32));
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              m0 = fmax3f(m0, xc[e], xc[e + 1]);
              m1 = fmax3f(m1, xc[e + 2], xc[e + 3]);
            }
          }
          float m_tile = fmaxf(m0, m1) * sl;
          if (m_tile < MASKED_MAX) m_tile = -INFINITY;
          const bool need = m_tile > m_acc;
          const float m_new = need ? m_tile : m_acc;
          if (t > 0) {
            if (!mbar_wait(B.o_full, (u - 1) & 1, p.err, 33)) { ok = false; break; }
            tc_fence_after();
            if (__any_sync(0xffffffffu, need)) {
              const float fac = need ? ex2_approx(m_acc - m_new) : 1.0f;
#pragma unroll 1
              for (int cc = 0; cc < HD / 16; ++cc) {
                uint32_t o[16];
                DSALT_TMEM_LD16(tO + cc * 16, o);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * fac);
                DSALT_TMEM_ST16(tO + cc * 16, o);
              }
              tmem_wait_st();
              l *= fac;
            }
          }
          m_acc = m_new;
          const float mu = (m_acc == -INFINITY) ? 0.0f : m_acc;
          const uint64_t sl2 = pk2(sl, sl), nmu2 = pk2(-mu, -mu);
          s0 = pk2(0.f, 0.f);
          s1 = s0;
#pragma unroll
          for (int cc = 0; cc < BN / 32; ++cc) {
            uint32_t pk[16];
            if ((none >> cc) & 1) {
#pragma unroll
              for (int e = 0; e < 16; ++e) pk[e] = 0u;
            } else {
              exp_chunk<BF>(x + cc * 32, sl2, nmu2, s0, s1, pk);  // masked above where needed
            }
            DSALT_TMEM_ST16(tP + cc * 16, pk);
          }
        }
        const float2 ss = up2(add2(s0, s1));
        l += ss.x + ss.y;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(B.p_full);
        ++u;
      }
      if (!ok) break;
      // the item's O, once its last P·V is done
      if (!mbar_wait(B.o_full, (u - 1) & 1, p.err, 34)) { ok = false; break; }
      tc_fence_after();
      float acc[HD];
#pragma unroll
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t* orr = reinterpret_cast<uint32_t*>(acc + cc * 32);
        DSALT_TMEM_LD32(tO + cc * 32, orr);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(B.o_empty);
      if (vrow) {
        const bool good = l > 1e-9f;
        float inv = 0.0f;  // 1 / l (MUFU approximation, ~1 ulp: far below the output rounding)
        if (good) asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv) : "f"(l));
        const int64_t row = (int64_t)f.qb + i;
        // the row's HD outputs, as 32-bit words (fp32 values or 16-bit pairs)
        const bool f32o = p.out_dtype == DSALT_F32;
        const uint64_t inv2 = pk2(inv, inv);
#pragma unroll
        for (int d = 0; d < HD; d += 2) {
          const float2 y = up2(mul2(pk2(acc[d], acc[d + 1]), inv2));
          acc[d] = y.x;
          acc[d + 1] = y.y;
        }
        if (!f32o) {
          const bool bo = p.out_dtype == DSALT_BF16;
#pragma unroll
          for (int d = 0; d < HD; d += 2) {
            const uint32_t w2 = bo ? pack_bf16x2(acc[d], acc[d + 1]) : pack_f16x2(acc[d], acc[d + 1]);
            acc[d / 2] = __uint_as_float(w2);
          }
        }
        const uint32_t* wv = reinterpret_cast<const uint32_t*>(acc);
        char* orow = reinterpret_cast<char*>(p.out) + (row * p.H + f.h) * (int64_t)HD * (f32o ? 4 : 2);
        const int nw = f32o ? HD : HD / 2;
        if (p.out_v8) {
#pragma unroll
          for (int q = 0; q < HD; q += 8)
            if (q < nw) st_global_v8(orow + q * 4, wv + q);
        } else {
#pragma unroll
          for (int q = 0; q < HD; q += 4)
            if (q < nw) *reinterpret_cast<uint4*>(orow + q * 4) = make_uint4(wv[q], wv[q + 1], wv[q + 2], wv[q + 3]);
        }
        const float mm = (m_acc == -INFINITY) ? 0.0f : m_acc;
        if (p.lse) p.lse[row * p.H + f.h] = good ? (mm + log2f(l)) * 0.6931471805599453f : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, TMEM_COLS);
}

// Sharded mode: the landmark K/V rows of every (local set, head) gathered into 128-row
// tiles, [set][head][tile][row][D], rows past the set's length or with position -1 zero.
// Rows are read from their owner rank's K/V shard (plain loads; peers' memory over NVLink).
// One CTA per (set, head, tile), 16 bytes per thread and row chunk.
template <int HD>
__global__ void __launch_bounds__(256) lmk_gather_kernel(const int32_t* __restrict__ lmk, int H, int rep,
                                                         int n_sets, int k, int nlt,
                                                         const uint16_t* const* __restrict__ ksrc,
                                                         const uint16_t* const* __restrict__ vsrc, int rows_per_src,
                                                         int64_t kv_stride, uint16_t* __restrict__ lk,
                                                         uint16_t* __restrict__ lv) {
  constexpr int CPR = HD / 8;
  const int lt = blockIdx.x % nlt, hs = blockIdx.x / nlt;  // hs = set * H + h
  const int h = hs % H, set = hs / H, hk = h / rep;
  const int32_t* P = lmk + ((int64_t)h * n_sets + set) * k;
  uint16_t* dk = lk + (int64_t)blockIdx.x * BN * HD;
  uint16_t* dv = lv + (int64_t)blockIdx.x * BN * HD;
  for (int e = threadIdx.x; e < BN * CPR; e += blockDim.x) {
    const int r = e / CPR, c = e - r * CPR;
    const int idx = lt * BN + r;
    const int pos = idx < k ? __ldg(P + idx) : -1;
    uint4 kv = make_uint4(0, 0, 0, 0), vv = kv;
    if (pos >= 0) {
      const int src = pos / rows_per_src;
      const int64_t off = (int64_t)(pos - src * rows_per_src) * kv_stride + (int64_t)hk * HD + c * 8;
      kv = *reinterpret_cast<const uint4*>(ksrc[src] + off);
      vv = *reinterpret_cast<const uint4*>(vsrc[src] + off);
    }
    reinterpret_cast<uint4*>(dk)[e] = kv;
    reinterpret_cast<uint4*>(dv)[e] = vv;
  }
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

// 2-D map over token rows of `cols` 16-bit elements (row stride row_stride elements), boxes of
// one row x 64 columns, 128-byte swizzle: the landmark gathers (tile::gather4)
static int make_gather_map(CUtensorMap* m, const void* base, int dtype, int64_t cols, int64_t rows,
                           int64_t row_stride) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return fail(DSALT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  const cuuint32_t box[2] = {64, 1};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dtype == DSALT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSALT_ERR_CUDA, "cuTensorMapEncodeTiled (gather) failed (%d)", (int)r);
  return DSALT_OK;
}

}  // namespace tc

int launch_attn_tc(const void* q, const void* k, const void* v, int dtype, int64_t T, int H, int Hkv, int HD,
                   int64_t q_stride, int64_t kv_stride, const int32_t* w, const int32_t* lmk, const float* lmk_bias,
                   int k_lmk, int lmk_block, const int32_t* cu, int n_seqs, int32_t* set_base, int32_t* tile_base,
                   int4* plan, int64_t max_tiles, void* out, int out_dtype, float* lse, int* err,
                   cudaStream_t stream, const ShardArgs* shard, const float* w_soft, float soft_edge,
                   float soft_tau) {
  using namespace tc;
  if (w_soft && (shard || !(soft_edge >= 0.0f && soft_edge <= 4.0f) || !(soft_tau > 0.0f)))
    return fail(DSALT_ERR_UNSUPPORTED, "attention (tensor cores): soft edge needs 0 <= win_edge <= 4, tau > 0");
  if (HD != 64 && HD != 128)
    return fail(DSALT_ERR_UNSUPPORTED, "attention (tensor cores): head_dim %d not supported (64, 128)", HD);
  if (k_lmk > MAX_LMK) return fail(DSALT_ERR_UNSUPPORTED, "attention: k_lmk %d above %d", k_lmk, MAX_LMK);
  if (lmk_block % BM) return fail(DSALT_ERR_UNSUPPORTED, "attention: lmk_block must be a multiple of %d", BM);
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15 || (q_stride * 2) % 16 ||
      (kv_stride * 2) % 16)
    return fail(DSALT_ERR_INVALID, "attention: q/k/v/out must be 16-byte aligned with 16-byte row strides");
  // q/out rows: T (packed) or the shard's query rows; k/v rows: T or the shard's key rows
  const int64_t q_rows = shard ? shard->q_rows : T, kv_rows = shard ? shard->kv_rows : T;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, q, dtype, HD, H, q_rows, q_stride))) return rc;
  if ((rc = make_map(&mk, k, dtype, HD, Hkv, kv_rows, kv_stride))) return rc;
  if ((rc = make_map(&mv, v, dtype, HD, Hkv, kv_rows, kv_stride))) return rc;
  const int shard_tiles = shard ? (int)(shard->q_rows / BM) : 0;
  if (shard) {
    tile_plan_kernel<<<(unsigned)((shard_tiles + 7) / 8), 256, 0, stream>>>(
        cu, n_seqs, tile_base, set_base, lmk_block, w, plan, shard_tiles, (int)shard->q_pos0, (int)shard->kv_pos0,
        (int)shard->seq_len, lmk_block ? (int)(shard->q_pos0 / lmk_block) : 0);
  } else {
    if ((rc = launch_chunk_table(cu, n_seqs, BM, tile_base, stream))) return rc;
    if (lmk_block > 0 && (rc = launch_chunk_table(cu, n_seqs, lmk_block, set_base, stream))) return rc;
    tile_plan_kernel<<<(unsigned)((max_tiles + 7) / 8), 256, 0, stream>>>(cu, n_seqs, tile_base, set_base, lmk_block,
                                                                         w, plan, 0, 0, 0, 0, 0);
  }
  if ((rc = check_cuda(cudaGetLastError(), "tile plan launch"))) return rc;
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
  p.plan = plan;
  CUtensorMap mlk, mlv;
  if (!shard) {
    // landmark rows: 2-D maps (rows = tokens, columns = all kv heads), one-row boxes, for
    // the four-row TMA gathers
    if ((rc = make_gather_map(&mlk, k, dtype, (int64_t)Hkv * HD, T, kv_stride))) return rc;
    if ((rc = make_gather_map(&mlv, v, dtype, (int64_t)Hkv * HD, T, kv_stride))) return rc;
  } else {
    mlk = mk;
    mlv = mv;
  }
  if (shard) {
    p.shard_tiles = shard_tiles;
    p.n_sets_local = lmk_block ? (int)((shard->q_rows + lmk_block - 1) / lmk_block) : 1;
    const int nlt = (k_lmk + BN - 1) / BN;
    const int64_t tiles = (int64_t)p.n_sets_local * H * nlt;
    if (tiles > 0) {
      auto gk = HD == 64 ? lmk_gather_kernel<64> : lmk_gather_kernel<128>;
      gk<<<(unsigned)tiles, 256, 0, stream>>>(
          lmk, H, H / Hkv, p.n_sets_local, k_lmk, nlt, reinterpret_cast<const uint16_t* const*>(shard->lmk_k_src),
          reinterpret_cast<const uint16_t* const*>(shard->lmk_v_src), (int)shard->rows_per_src, kv_stride,
          reinterpret_cast<uint16_t*>(shard->lmk_tiles_k), reinterpret_cast<uint16_t*>(shard->lmk_tiles_v));
      if ((rc = check_cuda(cudaGetLastError(), "landmark gather launch"))) return rc;
      if ((rc = make_map(&mlk, shard->lmk_tiles_k, dtype, HD, 1, tiles * BN, HD))) return rc;
      if ((rc = make_map(&mlv, shard->lmk_tiles_v, dtype, HD, 1, tiles * BN, HD))) return rc;
    }
  }
  p.w_soft = w_soft;
  p.soft_edge = soft_edge;
  p.soft_tau = soft_tau;
  p.scale_log2 = (float)(1.0 / sqrt((double)HD) * 1.4426950408889634);
  p.inv_scale = (float)sqrt((double)HD);
  const uint32_t ab = dtype == DSALT_BF16 ? 1u : 0u;
  p.idesc_qk = umma_idesc_f16(ab, 0, 0, BM, BN);
  p.idesc_pv = umma_idesc_f16(ab, 0, 1, BM, HD);
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_v8 = ((uintptr_t)out & 31) == 0 ? 1 : 0;
  p.lse = lse;
  p.err = err;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t max_items = (shard ? (int64_t)shard_tiles : T / BM + n_seqs) * (int64_t)H;
  const int np = HD == 64 ? Pipes<64>::N : Pipes<128>::N;
  const int64_t want = (max_items + np - 1) / np;
  const int grid = (int)(want < nsm ? want : nsm);
  if (grid <= 0) return DSALT_OK;
  const size_t smem = (HD == 64 ? Smem<64>::BYTES : Smem<128>::BYTES) + 1024;
  const int threads = HD == 64 ? Pipes<64>::THREADS : Pipes<128>::THREADS;
  const bool bf = dtype == DSALT_BF16;
  auto kern = w_soft ? (HD == 64 ? (bf ? attn_fwd_tc_kernel<64, true, true> : attn_fwd_tc_kernel<64, false, true>)
                                 : (bf ? attn_fwd_tc_kernel<128, true, true> : attn_fwd_tc_kernel<128, false, true>))
                     : (HD == 64 ? (bf ? attn_fwd_tc_kernel<64, true, false> : attn_fwd_tc_kernel<64, false, false>)
                                 : (bf ? attn_fwd_tc_kernel<128, true, false> : attn_fwd_tc_kernel<128, false, false>));
  if ((rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "attention smem attr")))
    return rc;
  kern<<<grid, threads, smem, stream>>>(mq, mk, mv, mlk, mlv, p);
  return check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace dsalt
