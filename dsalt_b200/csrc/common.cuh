// Shared device helpers for the DSALT B200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/dsalt_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "dsalt_b200 targets sm_100a only"
#endif

namespace dsalt {

// One rank's share of a sequence-sharded attention call (see dsalt_attention_fwd_sharded):
// q/out rows are positions [q_pos0, q_pos0 + q_rows) of one sequence of seq_len positions,
// k/v rows are positions [kv_pos0, kv_pos0 + kv_rows); landmark row of position p is row
// p - r * rows_per_src of rank r = p / rows_per_src's K/V (device arrays of pointers).
// lmk_tiles_k / lmk_tiles_v: workspace for the gathered landmark tiles of the local sets.
struct ShardArgs {
  int64_t q_pos0, q_rows, kv_pos0, kv_rows, seq_len, rows_per_src;
  const void* const* lmk_k_src;
  const void* const* lmk_v_src;
  void* lmk_tiles_k;
  void* lmk_tiles_v;
};

// --------------------------------------------------------------------------
// host-side error reporting (set by the C-ABI entry points)
// --------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int* device_status_ptr();  // device address of the status word of the current device

// device-side status word: the first kernel that gives up a bounded wait records a
// code here; the host reads it with dsalt_device_status().
__device__ __forceinline__ void report_device_error(int* flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

// --------------------------------------------------------------------------
// element access
// --------------------------------------------------------------------------
__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dt) {
  if (dt == DSALT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == DSALT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// round a float32 to bf16 / fp16 (ties to even), returned as float
__device__ __forceinline__ float round_bf16(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
__device__ __forceinline__ float round_f16(float f) { return __half2float(__float2half_rn(f)); }
__device__ __forceinline__ float round_to(float f, int dt) {
  return dt == DSALT_BF16 ? round_bf16(f) : (dt == DSALT_F16 ? round_f16(f) : f);
}

// correctly rounded float64 -> bf16 (no double rounding through float32)
__device__ __forceinline__ float f64_to_bf16(double a) {
  float f = __double2float_rn(a);
  uint32_t u = __float_as_uint(f);
  if ((u & 0xFFFFu) == 0x8000u && isfinite(f)) {
    // f sits on a bf16 midpoint: decide from the float64 value
    float lo = __uint_as_float(u & 0xFFFF0000u);
    float hi = __uint_as_float((u & 0xFFFF0000u) + 0x10000u);
    double dlo = fabs(a - (double)lo), dhi = fabs(a - (double)hi);
    if (dlo < dhi) return lo;
    if (dhi < dlo) return hi;
  }
  return round_bf16(f);
}
// float64 -> fp16 with a single rounding: the float32 intermediate can only mislead
// when it lands exactly on an fp16 midpoint, which is then decided from the float64.
__device__ __forceinline__ float f64_to_f16(double a) {
  float f = __double2float_rn(a);
  float r = round_f16(f);
  if (!isfinite(f)) return r;
  __half hz = __float2half_rz(f);
  float lo = __half2float(hz);
  if (lo == f) return f;
  float hi = __half2float(__ushort_as_half((unsigned short)(__half_as_ushort(hz) + 1)));
  if ((double)f * 2.0 == (double)lo + (double)hi) {
    double dlo = fabs(a - (double)lo), dhi = fabs(a - (double)hi);
    if (dlo < dhi) return lo;
    if (dhi < dlo) return hi;
  }
  return r;
}
__device__ __forceinline__ float f64_to(double a, int dt) {
  return dt == DSALT_BF16 ? f64_to_bf16(a) : (dt == DSALT_F16 ? f64_to_f16(a) : __double2float_rn(a));
}

// --------------------------------------------------------------------------
// double-double accumulation (Knuth two-sum): the rounded result of a dd sum is the
// correctly rounded float64 value of the exact sum except in cases within 2^-100
// (relative) of a float64 rounding boundary.
// --------------------------------------------------------------------------
struct DD {
  double hi, lo;
};
__device__ __forceinline__ DD two_sum(double a, double b) {
  double s = __dadd_rn(a, b);
  double bb = __dsub_rn(s, a);
  double err = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
  return DD{s, err};
}
__device__ __forceinline__ DD dd_add(DD a, DD b) {
  DD s = two_sum(a.hi, b.hi);
  DD t = two_sum(a.lo, b.lo);
  s.lo = __dadd_rn(s.lo, t.hi);
  DD u = two_sum(s.hi, s.lo);
  u.lo = __dadd_rn(u.lo, t.lo);
  return two_sum(u.hi, u.lo);
}
__device__ __forceinline__ DD dd_add_d(DD a, double b) {
  DD s = two_sum(a.hi, b);
  s.lo = __dadd_rn(s.lo, a.lo);
  return two_sum(s.hi, s.lo);
}
__device__ __forceinline__ double dd_round(DD a) { return __dadd_rn(a.hi, a.lo); }
__device__ __forceinline__ DD dd_shfl_xor(DD a, int off) {
  return DD{__shfl_xor_sync(0xffffffffu, a.hi, off), __shfl_xor_sync(0xffffffffu, a.lo, off)};
}
__device__ __forceinline__ DD dd_warp_sum(DD a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = dd_add(a, dd_shfl_xor(a, o));
  return a;
}

// --------------------------------------------------------------------------
// selection keys: 64-bit, larger = better (higher score, then lower position)
// --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t order_f32(float s) {
  uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint64_t make_key(float score, int32_t pos) {
  return ((uint64_t)order_f32(score) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)pos);
}
__device__ __forceinline__ int32_t key_pos(uint64_t key) {
  return (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

// --------------------------------------------------------------------------
// mbarrier / async-proxy helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: polls the barrier phase; after `timeout_ns` of wall time it records
// `code` in the device status word and returns false so the caller can wind down.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err_flag, int code,
                                          uint64_t timeout_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) break;
  }
  report_device_error(err_flag, code);
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory (no multicast); completion counted in
// bytes on the mbarrier. Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_dst),
               "l"(__cvta_generic_to_global(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// cp.async (16 bytes, zero-filled when src_bytes == 0) and its mbarrier tracking
__device__ __forceinline__ void cp_async_16(uint32_t smem_addr, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(__cvta_generic_to_global(gmem)),
               "r"(src_bytes)
               : "memory");
}
// 4-byte cp.async (zero-filled when src_bytes == 0)
__device__ __forceinline__ void cp_async_4(uint32_t smem_addr, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr), "l"(__cvta_generic_to_global(gmem)),
               "r"(src_bytes)
               : "memory");
}
// the mbarrier's pending count is raised by one now and lowered when this thread's prior
// cp.async operations have completed
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMA: 3-D tiled load into shared memory, completion on an mbarrier (no multicast)
__device__ __forceinline__ void tma_load_3d(uint32_t smem_addr, const void* tmap, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_addr),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// TMA gather of four rows of a 2-D tensor map (box: one row of 64 columns) into four
// consecutive 128-byte rows of shared memory, completion on an mbarrier (no multicast).
// col: first column (a multiple of 8 for 16-bit data); r0..r3: row coordinates.
__device__ __forceinline__ void tma_gather4(uint32_t smem_addr, const void* tmap, uint64_t* bar, int col, int r0,
                                            int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6, %7}], [%2];" ::"r"(smem_addr),
      "l"(tmap), "r"(smem_u32(bar)), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// --------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core) helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread
#define DSALT_TMEM_LD32(taddr, r)                                                                                  \
  asm volatile(                                                                                                    \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                               \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),     \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),    \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                  \
      : "r"(taddr))

// 32 lanes x 16 columns of 32-bit TMEM -> 16 registers per thread
#define DSALT_TMEM_LD16(taddr, r)                                                                              \
  asm volatile(                                                                                                \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];" \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),       \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])    \
      : "r"(taddr))

// 32 lanes x 16 columns of 32-bit registers -> TMEM
#define DSALT_TMEM_ST16(taddr, r)                                                                              \
  asm volatile(                                                                                                \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" \
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),   \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])             \
      : "memory")

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 format): start address >> 4 in bits [0,14),
// leading byte offset >> 4 in [16,30), stride byte offset >> 4 in [32,46), version 1 in
// [46,48), layout type in [61,64) (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16: fp32 accumulate, A/B of type `ab`
// (0 = f16, 1 = bf16), A/B major-ness (0 = K-major, 1 = MN-major), M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t ab, uint32_t a_mn_major, uint32_t b_mn_major,
                                                      uint32_t M, uint32_t N) {
  return (1u << 4)               // D format: f32
         | (ab << 7)             // A format
         | (ab << 10)            // B format
         | (a_mn_major << 15)    // A major
         | (b_mn_major << 16)    // B major
         | ((N >> 3) << 17)      // N
         | ((M >> 4) << 24);     // M
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "selp.b32 %0, 1, 0, px;\n\t}"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

}  // namespace dsalt
