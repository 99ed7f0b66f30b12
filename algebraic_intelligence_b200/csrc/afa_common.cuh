// Shared device helpers for the B200 (sm_100a) Algebraic FlashAttention library.
//
// * the octic weight map rho(s)^8 (reference: src/kernels/pallas_afa.py:32-49 and
//   src/attention.py:18-26) in the forms the kernels use;
// * thin inline-PTX wrappers for mbarriers, TMA tensor loads and the tcgen05
//   (5th-generation tensor core / tensor memory) instructions;
// * bounded waits: every spin on an mbarrier gives up after a wall-clock budget,
//   records where it gave up in a device status word and returns false, so a
//   logic error surfaces as a status code instead of a hung GPU.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "afa_problem.h"

namespace afa {

// ---------------------------------------------------------------------------
// Octic weight map
// ---------------------------------------------------------------------------

// Hardware reciprocal square root / reciprocal (MUFU), flush-to-zero forms.
__device__ __forceinline__ float rsqrt_approx(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Reference form (pallas_afa.py:39-49, attention.py:18-26): r = rsqrt(1+s^2),
// u = s*r, rho = (s < 0) ? r / (1 - u) : s + (1 + s^2) * r, then three
// squarings. The division is IEEE-rounded, as in the reference's XLA lowering.
__device__ __forceinline__ float octic_ref(float s) {
  const float rad = fmaf(s, s, 1.0f);
  const float r = rsqrtf(rad);
  const float u = s * r;
  const float rho = (s < 0.0f) ? __fdiv_rn(r, 1.0f - u) : fmaf(rad, r, s);
  const float k2 = rho * rho;
  const float k4 = k2 * k2;
  return k4 * k4;
}
__device__ __forceinline__ double octic_ref(double s) {
  const double rad = fma(s, s, 1.0);
  const double r = rsqrt(rad);
  const double u = s * r;
  const double rho = (s < 0.0) ? r / (1.0 - u) : fma(rad, r, s);
  const double k2 = rho * rho;
  const double k4 = k2 * k2;
  return k4 * k4;
}

// Hardware square root (MUFU), flush-to-zero form.
__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Tensor-core fast form: rho = s + sqrt(1 + s^2) for both signs -- the
// reference's positive branch (pallas_afa.py:46, which forms the square root
// as (1 + s^2) * rsqrt(1 + s^2)) applied to every s -- with one MUFU op per
// score, on a pair of scores with the sm_100 packed FP32 instructions
// (FFMA2 / FADD2 / FMUL2). The tensor-core kernels are bound by MUFU/issue
// throughput, and the conjugate negative branch costs a second MUFU op (a
// reciprocal) per score, which measured 30-45% slower. sqrt.approx then an
// add mapped 2.5% faster than rsqrt.approx then an FMA (+4% on an L = 4096
// prefill).
// Error: sqrt.approx measured relative error |d| <= 2^-23.3 (rsqrt.approx
// 2^-22.9) over 2^24 inputs in [1, 2^60], and 1 + s^2 is rounded once
// (2^-24), so rho(s) for s >= 0 is within ~2^-22.5; for s < 0 the sum
// cancels (rho ~ 1/(2|s|) against terms of size |s|) and the relative error of
// rho grows to ~ 2 s^2 (|d| + 2^-25), i.e. rho^8 to ~ 2.5e-6 s^2: 6.4e-4 at
// s = -16, 1% at s = -64, 16% at s = -256. The kernels therefore use this form
// only where that error cannot reach the result (see kTailChunkSum and
// kTailRowSum) and octic_exact2 elsewhere.
__device__ __forceinline__ float2 octic_fast2(float2 s) {
  const float2 rad = __ffma2_rn(s, s, make_float2(1.0f, 1.0f));
  const float2 rho = __fadd2_rn(make_float2(sqrt_approx(rad.x), sqrt_approx(rad.y)), s);
  const float2 k2 = __fmul2_rn(rho, rho);
  const float2 k4 = __fmul2_rn(k2, k2);
  return __fmul2_rn(k4, k4);
}

// The reference's branch form (pallas_afa.py:39-49) on a pair of scores, with
// hardware approximations: r = rsqrt.approx(1 + s^2), and for s < 0
// rho = r * rcp.approx(1 - s r), the conjugate that never cancels (1 - s r lies
// in [1, 2)); for s >= 0 rho = (1 + s^2) r + s. rho is within ~4 ulp for every
// s, so rho^8 is within ~4e-6 relative -- the negative tail included. Also
// returns r, which the backward reuses. Two MUFU ops per negative score: the
// tensor-core kernels run it only on chunks whose weights all lie in the tail.
__device__ __forceinline__ float2 octic_exact2(float2 s, float2& r) {
  const float2 rad = __ffma2_rn(s, s, make_float2(1.0f, 1.0f));
  r = make_float2(rsqrt_approx(rad.x), rsqrt_approx(rad.y));
  const float2 pos = __ffma2_rn(rad, r, s);
  const float2 u = __fmul2_rn(s, r);
  float2 rho;
  rho.x = s.x < 0.0f ? r.x * rcp_approx(1.0f - u.x) : pos.x;
  rho.y = s.y < 0.0f ? r.y * rcp_approx(1.0f - u.y) : pos.y;
  const float2 k2 = __fmul2_rn(rho, rho);
  const float2 k4 = __fmul2_rn(k2, k2);
  return __fmul2_rn(k4, k4);
}
__device__ __forceinline__ float2 octic_exact2(float2 s) {
  float2 r;
  return octic_exact2(s, r);
}

// When the fast form is exact enough. Errors below are relative to the sum of
// the weights they are part of; a weighted mean of values (the output) carries
// at most the same relative error.
//
// Per chunk (forward: one query row against 32 keys): if the chunk's weights
// sum to at least kTailChunkSum (= rho(-15.8)^8), every key at s >= -32
// carries relative error <= 2.6e-3, and the keys below -32 -- whose errors
// are larger but whose weights fall as s^-8 -- add at most
// 32 * 2.6e-3 * (16/32)^8 = 3.3e-4 of the chunk's sum. So a chunk with sum
// >= kTailChunkSum is within ~3e-3 of exact, under the bf16 rounding of P; a
// chunk below it is mapped again with octic_exact2.
constexpr float kTailChunkSum = 1e-12f;
// Per row (or any set of a row's keys): once the weights sum to at least
// kTailRowSum (= rho(-4.95)^8), a key at s < -16 adds error at most
// eps(s) rho(s)^8 <= 6.4e-4 * rho(-16)^8 = 5.8e-16, i.e. 5.8e-8 of the sum, so
// even 65536 such keys add < 4e-3, and keys at s >= -16 carry <= 6.4e-4 each.
// The forward therefore checks chunks only until every row of a warp has
// passed kTailRowSum, and the backward, which knows each row's sum from
// d_total - sink, takes the exact form for the rows below it.
constexpr float kTailRowSum = 1e-8f;

// ---------------------------------------------------------------------------
// Type helpers
// ---------------------------------------------------------------------------
template <typename T> struct AccOf { using type = float; };
template <> struct AccOf<double> { using type = double; };

__device__ __forceinline__ float to_acc(float x) { return x; }
__device__ __forceinline__ double to_acc(double x) { return x; }
__device__ __forceinline__ float to_acc(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_acc(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_acc(float x);
template <> __device__ __forceinline__ float from_acc<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_acc<__half>(float x) { return __float2half_rn(x); }
template <typename T> __device__ __forceinline__ T from_acc(double x);
template <> __device__ __forceinline__ double from_acc<double>(double x) { return x; }

// The value P takes in the P.V product: P.astype(v.dtype) (pallas_afa.py:133).
template <typename T> __device__ __forceinline__ float round_like(float x) { return to_acc(from_acc<T>(x)); }
template <> __device__ __forceinline__ float round_like<float>(float x) { return x; }
__device__ __forceinline__ double round_like_d(double x) { return x; }

// ---------------------------------------------------------------------------
// Device status word and bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wall-clock budget of one wait. Correct launches wait microseconds; only a
// logic error can reach this.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void flag_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}
__device__ __forceinline__ bool error_raised(const int* status) {
  return status && *reinterpret_cast<const volatile int*>(status) != 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits until the phase with the given parity has completed. Returns false
// (after flagging `code` in *status) when the budget runs out, or as soon as
// another thread of the launch has flagged an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          uint64_t budget_ns = kWaitBudgetNs) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(a, parity)) return true;
    if (error_raised(status)) return false;
    if (globaltimer_ns() - t0 > budget_ns) {
      flag_error(status, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tensor loads, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// TMA store of a shared-memory box to global memory (bulk-group completion;
// no multicast). The x coordinate c0 must be 16-byte aligned and no coordinate
// may be negative; rows outside the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and UMMA
// ---------------------------------------------------------------------------
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
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; kind::f16 covers bf16 inputs.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc].
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The mbarrier arrives once every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm100 layout: start>>4 in
// bits 0-13, leading byte offset>>4 in 16-29, stride byte offset>>4 in 32-45,
// version 1 in 46-47, swizzle mode 2 (128B) in 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// The descriptor of the operand `bytes` past the one `d` describes: the start
// field holds address >> 4 in bits 0-13, so for a 16-byte multiple that keeps
// the address below 256 KB (every shared-memory address does) the sum moves
// the start and leaves the other fields as they are.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }

// Instruction descriptor, kind::f16 with bf16 A/B and an fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, bool b_mn_major) {
  return (1u << 4)                                  // D format: F32
         | (1u << 7)                                // A format: BF16
         | (1u << 10)                               // B format: BF16
         | ((b_mn_major ? 1u : 0u) << 16)           // B major-ness
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// 32 lanes x 32 columns of 32-bit words: thread i of the warp receives lane
// (warp%4)*32+i, columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace afa
