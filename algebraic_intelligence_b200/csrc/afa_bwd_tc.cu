// AFA backward on the tcgen05 tensor cores (bf16 inputs, head_dim 64 or 128).
//
// Same math as afa_bwd.cu (tiled_afa_backward, src/kernels/pallas_afa.py:
// 409-522): w = rho(s)^8 / d_total, ds = 8 scale r w (g_out.v - E),
// dq = ds k, dk = ds^T q, dv = w^T g_out, with w and ds rounded to bf16 before
// the products (:440-448) and fp32 accumulation. rho uses a single-MUFU form,
// rho = (1+s^2) rsqrt(1+s^2) + s, whose rsqrt is also the r of the score
// derivative.
//
// Two kernels, each with the forward's warp roles (576 threads: 16 "grad"
// warps, 1 TMA warp, 1 MMA-issue warp) and one CTA per SM:
//
//   afa_bwd_dkv_tc_kernel  one 128-key tile per CTA, looping over the query
//     tiles that see it. TMEM holds S^T = K Q^T and dP^T = V dO^T (keys on the
//     lanes), then dV and dK. A thread owns one key (one TMEM lane); warpgroup g
//     owns query columns [32g, 32g+32). It turns its S^T and dP^T columns into
//     W^T and dS^T, written back as packed bf16 over its dP^T columns, which is
//     the A operand layout of the next two MMAs:
//     dV += W^T dO and dK += dS^T Q (B = the dO / Q tile read MN-major, the
//     same shared-memory tile the S^T MMA read K-major).
//   afa_bwd_dq_tc_kernel   one 128-query tile per CTA, looping over visible key
//     tiles: S = Q K^T and dP = dO V^T, then dQ += dS K with dS from TMEM
//     (queries on the lanes, per-row 1/d_total and E in registers).
//
// TMEM columns: X (S^T or S) [0,128), then one or two Y buffers (dP^T or dP,
// then the packed dS and W), then the accumulators (struct Tmem). The next
// tile's S (and, with two Y buffers, its dP) runs on the tensor core while the
// grad warps work on this tile. K/Q/V/dO tiles are TMA-loaded with 128-byte
// swizzle, no multicast.
// Every wait is bounded (afa_common.cuh) and reports to the device status word.
#include <cstdio>

#include "afa_b200.h"
#include "afa_common.cuh"
#include "afa_internal.h"
#include "afa_tmap.h"

namespace afa {
namespace {

template <int HD>
struct BwdCfg {
  static constexpr int kTmaWarp = 16;
  static constexpr int kMmaWarp = 17;
  static constexpr int kThreads = 18 * 32;
  static constexpr int KSUB = HD / 64;
  static constexpr int SUB_BYTES = 128 * 128;
  static constexpr int TILE_BYTES = KSUB * SUB_BYTES;  // 128 rows x HD bf16
  static constexpr int NST = 2;                        // stages of the streamed tile pair
  static constexpr int FIX_OFF = 0;                    // the CTA's two fixed tiles
  static constexpr int ST_OFF = 2 * TILE_BYTES;
  static constexpr int VEC_OFF = ST_OFF + NST * 2 * TILE_BYTES;  // per grad warp: 32 x (1/d, -8 scale E) floats
  static constexpr int BAR_OFF = VEC_OFF + 16 * 64 * 4;
  static constexpr int NBAR = 1 + 2 * NST + 6;  // fix_full, st_full[], st_empty[], s_full, x_read, g_full[2], o_full, drain
  static constexpr int SMEM_BYTES = BAR_OFF + NBAR * 8 + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t X_COL = 0;
  __device__ static constexpr uint32_t p_col(int kk) {
    return static_cast<uint32_t>((kk >> 1) * 32 + (kk & 1) * 8);
  }
};

// TMEM columns. X holds S (or S^T); Y holds dP (or dP^T) and then, packed as
// bf16 over each 32-column chunk, dS in the first 16 columns and W in the
// last 16 (the A operands of the accumulating products). With DBY there are
// two Y buffers, so the next tile's S and dP run while this tile's grad math
// does; without, only the next S does. Accumulators follow.
template <int HD, bool DBY>
struct Tmem {
  __device__ static constexpr uint32_t y(int b) { return 128u + (DBY ? 128u * static_cast<uint32_t>(b) : 0u); }
  static constexpr uint32_t ACC0 = DBY ? 384u : 256u;
  static constexpr uint32_t ACC1 = ACC0 + HD;
};

struct BwdTcArgs {
  const float* dtot;  // (B, H, L) d_total
  const float* e;     // (B, H, L) E
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int* status;
  int L, causal, valid;
  float scale;
  float sink;  // d_total - sink is a row's weight sum (the tail test)
};

// True when query row q's weights all lie in the negative tail of rho^8.
__device__ __forceinline__ bool tail_row(const BwdTcArgs& A, float dtot) { return dtot - A.sink < kTailRowSum; }

struct Bars {
  uint64_t *fix_full, *st_full, *st_empty, *s_full, *x_read, *g_full, *o_full, *drain;
  uint32_t* tmem_slot;
};

template <int HD>
__device__ __forceinline__ Bars carve(uint8_t* smem) {
  using C = BwdCfg<HD>;
  Bars b;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  b.fix_full = bars;
  b.st_full = bars + 1;
  b.st_empty = b.st_full + C::NST;
  b.s_full = b.st_empty + C::NST;
  b.x_read = b.s_full + 1;
  b.g_full = b.x_read + 1;  // two, by tile parity (see issue())
  b.o_full = b.g_full + 2;
  b.drain = b.o_full + 1;
  b.tmem_slot = reinterpret_cast<uint32_t*>(b.drain + 1);
  return b;
}

template <int HD>
__device__ __forceinline__ uint32_t setup(uint8_t* smem, const Bars& b, const CUtensorMap* t0, const CUtensorMap* t1,
                                          const CUtensorMap* t2, const CUtensorMap* t3) {
  using C = BwdCfg<HD>;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(b.fix_full, 1);
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(b.st_full + s, 1);
      mbar_init(b.st_empty + s, 1);
    }
    mbar_init(b.s_full, 1);
    mbar_init(b.x_read, 16);  // one elected arrive per grad warp
    mbar_init(b.g_full, 16);
    mbar_init(b.g_full + 1, 16);
    mbar_init(b.o_full, 1);
    mbar_init(b.drain, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(t0);
    prefetch_tmap(t1);
    prefetch_tmap(t2);
    prefetch_tmap(t3);
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(b.tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return *b.tmem_slot;
}

// TMA producer: the two fixed tiles (rows fix_row), then `niter` pairs of
// streamed tiles (rows st_row0 + 128 * it) through NST stages.
template <int HD>
__device__ __forceinline__ void produce(uint8_t* smem, const Bars& b, const CUtensorMap* fa, const CUtensorMap* fb,
                                        const CUtensorMap* sa, const CUtensorMap* sb, int fix_row, int st_row0,
                                        int niter, int bh, int* status) {
  using C = BwdCfg<HD>;
  if (niter <= 0) return;
  mbar_arrive_expect_tx(b.fix_full, 2 * C::TILE_BYTES);
  for (int h = 0; h < C::KSUB; ++h) {
    tma_load_3d(smem + C::FIX_OFF + h * C::SUB_BYTES, fa, b.fix_full, 64 * h, fix_row, bh);
    tma_load_3d(smem + C::FIX_OFF + C::TILE_BYTES + h * C::SUB_BYTES, fb, b.fix_full, 64 * h, fix_row, bh);
  }
  int issued = 0;
  for (int it = 0; it < niter; ++it) {
    const int s = it % C::NST;
    if (!mbar_wait(b.st_empty + s, ((it / C::NST) & 1) ^ 1, status, kDevTimeoutProducer)) break;
    mbar_arrive_expect_tx(b.st_full + s, 2 * C::TILE_BYTES);
    uint8_t* base = smem + C::ST_OFF + s * 2 * C::TILE_BYTES;
    for (int h = 0; h < C::KSUB; ++h) {
      tma_load_3d(base + h * C::SUB_BYTES, sa, b.st_full + s, 64 * h, st_row0 + 128 * it, bh);
      tma_load_3d(base + C::TILE_BYTES + h * C::SUB_BYTES, sb, b.st_full + s, 64 * h, st_row0 + 128 * it, bh);
    }
    issued = it + 1;
  }
  // Do not leave the CTA while loads into its shared memory are in flight.
  (void)mbar_wait(b.fix_full, 0, nullptr, 0);
  for (int it = issued - C::NST < 0 ? 0 : issued - C::NST; it < issued; ++it)
    (void)mbar_wait(b.st_full + (it % C::NST), (it / C::NST) & 1, nullptr, 0);
}

// MMA issuer. X = F0 S0^T and Y = F1 S1^T (F = the CTA's fixed tiles, S =
// the streamed pair, both read K-major); once the grad warps have written the
// packed operands into Y, the accumulating products read the streamed tiles
// MN-major:
//   dK/dV kernel (TWO): F = (K, V), S = (Q, dO); ACC0 = dV += W^T dO,
//                       ACC1 = dK += dS^T Q.
//   dQ kernel:          F = (Q, dO), S = (K, V); ACC0 = dQ += dS K.
// Order per tile j: [wait the grad warps' reads of X] next X (and next Y with
// DBY), [wait the packed operands] this tile's products, release the stage,
// next Y (without DBY). With DBY the grad warps may finish tile j+1 before
// this thread has seen tile j's operands ready, so that signal alternates
// between two barriers: reaching tile j+2 needs an s_full committed only after
// this thread passed tile j's wait, so no barrier gets two phases ahead.
template <int HD, bool TWO, bool DBY>
__device__ __forceinline__ void issue(uint8_t* smem, const Bars& b, uint32_t tmem, int niter, int* status) {
  using C = BwdCfg<HD>;
  using T = Tmem<HD, DBY>;
  if (niter <= 0) return;
  constexpr uint32_t idesc_x = idesc_bf16_f32(128, 128, false);
  constexpr uint32_t idesc_acc = idesc_bf16_f32(128, HD, true);
  // Base descriptors, built once; the loops add constant offsets (desc_add),
  // keeping this thread's instructions between MMAs few.
  const uint64_t fix_k = sw128_desc(smem_u32(smem + C::FIX_OFF), 16, 1024);
  const uint64_t st_k = sw128_desc(smem_u32(smem + C::ST_OFF), 16, 1024);
  const uint64_t st_mn = sw128_desc(smem_u32(smem + C::ST_OFF), C::SUB_BYTES, 1024);
  auto stage = [&](int j) { return static_cast<uint32_t>((j % C::NST) * 2 * C::TILE_BYTES); };
  auto score = [&](int t, int j, uint32_t dst) {  // t = 0: X = F0 S0^T, t = 1: Y = F1 S1^T
    const uint64_t sb = desc_add(st_k, stage(j) + t * C::TILE_BYTES);
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      const uint32_t off = (kk >> 2) * C::SUB_BYTES + (kk & 3) * 32;
      umma_ss(tmem + dst, desc_add(fix_k, t * C::TILE_BYTES + off), desc_add(sb, off), idesc_x, kk > 0 ? 1u : 0u);
    }
  };
  bool ok = mbar_wait(b.fix_full, 0, status, kDevTimeoutMma) && mbar_wait(b.st_full, 0, status, kDevTimeoutMma);
  if (ok) {
    tc_fence_after();
    score(0, 0, C::X_COL);
    score(1, 0, T::y(0));
    umma_commit(b.s_full);
  }
  for (int j = 0; ok && j < niter; ++j) {
    const int yb = DBY ? (j & 1) : 0;
    const bool more = j + 1 < niter;
    if (!(ok = mbar_wait(b.x_read, j & 1, status, kDevTimeoutMma))) break;
    if (more) {
      const int sn = (j + 1) % C::NST;
      if (!(ok = mbar_wait(b.st_full + sn, ((j + 1) / C::NST) & 1, status, kDevTimeoutMma))) break;
      tc_fence_after();
      score(0, j + 1, C::X_COL);
      if constexpr (DBY) {
        score(1, j + 1, T::y((j + 1) & 1));
        umma_commit(b.s_full);
      }
    }
    if (!(ok = mbar_wait(b.g_full + (j & 1), (j >> 1) & 1, status, kDevTimeoutMma))) break;
    tc_fence_after();
    const uint64_t sm = desc_add(st_mn, stage(j));
    const uint32_t ya = T::y(yb);
    if constexpr (TWO) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // dV += W^T dO
        const uint64_t m = desc_add(sm, C::TILE_BYTES + kk * 2048);
        umma_ts(tmem + T::ACC0, tmem + ya + C::p_col(kk) + 16, m, idesc_acc, (j > 0 || kk > 0) ? 1u : 0u);
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // dK += dS^T Q
        const uint64_t m = desc_add(sm, kk * 2048);
        umma_ts(tmem + T::ACC1, tmem + ya + C::p_col(kk), m, idesc_acc, (j > 0 || kk > 0) ? 1u : 0u);
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // dQ += dS K
        const uint64_t m = desc_add(sm, kk * 2048);
        umma_ts(tmem + T::ACC0, tmem + ya + C::p_col(kk), m, idesc_acc, (j > 0 || kk > 0) ? 1u : 0u);
      }
    }
    umma_commit(b.st_empty + (j % C::NST));
    if constexpr (!DBY) {
      if (more) {  // Y is single: after this tile's products have read it
        score(1, j + 1, T::y(0));
        umma_commit(b.s_full);
      }
    }
  }
  if (ok) umma_commit(b.o_full);
  // Every MMA this thread issued must finish before TMEM is released.
  umma_commit(b.drain);
  (void)mbar_wait(b.drain, 0, nullptr, 0);
}

// One 32-column chunk: scores x (raw S or S^T accumulator words), score
// gradients y (dP or dP^T); per-column (dK/dV kernel: vc[c/2] = (1/d_total of
// columns c, c+1, then -8 scale E of the same two)) or per-row (dQ kernel:
// inv_r, ne8_r) factors. ds = 8 scale r w (y - E) is formed as
// (r w) * fma(y, 8 scale, -8 scale E); w = p8 / d_total <= 1 keeps every
// product in range. Writes packed bf16 dS, and W per column (the dQ kernel
// needs no W). Element pairs go through the
// packed fp32x2 instructions (FFMA2 / FMUL2), which halve the issue slots of
// the map; the one MUFU op per element is the rsqrt. EXACT: the reference's
// branch form of rho (octic_exact2), for chunks that touch a query row whose
// weights all lie in the negative tail (d_total - sink < kTailRowSum), where
// the single-MUFU form cancels.
template <bool MASK, bool PER_COL, bool EXACT>
__device__ __forceinline__ void grad_chunk(const uint32_t (&x)[32], const uint32_t (&y)[32], uint32_t (&wp)[16],
                                           uint32_t (&dp)[16], float scale, const float4* vc, float inv_r,
                                           float ne8_r, int vis_lim, bool vis_row, int causal, int row_pos,
                                           int col_pos0, bool row_is_key) {
  const float2 sc = make_float2(scale, scale);
  const float2 c8 = make_float2(8.0f * scale, 8.0f * scale);
  const float2 invr = make_float2(inv_r, inv_r), ne8r = make_float2(ne8_r, ne8_r);
  const float2 one = make_float2(1.0f, 1.0f);
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    const float2 s = __fmul2_rn(make_float2(__uint_as_float(x[c]), __uint_as_float(x[c + 1])), sc);
    float2 r, p8;
    if constexpr (EXACT) {
      p8 = octic_exact2(s, r);
    } else {
      const float2 rad = __ffma2_rn(s, s, one);
      r = make_float2(rsqrt_approx(rad.x), rsqrt_approx(rad.y));
      const float2 rho = __ffma2_rn(rad, r, s);
      const float2 p2 = __fmul2_rn(rho, rho);
      const float2 p4 = __fmul2_rn(p2, p2);
      p8 = __fmul2_rn(p4, p4);
    }
    const float2 yv = make_float2(__uint_as_float(y[c]), __uint_as_float(y[c + 1]));
    float2 w = make_float2(0.f, 0.f), ds;
    if constexpr (PER_COL) {
      const float4 cv = vc[c >> 1];
      w = __fmul2_rn(p8, make_float2(cv.x, cv.y));
      ds = __fmul2_rn(__fmul2_rn(r, w), __ffma2_rn(yv, c8, make_float2(cv.z, cv.w)));
    } else {
      ds = __fmul2_rn(__fmul2_rn(r, __fmul2_rn(p8, invr)), __ffma2_rn(yv, c8, ne8r));
    }
    if (MASK) {
      // row_is_key: the row is a key, the columns queries; otherwise the reverse.
      const int col = col_pos0 + c;
      const int key0 = row_is_key ? row_pos : col, key1 = row_is_key ? row_pos : col + 1;
      const int qry0 = row_is_key ? col : row_pos, qry1 = row_is_key ? col + 1 : row_pos;
      const bool v0 = vis_row && key0 < vis_lim && (!causal || key0 <= qry0);
      const bool v1 = vis_row && key1 < vis_lim && (!causal || key1 <= qry1);
      w.x = v0 ? w.x : 0.0f;
      w.y = v1 ? w.y : 0.0f;
      ds.x = v0 ? ds.x : 0.0f;
      ds.y = v1 ? ds.y : 0.0f;
    }
    if constexpr (PER_COL) wp[c >> 1] = pack_bf16x2(w.x, w.y);
    dp[c >> 1] = pack_bf16x2(ds.x, ds.y);
  }
}

template <int HD>
__global__ void __launch_bounds__(576, 1)
    afa_bwd_dkv_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_g,
                          const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ BwdTcArgs A) {
  using C = BwdCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Bars b = carve<HD>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int k0 = blockIdx.y * 128;  // keys with the most causal queries first
  const int i_first = A.causal ? blockIdx.y : 0;
  const int nq = (A.L + 127) / 128;
  const int niter = k0 >= A.valid ? 0 : nq - i_first;
  const uint32_t tmem = setup<HD>(smem, b, &tm_q, &tm_g, &tm_k, &tm_v);

  constexpr bool DBY = HD == 64;  // two dP^T buffers fit next to dV and dK only at head_dim 64
  using T = Tmem<HD, DBY>;
  static_assert(T::ACC1 + HD <= C::TMEM_COLS, "TMEM budget");
  if (warp == C::kTmaWarp) {
    if (lane == 0) produce<HD>(smem, b, &tm_k, &tm_v, &tm_q, &tm_g, k0, 128 * i_first, niter, bh, A.status);
  } else if (warp == C::kMmaWarp) {
    if (lane == 0) issue<HD, true, DBY>(smem, b, tmem, niter, A.status);
  } else {
    const int g = warp >> 2, sub = warp & 3;
    const int row = sub * 32 + lane;
    const int key = k0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    float* vec = reinterpret_cast<float*>(smem + C::VEC_OFF) + warp * 64;
    const long long rbase = static_cast<long long>(bh) * A.L;
    bool ok = true;
    for (int it = 0; ok && it < niter; ++it) {
      const int q0 = 128 * (i_first + it);
      const int qc0 = q0 + 32 * g;
      bool tail;
      {  // 1/d_total and -8 scale E of this warp's 32 query columns, as float4s of two columns each
        const int qi = qc0 + lane;
        const bool in = qi < A.L;
        const float dt = in ? A.dtot[rbase + qi] : 1.0f;
        vec[(lane >> 1) * 4 + (lane & 1)] = in ? 1.0f / dt : 0.0f;
        vec[(lane >> 1) * 4 + 2 + (lane & 1)] = in ? -8.0f * A.scale * A.e[rbase + qi] : 0.0f;
        tail = __any_sync(0xffffffffu, in && tail_row(A, dt));
        __syncwarp();
      }
      const float4* vc = reinterpret_cast<const float4*>(vec);
      const uint32_t yb = T::y(DBY ? (it & 1) : 0) + lane_off + 32 * g;
      ok = mbar_wait(b.s_full, it & 1, A.status, kDevTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t x[32], y[32], wp[16], dp[16];
      tmem_ld32(tmem + C::X_COL + lane_off + 32 * g, x);
      tmem_ld32(tmem + yb, y);
      tmem_ld_wait();
      // Scores are in registers: the next tile's S may overwrite X.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b.x_read);
      const bool need_mask = k0 + 127 >= A.valid || q0 + 127 >= A.L || (A.causal && q0 < k0 + 127);
      // Columns past L read 1/d = 0, which zeroes W and dS; the mask covers
      // invisible keys and causal order.
      if (tail)
        grad_chunk<true, true, true>(x, y, wp, dp, A.scale, vc, 0.f, 0.f, A.valid, key < A.L, A.causal, key, qc0,
                                     true);
      else if (need_mask)
        grad_chunk<true, true, false>(x, y, wp, dp, A.scale, vc, 0.f, 0.f, A.valid, key < A.L, A.causal, key, qc0,
                                      true);
      else
        grad_chunk<false, true, false>(x, y, wp, dp, A.scale, vc, 0.f, 0.f, 0, true, 0, 0, 0, true);
      tmem_st16(tmem + yb, dp);       // dS^T over the chunk's first 16 columns
      tmem_st16(tmem + yb + 16, wp);  // W^T over its last 16
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b.g_full + (it & 1));
    }
    // Epilogue: warpgroup g stores columns [HD/4 g, HD/4 (g+1)) of dV and dK.
    constexpr int OC = HD / 4;
    bool have = niter > 0 && ok;
    if (have) {
      have = mbar_wait(b.o_full, 0, A.status, kDevTimeoutEpilogue);
      have = __all_sync(0xffffffffu, have);
    }
    tc_fence_after();
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      uint32_t ov[32];
      __syncwarp();
      if (have) {
        const uint32_t o_tm = tmem + (t ? T::ACC1 : T::ACC0) + lane_off + OC * g;
        if constexpr (OC == 32) {
          tmem_ld32(o_tm, ov);
        } else {
          uint32_t (&ov16)[16] = *reinterpret_cast<uint32_t(*)[16]>(ov);
          tmem_ld16(o_tm, ov16);
        }
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) ov[c] = 0u;
      }
      if (key < A.L && (have || niter == 0)) {
        __nv_bfloat16* dst = (t ? A.dk : A.dv) + (rbase + key) * HD + OC * g;
#pragma unroll
        for (int w8 = 0; w8 < OC / 8; ++w8) {
          uint4 pkt;
          pkt.x = pack_bf16x2(__uint_as_float(ov[8 * w8 + 0]), __uint_as_float(ov[8 * w8 + 1]));
          pkt.y = pack_bf16x2(__uint_as_float(ov[8 * w8 + 2]), __uint_as_float(ov[8 * w8 + 3]));
          pkt.z = pack_bf16x2(__uint_as_float(ov[8 * w8 + 4]), __uint_as_float(ov[8 * w8 + 5]));
          pkt.w = pack_bf16x2(__uint_as_float(ov[8 * w8 + 6]), __uint_as_float(ov[8 * w8 + 7]));
          reinterpret_cast<uint4*>(dst)[w8] = pkt;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int HD>
__global__ void __launch_bounds__(576, 1)
    afa_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_g,
                         const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ BwdTcArgs A) {
  using C = BwdCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Bars b = carve<HD>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int it_tile = gridDim.y - 1 - blockIdx.y;  // queries with the most causal keys first
  const int q0 = 128 * it_tile;
  int kend = A.valid;
  if (A.causal && q0 + 128 < kend) kend = q0 + 128;
  const int niter = (kend + 127) / 128;
  const uint32_t tmem = setup<HD>(smem, b, &tm_q, &tm_g, &tm_k, &tm_v);

  using T = Tmem<HD, true>;
  static_assert(T::ACC0 + HD <= C::TMEM_COLS, "TMEM budget");
  if (warp == C::kTmaWarp) {
    if (lane == 0) produce<HD>(smem, b, &tm_q, &tm_g, &tm_k, &tm_v, q0, 0, niter, bh, A.status);
  } else if (warp == C::kMmaWarp) {
    if (lane == 0) issue<HD, false, true>(smem, b, tmem, niter, A.status);
  } else {
    const int g = warp >> 2, sub = warp & 3;
    const int row = sub * 32 + lane;
    const int qry = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const long long rbase = static_cast<long long>(bh) * A.L;
    const bool in = qry < A.L;
    const float dt = in ? A.dtot[rbase + qry] : 1.0f;
    const float inv = in ? 1.0f / dt : 0.0f;
    const float ne8 = in ? -8.0f * A.scale * A.e[rbase + qry] : 0.0f;
    const bool tail = __any_sync(0xffffffffu, in && tail_row(A, dt));
    bool ok = true;
    for (int it = 0; ok && it < niter; ++it) {
      const int kc0 = 128 * it + 32 * g;
      const uint32_t yb = T::y(it & 1) + lane_off + 32 * g;
      ok = mbar_wait(b.s_full, it & 1, A.status, kDevTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t x[32], y[32], wp[16], dp[16];
      tmem_ld32(tmem + C::X_COL + lane_off + 32 * g, x);
      tmem_ld32(tmem + yb, y);
      tmem_ld_wait();
      // Scores are in registers: the next tile's S may overwrite X.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b.x_read);
      const bool need_mask = 128 * it + 127 >= A.valid || (A.causal && 128 * it + 127 > q0);
      if (tail)
        grad_chunk<true, false, true>(x, y, wp, dp, A.scale, nullptr, inv, ne8, A.valid, in, A.causal, qry, kc0,
                                      false);
      else if (need_mask)
        grad_chunk<true, false, false>(x, y, wp, dp, A.scale, nullptr, inv, ne8, A.valid, in, A.causal, qry, kc0,
                                       false);
      else
        grad_chunk<false, false, false>(x, y, wp, dp, A.scale, nullptr, inv, ne8, 0, true, 0, 0, 0, false);
      // dS over the chunk's first 16 dP columns: the A operand of dQ += dS K.
      tmem_st16(tmem + yb, dp);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b.g_full + (it & 1));
    }
    constexpr int OC = HD / 4;
    bool have = niter > 0 && ok;
    if (have) {
      have = mbar_wait(b.o_full, 0, A.status, kDevTimeoutEpilogue);
      have = __all_sync(0xffffffffu, have);
    }
    tc_fence_after();
    uint32_t ov[32];
    __syncwarp();
    if (have) {
      const uint32_t o_tm = tmem + T::ACC0 + lane_off + OC * g;
      if constexpr (OC == 32) {
        tmem_ld32(o_tm, ov);
      } else {
        uint32_t (&ov16)[16] = *reinterpret_cast<uint32_t(*)[16]>(ov);
        tmem_ld16(o_tm, ov16);
      }
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int c = 0; c < 32; ++c) ov[c] = 0u;
    }
    if (in && (have || niter == 0)) {
      __nv_bfloat16* dst = A.dq + (rbase + qry) * HD + OC * g;
#pragma unroll
      for (int w8 = 0; w8 < OC / 8; ++w8) {
        uint4 pkt;
        pkt.x = pack_bf16x2(__uint_as_float(ov[8 * w8 + 0]), __uint_as_float(ov[8 * w8 + 1]));
        pkt.y = pack_bf16x2(__uint_as_float(ov[8 * w8 + 2]), __uint_as_float(ov[8 * w8 + 3]));
        pkt.z = pack_bf16x2(__uint_as_float(ov[8 * w8 + 4]), __uint_as_float(ov[8 * w8 + 5]));
        pkt.w = pack_bf16x2(__uint_as_float(ov[8 * w8 + 6]), __uint_as_float(ov[8 * w8 + 7]));
        reinterpret_cast<uint4*>(dst)[w8] = pkt;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int HD>
cudaError_t launch_bwd_tc_hd(const void* q, const void* k, const void* v, const void* g, const BwdTcArgs& A, int bh,
                             cudaStream_t stream, const char** detail) {
  using C = BwdCfg<HD>;
  static PerDeviceOnce setup;
  int dev = 0;
  cudaError_t se = cudaGetDevice(&dev);
  if (se == cudaSuccess)
    se = setup.run(dev, [&] {
      cudaError_t e = cudaFuncSetAttribute(afa_bwd_dkv_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           C::SMEM_BYTES);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(afa_bwd_dq_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::SMEM_BYTES);
      return e;
    });
  if (se != cudaSuccess) {
    *detail = "cudaFuncSetAttribute(max dynamic shared memory) failed";
    return se;
  }
  CUtensorMap tq, tg, tk, tv;
  if (!make_tmap(&tq, q, HD, A.L, bh) || !make_tmap(&tg, g, HD, A.L, bh) || !make_tmap(&tk, k, HD, A.L, bh) ||
      !make_tmap(&tv, v, HD, A.L, bh)) {
    *detail = "cuTensorMapEncodeTiled failed (pointers must be 16-byte aligned)";
    return cudaErrorInvalidValue;
  }
  const int tiles = (A.L + 127) / 128;
  afa_bwd_dkv_tc_kernel<HD><<<dim3(bh, tiles), C::kThreads, C::SMEM_BYTES, stream>>>(tq, tg, tk, tv, A);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  afa_bwd_dq_tc_kernel<HD><<<dim3(bh, tiles), C::kThreads, C::SMEM_BYTES, stream>>>(tq, tg, tk, tv, A);
  return cudaGetLastError();
}

}  // namespace

bool tc_bwd_supported(int dtype, int d) { return dtype == kBF16 && (d == 64 || d == 128); }

cudaError_t launch_tc_bwd(const void* q, const void* k, const void* v, const void* g_out, const float* d_total,
                          const float* e, void* dq, void* dk, void* dv, int B, int H, int L, int D, int causal,
                          int valid, float scale, float sink, int* status, cudaStream_t stream, const char** detail) {
  BwdTcArgs A{};
  A.sink = sink;
  A.dtot = d_total;
  A.e = e;
  A.dq = static_cast<__nv_bfloat16*>(dq);
  A.dk = static_cast<__nv_bfloat16*>(dk);
  A.dv = static_cast<__nv_bfloat16*>(dv);
  A.status = status;
  A.L = L;
  A.causal = causal;
  A.valid = valid;
  A.scale = scale;
  return D == 128 ? launch_bwd_tc_hd<128>(q, k, v, g_out, A, B * H, stream, detail)
                  : launch_bwd_tc_hd<64>(q, k, v, g_out, A, B * H, stream, detail);
}

}  // namespace afa
