// AFA prefill forward on the B200 5th-generation tensor cores (tcgen05 + TMEM).
//
// Reference: afa_kernel / pallas_afa_forward (src/kernels/pallas_afa.py:52-151,
// :154-264). Per (batch, head, 128-row query tile) the reference accumulates
//     S = (Q K^T) * scale                (fp32 accumulation, :104-110)
//     P = rho(S)^8, masked               (:113-124)
//     O += P.astype(v.dtype) V           (fp32 accumulation, :132-137)
//     d += rowsum(P)                     (fp32 P, :139)
// and finishes with O / (d + sink) and d_total = d + sink (:142-151). There is
// no running maximum, so tiles add up with no rescaling.
//
// B200 design (one CTA per SM, 576 threads, two 128-row query tiles per CTA):
//   warp 16     TMA producer: Q once, then K_j / V_j tiles through a ring of
//               shared-memory slots (128-byte swizzle, no multicast).
//   warp 17     allocates 512 TMEM columns and issues every tcgen05.mma from one
//               thread: S_i = Q_i K_j^T (A, B from shared memory) and
//               O_i += P_i V_j (A = P from TMEM, B = V from shared memory), in
//               the order PV_0(t) S_0(t+1) PV_1(t) S_1(t+1). The tensor core
//               accepts only about two instructions ahead of the one executing,
//               so the issuer waits for the K/V fills of an iteration up front
//               and then issues each tile's 16 instructions back to back.
//   warps 0-15  "octic" warps: warps 0-7 map query tile 0, warps 8-15 tile 1.
//               Warp (h, sub) of a tile owns key columns [64h, 64h+64) of TMEM
//               lane quarter sub. Each thread owns one query row (one TMEM
//               lane): per 32-column chunk it reads its scores, applies the
//               octic map and masks in registers, keeps an fp32 partial row
//               sum, and writes P as packed bf16 to the first 16 of those
//               columns. One tile's map runs while the tensor core computes the
//               other tile's P.V and next S, and one tile's TMEM load/store
//               latency overlaps the other tile's MUFU work.
//   epilogue    the two row-sum partials (column halves) meet once in shared
//               memory; warpgroup g = warp / 4 reads its quarter of O's columns
//               of both tiles from TMEM, divides once by (d + sink) and stores
//               bf16 (or stores / adds / adds-and-divides the fp32 ring
//               accumulators).
// TMEM columns: S0/P0 [0,128), S1/P1 [128,256), O0 [256,256+D), O1 [256+D, ...).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "afa_common.cuh"
#include "afa_internal.h"
#include "afa_tc_shared.cuh"
#include "afa_tmap.h"

namespace afa {
namespace {

template <int HD>
struct TcCfg {
  static constexpr int kOcticWarps = 16;
  static constexpr int kTmaWarp = 16;
  static constexpr int kMmaWarp = 17;
  static constexpr int kThreads = 18 * 32;
  static constexpr int BN = 128;
  static constexpr int KSUB = HD / 64;             // 64-element (128 B) column blocks
  static constexpr int SUB_BYTES = 128 * 128;      // 128 rows x 128 B
  static constexpr int TILE_BYTES = KSUB * SUB_BYTES;
  static constexpr int NSLOT = (HD == 128) ? 5 : 8;
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = 2 * TILE_BYTES;
  static constexpr int BAR_OFF = KV_OFF + NSLOT * TILE_BYTES;
  static constexpr int NBAR = 1 + 2 * NSLOT + 2 + 2 + 2 + 1;
  // Past the common barriers: afa_tc_fwd_kernel keeps its TMEM address at
  // XBAR_OFF; afa_tc_sk_kernel keeps q_empty there, its TMEM address at +8,
  // the row-sum exchange barriers of its final-output mode at +16 (2 x 8) and
  // their fp32 row sums [tile][row] at XRED_OFF.
  static constexpr int XBAR_OFF = BAR_OFF + NBAR * 8;
  static constexpr int XRED_OFF = XBAR_OFF + 16 + 16 * 8;
  // fp32 row-sum partials [tile][column half][row] of the epilogue, in K/V
  // ring slot 2 (idle once every MMA has finished; slots 0-1 stage the output
  // tiles).
  static constexpr int RED_OFF = KV_OFF + 2 * TILE_BYTES;
  static constexpr int SMEM_BYTES = XRED_OFF + 2 * 128 * 4 + 1024;
  static_assert(NSLOT >= 3 && 2 * 2 * 128 * 4 <= TILE_BYTES, "row-sum partials fit in ring slot 2");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
  static constexpr uint32_t TMEM_COLS = 512;
  __device__ static constexpr uint32_t s_col(int i) { return static_cast<uint32_t>(i) * 128u; }
  __device__ static constexpr uint32_t o_col(int i) { return 256u + static_cast<uint32_t>(i) * HD; }
  // P of keys [16kk, 16kk+16): the 32-key chunk [32c, 32c+32) is packed into
  // columns [32c, 32c+16), 8 columns per 16 keys.
  __device__ static constexpr uint32_t p_col(int kk) {
    return static_cast<uint32_t>((kk >> 1) * 32 + (kk & 1) * 8);
  }
};

// Pairs per head in one block of the one-CTA-per-pair launch order, for
// launches with at least that many pairs per head. 256 (a whole head at
// L = 65536) cut DRAM reads from 8.07 GB to 811 MB per launch there and
// measured +2.4% over walking every head's longest pairs together (blocks of
// one pair), whose concurrent CTAs fetch 16 heads' K/V at once. Launches of
// fewer pairs per head (a few waves) walk all heads' pairs together: on the
// first hop of an 8-GPU ring (48 pairs per head) blocks of 256 ran 0.349 ms
// against 0.276 with blocks of one pair, as a head's long pairs started late.
constexpr int kPairGroup = 256;

template <int HD>
__global__ void __launch_bounds__(576, 1)
    afa_tc_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                      const __grid_constant__ Launch L) {
  using C = TcCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + C::NSLOT;
  uint64_t* s_full = kv_empty + C::NSLOT;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* drain = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  float* red = reinterpret_cast<float*>(smem + C::RED_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA order (1-D grid over B*H x pairs): heaviest work first -- pairs are
  // walked backwards, so the last (most causal keys) query tiles start first
  // -- in blocks of kPairGroup pairs per head when a head has that many, so
  // the CTAs that run together share each head's K/V tiles in L2; shorter
  // launches walk every head's pairs together (blocks of one pair).
  int bh, cta;
  {
    const int npair = L.prob[L.nprob - 1].cta0 + L.prob[L.nprob - 1].ncta;
    const int grp = npair >= kPairGroup ? kPairGroup : 1;
    const long long i = blockIdx.x;
    const long long per_block = static_cast<long long>(grp) * L.B * L.H;
    const int b = static_cast<int>(i / per_block);
    const int r = static_cast<int>(i - b * per_block);
    const int first = b * grp;  // in walk order (0 = last pair)
    const int size = npair - first < grp ? npair - first : grp;
    bh = r / size;
    cta = npair - 1 - (first + r % size);
  }
  int pi = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < L.nprob && cta >= L.prob[i].cta0) pi = i;
  const Problem& P = L.prob[pi];
  const int r0 = (cta - P.cta0) * 256;  // first row of query tile 0 in the q segment

  // Key tiles per query tile. Only the last key segment may be partially
  // visible, which makes tile 0's tiles a prefix of tile 1's.
  const bool q1_live = r0 + 128 < P.q.len;
  const int last0 = min(r0 + 127, P.q.len - 1);
  const int last1 = q1_live ? min(r0 + 255, P.q.len - 1) : last0;
  int cnt0[2] = {0, 0}, cnt1[2] = {0, 0};
#pragma unroll
  for (int s = 0; s < kMaxKSegs; ++s) {
    if (s < P.nk) {
      cnt0[s] = seg_tiles(P.k[s], L.causal, P.q.pos0 + last0);
      cnt1[s] = seg_tiles(P.k[s], L.causal, P.q.pos0 + last1);
    }
  }
  const int n1 = cnt1[0] + cnt1[1];
  const int n0 = (P.nk == 1 || cnt0[0] == cnt1[0]) ? cnt0[0] + cnt0[1] : n1;

  // The TMA thread sets up the barriers its loads complete and issues Q and
  // the first ring of K/V tiles (the slots start empty: no wait) before the
  // CTA-wide barrier, so their latency overlaps barrier and TMEM set-up.
  // Every load that needs a wait comes after it.
  const int early = n1 > 0 ? (2 * n1 < C::NSLOT ? 2 * n1 : C::NSLOT) : 0;
  if (warp == C::kTmaWarp && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NSLOT; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    fence_barrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    if (n1 > 0) {
      mbar_arrive_expect_tx(q_full, 2 * C::TILE_BYTES);
      for (int i = 0; i < 2; ++i)
        for (int h = 0; h < C::KSUB; ++h)
          tma_load_3d(smem + C::Q_OFF + (i * C::KSUB + h) * C::SUB_BYTES, &tm_q, q_full, 64 * h,
                      P.q.row0 + r0 + 128 * i, bh);
      for (int u = 0; u < early; ++u) {
        const KvTile kt = kv_tile(P, cnt1[0], u >> 1);
        mbar_arrive_expect_tx(kv_full + u, C::TILE_BYTES);
        for (int h = 0; h < C::KSUB; ++h)
          tma_load_3d(smem + C::KV_OFF + (u * C::KSUB + h) * C::SUB_BYTES, (u & 1) ? &tm_v : &tm_k, kv_full + u,
                      64 * h, kt.row, bh);
      }
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(p_full + i, 8);  // one elected arrive per octic warp of the tile
      mbar_init(o_full + i, 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tm_o);
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == C::kTmaWarp) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0 && n1 > 0) {
      int issued = early;
      for (int t = early >> 1; t < n1; ++t) {
        const KvTile kt = kv_tile(P, cnt1[0], t);
        bool ok = true;
        for (int kv = 0; kv < 2; ++kv) {
          const int u = 2 * t + kv;
          if (u < early) continue;  // issued before the CTA barrier
          const int slot = u % C::NSLOT;
          if (!mbar_wait(kv_empty + slot, ((u / C::NSLOT) & 1) ^ 1, L.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(kv_full + slot, C::TILE_BYTES);
          for (int h = 0; h < C::KSUB; ++h)
            tma_load_3d(smem + C::KV_OFF + (slot * C::KSUB + h) * C::SUB_BYTES, kv ? &tm_v : &tm_k,
                        kv_full + slot, 64 * h, kt.row, bh);
          issued = u + 1;
        }
        if (!ok) break;
      }
      // Do not leave the CTA while loads into its shared memory are in flight.
      (void)mbar_wait(q_full, 0, nullptr, 0);
      for (int u = issued - C::NSLOT < 0 ? 0 : issued - C::NSLOT; u < issued; ++u)
        (void)mbar_wait(kv_full + (u % C::NSLOT), (u / C::NSLOT) & 1, nullptr, 0);
    }
  } else if (warp == C::kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0 && n1 > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, HD, true);
      // Base descriptors, built once: the issue loops only add constant
      // offsets (desc_add), which keeps this thread's instructions between
      // MMAs few while the octic warps compete for the same issue slots.
      const uint64_t q_desc = sw128_desc(smem_u32(smem + C::Q_OFF), 16, 1024);
      const uint64_t k_desc = sw128_desc(smem_u32(smem + C::KV_OFF), 16, 1024);
      const uint64_t v_desc = sw128_desc(smem_u32(smem + C::KV_OFF), C::SUB_BYTES, 1024);
      auto issue_s = [&](int i, int slot) {
        const uint64_t kb = desc_add(k_desc, slot * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SUB_BYTES + (kk & 3) * 32;
          umma_ss(tmem + C::s_col(i), desc_add(q_desc, i * C::TILE_BYTES + off), desc_add(kb, off), idesc_s,
                  kk > 0 ? 1u : 0u);
        }
      };
      auto issue_o = [&](int i, int slot, bool acc) {
        const uint64_t vb = desc_add(v_desc, slot * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          umma_ts(tmem + C::o_col(i), tmem + C::s_col(i) + C::p_col(kk), desc_add(vb, kk * 2048), idesc_o,
                  (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(q_full, 0, L.status, kDevTimeoutMma) && mbar_wait(kv_full + 0, 0, L.status, kDevTimeoutMma);
      if (ok) {
        tc_fence_after();
        if (n0 > 0) {
          issue_s(0, 0);
          umma_commit(s_full + 0);
        }
        issue_s(1, 0);
        umma_commit(s_full + 1);
        umma_commit(kv_empty + 0);
      }
      for (int t = 0; ok && t < n1; ++t) {
        const int uv = 2 * t + 1, sv = uv % C::NSLOT;
        const int uk = 2 * t + 2, sk = uk % C::NSLOT;
        const bool more = t + 1 < n1;
        // Both fills of this iteration first (usually long complete), so the
        // only wait left between instruction blocks is the P dependency.
        if (!(ok = mbar_wait(kv_full + sv, (uv / C::NSLOT) & 1, L.status, kDevTimeoutMma))) break;
        if (more && !(ok = mbar_wait(kv_full + sk, (uk / C::NSLOT) & 1, L.status, kDevTimeoutMma))) break;
        if (t < n0) {
          if (!(ok = mbar_wait(p_full + 0, t & 1, L.status, kDevTimeoutMma))) break;
          tc_fence_after();
          issue_o(0, sv, t > 0);
          if (t + 1 == n0) umma_commit(o_full + 0);
          if (more && t + 1 < n0) {
            issue_s(0, sk);
            umma_commit(s_full + 0);
          }
        }
        if (!(ok = mbar_wait(p_full + 1, t & 1, L.status, kDevTimeoutMma))) break;
        tc_fence_after();
        issue_o(1, sv, t > 0);
        umma_commit(kv_empty + sv);
        if (t + 1 == n1) umma_commit(o_full + 1);
        if (more) {
          issue_s(1, sk);
          umma_commit(s_full + 1);
          umma_commit(kv_empty + sk);
        }
      }
      // Every MMA this thread issued must finish before TMEM is released.
      umma_commit(drain);
      (void)mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // --------------------------------------------------- octic map + epilogue
    // Map: warps 0-7 take query tile 0, warps 8-15 tile 1, so one tile's map
    // runs while the tensor core works on the other's P.V and next scores, and
    // the TMEM load/store latency of one overlaps the other's MUFU work. Warp
    // (mt, h, sub) maps key columns [64h, 64h+64) of TMEM lane quarter sub.
    // Epilogue: warpgroup g = warp / 4 takes O columns [OC g, OC g + OC) of
    // both tiles.
    const int g = warp >> 2;
    const int sub = warp & 3;          // TMEM lane quarter
    const int mt = warp >> 3;          // query tile this warp maps
    const int mh = (warp >> 2) & 1;    // its half of the key columns
    const int row = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float scale = L.scale;
    float dsum = 0.f;
    bool tail_check = true;  // warp-uniform: some row's weights so far < kTailRowSum
    bool ok = true;
    const int nmap = mt ? n1 : n0;
    for (int t = 0; t < nmap && ok; ++t) {
      const KvTile kt = kv_tile(P, cnt1[0], t);
      ok = mbar_wait(s_full + mt, t & 1, L.status, kDevTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int qfirst = P.q.pos0 + r0 + 128 * mt;
      const int qpos = qfirst + row;
      const bool need_mask = kt.lim < 128 || (L.causal && kt.pos + 127 > qfirst);
      const uint32_t s_base = tmem + C::s_col(mt) + lane_off;
      if (tail_check) {
        map_tile<true>(s_base, 64 * mh, need_mask, scale, kt.lim, L.causal, kt.pos, qpos, dsum);
        tail_check = __any_sync(0xffffffffu, dsum < kTailRowSum);
      } else {
        map_tile<false>(s_base, 64 * mh, need_mask, scale, kt.lim, L.causal, kt.pos, qpos, dsum);
      }
      // Every lane's P stores are complete (wait::st) and ordered before the
      // warp's single arrive.
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + mt);
    }
    bool have_o[2] = {false, false};
#pragma unroll
    for (int tile = 0; tile < 2; ++tile) {
      const int n = tile ? n1 : n0;
      if (ok && n > 0) {
        ok = mbar_wait(o_full + tile, 0, L.status, kDevTimeoutEpilogue);
        ok = __all_sync(0xffffffffu, ok);
        have_o[tile] = ok;
      }
    }
    // After both tiles' last MMAs (o_full), so nothing reads ring slot 2 now.
    red[(mt * 2 + mh) * 128 + row] = dsum;
    tc_fence_after();
    // The two column-half partials of every row meet here (fixed order).
    asm volatile("bar.sync 1, %0;" ::"r"(C::kOcticWarps * 32) : "memory");

    const bool fin = L.mode == kFinal || L.mode == kAccumFinal;
    const bool add_prev = L.mode == kAccumRaw || L.mode == kAccumFinal;
    constexpr int OC = HD / 4;  // O columns per warpgroup: 32 (D=128) or 16 (D=64)
    // A bf16 output tile leaves through a TMA store from shared memory (the
    // K/V ring is idle now) when its 128 rows all belong to this problem or
    // run past the end of the tensor, where TMA writes nothing; a direct store
    // from each thread would touch 32 rows per warp instruction. Other tiles
    // (a problem ending mid-tile next to another problem's rows) store directly.
    bool tma_tile[2];
#pragma unroll
    for (int tile = 0; tile < 2; ++tile)
      tma_tile[tile] = fin && r0 + 128 * tile < P.q.len &&
                       (r0 + 128 * (tile + 1) <= P.q.len || P.q.row0 + P.q.len == L.lq);
#pragma unroll
    for (int tile = 0; tile < 2; ++tile) {
      const float drow_tile = red[(tile * 2 + 0) * 128 + row] + red[(tile * 2 + 1) * 128 + row];
      const int rloc = r0 + 128 * tile + row;
      const bool row_ok = rloc < P.q.len;
      const long long grow = static_cast<long long>(bh) * L.lq + P.q.row0 + rloc;
      const float dprev = (row_ok && add_prev) ? static_cast<const float*>(L.d_acc)[grow] : 0.f;
      const float drow = drow_tile + dprev;
      const float denom = drow + L.sink;
      const float inv = 1.0f / denom;
      uint32_t ov[32];
      __syncwarp();  // tcgen05.ld is warp-collective
      if (have_o[tile]) {
        const uint32_t o_tm = tmem + C::o_col(tile) + lane_off + OC * g;
        if constexpr (OC == 32) {
          tmem_ld32(o_tm, ov);
        } else {
          uint32_t (&ov16)[16] = *reinterpret_cast<uint32_t(*)[16]>(ov);
          tmem_ld16(o_tm, ov16);
        }
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] = 0u;
      }
      constexpr int NCH = OC / 4;  // 16-byte chunks per row and warpgroup
      const int gi = lane % NCH;
      const int grow0 = r0 + 128 * tile + sub * 32 + (lane / NCH) * NCH;  // first row of the lane's group
      const long long gbase = static_cast<long long>(bh) * L.lq + P.q.row0;
      if (fin) {
        if (add_prev) {
          // The previous hops' rows are read transposed (NCH consecutive
          // chunks of one row per group and instruction, not one chunk of 32
          // rows), then the transpose is undone for the per-row epilogue.
          transpose_chunks<NCH>(ov, gi);
#pragma unroll
          for (int kr = 0; kr < NCH; ++kr) {
            if (grow0 + kr < P.q.len) {
              const float4 y = *reinterpret_cast<const float4*>(static_cast<const float*>(L.o_acc) +
                                                                (gbase + grow0 + kr) * HD + OC * g + 4 * gi);
              ov[4 * kr + 0] = __float_as_uint(__uint_as_float(ov[4 * kr + 0]) + y.x);
              ov[4 * kr + 1] = __float_as_uint(__uint_as_float(ov[4 * kr + 1]) + y.y);
              ov[4 * kr + 2] = __float_as_uint(__uint_as_float(ov[4 * kr + 2]) + y.z);
              ov[4 * kr + 3] = __float_as_uint(__uint_as_float(ov[4 * kr + 3]) + y.w);
            }
          }
          transpose_chunks<NCH>(ov, gi);
        }
        float x[OC];
#pragma unroll
        for (int e = 0; e < OC; ++e) x[e] = __uint_as_float(ov[e]);
        uint4 pk[OC / 8];
#pragma unroll
        for (int w = 0; w < OC / 8; ++w) {
          pk[w].x = pack_bf16x2(x[8 * w + 0] * inv, x[8 * w + 1] * inv);
          pk[w].y = pack_bf16x2(x[8 * w + 2] * inv, x[8 * w + 3] * inv);
          pk[w].z = pack_bf16x2(x[8 * w + 4] * inv, x[8 * w + 5] * inv);
          pk[w].w = pack_bf16x2(x[8 * w + 6] * inv, x[8 * w + 7] * inv);
        }
        if (tma_tile[tile]) {
          // 128-byte-swizzled staging: 64-column blocks of 128 rows x 128 B,
          // 16-byte chunk j of row r at (j ^ (r % 8)) * 16.
          uint8_t* stage = smem + C::KV_OFF + tile * C::TILE_BYTES;
#pragma unroll
          for (int w = 0; w < OC / 8; ++w) {
            const int col0 = OC * g + 8 * w;
            const int j = (col0 & 63) >> 3;
            st_shared_v4(smem_u32(stage + (col0 >> 6) * C::SUB_BYTES + row * 128 + ((j ^ (row & 7)) << 4)), pk[w]);
          }
        } else if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(L.out) + grow * HD + OC * g);
#pragma unroll
          for (int w = 0; w < OC / 8; ++w) dst[w] = pk[w];
        }
      } else {
        // Raw accumulator rows (store, or add the previous hops'): transposed
        // so the lanes of a group move NCH consecutive 16-byte chunks of one
        // row per instruction, rather than one chunk of 32 rows.
        // All loads are issued before the first store, which the compiler
        // could not move them past.
        transpose_chunks<NCH>(ov, gi);
        float* const acc0 = static_cast<float*>(L.o_acc) + (gbase + grow0) * HD + OC * g + 4 * gi;
        if (add_prev) {
#pragma unroll
          for (int kr = 0; kr < NCH; ++kr) {
            if (grow0 + kr < P.q.len) {
              const float4 y = *reinterpret_cast<const float4*>(acc0 + kr * HD);
              ov[4 * kr + 0] = __float_as_uint(__uint_as_float(ov[4 * kr + 0]) + y.x);
              ov[4 * kr + 1] = __float_as_uint(__uint_as_float(ov[4 * kr + 1]) + y.y);
              ov[4 * kr + 2] = __float_as_uint(__uint_as_float(ov[4 * kr + 2]) + y.z);
              ov[4 * kr + 3] = __float_as_uint(__uint_as_float(ov[4 * kr + 3]) + y.w);
            }
          }
        }
#pragma unroll
        for (int kr = 0; kr < NCH; ++kr) {
          if (grow0 + kr < P.q.len)
            *reinterpret_cast<uint4*>(acc0 + kr * HD) =
                make_uint4(ov[4 * kr + 0], ov[4 * kr + 1], ov[4 * kr + 2], ov[4 * kr + 3]);
        }
      }
      // d_acc / d_total: one writer per row (warpgroup 0); the others only
      // read d_acc above, in kAccumFinal, where nothing writes it.
      if (row_ok && g == 0) {
        if (fin) {
          if (L.dtot) static_cast<float*>(L.dtot)[grow] = denom;
        } else {
          static_cast<float*>(L.d_acc)[grow] = drow;
        }
      }
    }
    if (tma_tile[0] || tma_tile[1]) {  // uniform across the octic warps
      fence_proxy_async_shared();
      asm volatile("bar.sync 1, %0;" ::"r"(C::kOcticWarps * 32) : "memory");
      if (threadIdx.x == 0) {
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
          if (!tma_tile[tile]) continue;
          for (int h = 0; h < C::KSUB; ++h)
            tma_store_3d(&tm_o, smem + C::KV_OFF + tile * C::TILE_BYTES + h * C::SUB_BYTES, 64 * h,
                         P.q.row0 + r0 + 128 * tile, bh);
        }
        bulk_commit();
        bulk_wait_read();  // the staging area is released when the CTA exits
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

// ---------------------------------------------------------------------------
// Persistent stream-K kernel for the accumulate hop modes.
//
// A ring hop whose query pairs all see the same number of key tiles launches
// equal CTAs, and 256 or 512 of them on 148 SMs leave the last wave partly
// empty (about 13% of the hop); each CTA also ends with a read-modify-write of
// its fp32 accumulator rows. Accumulate-mode launches therefore run one CTA per
// SM (G CTAs) over a hybrid schedule. The (b, h, query pair) items are
// numbered with b*h varying fastest, as in the non-persistent grid. Whole
// rounds of items come first: CTA c takes items c, c+G, c+2G, ..., so the CTAs
// of a round sweep the same heads' keys together and share K/V tiles in L2.
// The key-tile iterations of the remaining items (less than one round) are
// then split evenly: CTA c takes the c-th of G equal contiguous ranges, and an
// item whose iterations straddle two ranges is computed in two pieces. AFA
// partial results only add (there is no running maximum to reconcile), so
// every piece adds its numerator and row sums into the fp32 accumulators with
// red.global.add: fire-and-forget reductions with no ordering between pieces.
// In kAccumFinal the divide runs afterwards over the problems' rows
// (sk_finalize_kernel). There is no named barrier and no inter-CTA wait; every
// wait is a bounded mbarrier wait as in afa_tc_fwd_kernel.
//
// Final-output mode (FINAL = true, kFinal prefills of many short pairs): the
// same CTAs walk whole pairs only, in snake order over a longest-first list,
// and each pair's octic warps write its bf16 output and d_total themselves,
// so a CTA's next pair loads and computes its first scores while the previous
// pair's last P.V and output run. There is no per-pair CTA launch, set-up or
// teardown.
// FINAL: the final-output mode (kFinal launches, snake plans, bf16 output and
// d_total written per pair); otherwise the accumulate hop modes.
template <int HD, bool FINAL>
__global__ void __launch_bounds__(576, 1)
    afa_tc_sk_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Launch L,
                     const __grid_constant__ SkPlan S) {
  using C = TcCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + C::NSLOT;
  uint64_t* s_full = kv_empty + C::NSLOT;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* drain = o_full + 2;
  uint64_t* q_empty = reinterpret_cast<uint64_t*>(smem + C::XBAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::XBAR_OFF + 8);
  uint64_t* xa = reinterpret_cast<uint64_t*>(smem + C::XBAR_OFF + 16);  // [tile * 4 + sub]: half 1's row sums written
  uint64_t* xb = xa + 8;                                                // [tile * 4 + sub]: row totals written
  float* xred = reinterpret_cast<float*>(smem + C::XRED_OFF);            // [tile][row]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  SkWalk<FINAL> walk;
  walk.init(S, gridDim.x, blockIdx.x);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::NSLOT; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(p_full + i, 8);  // one elected arrive per octic warp of the tile
      mbar_init(o_full + i, 1);
    }
    for (int i = 0; i < 8; ++i) {
      mbar_init(xa + i, 32);  // every lane of the writing warp arrives
      mbar_init(xb + i, 32);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == C::kTmaWarp) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      SkSeg sg;
      int u = 0, qn = 0;
      bool ok = true;
      while (ok && walk.next(sg)) {
        const PairGeom G = pair_geom(L, S.pair_of[sg.item]);
        const Problem& P = L.prob[G.pi];
        // The previous piece's last S = Q K^T must be done with the Q tiles.
        if (qn > 0 && !(ok = mbar_wait(q_empty, (qn - 1) & 1, L.status, kDevTimeoutProducer))) break;
        mbar_arrive_expect_tx(q_full, 2 * C::TILE_BYTES);
        for (int q = 0; q < 2; ++q)
          for (int h = 0; h < C::KSUB; ++h)
            tma_load_3d(smem + C::Q_OFF + (q * C::KSUB + h) * C::SUB_BYTES, &tm_q, q_full, 64 * h,
                        P.q.row0 + G.r0 + 128 * q, sg.bh);
        ++qn;
        for (int t = sg.t0; ok && t < sg.t1; ++t) {
          const KvTile kt = kv_tile(P, G.cnt1_0, t);
          for (int kv = 0; kv < 2; ++kv) {
            const int slot = u % C::NSLOT;
            if (!(ok = mbar_wait(kv_empty + slot, ((u / C::NSLOT) & 1) ^ 1, L.status, kDevTimeoutProducer))) break;
            mbar_arrive_expect_tx(kv_full + slot, C::TILE_BYTES);
            for (int h = 0; h < C::KSUB; ++h)
              tma_load_3d(smem + C::KV_OFF + (slot * C::KSUB + h) * C::SUB_BYTES, kv ? &tm_v : &tm_k,
                          kv_full + slot, 64 * h, kt.row, sg.bh);
            ++u;
          }
        }
      }
      // Do not leave the CTA while loads into its shared memory are in flight.
      if (qn > 0) (void)mbar_wait(q_full, (qn - 1) & 1, nullptr, 0);
      for (int x = u - C::NSLOT < 0 ? 0 : u - C::NSLOT; x < u; ++x)
        (void)mbar_wait(kv_full + (x % C::NSLOT), (x / C::NSLOT) & 1, nullptr, 0);
    }
  } else if (warp == C::kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, HD, true);
      // Base descriptors, built once: the issue loops only add constant
      // offsets (desc_add), which keeps this thread's instructions between
      // MMAs few while the octic warps compete for the same issue slots.
      const uint64_t q_desc = sw128_desc(smem_u32(smem + C::Q_OFF), 16, 1024);
      const uint64_t k_desc = sw128_desc(smem_u32(smem + C::KV_OFF), 16, 1024);
      const uint64_t v_desc = sw128_desc(smem_u32(smem + C::KV_OFF), C::SUB_BYTES, 1024);
      auto issue_s = [&](int q, int slot) {
        const uint64_t kb = desc_add(k_desc, slot * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SUB_BYTES + (kk & 3) * 32;
          umma_ss(tmem + C::s_col(q), desc_add(q_desc, q * C::TILE_BYTES + off), desc_add(kb, off), idesc_s,
                  kk > 0 ? 1u : 0u);
        }
      };
      auto issue_o = [&](int q, int slot, bool acc) {
        const uint64_t vb = desc_add(v_desc, slot * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          umma_ts(tmem + C::o_col(q), tmem + C::s_col(q) + C::p_col(kk), desc_add(vb, kk * 2048), idesc_o,
                  (acc || kk > 0) ? 1u : 0u);
      };
      SkSeg sg;
      int qn = 0, ub = 0, pc[2] = {0, 0};
      bool ok = true;
      while (ok && walk.next(sg)) {
        const PairGeom G = pair_geom(L, S.pair_of[sg.item]);
        const int t0 = sg.t0, t1 = sg.t1;
        const int e0 = t1 < G.n0 ? t1 : G.n0;  // query tile 0 is live for t in [t0, e0)
        const int sk0 = ub % C::NSLOT;
        if (!(ok = mbar_wait(q_full, qn & 1, L.status, kDevTimeoutMma) &&
                   mbar_wait(kv_full + sk0, (ub / C::NSLOT) & 1, L.status, kDevTimeoutMma)))
          break;
        ++qn;
        tc_fence_after();
        // The previous piece's O reads finished before its P arrivals of this
        // piece (the octic warps run the epilogue first), so the first P.V
        // below may overwrite O; S regions are free once the previous P.V ran,
        // which the in-order tensor pipe guarantees.
        if (t0 < e0) {
          issue_s(0, sk0);
          umma_commit(s_full + 0);
        }
        issue_s(1, sk0);
        umma_commit(s_full + 1);
        umma_commit(kv_empty + sk0);
        if (t1 - t0 == 1) umma_commit(q_empty);
        for (int t = t0; ok && t < t1; ++t) {
          const int uv = ub + 2 * (t - t0) + 1, sv = uv % C::NSLOT;
          const int uk = uv + 1, sk = uk % C::NSLOT;
          const bool more = t + 1 < t1;
          if (!(ok = mbar_wait(kv_full + sv, (uv / C::NSLOT) & 1, L.status, kDevTimeoutMma))) break;
          if (more && !(ok = mbar_wait(kv_full + sk, (uk / C::NSLOT) & 1, L.status, kDevTimeoutMma))) break;
          if (t < e0) {
            if (!(ok = mbar_wait(p_full + 0, pc[0] & 1, L.status, kDevTimeoutMma))) break;
            ++pc[0];
            tc_fence_after();
            issue_o(0, sv, t > t0);
            if (t + 1 == e0) umma_commit(o_full + 0);
            if (more && t + 1 < e0) {
              issue_s(0, sk);
              umma_commit(s_full + 0);
            }
          }
          if (!(ok = mbar_wait(p_full + 1, pc[1] & 1, L.status, kDevTimeoutMma))) break;
          ++pc[1];
          tc_fence_after();
          issue_o(1, sv, t > t0);
          umma_commit(kv_empty + sv);
          if (t + 1 == t1) umma_commit(o_full + 1);
          if (more) {
            issue_s(1, sk);
            umma_commit(s_full + 1);
            umma_commit(kv_empty + sk);
            if (t + 2 == t1) umma_commit(q_empty);
          }
        }
        ub += 2 * (t1 - t0);
      }
      // Every MMA this thread issued must finish before TMEM is released.
      umma_commit(drain);
      (void)mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------- octic map + accumulate epilogue
    // Warps 0-7 map query tile 0 and warps 8-15 tile 1 (as in the
    // non-persistent kernel); warp (mt, mh, sub) maps key columns
    // [64 mh, 64 mh + 64) and, after each piece, adds O columns
    // [HD/2 mh, HD/2 mh + HD/2) of its own tile, TMEM lane quarter sub. Reading
    // only its own tile's O keeps the overwrite of O by the next piece's first
    // P.V behind this warp's own next P arrival.
    const int sub = warp & 3;
    const int mt = warp >> 3;
    const int mh = (warp >> 2) & 1;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float scale = L.scale;
    SkSeg sg;
    int sc = 0, oc = 0, xc = 0;
    bool ok = true;
    while (ok && walk.next(sg)) {
      const PairGeom G = pair_geom(L, S.pair_of[sg.item]);
      const Problem& P = L.prob[G.pi];
      const int e0 = sg.t1 < G.n0 ? sg.t1 : G.n0;
      const int tend = mt ? sg.t1 : e0;  // this warp's tile: key tiles [sg.t0, tend)
      float dsum = 0.f;
      bool tail_check = true;  // warp-uniform: some row's weights so far < kTailRowSum
      for (int t = sg.t0; t < tend && ok; ++t) {
        const KvTile kt = kv_tile(P, G.cnt1_0, t);
        ok = mbar_wait(s_full + mt, sc & 1, L.status, kDevTimeoutSoftmax);
        ++sc;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const int qfirst = P.q.pos0 + G.r0 + 128 * mt;
        const int qpos = qfirst + row;
        const bool need_mask = kt.lim < 128 || (L.causal && kt.pos + 127 > qfirst);
        const uint32_t s_base = tmem + C::s_col(mt) + lane_off;
        if (tail_check) {
          map_tile<true>(s_base, 64 * mh, need_mask, scale, kt.lim, L.causal, kt.pos, qpos, dsum);
          tail_check = __any_sync(0xffffffffu, dsum < kTailRowSum);
        } else {
          map_tile<false>(s_base, 64 * mh, need_mask, scale, kt.lim, L.causal, kt.pos, qpos, dsum);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + mt);
      }
      if constexpr (FINAL) {
        // Final output of a whole item (snake plans): out = O / (d + sink) in
        // bf16 and d_total = d + sink, d being the two column halves' row sums
        // added in a fixed order, half 0 first, as afa_tc_fwd_kernel adds them.
        // Half 1 posts its sums, half 0 forms the totals and posts them back.
        const bool live = sg.t0 < tend;
        const int xi = mt * 4 + sub;
        float total = 0.f;
        if (ok && live) {
          float* const xr = xred + mt * 128 + row;
          if (mh == 1) {
            *xr = dsum;
            mbar_arrive(xa + xi);
            ok = mbar_wait(xb + xi, xc & 1, L.status, kDevTimeoutEpilogue);
            total = *xr;
          } else {
            ok = mbar_wait(xa + xi, xc & 1, L.status, kDevTimeoutEpilogue);
            total = dsum + *xr;
            *xr = total;
            mbar_arrive(xb + xi);
          }
          ++xc;
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            ok = mbar_wait(o_full + mt, oc & 1, L.status, kDevTimeoutEpilogue);
            ++oc;
            ok = __all_sync(0xffffffffu, ok);
          }
        }
        if (ok) {
          tc_fence_after();
          const float denom = total + L.sink;
          const float inv = 1.0f / denom;
          // Each lane packs 32 columns of its row into four 16-byte chunks;
          // transposed in groups of 4 lanes, a store instruction then writes 64
          // contiguous bytes of each of 8 rows.
          constexpr int NCH = 4;
          const int gi = lane % NCH;
          const int grow0 = G.r0 + 128 * mt + sub * 32 + (lane / NCH) * NCH;  // the group's first row
          const long long gbase = static_cast<long long>(sg.bh) * L.lq + P.q.row0;
#pragma unroll 1
          for (int c = 0; c < HD / 64; ++c) {
            const int col0 = (HD / 2) * mh + 32 * c;
            uint32_t ov[32];
            if (live) {
              __syncwarp();  // tcgen05.ld is warp-collective
              tmem_ld32(tmem + C::o_col(mt) + lane_off + col0, ov);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) ov[e] = 0u;
            }
            uint32_t pk[32];
#pragma unroll
            for (int w = 0; w < 16; ++w)
              pk[w] = pack_bf16x2(__uint_as_float(ov[2 * w]) * inv, __uint_as_float(ov[2 * w + 1]) * inv);
            transpose_chunks<NCH>(pk, gi);
#pragma unroll
            for (int kr = 0; kr < NCH; ++kr) {
              if (grow0 + kr < P.q.len)
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(L.out) + (gbase + grow0 + kr) * HD + col0 +
                                          8 * gi) = make_uint4(pk[4 * kr], pk[4 * kr + 1], pk[4 * kr + 2],
                                                               pk[4 * kr + 3]);
            }
          }
          const int rloc = G.r0 + 128 * mt + row;
          if (mh == 0 && L.dtot && rloc < P.q.len)
            static_cast<float*>(L.dtot)[static_cast<long long>(sg.bh) * L.lq + P.q.row0 + rloc] = denom;
        }
      } else if (ok && sg.t0 < tend) {  // accumulate modes
        // Add this piece into the accumulators: this warp's O columns of its
        // tile and its partial row sum (two adds per row).
        ok = mbar_wait(o_full + mt, oc & 1, L.status, kDevTimeoutEpilogue);
        ++oc;
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
          const int rloc = G.r0 + 128 * mt + row;
          const long long grow = static_cast<long long>(sg.bh) * L.lq + P.q.row0 + rloc;
          // Each thread holds 32 contiguous columns of one row per chunk.
          // Transposed in groups of 8 lanes, the lanes of a group then reduce
          // 8 consecutive 16-byte chunks of one row per instruction: full
          // 32-byte sectors, 128 contiguous bytes per row.
          constexpr int NCH = 8;
          const int gi = lane % NCH;
          const int grow0 = G.r0 + 128 * mt + sub * 32 + (lane / NCH) * NCH;  // the group's first row
          const long long gbase = static_cast<long long>(sg.bh) * L.lq + P.q.row0;
#pragma unroll 1
          for (int c = 0; c < HD / 64; ++c) {
            const int col0 = (HD / 2) * mh + 32 * c;
            uint32_t ov[32];
            __syncwarp();  // tcgen05.ld is warp-collective
            tmem_ld32(tmem + C::o_col(mt) + lane_off + col0, ov);
            tmem_ld_wait();
            transpose_chunks<NCH>(ov, gi);
#pragma unroll
            for (int kr = 0; kr < NCH; ++kr) {
              if (grow0 + kr < P.q.len) {
                float* dst = static_cast<float*>(L.o_acc) + (gbase + grow0 + kr) * HD + col0 + 4 * gi;
                red_add_v4(dst, __uint_as_float(ov[4 * kr + 0]), __uint_as_float(ov[4 * kr + 1]),
                           __uint_as_float(ov[4 * kr + 2]), __uint_as_float(ov[4 * kr + 3]));
              }
            }
          }
          if (rloc < P.q.len) red_add(static_cast<float*>(L.d_acc) + grow, dsum);
        }
      }
      // The O reads above are complete (wait::ld) before this warp's next
      // P arrival, which is what lets the MMA warp overwrite O.
      tc_fence_before();
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

// out = o_acc / (d_acc + sink) and d_total = d_acc + sink over the rows of the
// launch's problems: the divide of kAccumFinal after afa_tc_sk_kernel added the
// last hop in (pallas_afa.py:661). One warp per row.
template <int HD>
__global__ void __launch_bounds__(256) sk_finalize_kernel(const __grid_constant__ Launch L) {
  constexpr int VPL = HD / 32;  // fp32 columns per lane: 4 or 2
  int rows_bh = 0;
  for (int p = 0; p < L.nprob; ++p) rows_bh += L.prob[p].q.len;
  const long long total = static_cast<long long>(L.B) * L.H * rows_bh;
  const int lane = threadIdx.x & 31;
  for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < total;
       r += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const int bh = static_cast<int>(r / rows_bh);
    int w = static_cast<int>(r - static_cast<long long>(bh) * rows_bh);
    int p = 0;
    while (w >= L.prob[p].q.len) w -= L.prob[p++].q.len;
    const long long grow = static_cast<long long>(bh) * L.lq + L.prob[p].q.row0 + w;
    const float d = static_cast<const float*>(L.d_acc)[grow];
    const float denom = d + L.sink;
    const float inv = 1.0f / denom;
    const float* src = static_cast<const float*>(L.o_acc) + grow * HD + VPL * lane;
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(L.out) + grow * HD + VPL * lane;
    if constexpr (VPL == 4) {
      const float4 x = *reinterpret_cast<const float4*>(src);
      uint2 pkt;
      pkt.x = pack_bf16x2(x.x * inv, x.y * inv);
      pkt.y = pack_bf16x2(x.z * inv, x.w * inv);
      *reinterpret_cast<uint2*>(dst) = pkt;
    } else {
      const float2 x = *reinterpret_cast<const float2*>(src);
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(x.x * inv, x.y * inv);
    }
    if (lane == 0 && L.dtot) static_cast<float*>(L.dtot)[grow] = denom;
  }
}

template <int HD>
cudaError_t launch_hd(const Launch& L, cudaStream_t stream, const char** detail) {
  using C = TcCfg<HD>;
  static PerDeviceOnce setup;
  static int sm_count[kMaxDevices] = {};
  int dev = 0;
  cudaError_t se = cudaGetDevice(&dev);
  if (se == cudaSuccess)
    se = setup.run(dev, [&] {
      cudaError_t e = cudaFuncSetAttribute(afa_tc_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           C::SMEM_BYTES);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(afa_tc_sk_kernel<HD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::SMEM_BYTES);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(afa_tc_sk_kernel<HD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::SMEM_BYTES);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
      return e;
    });
  if (se != cudaSuccess) {
    *detail = "kernel set-up failed (max dynamic shared memory attribute or SM count)";
    return se;
  }
  CUtensorMap tq, tk, tv, to;
  const int bh = L.B * L.H;
  if (!make_tmap(&tq, L.q, HD, L.lq, bh) || !make_tmap(&tk, L.k, HD, L.lk, bh) ||
      !make_tmap(&tv, L.v, HD, L.lk, bh) || (L.out && !make_tmap(&to, L.out, HD, L.lq, bh))) {
    *detail = "cuTensorMapEncodeTiled failed (pointer must be 16-byte aligned)";
    return cudaErrorInvalidValue;
  }
  Launch LL = L;
  const int total = assign_ctas(LL, 256);
  if (total == 0) return cudaSuccess;
  // The pairs with key tiles, longest first (stable): whole-item rounds then
  // hold items of similar length.
  auto make_plan = [&](SkPlan& S) {
    int len[kMaxSkItems];
    S.nitems = 0;
    for (int c = 0; c < total; ++c) {
      len[c] = pair_geom(LL, c).n1;
      if (len[c] > 0) S.pair_of[S.nitems++] = c;
    }
    std::stable_sort(S.pair_of, S.pair_of + S.nitems, [&](int a, int b) { return len[a] > len[b]; });
    S.nbh = bh;
    S.prefix[0] = 0;
    for (int i = 0; i < S.nitems; ++i) S.prefix[i + 1] = S.prefix[i] + len[S.pair_of[i]];
  };
  if (LL.mode == kFinal && LL.out && total <= kMaxSkItems && static_cast<long long>(bh) * total > sm_count[dev]) {
    // More query pairs than SMs, and not long ones: one persistent CTA per SM
    // walks whole pairs, longest first in snake order, so a CTA's next pair
    // starts (Q load, first scores) while its previous pair's last P.V and
    // output run. Measured on B200: +5% at L=2048 causal (9 key tiles per
    // pair on average), +3.7% at L=4096 (17), even at L=65536 (257), where
    // per-CTA set-up is already negligible; pairs of more than
    // kSkFinalMaxAvgTiles key tiles on average keep one CTA per pair. Every
    // pair must have key tiles: a pair the plan leaves out would leave its
    // output rows unwritten.
    SkPlan S;
    make_plan(S);
    if (S.nitems == total && S.prefix[S.nitems] <= kSkFinalMaxAvgTiles * S.nitems) {
      const long long items = static_cast<long long>(bh) * S.nitems;
      const int G = static_cast<int>(items < sm_count[dev] ? items : sm_count[dev]);
      S.waves = static_cast<int>((items + G - 1) / G);
      afa_tc_sk_kernel<HD, true><<<G, C::kThreads, C::SMEM_BYTES, stream>>>(tq, tk, tv, LL, S);
      return cudaGetLastError();
    }
  }
  if ((LL.mode == kAccumRaw || LL.mode == kAccumFinal) && total <= kMaxSkItems) {
    // Accumulate modes: persistent stream-K over equal shares of the key-tile
    // iterations, pieces added with reductions; then the divide for kAccumFinal.
    SkPlan S;
    make_plan(S);
    const long long W = static_cast<long long>(bh) * S.prefix[S.nitems];
    if (W > 0) {
      long long G = W / 8;  // at least 8 key tiles per CTA
      if (G > sm_count[dev]) G = sm_count[dev];
      if (G < 1) G = 1;
      S.waves = static_cast<int>(static_cast<long long>(bh) * S.nitems / G);
      afa_tc_sk_kernel<HD, false><<<static_cast<int>(G), C::kThreads, C::SMEM_BYTES, stream>>>(tq, tk, tv, LL,
                                                                                               S);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return e;
    }
    if (LL.mode == kAccumFinal) {
      long long rows = 0;
      for (int p = 0; p < LL.nprob; ++p) rows += LL.prob[p].q.len;
      rows *= bh;
      long long blocks = (rows + 7) / 8;  // 8 warps (rows) per block
      if (blocks > 8LL * sm_count[dev]) blocks = 8LL * sm_count[dev];
      sk_finalize_kernel<HD><<<static_cast<int>(blocks), 256, 0, stream>>>(LL);
    }
    return cudaGetLastError();
  }
  if (!L.out) to = tq;  // raw modes store no bf16 output
  const long long ctas = static_cast<long long>(bh) * total;
  if (ctas > 0x7fffffffLL) {
    *detail = "too many query tiles for one launch";
    return cudaErrorInvalidValue;
  }
  afa_tc_fwd_kernel<HD><<<static_cast<unsigned>(ctas), C::kThreads, C::SMEM_BYTES, stream>>>(tq, tk, tv, to, LL);
  return cudaGetLastError();
}

}  // namespace

bool tc_fwd_supported(int dtype, int d) { return dtype == kBF16 && (d == 64 || d == 128); }

bool tc_accum_reduces(const Launch& L, int dtype) {
  if (!tc_fwd_supported(dtype, L.d) || L.mode != kAccumRaw) return false;
  Launch LL = L;
  return assign_ctas(LL, 256) <= kMaxSkItems;  // the condition launch_hd takes the persistent kernel on
}

cudaError_t launch_tc_fwd(Launch L, int dtype, cudaStream_t stream, const char** detail) {
  if (!tc_fwd_supported(dtype, L.d)) {
    *detail = "tensor-core path needs bf16 and head_dim 64 or 128";
    return cudaErrorInvalidValue;
  }
  return L.d == 128 ? launch_hd<128>(L, stream, detail) : launch_hd<64>(L, stream, detail);
}

}  // namespace afa
