// Device pieces of the tensor-core AFA forward kernels (afa_tc_sm100.cu):
// work-unit geometry on global positions, the octic map of a TMEM score chunk
// (with its negative-tail switch), the chunk transpose of the epilogues, and
// the persistent walk over a longest-first item list.
//
// Reference: afa_kernel (src/kernels/pallas_afa.py:52-151): the causal key-tile
// skip (:91-95), the valid-length and causal masks (:116-124) and the weight
// map (:113) that these helpers implement.
#pragma once

#include "afa_common.cuh"
#include "afa_problem.h"

namespace afa {

// Key tiles of one segment visible from a query tile whose last valid row sits
// at global position qpos_last.
__host__ __device__ __forceinline__ int seg_tiles(const Segment& ks, int causal, int qpos_last) {
  int n = ks.len;
  if (causal) {
    const int m = qpos_last - ks.pos0 + 1;
    n = m < n ? m : n;
  }
  return n <= 0 ? 0 : (n + 127) / 128;
}

struct KvTile {
  int row;  // first row of the tile in the per-(b,h) K/V tensor
  int pos;  // global position of that row
  int lim;  // valid keys in the tile (1..128)
};

__host__ __device__ __forceinline__ KvTile kv_tile(const Problem& P, int cnt_seg0, int t) {
  const int s = (t < cnt_seg0) ? 0 : 1;
  const int jj = s ? t - cnt_seg0 : t;
  const Segment& ks = P.k[s];
  KvTile kt;
  kt.row = ks.row0 + jj * 128;
  kt.pos = ks.pos0 + jj * 128;
  const int lim = ks.len - jj * 128;
  kt.lim = lim < 128 ? lim : 128;
  return kt;
}

// Geometry of work unit `cta` of a launch: two query tiles of TILE rows each
// (a "pair" of 128-row tiles for one CTA): its problem, first row, and
// key-tile counts. Only the last key segment may be partially visible, which
// makes tile 0's key tiles a prefix of tile 1's.
struct PairGeom {
  int pi;      // problem index
  int r0;      // first row of query tile 0 in the problem's q segment
  int n0, n1;  // key tiles of query tile 0 / 1
  int cnt1_0;  // tile 1's key tiles in key segment 0
};

template <int TILE>
__host__ __device__ __forceinline__ PairGeom unit_geom(const Launch& L, int cta) {
  PairGeom G;
  int pi = 0;
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < L.nprob && cta >= L.prob[i].cta0) pi = i;
  const Problem& P = L.prob[pi];
  G.pi = pi;
  G.r0 = (cta - P.cta0) * 2 * TILE;
  const bool q1_live = G.r0 + TILE < P.q.len;
  const int last0 = (G.r0 + TILE - 1 < P.q.len - 1) ? G.r0 + TILE - 1 : P.q.len - 1;
  const int last1 = q1_live ? ((G.r0 + 2 * TILE - 1 < P.q.len - 1) ? G.r0 + 2 * TILE - 1 : P.q.len - 1) : last0;
  int cnt0[2] = {0, 0}, cnt1[2] = {0, 0};
  for (int s = 0; s < kMaxKSegs; ++s) {
    if (s < P.nk) {
      cnt0[s] = seg_tiles(P.k[s], L.causal, P.q.pos0 + last0);
      cnt1[s] = seg_tiles(P.k[s], L.causal, P.q.pos0 + last1);
    }
  }
  G.n1 = cnt1[0] + cnt1[1];
  G.n0 = (P.nk == 1 || cnt0[0] == cnt1[0]) ? cnt0[0] + cnt0[1] : G.n1;
  G.cnt1_0 = cnt1[0];
  return G;
}

// Query pair `cta` of a one-CTA launch (two 128-row tiles).
__host__ __device__ __forceinline__ PairGeom pair_geom(const Launch& L, int cta) { return unit_geom<128>(L, cta); }

// Octic map of one 32-column chunk of a score row, written back as 16 packed
// bf16 pairs; returns the chunk's fp32 row sum. MASK selects the per-element
// visibility test (diagonal and partial tiles only); EXACT the reference's
// branch form of rho (octic_exact2) instead of the single-MUFU one.
template <bool MASK, bool EXACT>
__device__ __forceinline__ float map_chunk(const uint32_t (&sv)[32], uint32_t (&pk)[16], float scale, int key0,
                                           int lim, int causal, int kpos0, int qpos) {
  float2 acc = make_float2(0.f, 0.f);
  const float2 sc = make_float2(scale, scale);
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const float2 s = __fmul2_rn(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), sc);
    float2 p = EXACT ? octic_exact2(s) : octic_fast2(s);
    if (MASK) {
      const int c0 = key0 + e, c1 = c0 + 1;
      const bool v0 = (c0 < lim) && (!causal || kpos0 + c0 <= qpos);
      const bool v1 = (c1 < lim) && (!causal || kpos0 + c1 <= qpos);
      p.x = v0 ? p.x : 0.f;
      p.y = v1 ? p.y : 0.f;
    }
    acc = __fadd2_rn(acc, p);
    pk[e >> 1] = pack_bf16x2(p.x, p.y);
  }
  return acc.x + acc.y;
}

// Maps the 32-column chunk of TMEM scores at s_tm into pk and returns its row
// sum with the single-MUFU form. CHECK: a warp with a lane that sees a key
// and whose chunk weights sum below kTailChunkSum (every score of that row
// chunk deep in the negative tail, where the fast form cancels) maps the
// chunk again with the exact form, from the scores still in TMEM.
template <bool CHECK>
__device__ __forceinline__ float map_chunk_tmem(uint32_t s_tm, uint32_t (&pk)[16], bool need_mask, float scale,
                                                int key0, int lim, int causal, int kpos0, int qpos) {
  uint32_t sv[32];
  tmem_ld32(s_tm, sv);
  tmem_ld_wait();
  float part = need_mask ? map_chunk<true, false>(sv, pk, scale, key0, lim, causal, kpos0, qpos)
                         : map_chunk<false, false>(sv, pk, scale, key0, lim, causal, kpos0, qpos);
  if constexpr (CHECK) {
    // Visible keys of a chunk form a prefix, so it sees one iff it sees key0.
    const bool sees = !need_mask || (key0 < lim && (!causal || kpos0 + key0 <= qpos));
    if (__any_sync(0xffffffffu, sees && part < kTailChunkSum)) {
      tmem_ld32(s_tm, sv);
      tmem_ld_wait();
      part = need_mask ? map_chunk<true, true>(sv, pk, scale, key0, lim, causal, kpos0, qpos)
                       : map_chunk<false, true>(sv, pk, scale, key0, lim, causal, kpos0, qpos);
    }
  }
  return part;
}

// Maps one key tile's two 32-column chunks of this warp (columns
// [key_base, key_base + 64)), stores P and adds the chunk sums to dsum. The
// chunk check (CHECK) is needed only while the warp holds a row whose weights
// so far sum below kTailRowSum: past that, the errors of later tail chunks are
// bounded by the row sum they add to (see kTailRowSum), so the loop drops the
// check once every lane has passed it -- after the first key tile, for all
// but rows wholly in the tail. (The checked path's code alone, never run,
// measured about 1% on short prefills; the check itself adds little.)
//
// In a masked tile (need_mask: the diagonal of a causal launch, or a partial
// key tile) each chunk is classed for the warp's 32 rows as a whole (the rows
// are consecutive, so the visible keys of row i are a prefix no shorter than
// row i-1's): a chunk no row of the warp sees gets P = 0 without loading or
// mapping its scores, a chunk every row sees in full takes the unmasked map,
// and only the chunks crossing the diagonal (or the valid length) run the
// per-element mask. The unmasked tiles keep a loop of their own: with the
// classes inside one shared loop the long-sequence launch measured 1-2% slower.
template <bool CHECK>
__device__ __forceinline__ void map_tile(uint32_t s_base, int key_base, bool need_mask, float scale, int lim,
                                         int causal, int kpos0, int qpos, float& dsum) {
  if (!need_mask) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int key0 = key_base + 32 * c;
      const uint32_t s_tm = s_base + key0;
      uint32_t pk[16];
      const float part = map_chunk_tmem<CHECK>(s_tm, pk, false, scale, key0, lim, causal, kpos0, qpos);
      // P of these 32 keys -> the first 16 of the 32 columns just read.
      tmem_st16(s_tm, pk);
      dsum += part;
    }
    return;
  }
  // Last key index (tile-relative) the warp's first / last row sees.
  const int row_first = qpos - static_cast<int>(threadIdx.x & 31);
  const int vis_first = causal ? row_first - kpos0 : 0x7fffffff;
  const int vis_last = causal ? row_first + 31 - kpos0 : 0x7fffffff;
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    const int key0 = key_base + 32 * c;
    const uint32_t s_tm = s_base + key0;
    uint32_t pk[16];
    float part = 0.f;
    if (key0 >= lim || key0 > vis_last) {  // no row of the warp sees a key of the chunk
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = 0u;
    } else {
      const bool full = key0 + 31 < lim && key0 + 31 <= vis_first;
      part = map_chunk_tmem<CHECK>(s_tm, pk, !full, scale, key0, lim, causal, kpos0, qpos);
    }
    tmem_st16(s_tm, pk);
    dsum += part;
  }
}

// Transposes NCH x NCH blocks of float4 chunks within groups of NCH lanes:
// lane i of a group holds chunks j = 0..NCH-1 (v[4j..4j+3]) of its own row;
// afterwards it holds chunk i of the group's rows 0..NCH-1 (slot k = row k).
// log2(NCH) exchange stages: at stage m a lane swaps, with lane i^m, the
// chunks whose index differs from its own index in bit m.
template <int NCH>
__device__ __forceinline__ void transpose_chunks(uint32_t (&v)[32], int i) {
#pragma unroll
  for (int m = NCH / 2; m >= 1; m >>= 1) {
    const bool hi = (i & m) != 0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      if (j & m) continue;  // pair (j, j | m)
      const int jh = j | m;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t send = hi ? v[4 * j + e] : v[4 * jh + e];
        const uint32_t got = __shfl_xor_sync(0xffffffffu, send, m);
        if (hi)
          v[4 * j + e] = got;
        else
          v[4 * jh + e] = got;
      }
    }
  }
}

constexpr int kMaxSkItems = 1024;
// Final-output launches use the persistent kernel only while their query pairs
// average at most this many key tiles.
constexpr int kSkFinalMaxAvgTiles = 32;

struct SkPlan {
  int nitems;                   // listed query pairs per (b, h)
  int nbh;                      // B * H
  int waves;                    // rounds of whole items
  int prefix[kMaxSkItems + 1];  // key-tile iterations before listed pair i; prefix[nitems] = per (b, h)
  int pair_of[kMaxSkItems];     // launch pair (pair_geom index) of listed pair i
};

struct SkSeg {
  int bh, item, t0, t1;  // key tiles [t0, t1) of listed pair `item` of head bh
};

// Iterations of linear items [0, j) (item j = pair j / nbh of head j % nbh).
__host__ __device__ __forceinline__ long long sk_before(const SkPlan& S, long long j) {
  const int pair = static_cast<int>(j / S.nbh);
  const int hh = static_cast<int>(j - static_cast<long long>(pair) * S.nbh);
  const long long base = static_cast<long long>(S.nbh) * S.prefix[pair];
  return pair >= S.nitems ? base : base + static_cast<long long>(hh) * (S.prefix[pair + 1] - S.prefix[pair]);
}

// The pieces CTA c of G computes, in order; every role of the CTA walks the
// same sequence. SNAKE (the final-output mode): whole items only, and in odd
// rounds CTA c takes the round's (G-1-c)-th item, so over the rounds of a
// longest-first list every CTA gets a like share. Otherwise whole-item rounds
// are followed by the even split of the remaining iterations.
template <bool SNAKE>
struct SkWalk;

template <>
struct SkWalk<true> {
  const SkPlan* S;
  int G, c, k, total;

  __device__ __forceinline__ void init(const SkPlan& s, int G_, int c_) {
    S = &s;
    G = G_;
    c = c_;
    k = 0;
    total = s.nbh * s.nitems;
  }

  __device__ __forceinline__ bool next(SkSeg& sg) {
    while (k < S->waves) {
      const int j = k * G + ((k & 1) ? G - 1 - c : c);
      ++k;
      if (j >= total) continue;
      const int item = j / S->nbh;
      const int n = S->prefix[item + 1] - S->prefix[item];
      if (n > 0) {
        sg.bh = j - item * S->nbh;
        sg.item = item;
        sg.t0 = 0;
        sg.t1 = n;
        return true;
      }
    }
    return false;
  }
};

template <>
struct SkWalk<false> {
  const SkPlan* S;
  int G, c, k;
  long long j0, total, i, hi;

  __device__ __forceinline__ void init(const SkPlan& s, int G_, int c_) {
    S = &s;
    G = G_;
    c = c_;
    k = 0;
    total = static_cast<long long>(s.nbh) * s.nitems;
    j0 = static_cast<long long>(s.waves) * G;
    const long long i0 = sk_before(s, j0);
    const long long tail = sk_before(s, total) - i0;
    i = i0 + tail * c / G;
    hi = i0 + tail * (c + 1) / G;
  }

  __device__ __forceinline__ bool next(SkSeg& sg) {
    while (k < S->waves) {  // whole items
      const long long j = static_cast<long long>(k++) * G + c;
      const int item = static_cast<int>(j / S->nbh);
      const int n = S->prefix[item + 1] - S->prefix[item];
      if (n > 0) {
        sg.bh = static_cast<int>(j - static_cast<long long>(item) * S->nbh);
        sg.item = item;
        sg.t0 = 0;
        sg.t1 = n;
        return true;
      }
    }
    if (i >= hi) return false;  // split tail: the item holding iteration i
    long long lo = j0, up = total;  // sk_before(lo) <= i < sk_before(up)
    while (up - lo > 1) {
      const long long mid = (lo + up) >> 1;
      if (sk_before(*S, mid) <= i) lo = mid; else up = mid;
    }
    const int item = static_cast<int>(lo / S->nbh);
    sg.bh = static_cast<int>(lo - static_cast<long long>(item) * S->nbh);
    sg.item = item;
    sg.t0 = static_cast<int>(i - sk_before(*S, lo));
    const int n = S->prefix[item + 1] - S->prefix[item];
    const long long rem = hi - i;
    sg.t1 = rem < static_cast<long long>(n - sg.t0) ? sg.t0 + static_cast<int>(rem) : n;
    i += sg.t1 - sg.t0;
    return true;
  }
};

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ void red_add(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}


}  // namespace afa
