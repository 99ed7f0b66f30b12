// AFA decode step: one query token per (batch, head) attending to its KV cache.
//
// The reference has no decode kernel; its math is pallas_afa_forward with a
// single query row, non-causal (src/kernels/pallas_afa.py:104-151): s = q.k *
// scale in fp32, p = rho(s)^8, O += p.astype(v.dtype) * v, d += p, out =
// O / (d + sink). The oracle is reference_afa with Lq = 1
// (tests/reference_attention.py:44-59).
//
// The step is HBM-bound: every cache byte is read once. Design:
//   * grid (batch*heads, splits); a CTA of 8 warps streams one contiguous key
//     range of one head;
//   * a row of D elements is read by D*sizeof(T)/16 lanes with 16-byte
//     (128-bit) loads, so a warp load instruction covers whole rows,
//     consecutive in memory (fully coalesced); UNROLL independent K and V loads
//     per lane are in flight before any arithmetic;
//   * the dot product is reduced across the row's lanes with xor shuffles;
//     every lane then holds s, maps it with the reference's branch form of rho
//     (octic_ref: exact in the negative tail; its second MUFU op is free in a
//     kernel bound by HBM) and accumulates p*v on its own columns;
//   * warp partials combine by xor shuffle, CTA partials through shared memory;
//   * with more than one split, per-split (numerator, row sum) partials go to a
//     workspace and a second kernel adds them -- plain addition, since AFA needs
//     no running-max rescale -- and divides once.
#include "afa_common.cuh"
#include "afa_internal.h"

namespace afa {
namespace {

constexpr int kDecWarps = 8;
constexpr int kDecThreads = kDecWarps * 32;

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float (&f)[16 / sizeof(T)]);

template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& u, float (&f)[4]) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename T, int D, int UNROLL>
__global__ void __launch_bounds__(kDecThreads) afa_decode_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                 const T* __restrict__ v, T* __restrict__ out,
                                                                 float* __restrict__ dtot, float* __restrict__ ws_o,
                                                                 float* __restrict__ ws_d, int H, int lkv,
                                                                 const int* __restrict__ kv_lens, int kv_len,
                                                                 int nsplit, int chunk, float scale, float sink) {
  constexpr int VEC = 16 / sizeof(T);  // elements per 16-byte load
  constexpr int LPR = D / VEC;         // lanes per row
  constexpr int RPW = 32 / LPR;        // rows per warp-wide load
  static_assert(LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "unsupported head_dim");
  __shared__ float s_o[kDecWarps][D];
  __shared__ float s_d[kDecWarps];

  const int bh = blockIdx.x;
  const int split = blockIdx.y;
  const int b = bh / H;
  // Visible prefix of the cache, clamped to [0, lkv]; an empty row gives
  // output 0 and d_total = sink.
  int len = kv_lens ? kv_lens[b] : kv_len;
  len = len < lkv ? len : lkv;
  len = len > 0 ? len : 0;
  const int kbeg = split * chunk;
  const int kend = min(len, kbeg + chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sl = lane % LPR;
  const int rsub = lane / LPR;

  float qf[VEC];
  {
    const uint4 qq = *reinterpret_cast<const uint4*>(q + static_cast<long long>(bh) * D + sl * VEC);
    unpack16<T>(qq, qf);
  }
  float o[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) o[e] = 0.f;
  float dsum = 0.f;

  const T* kb = k + static_cast<long long>(bh) * lkv * D + sl * VEC;
  const T* vb = v + static_cast<long long>(bh) * lkv * D + sl * VEC;
  constexpr int STEP = kDecWarps * RPW * UNROLL;
  for (int base = kbeg + warp * RPW * UNROLL; base < kend; base += STEP) {
    uint4 kr[UNROLL], vr[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int key = base + u * RPW + rsub;
      if (key < kend) {
        kr[u] = ldg_stream(kb + static_cast<long long>(key) * D);
        vr[u] = ldg_stream(vb + static_cast<long long>(key) * D);
      } else {
        kr[u] = make_uint4(0, 0, 0, 0);
        vr[u] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      float kf[VEC], vf[VEC];
      unpack16<T>(kr[u], kf);
      unpack16<T>(vr[u], vf);
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; ++e) dot = fmaf(qf[e], kf[e], dot);
#pragma unroll
      for (int off = LPR / 2; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      const int key = base + u * RPW + rsub;
      float p = octic_ref(dot * scale);
      p = key < kend ? p : 0.f;
      dsum += p;
      const float pr = round_like<T>(p);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = fmaf(pr, vf[e], o[e]);
    }
  }
  // Lanes with the same column slice (different row slots) hold partials of
  // the same columns; every lane of a row group holds the same dsum.
#pragma unroll
  for (int off = LPR; off < 32; off <<= 1) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
    dsum += __shfl_xor_sync(0xffffffffu, dsum, off);
  }
  if (rsub == 0) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) s_o[warp][sl * VEC + e] = o[e];
  }
  if (lane == 0) s_d[warp] = dsum;
  __syncthreads();
  float dtotal = 0.f;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) dtotal += s_d[w];
  if (nsplit == 1) {
    const float denom = dtotal + sink;
    for (int c = threadIdx.x; c < D; c += kDecThreads) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) acc += s_o[w][c];
      out[static_cast<long long>(bh) * D + c] = from_acc<T>(denom > 0.f ? acc / denom : 0.f);
    }
    if (threadIdx.x == 0 && dtot) dtot[bh] = denom;
  } else {
    const long long slot = static_cast<long long>(bh) * nsplit + split;
    for (int c = threadIdx.x; c < D; c += kDecThreads) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) acc += s_o[w][c];
      ws_o[slot * D + c] = acc;
    }
    if (threadIdx.x == 0) ws_d[slot] = dtotal;
  }
}

template <typename T>
__global__ void afa_decode_combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_d,
                                          T* __restrict__ out, float* __restrict__ dtot, int d, int nsplit,
                                          float sink) {
  const int bh = blockIdx.x;
  float den = 0.f;
  for (int s = 0; s < nsplit; ++s) den += ws_d[static_cast<long long>(bh) * nsplit + s];
  den += sink;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s) acc += ws_o[(static_cast<long long>(bh) * nsplit + s) * d + c];
    out[static_cast<long long>(bh) * d + c] = from_acc<T>(den > 0.f ? acc / den : 0.f);
  }
  if (threadIdx.x == 0 && dtot) dtot[bh] = den;
}

template <typename T, int D>
cudaError_t launch_dec(const void* q, const void* k, const void* v, void* out, void* dtot, int B, int H, int lkv,
                       float sink, const int* kv_lens, int kv_len, float* ws_o, float* ws_d, int nsplit,
                       cudaStream_t stream) {
  constexpr int UNROLL = 4;
  const int bh = B * H;
  const int chunk = (lkv + nsplit - 1) / nsplit;
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(D)));
  dim3 grid(bh, nsplit);
  afa_decode_kernel<T, D, UNROLL><<<grid, kDecThreads, 0, stream>>>(
      static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<T*>(out),
      static_cast<float*>(dtot), ws_o, ws_d, H, lkv, kv_lens, kv_len, nsplit, chunk, scale, sink);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || nsplit == 1) return e;
  afa_decode_combine_kernel<T><<<bh, 128, 0, stream>>>(ws_o, ws_d, static_cast<T*>(out), static_cast<float*>(dtot),
                                                       D, nsplit, sink);
  return cudaGetLastError();
}

}  // namespace

// Splits per head: enough CTAs to cover the 148 SMs about four times over, no
// split shorter than 512 keys.
int decode_splits(int bh, int lkv) {
  const int target = 148 * 4;
  int s = (target + bh - 1) / bh;
  const int max_s = (lkv + 511) / 512;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  return s;
}

bool decode_fast_supported(int dtype, int d) {
  return (dtype == kBF16 && (d == 64 || d == 128 || d == 256)) || (dtype == kF32 && (d == 64 || d == 128));
}

cudaError_t launch_decode(const void* q, const void* k, const void* v, void* out, void* dtot, int B, int H,
                          int lkv, int d, int dtype, double sink, const int* kv_lens, int kv_len, float* ws_o,
                          float* ws_d, int nsplit, int* /*status*/, cudaStream_t stream) {
  const float fs = static_cast<float>(sink);
  if (dtype == kBF16) {
    if (d == 64) return launch_dec<__nv_bfloat16, 64>(q, k, v, out, dtot, B, H, lkv, fs, kv_lens, kv_len, ws_o, ws_d, nsplit, stream);
    if (d == 128) return launch_dec<__nv_bfloat16, 128>(q, k, v, out, dtot, B, H, lkv, fs, kv_lens, kv_len, ws_o, ws_d, nsplit, stream);
    if (d == 256) return launch_dec<__nv_bfloat16, 256>(q, k, v, out, dtot, B, H, lkv, fs, kv_lens, kv_len, ws_o, ws_d, nsplit, stream);
  } else if (dtype == kF32) {
    if (d == 64) return launch_dec<float, 64>(q, k, v, out, dtot, B, H, lkv, fs, kv_lens, kv_len, ws_o, ws_d, nsplit, stream);
    if (d == 128) return launch_dec<float, 128>(q, k, v, out, dtot, B, H, lkv, fs, kv_lens, kv_len, ws_o, ws_d, nsplit, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace afa
