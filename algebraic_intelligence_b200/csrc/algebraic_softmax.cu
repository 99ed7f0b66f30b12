// algebraic_softmax forward and the elementwise octic map.
//
// algebraic_softmax (reference src/attention.py:59-67, 88-91 with
// src/primitives.py:17-21, 56-65): per row of length K
//     z   = x in the accumulation dtype (fp32 for half inputs, fp64 kept)
//     tau = rsqrt(sum(z^2) * (1/K) + eps)                       (AVN)
//     k   = rho(tau * z)^8            (branch form, attention.py:18-26)
//     p   = k / (sum(k) + sink)   -> input dtype
// A row is read once and written once: it is memory-bound. Rows of up to 1024
// elements are held in the registers of one warp; longer rows use a CTA per
// row and three sweeps that hit L2 after the first.
//
// Backward (the custom VJP of attention.py:70-85 with primitives.py:73-79):
// with y = tau z, r = rsqrt(1 + y^2), p as above and upstream g,
//     ng = 8 r p (g - sum(p g))                (attention.py:77-79)
//     dx = tau (ng - y sum(ng y) / K)          (AVN backward)
// in the accumulation dtype, returned in g's dtype. The forward quantities
// are recomputed from x, so the backward reads x and g and writes dx.
//
// octic_kernel (attention.py:47-50): y = rho(x)^8 elementwise in the
// accumulation dtype, returned in the input dtype; its VJP (attention.py:38-44)
// dx = 8 r rho(x)^8 g with r = rsqrt(1 + x^2), returned in g's dtype.
#include "afa_common.cuh"
#include "afa_internal.h"

namespace afa {
namespace {

template <typename A>
__device__ __forceinline__ A warp_sum(A x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

template <typename A>
__device__ __forceinline__ A rsqrt_acc(A x);
template <>
__device__ __forceinline__ float rsqrt_acc<float>(float x) { return rsqrtf(x); }
template <>
__device__ __forceinline__ double rsqrt_acc<double>(double x) { return rsqrt(x); }

template <typename T, int VPT>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const T* __restrict__ x, T* __restrict__ y, long long rows,
                                                           int cols, double sink_d, double eps_d) {
  using A = typename AccOf<T>::type;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * cols;
  T* yr = y + row * cols;
  const A inv_width = static_cast<A>(1.0 / cols);
  const A eps = static_cast<A>(eps_d), sink = static_cast<A>(sink_d);
  A z[VPT];
  A ss = A(0);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    z[i] = c < cols ? static_cast<A>(to_acc(xr[c])) : A(0);
    ss = fma(z[i], z[i], ss);
  }
  ss = warp_sum(ss);
  const A tau = rsqrt_acc<A>(ss * inv_width + eps);
  A ks = A(0);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    const A kv = octic_ref(z[i] * tau);
    z[i] = kv;
    ks += c < cols ? kv : A(0);
  }
  ks = warp_sum(ks);
  const A den = ks + sink;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < cols) yr[c] = from_acc<T>(z[i] / den);
  }
}

template <typename A>
__device__ __forceinline__ A block_sum(A x, A* red) {
  x = warp_sum(x);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = x;
  __syncthreads();
  A t = A(0);
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

template <typename T>
__global__ void __launch_bounds__(256) softmax_block_kernel(const T* __restrict__ x, T* __restrict__ y, int cols,
                                                            double sink_d, double eps_d) {
  using A = typename AccOf<T>::type;
  __shared__ A red[8];
  const long long row = blockIdx.x;
  const T* xr = x + row * cols;
  T* yr = y + row * cols;
  const A inv_width = static_cast<A>(1.0 / cols);
  A ss = A(0);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const A z = static_cast<A>(to_acc(xr[c]));
    ss = fma(z, z, ss);
  }
  ss = block_sum(ss, red);
  const A tau = rsqrt_acc<A>(ss * inv_width + static_cast<A>(eps_d));
  A ks = A(0);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) ks += octic_ref(static_cast<A>(to_acc(xr[c])) * tau);
  ks = block_sum(ks, red);
  const A den = ks + static_cast<A>(sink_d);
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    yr[c] = from_acc<T>(octic_ref(static_cast<A>(to_acc(xr[c])) * tau) / den);
}

// Backward, one warp per row (rows of at most 32 * VPT elements).
template <typename T, int VPT>
__global__ void __launch_bounds__(256) softmax_bwd_warp_kernel(const T* __restrict__ x, const T* __restrict__ g,
                                                               T* __restrict__ dx, long long rows, int cols,
                                                               double sink_d, double eps_d) {
  using A = typename AccOf<T>::type;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * cols;
  const T* gr = g + row * cols;
  T* dr = dx + row * cols;
  const A inv_width = static_cast<A>(1.0 / cols);
  A y[VPT], p[VPT], gv[VPT];
  A ss = A(0);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    y[i] = c < cols ? static_cast<A>(to_acc(xr[c])) : A(0);
    gv[i] = c < cols ? static_cast<A>(to_acc(gr[c])) : A(0);
    ss = fma(y[i], y[i], ss);
  }
  const A tau = rsqrt_acc<A>(warp_sum(ss) * inv_width + static_cast<A>(eps_d));
  A ks = A(0);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    y[i] *= tau;
    p[i] = c < cols ? octic_ref(y[i]) : A(0);
    ks += p[i];
  }
  const A inv_den = A(1) / (warp_sum(ks) + static_cast<A>(sink_d));
  A pg = A(0);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    p[i] *= inv_den;
    pg = fma(p[i], gv[i], pg);
  }
  pg = warp_sum(pg);
  A ny = A(0);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const A r = rsqrt_acc<A>(fma(y[i], y[i], A(1)));
    gv[i] = A(8) * r * p[i] * (gv[i] - pg);  // ng
    ny = fma(gv[i], y[i], ny);
  }
  const A radial = warp_sum(ny) * inv_width;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < cols) dr[c] = from_acc<T>(tau * (gv[i] - radial * y[i]));
  }
}

// Backward, one CTA per row (longer rows): five sweeps over the row, all but
// the first from L2.
template <typename T>
__global__ void __launch_bounds__(256) softmax_bwd_block_kernel(const T* __restrict__ x, const T* __restrict__ g,
                                                                T* __restrict__ dx, int cols, double sink_d,
                                                                double eps_d) {
  using A = typename AccOf<T>::type;
  __shared__ A red[8];
  const long long row = blockIdx.x;
  const T* xr = x + row * cols;
  const T* gr = g + row * cols;
  T* dr = dx + row * cols;
  const A inv_width = static_cast<A>(1.0 / cols);
  A ss = A(0);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const A z = static_cast<A>(to_acc(xr[c]));
    ss = fma(z, z, ss);
  }
  const A tau = rsqrt_acc<A>(block_sum(ss, red) * inv_width + static_cast<A>(eps_d));
  A ks = A(0);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) ks += octic_ref(static_cast<A>(to_acc(xr[c])) * tau);
  const A inv_den = A(1) / (block_sum(ks, red) + static_cast<A>(sink_d));
  A pg = A(0);
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    pg = fma(octic_ref(static_cast<A>(to_acc(xr[c])) * tau) * inv_den, static_cast<A>(to_acc(gr[c])), pg);
  pg = block_sum(pg, red);
  auto ng_of = [&](int c, A& yv) {
    yv = static_cast<A>(to_acc(xr[c])) * tau;
    const A pv = octic_ref(yv) * inv_den;
    return A(8) * rsqrt_acc<A>(fma(yv, yv, A(1))) * pv * (static_cast<A>(to_acc(gr[c])) - pg);
  };
  A ny = A(0);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    A yv;
    const A ng = ng_of(c, yv);
    ny = fma(ng, yv, ny);
  }
  const A radial = block_sum(ny, red) * inv_width;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    A yv;
    const A ng = ng_of(c, yv);
    dr[c] = from_acc<T>(tau * (ng - radial * yv));
  }
}

template <typename T>
cudaError_t softmax_bwd_t(const void* x, const void* g, void* dx, long long rows, int cols, double sink, double eps,
                          cudaStream_t stream) {
  using A = typename AccOf<T>::type;
  const T* xp = static_cast<const T*>(x);
  const T* gp = static_cast<const T*>(g);
  T* dp = static_cast<T*>(dx);
  // Three row arrays stay in registers: up to 1024 float32 or 512 float64 columns.
  const int warp_limit = sizeof(A) == 8 ? 512 : 1024;
  if (cols <= warp_limit) {
    const long long blocks = (rows * 32 + 255) / 256;
    if (blocks > 2147483647LL) return cudaErrorInvalidValue;
    const int vpt = (cols + 31) / 32;
    const dim3 b(static_cast<unsigned>(blocks));
    if (vpt <= 1) softmax_bwd_warp_kernel<T, 1><<<b, 256, 0, stream>>>(xp, gp, dp, rows, cols, sink, eps);
    else if (vpt <= 2) softmax_bwd_warp_kernel<T, 2><<<b, 256, 0, stream>>>(xp, gp, dp, rows, cols, sink, eps);
    else if (vpt <= 4) softmax_bwd_warp_kernel<T, 4><<<b, 256, 0, stream>>>(xp, gp, dp, rows, cols, sink, eps);
    else if (vpt <= 8) softmax_bwd_warp_kernel<T, 8><<<b, 256, 0, stream>>>(xp, gp, dp, rows, cols, sink, eps);
    else if (vpt <= 16) softmax_bwd_warp_kernel<T, 16><<<b, 256, 0, stream>>>(xp, gp, dp, rows, cols, sink, eps);
    else if constexpr (sizeof(A) == 4)
      softmax_bwd_warp_kernel<T, 32><<<b, 256, 0, stream>>>(xp, gp, dp, rows, cols, sink, eps);
  } else {
    if (rows > 2147483647LL) return cudaErrorInvalidValue;
    softmax_bwd_block_kernel<T><<<static_cast<unsigned>(rows), 256, 0, stream>>>(xp, gp, dp, cols, sink, eps);
  }
  return cudaGetLastError();
}

template <typename T>
__global__ void octic_kernel(const T* __restrict__ x, T* __restrict__ y, long long n) {
  using A = typename AccOf<T>::type;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = from_acc<T>(octic_ref(static_cast<A>(to_acc(x[i]))));
}

template <typename T>
cudaError_t softmax_t(const void* x, void* y, long long rows, int cols, double sink, double eps,
                      cudaStream_t stream) {
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  if (cols <= 1024) {
    const long long blocks = (rows * 32 + 255) / 256;
    if (blocks > 2147483647LL) return cudaErrorInvalidValue;
    const int vpt = (cols + 31) / 32;
    const dim3 g(static_cast<unsigned>(blocks));
    if (vpt <= 1) softmax_warp_kernel<T, 1><<<g, 256, 0, stream>>>(xp, yp, rows, cols, sink, eps);
    else if (vpt <= 2) softmax_warp_kernel<T, 2><<<g, 256, 0, stream>>>(xp, yp, rows, cols, sink, eps);
    else if (vpt <= 4) softmax_warp_kernel<T, 4><<<g, 256, 0, stream>>>(xp, yp, rows, cols, sink, eps);
    else if (vpt <= 8) softmax_warp_kernel<T, 8><<<g, 256, 0, stream>>>(xp, yp, rows, cols, sink, eps);
    else if (vpt <= 16) softmax_warp_kernel<T, 16><<<g, 256, 0, stream>>>(xp, yp, rows, cols, sink, eps);
    else softmax_warp_kernel<T, 32><<<g, 256, 0, stream>>>(xp, yp, rows, cols, sink, eps);
  } else {
    if (rows > 2147483647LL) return cudaErrorInvalidValue;
    softmax_block_kernel<T><<<static_cast<unsigned>(rows), 256, 0, stream>>>(xp, yp, cols, sink, eps);
  }
  return cudaGetLastError();
}

template <typename T>
__global__ void octic_bwd_kernel(const T* __restrict__ x, const T* __restrict__ g, T* __restrict__ dx, long long n) {
  using A = typename AccOf<T>::type;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const A xv = static_cast<A>(to_acc(x[i]));
    const A r = rsqrt_acc<A>(fma(xv, xv, A(1)));
    dx[i] = from_acc<T>(A(8) * r * octic_ref(xv) * static_cast<A>(to_acc(g[i])));
  }
}

template <typename T>
cudaError_t octic_bwd_t(const void* x, const void* g, void* dx, long long n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const long long want = (n + 255) / 256;
  const int blocks = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
  octic_bwd_kernel<T><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), static_cast<const T*>(g),
                                                  static_cast<T*>(dx), n);
  return cudaGetLastError();
}

template <typename T>
cudaError_t octic_t(const void* x, void* y, long long n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const long long want = (n + 255) / 256;
  const int blocks = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
  octic_kernel<T><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), static_cast<T*>(y), n);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_softmax(const void* x, void* y, long long rows, int cols, int dtype, double sink, double eps,
                           cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  switch (dtype) {
    case kF32: return softmax_t<float>(x, y, rows, cols, sink, eps, stream);
    case kBF16: return softmax_t<__nv_bfloat16>(x, y, rows, cols, sink, eps, stream);
    case kF16: return softmax_t<__half>(x, y, rows, cols, sink, eps, stream);
    case kF64: return softmax_t<double>(x, y, rows, cols, sink, eps, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_softmax_bwd(const void* x, const void* g, void* dx, long long rows, int cols, int dtype, double sink,
                               double eps, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  switch (dtype) {
    case kF32: return softmax_bwd_t<float>(x, g, dx, rows, cols, sink, eps, stream);
    case kBF16: return softmax_bwd_t<__nv_bfloat16>(x, g, dx, rows, cols, sink, eps, stream);
    case kF16: return softmax_bwd_t<__half>(x, g, dx, rows, cols, sink, eps, stream);
    case kF64: return softmax_bwd_t<double>(x, g, dx, rows, cols, sink, eps, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_octic_bwd(const void* x, const void* g, void* dx, long long n, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case kF32: return octic_bwd_t<float>(x, g, dx, n, stream);
    case kBF16: return octic_bwd_t<__nv_bfloat16>(x, g, dx, n, stream);
    case kF16: return octic_bwd_t<__half>(x, g, dx, n, stream);
    case kF64: return octic_bwd_t<double>(x, g, dx, n, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_octic(const void* x, void* y, long long n, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case kF32: return octic_t<float>(x, y, n, stream);
    case kBF16: return octic_t<__nv_bfloat16>(x, y, n, stream);
    case kF16: return octic_t<__half>(x, y, n, stream);
    case kF64: return octic_t<double>(x, y, n, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace afa
