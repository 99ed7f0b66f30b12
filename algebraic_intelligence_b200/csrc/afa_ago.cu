// AGO rotary position rotations: the Q/K prologue of the attention layer
// (src/model.py:262-264).
//
//   afa_ago_table   build_cayley_rotary_matrix (src/attention.py:156-207): per
//                   channel pair k a rational frequency w_k, the Cayley step
//                   rotation ((1-w^2)/(1+w^2), 2w/(1+w^2)), and the tables
//                   (c, s)[m] = the m-fold product, renormalised after every
//                   step. One thread per pair walks the positions in order, in
//                   the reference's calc dtype (float32 for bf16 / float32
//                   tables, float64 for float64). Products are rounded one by
//                   one (no fused multiply-add) and sqrt / divide are IEEE, as
//                   in the float64 oracle (tests/reference_ago.py:21-53), so the
//                   float64 tables reproduce it.
//   afa_ago_rotate  apply_ago_rotations / _rotate_tensor (src/attention.py:
//                   142-152, :210-240): (x0, x1) at position m ->
//                   (c x0 - s x1, s x0 + c x1), with c, s first cast to the
//                   tensor dtype (:148-149). Q and K go through one launch: one
//                   HBM pass reading both and writing both, four channel pairs
//                   per thread with 8- or 16-byte accesses.
//
// Why a separate pass and not the attention kernel's prologue: a K tile is read
// by every CTA that owns a query pair of its head (16 to 256 of them), so
// rotating K there would repeat the work that many times on the warps that
// already bound that kernel, while this pass costs one read and one write of Q
// and K, a few percent of the attention time.
#include <cmath>
#include <cstdio>

#include "afa_b200.h"
#include "afa_common.cuh"
#include "afa_internal.h"

namespace afa {
namespace {

constexpr int kMaxAgoPairs = 256;

struct AgoTableArgs {
  void* c;
  void* s;
  int pairs, len, has_freqs;
  double base;
  double freqs[kMaxAgoPairs];
};

template <typename A> __device__ __forceinline__ A mul_rn(A a, A b);
template <> __device__ __forceinline__ float mul_rn<float>(float a, float b) { return __fmul_rn(a, b); }
template <> __device__ __forceinline__ double mul_rn<double>(double a, double b) { return __dmul_rn(a, b); }

template <typename T, typename A>
__global__ void ago_table_kernel(const __grid_constant__ AgoTableArgs a) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= a.pairs) return;
  A w;
  if (a.has_freqs) {
    w = static_cast<A>(a.freqs[k]);
  } else {
    const A base = static_cast<A>(a.base);
    const A denom = a.pairs - 1 > 1 ? static_cast<A>(a.pairs - 1) : A(1);
    const A alpha = (sqrt(base) - A(1)) / denom;
    const A lin = A(1) + mul_rn<A>(alpha, static_cast<A>(k));
    w = A(1) / mul_rn<A>(lin, lin);
  }
  const A w2 = mul_rn<A>(w, w);
  const A cb = (A(1) - w2) / (A(1) + w2);
  const A sb = mul_rn<A>(A(2), w) / (A(1) + w2);
  A c = A(1), s = A(0);
  T* co = static_cast<T*>(a.c) + k;
  T* so = static_cast<T*>(a.s) + k;
  for (int m = 0; m < a.len; ++m) {
    co[static_cast<long long>(m) * a.pairs] = from_acc<T>(c);
    so[static_cast<long long>(m) * a.pairs] = from_acc<T>(s);
    const A cn = mul_rn<A>(cb, c) - mul_rn<A>(sb, s);
    const A sn = mul_rn<A>(sb, c) + mul_rn<A>(cb, s);
    const A r = A(1) / sqrt(mul_rn<A>(cn, cn) + mul_rn<A>(sn, sn));
    c = mul_rn<A>(cn, r);
    s = mul_rn<A>(sn, r);
  }
}

// Table value cast to the tensor dtype (src/attention.py:148-149), in the
// arithmetic type of the rotation.
template <typename T, typename TT, typename A>
__device__ __forceinline__ A table_as(const TT* p, long long i) {
  return static_cast<A>(to_acc(from_acc<T>(static_cast<A>(to_acc(p[i])))));
}

struct AgoRotateArgs {
  const void* q;
  const void* k;
  void* qo;
  void* ko;
  const void* c;
  const void* s;
  long long rows;   // elements / dim
  long long inner;  // rows per position step (product of the axes between the sequence axis and the last)
  int pairs, seq_len;
};

// V channel pairs per thread (pairs % V == 0).
template <typename T, typename TT, typename A, int V>
__global__ void __launch_bounds__(256) ago_rotate_kernel(const __grid_constant__ AgoRotateArgs a) {
  const long long groups = a.rows * (a.pairs / V);
  const int gpr = a.pairs / V;
  for (long long gi = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; gi < groups;
       gi += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = gi / gpr;
    const int p0 = static_cast<int>(gi - row * gpr) * V;
    const int pos = static_cast<int>((row / a.inner) % a.seq_len);
    const long long e0 = row * (2LL * a.pairs) + 2LL * p0;  // first element
    const long long t0 = static_cast<long long>(pos) * a.pairs + p0;
    // V == 4: 16-byte chunks (the host picks it only for 16-byte-aligned
    // rows); V == 1: element accesses. Both tensors' chunks are loaded before
    // either is stored (the compiler may not move a load of k past a store to
    // qo), which doubles the bytes each thread has in flight.
    constexpr int N16 = V == 4 ? static_cast<int>(sizeof(T)) * 2 * V / 16 : 0;
    alignas(16) T in[2][2 * V];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const T* x = static_cast<const T*>(t ? a.k : a.q) + e0;
      if constexpr (N16 > 0) {
#pragma unroll
        for (int i = 0; i < N16; ++i) reinterpret_cast<uint4*>(in[t])[i] = reinterpret_cast<const uint4*>(x)[i];
      } else {
#pragma unroll
        for (int i = 0; i < 2 * V; ++i) in[t][i] = x[i];
      }
    }
    A cc[V], ss[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      cc[v] = table_as<T, TT, A>(static_cast<const TT*>(a.c), t0 + v);
      ss[v] = table_as<T, TT, A>(static_cast<const TT*>(a.s), t0 + v);
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      T* y = static_cast<T*>(t ? a.ko : a.qo) + e0;
      alignas(16) T out[2 * V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const A x0 = static_cast<A>(to_acc(in[t][2 * v])), x1 = static_cast<A>(to_acc(in[t][2 * v + 1]));
        out[2 * v] = from_acc<T>(cc[v] * x0 - ss[v] * x1);
        out[2 * v + 1] = from_acc<T>(ss[v] * x0 + cc[v] * x1);
      }
      if constexpr (N16 > 0) {
#pragma unroll
        for (int i = 0; i < N16; ++i) reinterpret_cast<uint4*>(y)[i] = reinterpret_cast<const uint4*>(out)[i];
      } else {
#pragma unroll
        for (int i = 0; i < 2 * V; ++i) y[i] = out[i];
      }
    }
  }
}

template <typename T, typename TT, typename A>
cudaError_t launch_rotate_tt(const AgoRotateArgs& a, bool aligned, cudaStream_t stream) {
  // Four pairs per thread (16 bytes of bf16, 32 of float32, 64 of float64 per
  // tensor) in 16-byte accesses, which need 16-byte-aligned rows: a
  // contiguous tensor with dim % 8 == 0 and 16-byte-aligned base pointers.
  const bool vec = aligned && a.pairs % 4 == 0;
  const long long groups = a.rows * (a.pairs / (vec ? 4 : 1));
  long long blocks = (groups + 255) / 256;
  if (blocks > 148LL * 32) blocks = 148LL * 32;
  if (blocks < 1) blocks = 1;
  if (vec)
    ago_rotate_kernel<T, TT, A, 4><<<static_cast<int>(blocks), 256, 0, stream>>>(a);
  else
    ago_rotate_kernel<T, TT, A, 1><<<static_cast<int>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

template <typename T, typename A>
cudaError_t launch_rotate_t(const AgoRotateArgs& a, int table_dtype, bool aligned, cudaStream_t stream) {
  switch (table_dtype) {
    case kF32: return launch_rotate_tt<T, float, A>(a, aligned, stream);
    case kBF16: return launch_rotate_tt<T, __nv_bfloat16, A>(a, aligned, stream);
    case kF64: return launch_rotate_tt<T, double, A>(a, aligned, stream);
    default: return cudaErrorInvalidValue;
  }
}

bool ok_dtype(int dt) { return dt == kF32 || dt == kBF16 || dt == kF64; }

int fail_cuda(const char* what, cudaError_t e) {
  char msg[200];
  snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
  return set_last_error(AFA_ERR_CUDA, msg);
}

}  // namespace
}  // namespace afa

extern "C" int afa_ago_table(void* c, void* s, int dim, int max_seq_len, const double* freqs, double base, int dtype,
                             void* stream) {
  using namespace afa;
  if (!ok_dtype(dtype)) return set_last_error(AFA_ERR_DTYPE, "afa_ago_table: dtype must be float32, bfloat16 or float64");
  if (dim <= 0 || dim % 2 != 0) return set_last_error(AFA_ERR_INVALID, "dim must be a positive even integer");
  if (max_seq_len <= 0) return set_last_error(AFA_ERR_INVALID, "max_seq_len must be a positive integer");
  if (dim / 2 > kMaxAgoPairs) return set_last_error(AFA_ERR_INVALID, "afa_ago_table: dim above 512 is not supported");
  if (!c || !s) return set_last_error(AFA_ERR_INVALID, "afa_ago_table: c and s must be non-null device pointers");
  if (!freqs && !(std::isfinite(base) && base > 0.0))
    return set_last_error(AFA_ERR_INVALID, "afa_ago_table: base must be finite and positive");
  AgoTableArgs a{};
  a.c = c;
  a.s = s;
  a.pairs = dim / 2;
  a.len = max_seq_len;
  a.base = base;
  a.has_freqs = freqs ? 1 : 0;
  if (freqs)
    for (int i = 0; i < a.pairs; ++i) a.freqs[i] = freqs[i];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int blocks = (a.pairs + 127) / 128;
  if (dtype == kF64)
    ago_table_kernel<double, double><<<blocks, 128, 0, st>>>(a);
  else if (dtype == kF32)
    ago_table_kernel<float, float><<<blocks, 128, 0, st>>>(a);
  else
    ago_table_kernel<__nv_bfloat16, float><<<blocks, 128, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AFA_OK : fail_cuda("afa_ago_table launch", e);
}

extern "C" int afa_ago_rotate(const void* q, const void* k, void* q_out, void* k_out, const void* c, const void* s,
                              int table_dtype, long long rows, int dim, int seq_len, long long inner, int dtype,
                              void* stream) {
  using namespace afa;
  if (!ok_dtype(dtype) || !ok_dtype(table_dtype))
    return set_last_error(AFA_ERR_DTYPE, "afa_ago_rotate: dtypes must be float32, bfloat16 or float64");
  if (!q || !k || !q_out || !k_out || !c || !s)
    return set_last_error(AFA_ERR_INVALID, "afa_ago_rotate: null pointer");
  if (dim <= 0 || dim % 2 != 0) return set_last_error(AFA_ERR_INVALID, "Feature dimension must be even");
  if (rows < 0 || seq_len <= 0 || inner <= 0) return set_last_error(AFA_ERR_INVALID, "afa_ago_rotate: bad shape");
  if (rows == 0) return AFA_OK;
  AgoRotateArgs a{};
  a.q = q;
  a.k = k;
  a.qo = q_out;
  a.ko = k_out;
  a.c = c;
  a.s = s;
  a.rows = rows;
  a.inner = inner;
  a.pairs = dim / 2;
  a.seq_len = seq_len;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool aligned = al(q) && al(k) && al(q_out) && al(k_out) && dim % 8 == 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == kF64)
    e = launch_rotate_t<double, double>(a, table_dtype, aligned, st);
  else if (dtype == kF32)
    e = launch_rotate_t<float, float>(a, table_dtype, aligned, st);
  else
    e = launch_rotate_t<__nv_bfloat16, float>(a, table_dtype, aligned, st);
  return e == cudaSuccess ? AFA_OK : fail_cuda("afa_ago_rotate launch", e);
}
