// AFA forward on the CUDA cores (FFMA), for float32 / float64 inputs and for
// bf16 head dimensions the tensor-core kernel does not cover.
//
// Same math and problem descriptors as afa_tc_sm100.cu (reference
// src/kernels/pallas_afa.py:52-151): fp32 (fp64 for float64) dot products, the
// reference's branch form of rho (pallas_afa.py:39-49), P rounded to the value
// dtype before P.V (:133), the row sum over unrounded P (:139), one divide at
// the end (:149). tcgen05 has no full-precision fp32 MMA, so the float32 path
// (the reference runs it at Precision.HIGHEST, :224-228) is computed here.
//
// Tiling: BM query rows x BN keys per step, 256 threads, 16x16 thread grid;
// thread (ty, tx) owns S elements (ty+16i, tx+16j) and O elements
// (ty+16i, tx+16j'), so shared-memory reads are bank-conflict free (row pitch
// DMAX+1) and each half-warp shares one query row.
#include "afa_common.cuh"
#include "afa_internal.h"

namespace afa {
namespace {

template <typename A>
__device__ __forceinline__ A octic_simt(A s) {
  return octic_ref(s);
}

// Accumulator of the P.V numerator and the row sum. Float32 inputs accumulate
// in float64 here: the result is then the correctly rounded float32 of a
// nearly exact sum, so the single-device forward and a ring that splits the
// same sum over hops agree to one float32 rounding per hop.
template <typename T> struct SumOf { using type = float; };
template <> struct SumOf<float> { using type = double; };
template <> struct SumOf<double> { using type = double; };

template <typename T, typename A>
__device__ __forceinline__ A round_p(A p) {
  if constexpr (sizeof(A) == 8) {
    return p;
  } else {
    return round_like<T>(p);
  }
}

template <typename T, typename A, int BM, int BN, int DMAX>
__global__ void __launch_bounds__(256) afa_simt_fwd_kernel(const __grid_constant__ Launch L) {
  constexpr int LD = DMAX + 1;
  constexpr int PLD = BN + 1;
  constexpr int TR = BM / 16;
  constexpr int TC = BN / 16;
  constexpr int OC = DMAX / 16;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  A* Qs = reinterpret_cast<A*>(smem_raw);
  A* Ks = Qs + BM * LD;
  A* Vs = Ks + BN * LD;
  A* Ps = Vs + BN * LD;

  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int bh = blockIdx.x;
  const int cta = gridDim.y - 1 - blockIdx.y;
  int pi = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < L.nprob && cta >= L.prob[i].cta0) pi = i;
  const Problem& P = L.prob[pi];
  const int r0 = (cta - P.cta0) * BM;
  const int D = L.d;
  const T* q = static_cast<const T*>(L.q) + static_cast<long long>(bh) * L.lq * D;
  const T* k = static_cast<const T*>(L.k) + static_cast<long long>(bh) * L.lk * D;
  const T* v = static_cast<const T*>(L.v) + static_cast<long long>(bh) * L.lk * D;
  const A scale = sizeof(A) == 8 ? static_cast<A>(L.scale_d) : static_cast<A>(L.scale);
  const A sink = sizeof(A) == 8 ? static_cast<A>(L.sink_d) : static_cast<A>(L.sink);

  for (int idx = tid; idx < BM * D; idx += 256) {
    const int r = idx / D, c = idx - r * D;
    const int rl = r0 + r;
    Qs[r * LD + c] = rl < P.q.len ? static_cast<A>(to_acc(q[static_cast<long long>(P.q.row0 + rl) * D + c])) : A(0);
  }
  const int last = min(r0 + BM - 1, P.q.len - 1);
  const int qpos_first = P.q.pos0 + r0;

  using W = typename SumOf<T>::type;
  W o[TR][OC];
  W rs[TR];
#pragma unroll
  for (int i = 0; i < TR; ++i) {
    rs[i] = W(0);
#pragma unroll
    for (int j = 0; j < OC; ++j) o[i][j] = W(0);
  }

  for (int s = 0; s < P.nk; ++s) {
    const Segment ks = P.k[s];
    int nvis = ks.len;
    if (L.causal) nvis = min(nvis, P.q.pos0 + last - ks.pos0 + 1);
    const int ntile = nvis <= 0 ? 0 : (nvis + BN - 1) / BN;
    for (int jj = 0; jj < ntile; ++jj) {
      const int kbase = jj * BN;
      __syncthreads();
      for (int idx = tid; idx < BN * D; idx += 256) {
        const int r = idx / D, c = idx - r * D;
        const int key = kbase + r;
        const bool ok = key < ks.len;
        const long long off = static_cast<long long>(ks.row0 + key) * D + c;
        Ks[r * LD + c] = ok ? static_cast<A>(to_acc(k[off])) : A(0);
        Vs[r * LD + c] = ok ? static_cast<A>(to_acc(v[off])) : A(0);
      }
      __syncthreads();
      A sacc[TR][TC];
#pragma unroll
      for (int i = 0; i < TR; ++i)
#pragma unroll
        for (int j = 0; j < TC; ++j) sacc[i][j] = A(0);
      for (int d = 0; d < D; ++d) {
        A a[TR], b[TC];
#pragma unroll
        for (int i = 0; i < TR; ++i) a[i] = Qs[(ty + 16 * i) * LD + d];
#pragma unroll
        for (int j = 0; j < TC; ++j) b[j] = Ks[(tx + 16 * j) * LD + d];
#pragma unroll
        for (int i = 0; i < TR; ++i)
#pragma unroll
          for (int j = 0; j < TC; ++j) sacc[i][j] = fma(a[i], b[j], sacc[i][j]);
      }
      const int kpos0 = ks.pos0 + kbase;
      const bool need_mask = (kbase + BN > ks.len) || (L.causal && kpos0 + BN - 1 > qpos_first);
#pragma unroll
      for (int i = 0; i < TR; ++i) {
        const int qpos = P.q.pos0 + r0 + ty + 16 * i;
#pragma unroll
        for (int j = 0; j < TC; ++j) {
          const int c = tx + 16 * j;
          A p = octic_simt<A>(sacc[i][j] * scale);
          if (need_mask) {
            const bool vis = (kbase + c < ks.len) && (!L.causal || kpos0 + c <= qpos);
            p = vis ? p : A(0);
          }
          rs[i] += static_cast<W>(p);
          Ps[(ty + 16 * i) * PLD + c] = round_p<T, A>(p);
        }
      }
      __syncthreads();
#pragma unroll 4
      for (int kk = 0; kk < BN; ++kk) {
        W pv[TR];
#pragma unroll
        for (int i = 0; i < TR; ++i) pv[i] = static_cast<W>(Ps[(ty + 16 * i) * PLD + kk]);
#pragma unroll
        for (int j = 0; j < OC; ++j) {
          const int col = tx + 16 * j;
          if (col < D) {
            const W vv = static_cast<W>(Vs[kk * LD + col]);
#pragma unroll
            for (int i = 0; i < TR; ++i) o[i][j] = fma(pv[i], vv, o[i][j]);
          }
        }
      }
    }
  }

  // Row sums: the 16 threads of a half-warp share the same rows.
#pragma unroll
  for (int i = 0; i < TR; ++i)
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], off);

  const bool fin = L.mode == kFinal || L.mode == kAccumFinal;
  const bool add_prev = L.mode == kAccumRaw || L.mode == kAccumFinal;
#pragma unroll
  for (int i = 0; i < TR; ++i) {
    const int rl = r0 + ty + 16 * i;
    if (rl >= P.q.len) continue;
    const long long grow = static_cast<long long>(bh) * L.lq + P.q.row0 + rl;
    A* arow = static_cast<A*>(L.o_acc) + grow * D;
    const W drow = rs[i] + (add_prev ? static_cast<W>(static_cast<const A*>(L.d_acc)[grow]) : W(0));
    const W denom = drow + static_cast<W>(sink);
#pragma unroll
    for (int j = 0; j < OC; ++j) {
      const int col = tx + 16 * j;
      if (col >= D) continue;
      const W x = o[i][j] + (add_prev ? static_cast<W>(arow[col]) : W(0));
      if (fin)
        static_cast<T*>(L.out)[grow * D + col] = from_acc<T>(static_cast<A>(x / denom));
      else
        arow[col] = static_cast<A>(x);
    }
    if (tx == 0) {
      if (fin) {
        if (L.dtot) static_cast<A*>(L.dtot)[grow] = static_cast<A>(denom);
      } else {
        static_cast<A*>(L.d_acc)[grow] = static_cast<A>(drow);
      }
    }
  }
}

template <typename T, typename A, int BM, int BN, int DMAX>
cudaError_t launch_cfg(Launch L, cudaStream_t stream) {
  constexpr size_t smem = sizeof(A) * (static_cast<size_t>(BM + 2 * BN) * (DMAX + 1) + static_cast<size_t>(BM) * (BN + 1));
  auto kern = afa_simt_fwd_kernel<T, A, BM, BN, DMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int total = assign_ctas(L, BM);
  if (total == 0) return cudaSuccess;
  dim3 grid(L.B * L.H, total);
  kern<<<grid, 256, smem, stream>>>(L);
  return cudaGetLastError();
}

template <typename T, typename A>
cudaError_t launch_type(const Launch& L, cudaStream_t stream) {
  if constexpr (sizeof(A) == 8) {
    if (L.d <= 128) return launch_cfg<T, A, 32, 32, 128>(L, stream);
    return launch_cfg<T, A, 16, 16, 256>(L, stream);
  } else {
    if (L.d <= 64) return launch_cfg<T, A, 64, 64, 64>(L, stream);
    if (L.d <= 128) return launch_cfg<T, A, 64, 64, 128>(L, stream);
    return launch_cfg<T, A, 32, 32, 256>(L, stream);
  }
}

// Final normalisation of ring accumulators: out = o_acc / (d_acc + sink)
// (src/kernels/pallas_afa.py:661), d_total = d_acc + sink.
template <typename T, typename A>
__global__ void finalize_kernel(const A* o_acc, const A* d_acc, T* out, A* dtot, long long rows, int d, A sink) {
  const long long n = rows * d;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / d;
    const A den = d_acc[r] + sink;
    out[i] = from_acc<T>(o_acc[i] / den);
    if (dtot && i - r * d == 0) dtot[r] = den;
  }
}

}  // namespace

cudaError_t launch_simt_fwd(Launch L, int dtype, cudaStream_t stream, const char** detail) {
  if (L.d > 256) {
    *detail = "head_dim above 256 is not supported";
    return cudaErrorInvalidValue;
  }
  switch (dtype) {
    case kF32: return launch_type<float, float>(L, stream);
    case kBF16: return launch_type<__nv_bfloat16, float>(L, stream);
    case kF64: return launch_type<double, double>(L, stream);
    default: *detail = "unsupported dtype"; return cudaErrorInvalidValue;
  }
}

cudaError_t launch_finalize(const void* o_acc, const void* d_acc, void* out, void* dtot, long long rows, int d,
                            int dtype, double sink, cudaStream_t stream) {
  const long long n = rows * d;
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  const long long want = (n + threads - 1) / threads;
  const int blocks = static_cast<int>(want < 148 * 16 ? want : 148 * 16);
  switch (dtype) {
    case kF32:
      finalize_kernel<float, float><<<blocks, threads, 0, stream>>>(
          static_cast<const float*>(o_acc), static_cast<const float*>(d_acc), static_cast<float*>(out),
          static_cast<float*>(dtot), rows, d, static_cast<float>(sink));
      break;
    case kBF16:
      finalize_kernel<__nv_bfloat16, float><<<blocks, threads, 0, stream>>>(
          static_cast<const float*>(o_acc), static_cast<const float*>(d_acc), static_cast<__nv_bfloat16*>(out),
          static_cast<float*>(dtot), rows, d, static_cast<float>(sink));
      break;
    case kF64:
      finalize_kernel<double, double><<<blocks, threads, 0, stream>>>(
          static_cast<const double*>(o_acc), static_cast<const double*>(d_acc), static_cast<double*>(out),
          static_cast<double*>(dtot), rows, d, sink);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace afa
