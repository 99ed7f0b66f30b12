// AFA backward: gradients of sum(out * g_out) for out = AFA(q, k, v).
//
// Reference: tiled_afa_backward (src/kernels/pallas_afa.py:409-522), the
// analytical single-pass VJP of pallas_afa (:579-612):
//   E_i   = sum_d g_out[i,d] * out[i,d]                         (:459)
//   w_ij  = rho(s_ij)^8 / D_i, D_i = d_total (row sum + sink)   (:475-499)
//   g_ij  = g_out_i . v_j                                       (:500)
//   ds_ij = 8 * scale * r_ij * w_ij * (g_ij - E_i), r = rsqrt(1 + s^2)   (:502)
//   dq = ds k, dk = ds^T q, dv = w^T g_out                      (:507-510)
// with the forward's masks. For bf16 inputs w and ds are rounded to bf16
// before the three products (the reference casts both matmul operands to the
// input dtype, :440-448); float32 and float64 stay at full precision.
//
// bf16 with head_dim 64 or 128 runs on the tensor cores (afa_bwd_tc.cu); this
// file holds the CUDA-core path (every dtype and head dimension up to 256),
// the row-dot kernel both paths use, and the C ABI. Two kernels, no
// atomics: a query-parallel kernel recomputes S and g = g_out v^T for its rows
// against every visible key tile and accumulates dq; a key-parallel kernel
// recomputes them for its keys against every query tile that sees them and
// accumulates dk and dv. E comes from a row-dot kernel into the caller's
// workspace. Thread layout as the forward (afa_simt.cu): 16x16 threads, thread
// (ty, tx) owns rows ty+16i and columns tx+16j, shared-memory row pitch DMAX+1.
#include <cmath>
#include <cstdio>

#include "afa_b200.h"
#include "afa_common.cuh"
#include "afa_internal.h"

namespace afa {
namespace {

struct BwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* g;     // g_out (B, H, L, D)
  const void* out;   // forward output (B, H, L, D)
  const void* dtot;  // forward d_total (B, H, L), accumulation dtype
  void* e;           // E (B, H, L), accumulation dtype (workspace)
  void* dq;
  void* dk;
  void* dv;
  int L, D, causal, valid;
  long long rows;    // B * H * L
  float scale;
  double scale_d;
};

template <typename A>
__device__ __forceinline__ A inv_sqrt(A x) {
  if constexpr (sizeof(A) == 8) {
    return 1.0 / sqrt(x);
  } else {
    return rsqrtf(x);
  }
}

template <typename T, typename A>
__device__ __forceinline__ A round_operand(A x) {
  if constexpr (sizeof(A) == 8) {
    return x;
  } else {
    return round_like<T>(x);
  }
}

// E_i = sum_d g_out[i,d] * out[i,d], one warp per row.
template <typename T, typename A>
__global__ void __launch_bounds__(256) bwd_rowdot_kernel(const __grid_constant__ BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < a.rows; r += nwarps) {
    const T* g = static_cast<const T*>(a.g) + r * a.D;
    const T* o = static_cast<const T*>(a.out) + r * a.D;
    A s = A(0);
    for (int c = lane; c < a.D; c += 32) s += static_cast<A>(to_acc(g[c])) * static_cast<A>(to_acc(o[c]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) static_cast<A*>(a.e)[r] = s;
  }
}

// The weight and score gradient of one visible (query, key) pair.
template <typename A>
__device__ __forceinline__ void pair_grad(A sacc, A gacc, A scale, A inv_d, A e, A& w, A& ds) {
  const A s = sacc * scale;
  w = octic_ref(s) * inv_d;
  const A r = inv_sqrt<A>(A(1) + s * s);
  ds = A(8) * scale * r * w * (gacc - e);
}

// dq for BM query rows of one (b, h).
template <typename T, typename A, int BM, int BN, int DMAX>
__global__ void __launch_bounds__(256) bwd_dq_simt_kernel(const __grid_constant__ BwdArgs a) {
  constexpr int LD = DMAX + 1, DLD = BN + 1, TR = BM / 16, TC = BN / 16, OC = DMAX / 16;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  A* Qs = reinterpret_cast<A*>(smem_raw);
  A* Gs = Qs + BM * LD;
  A* Ks = Gs + BM * LD;
  A* Vs = Ks + BN * LD;
  A* Ds = Vs + BN * LD;

  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int bh = blockIdx.x;
  const int r0 = (gridDim.y - 1 - blockIdx.y) * BM;  // rows with the most causal keys first
  const int D = a.D, L = a.L;
  const long long base = static_cast<long long>(bh) * L;
  const T* q = static_cast<const T*>(a.q) + base * D;
  const T* g = static_cast<const T*>(a.g) + base * D;
  const T* k = static_cast<const T*>(a.k) + base * D;
  const T* v = static_cast<const T*>(a.v) + base * D;
  const A scale = sizeof(A) == 8 ? static_cast<A>(a.scale_d) : static_cast<A>(a.scale);

  for (int idx = tid; idx < BM * D; idx += 256) {
    const int r = idx / D, c = idx - r * D;
    const bool ok = r0 + r < L;
    const long long off = static_cast<long long>(r0 + r) * D + c;
    Qs[r * LD + c] = ok ? static_cast<A>(to_acc(q[off])) : A(0);
    Gs[r * LD + c] = ok ? static_cast<A>(to_acc(g[off])) : A(0);
  }
  A inv_d[TR], e[TR];
#pragma unroll
  for (int i = 0; i < TR; ++i) {
    const int row = r0 + ty + 16 * i;
    inv_d[i] = row < L ? A(1) / static_cast<const A*>(a.dtot)[base + row] : A(0);
    e[i] = row < L ? static_cast<const A*>(a.e)[base + row] : A(0);
  }
  A acc[TR][OC];
#pragma unroll
  for (int i = 0; i < TR; ++i)
#pragma unroll
    for (int j = 0; j < OC; ++j) acc[i][j] = A(0);

  int kend = a.valid;
  if (a.causal) kend = min(kend, r0 + BM);
  const int ntile = kend <= 0 ? 0 : (kend + BN - 1) / BN;
  for (int jt = 0; jt < ntile; ++jt) {
    const int kbase = jt * BN;
    __syncthreads();
    for (int idx = tid; idx < BN * D; idx += 256) {
      const int r = idx / D, c = idx - r * D;
      const bool ok = kbase + r < L;
      const long long off = static_cast<long long>(kbase + r) * D + c;
      Ks[r * LD + c] = ok ? static_cast<A>(to_acc(k[off])) : A(0);
      Vs[r * LD + c] = ok ? static_cast<A>(to_acc(v[off])) : A(0);
    }
    __syncthreads();
    A sacc[TR][TC], gacc[TR][TC];
#pragma unroll
    for (int i = 0; i < TR; ++i)
#pragma unroll
      for (int j = 0; j < TC; ++j) sacc[i][j] = gacc[i][j] = A(0);
    for (int d = 0; d < D; ++d) {
      A aq[TR], ag[TR], bk[TC], bv[TC];
#pragma unroll
      for (int i = 0; i < TR; ++i) {
        aq[i] = Qs[(ty + 16 * i) * LD + d];
        ag[i] = Gs[(ty + 16 * i) * LD + d];
      }
#pragma unroll
      for (int j = 0; j < TC; ++j) {
        bk[j] = Ks[(tx + 16 * j) * LD + d];
        bv[j] = Vs[(tx + 16 * j) * LD + d];
      }
#pragma unroll
      for (int i = 0; i < TR; ++i)
#pragma unroll
        for (int j = 0; j < TC; ++j) {
          sacc[i][j] = fma(aq[i], bk[j], sacc[i][j]);
          gacc[i][j] = fma(ag[i], bv[j], gacc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < TR; ++i) {
      const int row = r0 + ty + 16 * i;
#pragma unroll
      for (int j = 0; j < TC; ++j) {
        const int key = kbase + tx + 16 * j;
        const bool vis = key < a.valid && row < L && (!a.causal || key <= row);
        A w = A(0), ds = A(0);
        if (vis) pair_grad<A>(sacc[i][j], gacc[i][j], scale, inv_d[i], e[i], w, ds);
        Ds[(ty + 16 * i) * DLD + tx + 16 * j] = round_operand<T, A>(ds);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < BN; ++kk) {
      A dsr[TR];
#pragma unroll
      for (int i = 0; i < TR; ++i) dsr[i] = Ds[(ty + 16 * i) * DLD + kk];
#pragma unroll
      for (int j = 0; j < OC; ++j) {
        const int col = tx + 16 * j;
        if (col < D) {
          const A kv = Ks[kk * LD + col];
#pragma unroll
          for (int i = 0; i < TR; ++i) acc[i][j] = fma(dsr[i], kv, acc[i][j]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < TR; ++i) {
    const int row = r0 + ty + 16 * i;
    if (row >= L) continue;
#pragma unroll
    for (int j = 0; j < OC; ++j) {
      const int col = tx + 16 * j;
      if (col < D) static_cast<T*>(a.dq)[(base + row) * D + col] = from_acc<T>(acc[i][j]);
    }
  }
}

// dk and dv for BN keys of one (b, h).
template <typename T, typename A, int BM, int BN, int DMAX>
__global__ void __launch_bounds__(256) bwd_dkv_simt_kernel(const __grid_constant__ BwdArgs a) {
  constexpr int LD = DMAX + 1, WLD = BM + 1, TR = BN / 16, TC = BM / 16, OC = DMAX / 16;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  A* Ks = reinterpret_cast<A*>(smem_raw);
  A* Vs = Ks + BN * LD;
  A* Qs = Vs + BN * LD;
  A* Gs = Qs + BM * LD;
  A* Wt = Gs + BM * LD;
  A* Dt = Wt + BN * WLD;
  A* Is = Dt + BN * WLD;
  A* Es = Is + BM;

  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int bh = blockIdx.x;
  const int k0 = blockIdx.y * BN;  // keys with the most causal queries first
  const int D = a.D, L = a.L;
  const long long base = static_cast<long long>(bh) * L;
  const T* q = static_cast<const T*>(a.q) + base * D;
  const T* g = static_cast<const T*>(a.g) + base * D;
  const T* k = static_cast<const T*>(a.k) + base * D;
  const T* v = static_cast<const T*>(a.v) + base * D;
  const A scale = sizeof(A) == 8 ? static_cast<A>(a.scale_d) : static_cast<A>(a.scale);

  for (int idx = tid; idx < BN * D; idx += 256) {
    const int r = idx / D, c = idx - r * D;
    const bool ok = k0 + r < L;
    const long long off = static_cast<long long>(k0 + r) * D + c;
    Ks[r * LD + c] = ok ? static_cast<A>(to_acc(k[off])) : A(0);
    Vs[r * LD + c] = ok ? static_cast<A>(to_acc(v[off])) : A(0);
  }
  A dk[TR][OC], dv[TR][OC];
#pragma unroll
  for (int i = 0; i < TR; ++i)
#pragma unroll
    for (int j = 0; j < OC; ++j) dk[i][j] = dv[i][j] = A(0);

  // Keys at index >= valid_len get no weight from any query.
  const int qfirst = a.causal ? (k0 / BM) * BM : 0;
  const int ntile = k0 >= a.valid ? 0 : (L - qfirst + BM - 1) / BM;
  for (int it = 0; it < ntile; ++it) {
    const int q0 = qfirst + it * BM;
    __syncthreads();
    for (int idx = tid; idx < BM * D; idx += 256) {
      const int r = idx / D, c = idx - r * D;
      const bool ok = q0 + r < L;
      const long long off = static_cast<long long>(q0 + r) * D + c;
      Qs[r * LD + c] = ok ? static_cast<A>(to_acc(q[off])) : A(0);
      Gs[r * LD + c] = ok ? static_cast<A>(to_acc(g[off])) : A(0);
    }
    for (int r = tid; r < BM; r += 256) {
      const bool ok = q0 + r < L;
      Is[r] = ok ? A(1) / static_cast<const A*>(a.dtot)[base + q0 + r] : A(0);
      Es[r] = ok ? static_cast<const A*>(a.e)[base + q0 + r] : A(0);
    }
    __syncthreads();
    A sacc[TR][TC], gacc[TR][TC];
#pragma unroll
    for (int i = 0; i < TR; ++i)
#pragma unroll
      for (int j = 0; j < TC; ++j) sacc[i][j] = gacc[i][j] = A(0);
    for (int d = 0; d < D; ++d) {
      A ak[TR], av[TR], bq[TC], bg[TC];
#pragma unroll
      for (int i = 0; i < TR; ++i) {
        ak[i] = Ks[(ty + 16 * i) * LD + d];
        av[i] = Vs[(ty + 16 * i) * LD + d];
      }
#pragma unroll
      for (int j = 0; j < TC; ++j) {
        bq[j] = Qs[(tx + 16 * j) * LD + d];
        bg[j] = Gs[(tx + 16 * j) * LD + d];
      }
#pragma unroll
      for (int i = 0; i < TR; ++i)
#pragma unroll
        for (int j = 0; j < TC; ++j) {
          sacc[i][j] = fma(ak[i], bq[j], sacc[i][j]);
          gacc[i][j] = fma(av[i], bg[j], gacc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < TR; ++i) {
      const int key = k0 + ty + 16 * i;
#pragma unroll
      for (int j = 0; j < TC; ++j) {
        const int qc = tx + 16 * j;
        const int row = q0 + qc;
        const bool vis = key < a.valid && row < L && (!a.causal || key <= row);
        A w = A(0), ds = A(0);
        if (vis) pair_grad<A>(sacc[i][j], gacc[i][j], scale, Is[qc], Es[qc], w, ds);
        Wt[(ty + 16 * i) * WLD + qc] = round_operand<T, A>(w);
        Dt[(ty + 16 * i) * WLD + qc] = round_operand<T, A>(ds);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int qq = 0; qq < BM; ++qq) {
      A wr[TR], dr[TR];
#pragma unroll
      for (int i = 0; i < TR; ++i) {
        wr[i] = Wt[(ty + 16 * i) * WLD + qq];
        dr[i] = Dt[(ty + 16 * i) * WLD + qq];
      }
#pragma unroll
      for (int j = 0; j < OC; ++j) {
        const int col = tx + 16 * j;
        if (col < D) {
          const A gv = Gs[qq * LD + col];
          const A qv = Qs[qq * LD + col];
#pragma unroll
          for (int i = 0; i < TR; ++i) {
            dv[i][j] = fma(wr[i], gv, dv[i][j]);
            dk[i][j] = fma(dr[i], qv, dk[i][j]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < TR; ++i) {
    const int key = k0 + ty + 16 * i;
    if (key >= L) continue;
#pragma unroll
    for (int j = 0; j < OC; ++j) {
      const int col = tx + 16 * j;
      if (col < D) {
        static_cast<T*>(a.dk)[(base + key) * D + col] = from_acc<T>(dk[i][j]);
        static_cast<T*>(a.dv)[(base + key) * D + col] = from_acc<T>(dv[i][j]);
      }
    }
  }
}

template <typename T, typename A, int BM, int BN, int DMAX>
cudaError_t launch_bwd_cfg(const BwdArgs& a, int bh, cudaStream_t stream) {
  constexpr size_t dq_smem = sizeof(A) * (static_cast<size_t>(2 * BM + 2 * BN) * (DMAX + 1) +
                                          static_cast<size_t>(BM) * (BN + 1));
  constexpr size_t dkv_smem = sizeof(A) * (static_cast<size_t>(2 * BM + 2 * BN) * (DMAX + 1) +
                                           2 * static_cast<size_t>(BN) * (BM + 1) + 2 * BM);
  auto kdq = bwd_dq_simt_kernel<T, A, BM, BN, DMAX>;
  auto kdkv = bwd_dkv_simt_kernel<T, A, BM, BN, DMAX>;
  cudaError_t e = cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dq_smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kdkv, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dkv_smem));
  if (e != cudaSuccess) return e;
  kdq<<<dim3(bh, (a.L + BM - 1) / BM), 256, dq_smem, stream>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  kdkv<<<dim3(bh, (a.L + BN - 1) / BN), 256, dkv_smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename T, typename A>
cudaError_t launch_rowdot(const BwdArgs& a, cudaStream_t stream) {
  long long blocks = (a.rows * 32 + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  bwd_rowdot_kernel<T, A><<<static_cast<int>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

template <typename T, typename A>
cudaError_t launch_bwd_typed(const BwdArgs& a, int bh, cudaStream_t stream) {
  if (cudaError_t e = launch_rowdot<T, A>(a, stream); e != cudaSuccess) return e;
  if constexpr (sizeof(A) == 8) {
    if (a.D <= 128) return launch_bwd_cfg<T, A, 32, 32, 128>(a, bh, stream);
    return launch_bwd_cfg<T, A, 16, 16, 256>(a, bh, stream);
  } else {
    if (a.D <= 64) return launch_bwd_cfg<T, A, 64, 64, 64>(a, bh, stream);
    if (a.D <= 128) return launch_bwd_cfg<T, A, 32, 32, 128>(a, bh, stream);
    return launch_bwd_cfg<T, A, 32, 32, 256>(a, bh, stream);
  }
}

size_t acc_size(int dtype) { return dtype == kF64 ? 8 : 4; }

}  // namespace
}  // namespace afa

extern "C" size_t afa_bwd_workspace_bytes(int B, int H, int L, int D, int dtype) {
  (void)D;
  if (B <= 0 || H <= 0 || L <= 0) return 0;
  return static_cast<size_t>(B) * H * L * afa::acc_size(dtype);
}

extern "C" int afa_bwd(const void* q, const void* k, const void* v, const void* out, const void* d_total,
                       const void* g_out, void* dq, void* dk, void* dv, int B, int H, int L, int D, int dtype,
                       float sink_omega, int causal, int valid_len, void* workspace, size_t workspace_bytes,
                       void* stream) {
  using namespace afa;
  if (dtype == AFA_F16)
    return set_last_error(AFA_ERR_DTYPE, "float16 is not supported (the forward rejects it); use bfloat16 or float32");
  if (dtype != AFA_F32 && dtype != AFA_BF16 && dtype != AFA_F64)
    return set_last_error(AFA_ERR_DTYPE, "afa_bwd: unsupported dtype code");
  if (!q || !k || !v || !out || !d_total || !g_out || !dq || !dk || !dv)
    return set_last_error(AFA_ERR_INVALID, "afa_bwd: q, k, v, out, d_total, g_out, dq, dk and dv must be non-null");
  if (B <= 0 || H <= 0 || L <= 0) return set_last_error(AFA_ERR_INVALID, "batch, heads and sequence must be positive");
  if (D <= 0 || D > 256) return set_last_error(AFA_ERR_INVALID, "afa_bwd: head dimension must be in [1, 256]");
  if (valid_len < 0 || valid_len > L) return set_last_error(AFA_ERR_INVALID, "valid_seq_len must be in [1, seq_len]");
  if (!(sink_omega >= 0.0f) || !std::isfinite(sink_omega))
    return set_last_error(AFA_ERR_INVALID, "sink_omega must be finite and nonnegative");
  const size_t need = afa_bwd_workspace_bytes(B, H, L, D, dtype);
  if (!workspace || workspace_bytes < need) {
    char msg[160];
    snprintf(msg, sizeof(msg), "afa_bwd: workspace of %zu bytes needed (afa_bwd_workspace_bytes), got %zu", need,
             workspace ? workspace_bytes : static_cast<size_t>(0));
    return set_last_error(AFA_ERR_INVALID, msg);
  }
  BwdArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.g = g_out;
  a.out = out;
  a.dtot = d_total;
  a.e = workspace;
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.L = L;
  a.D = D;
  a.causal = causal ? 1 : 0;
  a.valid = valid_len > 0 ? valid_len : L;
  a.rows = static_cast<long long>(B) * H * L;
  a.scale_d = 1.0 / std::sqrt(static_cast<double>(D));
  a.scale = static_cast<float>(a.scale_d);
  const int bh = B * H;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (tc_bwd_supported(dtype, D)) {
    // Tensor cores: E first, then the key-parallel dK/dV and query-parallel dQ kernels.
    int* status = device_status_ptr();
    if (!status) return set_last_error(AFA_ERR_CUDA, "afa_bwd: could not resolve the device status word");
    const char* detail = nullptr;
    e = launch_rowdot<__nv_bfloat16, float>(a, s);
    if (e == cudaSuccess)
      e = launch_tc_bwd(q, k, v, g_out, static_cast<const float*>(d_total), static_cast<const float*>(workspace), dq,
                        dk, dv, B, H, L, D, a.causal, a.valid, a.scale, sink_omega, status, s, &detail);
    if (e != cudaSuccess) {
      char msg[256];
      snprintf(msg, sizeof(msg), "afa_bwd tensor-core launch: %s%s%s", cudaGetErrorString(e), detail ? " -- " : "",
               detail ? detail : "");
      return set_last_error(AFA_ERR_CUDA, msg);
    }
    return AFA_OK;
  }
  if (dtype == AFA_F64)
    e = launch_bwd_typed<double, double>(a, bh, s);
  else if (dtype == AFA_F32)
    e = launch_bwd_typed<float, float>(a, bh, s);
  else
    e = launch_bwd_typed<__nv_bfloat16, float>(a, bh, s);
  if (e != cudaSuccess) {
    char msg[200];
    snprintf(msg, sizeof(msg), "afa_bwd kernel launch: %s", cudaGetErrorString(e));
    return set_last_error(AFA_ERR_CUDA, msg);
  }
  return AFA_OK;
}
