// C ABI of libafa_b200.so (declared in include/afa_b200.h): argument checks,
// dispatch to the kernels, error reporting.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "afa_b200.h"
#include "afa_common.cuh"
#include "afa_internal.h"

// One status word per device: kernels record where a bounded wait ran out.
__device__ int g_afa_device_status;

namespace {

// Failure-detection self-test: one thread waits on an mbarrier that nothing
// ever arrives at. The bounded wait must give up after `budget_ns`, record
// kDevTimeoutSelftest in the status word and return, leaving the context usable.
__global__ void selftest_wait_kernel(int* status, unsigned long long budget_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    afa::mbar_init(&bar, 1);
    afa::fence_barrier_init();
    (void)afa::mbar_wait(&bar, 0, status, afa::kDevTimeoutSelftest, budget_ns);
  }
}

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what, const char* detail = nullptr) {
  return fail(AFA_ERR_CUDA, "%s: %s%s%s", what, cudaGetErrorString(e), detail ? " -- " : "", detail ? detail : "");
}

int* status_ptr() {
  static afa::PerDeviceOnce setup;
  static int* ptrs[afa::kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  const cudaError_t e = setup.run(dev, [&] {
    void* p = nullptr;
    const cudaError_t r = cudaGetSymbolAddress(&p, g_afa_device_status);
    ptrs[dev] = static_cast<int*>(p);
    return r;
  });
  return e == cudaSuccess ? ptrs[dev] : nullptr;
}

bool finite_nonneg(double x) { return std::isfinite(x) && x >= 0.0; }

int check_attn_dtype(int dtype) {
  if (dtype == AFA_F16)
    return fail(AFA_ERR_DTYPE,
                "float16 is not supported: P is cast to the value dtype before P.V "
                "(pallas_afa.py:133) and rho(s)^8 overflows float16 for s > 2.4; use bfloat16 or float32");
  if (dtype != AFA_F32 && dtype != AFA_BF16 && dtype != AFA_F64)
    return fail(AFA_ERR_DTYPE, "unsupported dtype code %d", dtype);
  return AFA_OK;
}

afa::Launch base_launch(int B, int H, int lq, int lk, int D, int dtype, float sink, int causal) {
  afa::Launch L{};
  L.B = B;
  L.H = H;
  L.lq = lq;
  L.lk = lk;
  L.d = D;
  L.causal = causal ? 1 : 0;
  L.scale_d = 1.0 / std::sqrt(static_cast<double>(D));
  L.scale = static_cast<float>(L.scale_d);
  L.sink = sink;
  L.sink_d = static_cast<double>(sink);
  (void)dtype;
  return L;
}

int run_launch(afa::Launch& L, int dtype, cudaStream_t stream) {
  L.status = status_ptr();
  if (!L.status) return fail(AFA_ERR_CUDA, "could not resolve the device status word");
  const char* detail = nullptr;
  cudaError_t e;
  if (afa::tc_fwd_supported(dtype, L.d))
    e = afa::launch_tc_fwd(L, dtype, stream, &detail);
  else
    e = afa::launch_simt_fwd(L, dtype, stream, &detail);
  if (e != cudaSuccess) return cuda_fail(e, "AFA kernel launch", detail);
  return AFA_OK;
}

}  // namespace

namespace afa {
int set_last_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}
int* device_status_ptr() { return status_ptr(); }
}  // namespace afa

extern "C" {

const char* afa_version(void) { return "afa_b200 0.1.0 sm_100a"; }

const char* afa_last_error(void) { return g_last_error.c_str(); }

int afa_fwd(const void* q, const void* k, const void* v, void* out, void* d_total, int B, int H, int L, int D,
            int dtype, float sink_omega, int causal, int valid_len, void* stream) {
  if (int rc = check_attn_dtype(dtype)) return rc;
  if (!q || !k || !v || !out) return fail(AFA_ERR_INVALID, "q, k, v and out must be non-null device pointers");
  if (B <= 0 || H <= 0 || L <= 0) return fail(AFA_ERR_INVALID, "batch, heads and sequence must be positive");
  if (D <= 0) return fail(AFA_ERR_INVALID, "head dimension must be positive");
  if (D > 256) return fail(AFA_ERR_INVALID, "head dimension above 256 is not supported");
  if (!finite_nonneg(sink_omega)) return fail(AFA_ERR_INVALID, "sink_omega must be finite and nonnegative");
  if (valid_len < 0 || valid_len > L) return fail(AFA_ERR_INVALID, "valid_seq_len must be in [1, seq_len]");
  afa::Launch Lc = base_launch(B, H, L, L, D, dtype, sink_omega, causal);
  Lc.nprob = 1;
  Lc.prob[0].q = {0, L, 0};
  Lc.prob[0].k[0] = {0, valid_len > 0 ? valid_len : L, 0};
  Lc.prob[0].nk = 1;
  Lc.mode = afa::kFinal;
  Lc.q = q;
  Lc.k = k;
  Lc.v = v;
  Lc.out = out;
  Lc.dtot = d_total;
  return run_launch(Lc, dtype, static_cast<cudaStream_t>(stream));
}

int afa_fwd_hop(const void* q, const void* k, const void* v, void* o_acc, void* d_acc, void* out, void* d_total,
                int B, int H, int Lq, int Lk, int D, int dtype, const int* problems, int nproblems, int causal,
                int mode, float sink_omega, void* stream) {
  if (int rc = check_attn_dtype(dtype)) return rc;
  if (!q || !k || !v || !problems) return fail(AFA_ERR_INVALID, "q, k, v and problems must be non-null");
  if (mode < AFA_HOP_STORE || mode > AFA_HOP_ONLY) return fail(AFA_ERR_INVALID, "unknown hop mode %d", mode);
  if (mode != AFA_HOP_ONLY && (!o_acc || !d_acc))
    return fail(AFA_ERR_INVALID, "o_acc and d_acc must be non-null for this hop mode");
  if ((mode == AFA_HOP_FINALIZE || mode == AFA_HOP_ONLY) && !out)
    return fail(AFA_ERR_INVALID, "out must be non-null for this hop mode");
  if (!finite_nonneg(sink_omega)) return fail(AFA_ERR_INVALID, "sink_omega must be finite and nonnegative");
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0 || D <= 0 || D > 256)
    return fail(AFA_ERR_INVALID, "invalid shape B=%d H=%d Lq=%d Lk=%d D=%d", B, H, Lq, Lk, D);
  if (nproblems < 1 || nproblems > afa::kMaxProblems)
    return fail(AFA_ERR_INVALID, "nproblems must be in [1, %d]", afa::kMaxProblems);
  afa::Launch Lc = base_launch(B, H, Lq, Lk, D, dtype, sink_omega, causal);
  Lc.nprob = nproblems;
  for (int i = 0; i < nproblems; ++i) {
    const int* p = problems + 10 * i;
    afa::Problem& P = Lc.prob[i];
    P.q = {p[0], p[1], p[2]};
    P.nk = p[3];
    P.k[0] = {p[4], p[5], p[6]};
    P.k[1] = {p[7], p[8], p[9]};
    if (P.nk < 1 || P.nk > 2) return fail(AFA_ERR_INVALID, "problem %d: nk must be 1 or 2", i);
    if (P.q.row0 < 0 || P.q.len <= 0 || P.q.row0 + P.q.len > Lq)
      return fail(AFA_ERR_INVALID, "problem %d: query rows out of range", i);
    for (int s = 0; s < P.nk; ++s)
      if (P.k[s].row0 < 0 || P.k[s].len <= 0 || P.k[s].row0 + P.k[s].len > Lk)
        return fail(AFA_ERR_INVALID, "problem %d: key segment %d out of range", i, s);
    if (P.nk == 1) P.k[1] = {0, 0, 0};
    if (causal && P.nk == 2 && P.k[0].pos0 + P.k[0].len - 1 > P.q.pos0)
      return fail(AFA_ERR_INVALID,
                  "problem %d: with causal masking the first key segment must be visible to every query row", i);
  }
  static const int kModeMap[4] = {afa::kStoreRaw, afa::kAccumRaw, afa::kAccumFinal, afa::kFinal};
  Lc.mode = kModeMap[mode];
  // Query rows shared by two problems only add up where the launch adds its
  // pieces with reductions (merged accumulate hops on the tensor cores).
  if (!afa::tc_accum_reduces(Lc, dtype)) {
    for (int i = 0; i < nproblems; ++i)
      for (int j = 0; j < i; ++j) {
        const afa::Segment& a = Lc.prob[j].q;
        const afa::Segment& b = Lc.prob[i].q;
        if (a.row0 < b.row0 + b.len && b.row0 < a.row0 + a.len)
          return fail(AFA_ERR_INVALID, "problems %d and %d write overlapping query rows", j, i);
      }
  }
  Lc.q = q;
  Lc.k = k;
  Lc.v = v;
  Lc.o_acc = o_acc;
  Lc.d_acc = d_acc;
  Lc.out = out;
  Lc.dtot = d_total;
  return run_launch(Lc, dtype, static_cast<cudaStream_t>(stream));
}

int afa_finalize(const void* o_acc, const void* d_acc, void* out, void* d_total, long long rows, int D, int dtype,
                 float sink_omega, void* stream) {
  if (int rc = check_attn_dtype(dtype)) return rc;
  if (!o_acc || !d_acc || !out) return fail(AFA_ERR_INVALID, "o_acc, d_acc and out must be non-null");
  if (rows < 0 || D <= 0) return fail(AFA_ERR_INVALID, "invalid shape");
  if (!finite_nonneg(sink_omega)) return fail(AFA_ERR_INVALID, "sink_omega must be finite and nonnegative");
  cudaError_t e = afa::launch_finalize(o_acc, d_acc, out, d_total, rows, D, dtype, sink_omega,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "afa_finalize launch");
  return AFA_OK;
}

size_t afa_decode_workspace_bytes(int B, int H, int Lkv, int D) {
  if (B <= 0 || H <= 0 || Lkv <= 0 || D <= 0) return 0;
  const int bh = B * H;
  const int ns = afa::decode_splits(bh, Lkv);
  if (ns <= 1) return 0;
  return static_cast<size_t>(bh) * ns * (static_cast<size_t>(D) + 1) * sizeof(float);
}

int afa_decode(const void* q, const void* k_cache, const void* v_cache, void* out, void* d_total, int B, int H,
               int Lkv, int D, int dtype, float sink_omega, const int* kv_lens, int kv_len, void* workspace,
               size_t workspace_bytes, void* stream) {
  if (int rc = check_attn_dtype(dtype)) return rc;
  if (!q || !k_cache || !v_cache || !out) return fail(AFA_ERR_INVALID, "q, caches and out must be non-null");
  if (B <= 0 || H <= 0 || Lkv <= 0 || D <= 0 || D > 256)
    return fail(AFA_ERR_INVALID, "invalid shape B=%d H=%d Lkv=%d D=%d", B, H, Lkv, D);
  if (!finite_nonneg(sink_omega)) return fail(AFA_ERR_INVALID, "sink_omega must be finite and nonnegative");
  if (kv_len < 0 || kv_len > Lkv) return fail(AFA_ERR_INVALID, "kv_len must be in [0, Lkv]");
  const int len = kv_len > 0 ? kv_len : Lkv;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (afa::decode_fast_supported(dtype, D)) {
    const int bh = B * H;
    const int ns = afa::decode_splits(bh, Lkv);
    const size_t need = afa_decode_workspace_bytes(B, H, Lkv, D);
    if (need > 0 && (!workspace || workspace_bytes < need))
      return fail(AFA_ERR_INVALID, "decode needs a workspace of %zu bytes (got %zu)", need, workspace_bytes);
    float* ws_o = static_cast<float*>(workspace);
    float* ws_d = ws_o ? ws_o + static_cast<size_t>(bh) * ns * D : nullptr;
    cudaError_t e = afa::launch_decode(q, k_cache, v_cache, out, d_total, B, H, Lkv, D, dtype, sink_omega, kv_lens,
                                       len, ws_o, ws_d, ns, status_ptr(), st);
    if (e != cudaSuccess) return cuda_fail(e, "afa_decode launch");
    return AFA_OK;
  }
  if (kv_lens) return fail(AFA_ERR_INVALID, "per-batch kv_lens needs bf16 (D 64/128/256) or f32 (D 64/128)");
  // General shapes: the forward kernel with one query row per (batch, head).
  afa::Launch Lc = base_launch(B, H, 1, Lkv, D, dtype, sink_omega, 0);
  Lc.nprob = 1;
  Lc.prob[0].q = {0, 1, 0};
  Lc.prob[0].k[0] = {0, len, 0};
  Lc.prob[0].nk = 1;
  Lc.mode = afa::kFinal;
  Lc.q = q;
  Lc.k = k_cache;
  Lc.v = v_cache;
  Lc.out = out;
  Lc.dtot = d_total;
  Lc.status = status_ptr();
  const char* detail = nullptr;
  cudaError_t e = afa::launch_simt_fwd(Lc, dtype, st, &detail);
  if (e != cudaSuccess) return cuda_fail(e, "afa_decode launch", detail);
  return AFA_OK;
}

int algebraic_softmax_fwd(const void* x, void* y, long long rows, int cols, int dtype, double sink_omega,
                          double eps, void* stream) {
  if (!(std::isfinite(sink_omega) && sink_omega >= 0.0))
    return fail(AFA_ERR_INVALID, "sink_omega must be finite and nonnegative");
  if (!(std::isfinite(eps) && eps > 0.0)) return fail(AFA_ERR_INVALID, "eps must be finite and positive");
  if (dtype != AFA_F32 && dtype != AFA_BF16 && dtype != AFA_F16 && dtype != AFA_F64)
    return fail(AFA_ERR_DTYPE, "expected a floating point array");
  if (cols <= 0 || rows < 0) return fail(AFA_ERR_INVALID, "AVN needs a nonempty feature axis");
  if (rows > 0 && (!x || !y)) return fail(AFA_ERR_INVALID, "x and y must be non-null device pointers");
  cudaError_t e = afa::launch_softmax(x, y, rows, cols, dtype, sink_omega, eps, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "algebraic_softmax launch");
  return AFA_OK;
}

int algebraic_softmax_bwd(const void* x, const void* g, void* dx, long long rows, int cols, int dtype,
                          double sink_omega, double eps, void* stream) {
  if (!(std::isfinite(sink_omega) && sink_omega >= 0.0))
    return fail(AFA_ERR_INVALID, "sink_omega must be finite and nonnegative");
  if (!(std::isfinite(eps) && eps > 0.0)) return fail(AFA_ERR_INVALID, "eps must be finite and positive");
  if (dtype != AFA_F32 && dtype != AFA_BF16 && dtype != AFA_F16 && dtype != AFA_F64)
    return fail(AFA_ERR_DTYPE, "expected a floating point array");
  if (cols <= 0 || rows < 0) return fail(AFA_ERR_INVALID, "AVN needs a nonempty feature axis");
  if (rows > 0 && (!x || !g || !dx)) return fail(AFA_ERR_INVALID, "x, g and dx must be non-null device pointers");
  cudaError_t e = afa::launch_softmax_bwd(x, g, dx, rows, cols, dtype, sink_omega, eps,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "algebraic_softmax backward launch");
  return AFA_OK;
}

int afa_octic_bwd(const void* x, const void* g, void* dx, long long n, int dtype, void* stream) {
  if (dtype != AFA_F32 && dtype != AFA_BF16 && dtype != AFA_F16 && dtype != AFA_F64)
    return fail(AFA_ERR_DTYPE, "expected a floating point array");
  if (n < 0) return fail(AFA_ERR_INVALID, "negative element count");
  if (n > 0 && (!x || !g || !dx)) return fail(AFA_ERR_INVALID, "x, g and dx must be non-null device pointers");
  cudaError_t e = afa::launch_octic_bwd(x, g, dx, n, dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "afa_octic_bwd launch");
  return AFA_OK;
}

int afa_octic(const void* x, void* y, long long n, int dtype, void* stream) {
  if (dtype != AFA_F32 && dtype != AFA_BF16 && dtype != AFA_F16 && dtype != AFA_F64)
    return fail(AFA_ERR_DTYPE, "expected a floating point array");
  if (n < 0) return fail(AFA_ERR_INVALID, "negative element count");
  if (n > 0 && (!x || !y)) return fail(AFA_ERR_INVALID, "x and y must be non-null device pointers");
  cudaError_t e = afa::launch_octic(x, y, n, dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "afa_octic launch");
  return AFA_OK;
}

int afa_selftest_bounded_wait(long long budget_ns, void* stream) {
  if (budget_ns <= 0 || budget_ns > 2000000000LL)
    return fail(AFA_ERR_INVALID, "budget_ns must be in (0, 2e9]");
  int* st = status_ptr();
  if (!st) return fail(AFA_ERR_CUDA, "could not resolve the device status word");
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(st, static_cast<unsigned long long>(budget_ns));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "self-test launch");
  return AFA_OK;
}

int afa_device_status(void* stream, int* status, int clear) {
  if (!status) return fail(AFA_ERR_INVALID, "status must be non-null");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_afa_device_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
  *status = v;
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_afa_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device status word");
  }
  return AFA_OK;
}

}  // extern "C"
