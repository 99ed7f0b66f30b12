// Host-side interfaces between the C-ABI layer (afa_capi.cu) and the kernel
// translation units. Not part of the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include <mutex>

#include "afa_problem.h"

namespace afa {

constexpr int kMaxDevices = 64;

// Host set-up that runs once per device (kernel attributes, device
// properties), safe when several host threads make their first call on one
// device at the same time. The set-up's status is kept and returned to every
// caller; a device index outside [0, kMaxDevices) is an error.
class PerDeviceOnce {
 public:
  template <class F>
  cudaError_t run(int dev, F&& init) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once_[dev], [&] { status_[dev] = init(); });
    return status_[dev];
  }

 private:
  std::once_flag once_[kMaxDevices];
  cudaError_t status_[kMaxDevices] = {};
};

enum Dtype : int { kF32 = 0, kBF16 = 1, kF16 = 2, kF64 = 3 };

inline size_t dtype_size(int dt) {
  switch (dt) {
    case kF32: return 4;
    case kBF16: return 2;
    case kF16: return 2;
    case kF64: return 8;
    default: return 0;
  }
}

// Number of CTAs along the problem axis that a problem needs for the given
// query rows per CTA; fills Problem::cta0/ncta and returns the total.
inline int assign_ctas(Launch& L, int rows_per_cta) {
  int total = 0;
  for (int i = 0; i < L.nprob; ++i) {
    L.prob[i].cta0 = total;
    L.prob[i].ncta = (L.prob[i].q.len + rows_per_cta - 1) / rows_per_cta;
    total += L.prob[i].ncta;
  }
  return total;
}

// Each returns cudaSuccess or the launch error; `detail` receives a short
// message on failure.
bool tc_fwd_supported(int dtype, int d);
// True when an accumulate launch of these problems runs the persistent
// tensor-core kernel, whose pieces add into the accumulators with reductions,
// so two problems may share query rows (their partial sums add).
bool tc_accum_reduces(const Launch& L, int dtype);
cudaError_t launch_tc_fwd(Launch L, int dtype, cudaStream_t stream, const char** detail);

cudaError_t launch_simt_fwd(Launch L, int dtype, cudaStream_t stream, const char** detail);

bool tc_bwd_supported(int dtype, int d);
cudaError_t launch_tc_bwd(const void* q, const void* k, const void* v, const void* g_out, const float* d_total,
                          const float* e, void* dq, void* dk, void* dv, int B, int H, int L, int D, int causal,
                          int valid, float scale, float sink, int* status, cudaStream_t stream, const char** detail);

cudaError_t launch_finalize(const void* o_acc, const void* d_acc, void* out, void* dtot, long long rows, int d,
                            int dtype, double sink, cudaStream_t stream);

int decode_splits(int bh, int lkv);
bool decode_fast_supported(int dtype, int d);
cudaError_t launch_decode(const void* q, const void* k, const void* v, void* out, void* dtot, int B, int H,
                          int lkv, int d, int dtype, double sink, const int* kv_lens, int kv_len, float* ws_o,
                          float* ws_d, int nsplit, int* status, cudaStream_t stream);

cudaError_t launch_softmax(const void* x, void* y, long long rows, int cols, int dtype, double sink, double eps,
                           cudaStream_t stream);
cudaError_t launch_softmax_bwd(const void* x, const void* g, void* dx, long long rows, int cols, int dtype, double sink,
                               double eps, cudaStream_t stream);
cudaError_t launch_octic(const void* x, void* y, long long n, int dtype, cudaStream_t stream);
cudaError_t launch_octic_bwd(const void* x, const void* g, void* dx, long long n, int dtype, cudaStream_t stream);

// Records `msg` as the calling thread's afa_last_error() and returns `code`.
int set_last_error(int code, const char* msg);

// The calling device's status word (where bounded waits report), or nullptr.
int* device_status_ptr();

}  // namespace afa
