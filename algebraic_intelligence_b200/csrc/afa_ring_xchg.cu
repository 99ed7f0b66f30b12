// Ring K/V exchange: CUDA IPC mappings of each rank's published K/V buffer and
// copy-engine pulls from them.
//
// The reference moves K/V around the ring with lax.ppermute
// (src/kernels/pallas_afa.py:651-652), one send/receive per hop. On one B200
// node every GPU reaches every other over NVSwitch at full bandwidth, so a hop
// does not need the shard to travel through the ranks in between: each rank
// publishes its shard once per call and every hop pulls the shard it needs
// from the rank that owns it. The pull is a cudaMemcpyAsync between a peer
// mapping and local memory, which the copy engines carry over NVLink. No SM
// takes part, so the transfer runs beside the attention kernel, which keeps
// every SM busy; an SM-driven transfer (a collective library's send/receive
// kernel) would instead wait for the attention kernel's last wave.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>
#include <cstring>

#include "afa_b200.h"
#include "afa_internal.h"

static_assert(sizeof(cudaIpcMemHandle_t) == AFA_RING_HANDLE_BYTES, "IPC handle size");

namespace {

// Resolved once (a function-local static is initialised once, thread-safely).
PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static const PFN_cuMemGetAddressRange_v3020 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    const bool ok = cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
                    q == cudaDriverEntryPointSuccess;
    return ok ? reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p) : nullptr;
  }();
  return fn;
}

int cuda_fail(const char* what, cudaError_t e) {
  char msg[256];
  snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
  return afa::set_last_error(AFA_ERR_CUDA, msg);
}

}  // namespace

extern "C" int afa_ring_export(const void* ptr, void* handle_out, unsigned long long* offset_out) {
  if (!ptr || !handle_out || !offset_out) return afa::set_last_error(AFA_ERR_INVALID, "afa_ring_export: null pointer");
  auto range = address_range_fn();
  if (!range) return afa::set_last_error(AFA_ERR_CUDA, "afa_ring_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS || base == 0)
    return afa::set_last_error(AFA_ERR_INVALID, "afa_ring_export: pointer is not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail("afa_ring_export: cudaIpcGetMemHandle (the buffer must come from cudaMalloc, not a "
                     "virtual-memory or expandable-segment allocator)", e);
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(ptr) - base);
  return AFA_OK;
}

extern "C" int afa_ring_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return afa::set_last_error(AFA_ERR_INVALID, "afa_ring_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail("afa_ring_open: cudaIpcOpenMemHandle", e);
  }
  *base_out = p;
  return AFA_OK;
}

extern "C" int afa_ring_close(void* base) {
  if (!base) return afa::set_last_error(AFA_ERR_INVALID, "afa_ring_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail("afa_ring_close: cudaIpcCloseMemHandle", e);
  }
  return AFA_OK;
}

extern "C" int afa_ring_pull(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return AFA_OK;
  if (!dst || !src) return afa::set_last_error(AFA_ERR_INVALID, "afa_ring_pull: null pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("afa_ring_pull: cudaMemcpyAsync", e);
  return AFA_OK;
}

extern "C" int afa_ring_pull2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t row_bytes,
                               size_t rows, void* stream) {
  if (row_bytes == 0 || rows == 0) return AFA_OK;
  if (!dst || !src) return afa::set_last_error(AFA_ERR_INVALID, "afa_ring_pull2d: null pointer");
  if (dst_pitch < row_bytes || src_pitch < row_bytes)
    return afa::set_last_error(AFA_ERR_INVALID, "afa_ring_pull2d: a pitch is shorter than a row");
  cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, row_bytes, rows, cudaMemcpyDefault,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("afa_ring_pull2d: cudaMemcpy2DAsync", e);
  return AFA_OK;
}
