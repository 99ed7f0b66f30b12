// afa_decode_noalloc: the decode step for callers that cannot allocate device
// memory.
//
// afa_decode takes its split-KV scratch from the caller (sized by
// afa_decode_workspace_bytes). Some callers have no way to provide it:
// - plugin hosts whose device allocator belongs to another runtime and is not
//   reachable from the plugin (an XLA custom call that was not handed a scratch
//   buffer, for instance);
// - serving loops that forbid allocation on the per-token path, where a
//   cudaMalloc would synchronise the device and stall every stream.
// This entry point runs the same kernels with the scratch placed in a
// fixed-size array in this library's device memory instead.
//
// Contract:
// - The array is kNoallocScratchBytes (1 MiB) per GPU. Every GPU that loads
//   the library holds it until the process exits.
// - Shapes whose scratch would exceed that are rejected with AFA_ERR_INVALID.
//   Shapes that fill the GPU need no scratch at all: (batch x heads) >= 592,
//   or caches of at most 512 keys.
// - Every call shares the one array. Calls that overlap on the GPU (concurrent
//   streams, or several host threads using one device) race on it; serialise
//   them on one stream. Each call overwrites every scratch element it later
//   reads, so nothing needs clearing between calls.
// - Only shapes that run the split-KV kernels use the array (bf16 with head
//   dim 64/128/256, f32 with 64/128); other shapes run without scratch.
// - The first call on a device resolves the array's device address
//   (cudaGetSymbolAddress) and caches it. Make that first call before any
//   stream capture.
// - The cached address belongs to the device's current context: do not use
//   the library across cudaDeviceReset (or a reset of the primary context),
//   after which the address is stale.
#include <cstdio>
#include <mutex>

#include "afa_b200.h"
#include "afa_common.cuh"
#include "afa_internal.h"

namespace {

constexpr size_t kNoallocScratchBytes = size_t(1) << 20;  // 1 MiB

// Device-side scratch. In host code this name is only a host-side stand-in: its
// device address must come from cudaGetSymbolAddress (below), never from taking
// the address of the symbol on the host.
static __device__ __align__(256) unsigned char g_decode_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

}  // namespace

extern "C" int afa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out, void* d_total,
                                  int B, int H, int Lkv, int D, int dtype, float sink_omega, const int* kv_lens,
                                  int kv_len, void* stream) {
  // Only the split-KV kernels use scratch; afa_decode checks the dtype.
  const size_t need = afa::decode_fast_supported(dtype, D) ? afa_decode_workspace_bytes(B, H, Lkv, D) : 0;
  if (need > kNoallocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "afa_decode_noalloc: this shape needs %zu bytes of split-KV scratch, above the fixed %zu-byte "
             "scratch of the allocation-free entry point; use afa_decode with a caller workspace",
             need, kNoallocScratchBytes);
    return afa::set_last_error(AFA_ERR_INVALID, msg);
  }
  void* scratch = nullptr;
  if (need > 0) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return afa::set_last_error(AFA_ERR_CUDA, "afa_decode_noalloc: no current CUDA device");
    {
      std::lock_guard<std::mutex> lock(g_scratch_mu);
      if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess || p == nullptr)
          return afa::set_last_error(AFA_ERR_CUDA, "afa_decode_noalloc: cudaGetSymbolAddress of the scratch array failed");
        g_scratch_ptr[dev] = p;
      }
      scratch = g_scratch_ptr[dev];
    }
  }
  return afa_decode(q, k_cache, v_cache, out, d_total, B, H, Lkv, D, dtype, sink_omega, kv_lens, kv_len, scratch,
                    need, stream);
}
