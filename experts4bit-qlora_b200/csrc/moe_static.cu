// Allocation-free variant of e4b_moe_forward.
//
// Some callers cannot allocate device memory at call time: code running under a
// host framework that owns every device allocation (a serving runtime with a
// fixed memory plan, a plugin host that forbids cudaMalloc after start-up), or a
// caller with no allocator of its own at all. This entry point runs the same
// fused expert layer with its scratch in a fixed, file-scope device array
// instead of a caller-provided workspace.
//
// Limits and behaviour:
//  * The array is E4B_STATIC_SCRATCH_BYTES (16 MiB) and lives on every GPU that
//    loads this library until the process exits.
//  * A layer whose scratch need (e4b_moe_workspace_bytes) exceeds it is refused
//    with E4B_ERR_STATIC_SCRATCH before anything is launched.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture on the device.
//  * Every call on a device shares the one array and it keeps the previous
//    call's contents. What must start at zero is the array's header: the decode
//    kernel's counter block, zero at load (a static device array is zero-filled)
//    and left zero by every launch, and the device error word, which keeps the
//    first error any call records (nothing reads it back here). Calls that
//    overlap on the GPU (different streams, no ordering between them) race on the
//    array.
#include <mutex>

#include "common.cuh"

static __device__ __align__(256) unsigned char g_e4b_static_scratch[E4B_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_mu;
void* g_addr[64] = {nullptr};
}  // namespace

extern "C" e4b_status e4b_moe_forward_static(const e4b_moe_desc* desc, const e4b_moe_tensors* t, void* stream) {
  if (!desc || !t) return E4B_ERR_INVALID_ARG;
  const size_t need = e4b_moe_workspace_bytes(desc);
  if (need == 0) return E4B_ERR_INVALID_ARG;
  if (need > (size_t)E4B_STATIC_SCRATCH_BYTES) return E4B_ERR_STATIC_SCRATCH;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return E4B_ERR_CUDA;
  void* p;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
      void* a = nullptr;
      if (cudaGetSymbolAddress(&a, g_e4b_static_scratch) != cudaSuccess || !a) return E4B_ERR_CUDA;
      g_addr[dev] = a;
    }
    p = g_addr[dev];
  }
  return e4b_moe_forward(desc, t, p, (size_t)E4B_STATIC_SCRATCH_BYTES, stream);
}
