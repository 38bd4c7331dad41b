// dcr_noalloc.cu — dcr_decode_noalloc: the full decode step with library-owned scratch.
//
// Why it exists: dcr_decode needs a workspace (scores, selected indices, split-K
// partials, tickets) that the caller allocates. Some callers cannot allocate device memory
// at the point where they run a decode step: an inference-engine plugin whose enqueue
// function must not allocate (the engine owns all device memory), or a latency-critical
// serving loop that cannot afford cudaMalloc's implicit device synchronisation. For them
// this entry point runs the same three kernels on scratch memory that lives in a
// file-scope __device__ array of this library.
//
// Limits and sharing rules:
//  - The array holds DCR_NOALLOC_SCRATCH_BYTES (16 MiB). Every GPU on which the library's
//    device code is loaded holds this array until the process exits. A shape whose
//    workspace (dcr_workspace_bytes) is larger is rejected with DCR_ERR_NOALLOC_LIMIT
//    before anything is launched.
//  - All calls on a device share the one array, and it keeps whatever the previous call
//    left there. Two calls whose kernels overlap on the GPU (different streams without an
//    ordering between them) race on it and may return wrong results. Calls ordered on one
//    stream are safe.
//  - The only state that must start at zero, the split-K tickets, is cleared by Pass 2 of
//    every call before Pass 3 uses it; scores, indices and partials are fully written
//    before they are read.
//  - The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current; the driver may load the library's
//    module then) and sets the kernels' shared-memory attributes. Make that first call a
//    warm-up during the caller's initialisation, outside its no-allocation region and
//    before any stream capture begins; later calls allocate nothing.
//  - The entry point calls no cudaMalloc, cudaFree or other device allocator.
#include <cuda_runtime.h>

#include <mutex>

#include "dcr_b200.h"
#include "dcr_internal.h"

namespace dcr {

constexpr size_t kNoAllocScratchBytes = DCR_NOALLOC_SCRATCH_BYTES;

// The scratch itself. In host code this name is only a handle for the runtime API, not a
// device address; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kNoAllocMaxDevices = 128;

struct NoAllocDevice {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};

NoAllocDevice g_noalloc_devices[kNoAllocMaxDevices];

// Device address of the scratch array on the current device (looked up once per device,
// with that device current). Returns nullptr on failure.
void* noalloc_scratch_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return nullptr;
  NoAllocDevice& d = g_noalloc_devices[dev];
  std::call_once(d.once, [&d] {
    void* p = nullptr;
    d.err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    d.ptr = (d.err == cudaSuccess) ? p : nullptr;
  });
  return d.ptr;
}

}  // namespace
}  // namespace dcr

extern "C" int dcr_decode_noalloc(const void* Q, const void* K, const void* V, int dtype,
                                  int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                                  int64_t v_stride_h, int B, int H, int H_kv, int N, int D,
                                  int k_eff, float eps, void* O, void* stream) {
  using namespace dcr;
  int st = check_heads(B, H, H_kv, N, D);
  if (st) return st;
  if ((st = check_k(k_eff, N))) return st;
  if (workspace_layout(B * H, N, k_eff).total > kNoAllocScratchBytes) return DCR_ERR_NOALLOC_LIMIT;
  void* scratch = noalloc_scratch_ptr();
  if (scratch == nullptr) return DCR_ERR_CUDA;
  return decode_impl(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, B, H, H_kv,
                     N, D, k_eff, eps, O, scratch, kNoAllocScratchBytes, stream, nullptr);
}
