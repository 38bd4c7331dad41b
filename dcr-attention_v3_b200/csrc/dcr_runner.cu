// dcr_runner.cu — a native decode-step runner: one step (the H2D copy of the step's query,
// the three passes, the D2H copy of O) captured once as a CUDA graph and replayed per call.
//
// The reference's hook calls its kernels from Python every step (dcr_attention/models/
// llama/attention.py:805-813): launches, argument checks and allocations per call, and a
// host round trip through torch for the copies. A serving loop over fixed caches needs a
// step that costs one graph launch and one synchronisation: dcr_runner_create captures the
// step for one (K, V, N, k_eff) binding, on a stream and with device buffers, pinned host
// staging and a workspace that the runner owns; dcr_runner_step copies the caller's query
// into the pinned staging, replays the graph, waits for it, and copies O out. No device
// memory is allocated after creation.
//
// The staging is mapped into the device's address space, and the graph moves Q in and O out
// with a small copy kernel each (16-byte loads and stores over the bus) instead of copy-engine
// nodes: a memcpy node costs several microseconds to start, the kernel about one.
#include <cuda_runtime.h>
#include <string.h>

#include "dcr_b200.h"
#include "dcr_internal.h"

namespace {

struct Runner {
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  void* q_pinned = nullptr;
  void* o_pinned = nullptr;
  void* q_mapped = nullptr;  // device addresses of the pinned staging
  void* o_mapped = nullptr;
  void* q_dev = nullptr;
  void* o_dev = nullptr;
  void* ws = nullptr;
  size_t q_bytes = 0;
};

void runner_free(Runner* r) {
  if (r == nullptr) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(r->device);
  if (r->exec) cudaGraphExecDestroy(r->exec);
  if (r->graph) cudaGraphDestroy(r->graph);
  if (r->stream) cudaStreamDestroy(r->stream);
  if (r->q_pinned) cudaFreeHost(r->q_pinned);
  if (r->o_pinned) cudaFreeHost(r->o_pinned);
  if (r->q_dev) cudaFree(r->q_dev);
  if (r->o_dev) cudaFree(r->o_dev);
  if (r->ws) cudaFree(r->ws);
  cudaSetDevice(prev);
  delete r;
}

}  // namespace

namespace dcr {

// dst[i] = src[i] for n 16-byte words; either side may be mapped host memory.
__global__ void __launch_bounds__(256) runner_copy16(const uint4* __restrict__ src,
                                                     uint4* __restrict__ dst, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i];
}

static cudaError_t copy16(const void* src, void* dst, size_t bytes, cudaStream_t st) {
  const int n = static_cast<int>(bytes / 16);
  runner_copy16<<<(n + 255) / 256, 256, 0, st>>>(static_cast<const uint4*>(src),
                                                 static_cast<uint4*>(dst), n);
  return cudaGetLastError();
}

}  // namespace dcr

extern "C" {

int dcr_runner_create(const void* K, const void* V, const void* KP, const float* P, int dtype,
                      int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                      int64_t v_stride_h, int64_t p_stride_b, int64_t p_stride_h, int B, int H,
                      int H_kv, int N, int D, int k_eff, float eps, void** runner_out) {
  if (runner_out == nullptr) return DCR_ERR_NULL;
  *runner_out = nullptr;
  const size_t eb = dtype == DCR_DTYPE_F32 ? 4 : (dtype == DCR_DTYPE_BF16 || dtype == DCR_DTYPE_F16 ? 2 : 0);
  if (eb == 0) return DCR_ERR_DTYPE;
  if (B <= 0 || H <= 0 || D != DCR_HEAD_DIM) return DCR_ERR_SHAPE;
  const size_t ws_bytes = dcr_workspace_bytes(B, H, H_kv, N, D, k_eff);
  if (ws_bytes == 0) return DCR_ERR_SHAPE;
  Runner* r = new Runner();
  cudaGetDevice(&r->device);
  r->q_bytes = static_cast<size_t>(B) * H * D * eb;
  auto fail = [&](int st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (r->stream && cudaStreamIsCapturing(r->stream, &cs) == cudaSuccess &&
        cs != cudaStreamCaptureStatusNone) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(r->stream, &g);
      if (g) cudaGraphDestroy(g);
    }
    cudaGetLastError();
    runner_free(r);
    return st;
  };
  if (cudaStreamCreateWithFlags(&r->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaHostAlloc(&r->q_pinned, r->q_bytes, cudaHostAllocPortable | cudaHostAllocMapped) !=
          cudaSuccess ||
      cudaHostAlloc(&r->o_pinned, r->q_bytes, cudaHostAllocPortable | cudaHostAllocMapped) !=
          cudaSuccess ||
      cudaHostGetDevicePointer(&r->q_mapped, r->q_pinned, 0) != cudaSuccess ||
      cudaHostGetDevicePointer(&r->o_mapped, r->o_pinned, 0) != cudaSuccess ||
      cudaMalloc(&r->q_dev, r->q_bytes) != cudaSuccess ||
      cudaMalloc(&r->o_dev, r->q_bytes) != cudaSuccess ||
      cudaMalloc(&r->ws, ws_bytes) != cudaSuccess)
    return fail(DCR_ERR_CUDA);
  memset(r->q_pinned, 0, r->q_bytes);
  if (cudaMemsetAsync(r->q_dev, 0, r->q_bytes, r->stream) != cudaSuccess) return fail(DCR_ERR_CUDA);
  auto step = [&]() -> int {
    if (KP != nullptr)
      return dcr_decode_projected(r->q_dev, K, V, KP, dtype, k_stride_b, k_stride_h, v_stride_b,
                                  v_stride_h, p_stride_b, p_stride_h, P, DCR_PROJ_RANK, nullptr,
                                  B, H, H_kv, N, D, k_eff, eps, r->o_dev, r->ws, ws_bytes,
                                  r->stream);
    return dcr_decode(r->q_dev, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, B,
                      H, H_kv, N, D, k_eff, eps, r->o_dev, r->ws, ws_bytes, r->stream);
  };
  // one eager step first: argument checks and the kernels' one-time setup run outside the
  // capture, and an invalid binding fails here with its own status
  int st = step();
  if (st != DCR_OK) return fail(st);
  if (cudaStreamSynchronize(r->stream) != cudaSuccess) return fail(DCR_ERR_CUDA);
  if (cudaStreamBeginCapture(r->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
    return fail(DCR_ERR_CUDA);
  if (dcr::copy16(r->q_mapped, r->q_dev, r->q_bytes, r->stream) != cudaSuccess)
    return fail(DCR_ERR_CUDA);
  if ((st = step()) != DCR_OK) return fail(st);
  if (dcr::copy16(r->o_dev, r->o_mapped, r->q_bytes, r->stream) != cudaSuccess)
    return fail(DCR_ERR_CUDA);
  if (cudaStreamEndCapture(r->stream, &r->graph) != cudaSuccess) return fail(DCR_ERR_CUDA);
  if (cudaGraphInstantiate(&r->exec, r->graph, 0) != cudaSuccess) return fail(DCR_ERR_CUDA);
  *runner_out = r;
  return DCR_OK;
}

int dcr_runner_step(void* runner, const void* q_host, void* o_host) {
  Runner* r = static_cast<Runner*>(runner);
  if (r == nullptr || q_host == nullptr || o_host == nullptr) return DCR_ERR_NULL;
  if (q_host != r->q_pinned) memcpy(r->q_pinned, q_host, r->q_bytes);
  if (cudaGraphLaunch(r->exec, r->stream) != cudaSuccess) return DCR_ERR_CUDA;
  if (cudaStreamSynchronize(r->stream) != cudaSuccess) return DCR_ERR_CUDA;
  if (o_host != r->o_pinned) memcpy(o_host, r->o_pinned, r->q_bytes);
  return DCR_OK;
}

void* dcr_runner_query_buffer(void* runner) {
  return runner == nullptr ? nullptr : static_cast<Runner*>(runner)->q_pinned;
}

void* dcr_runner_output_buffer(void* runner) {
  return runner == nullptr ? nullptr : static_cast<Runner*>(runner)->o_pinned;
}

int dcr_runner_destroy(void* runner) {
  runner_free(static_cast<Runner*>(runner));
  return DCR_OK;
}

}  // extern "C"
