// dcr_decode_ops.cu — the non-attention kernels of a decode step (sm_100a): residual add +
// RMSNorm and the SiLU-gated product.
//
// These serve the decode model around the attention layer (the reference runs them as HF
// LlamaRMSNorm and LlamaMLP in torch, transformers' modeling_llama). In a decode step the
// norms and activations are a few kilobytes each and cost their launches: one kernel
// replaces each chain of small torch kernels. (The linear layers stay library GEMMs: cuBLAS
// streams the large decode-step weights at 5-7 TB/s.) Numerics follow torch's composition
// of the same ops: values rounded to the model dtype where torch stores a tensor, fp32 in
// between.
//
// add_rmsnorm (one CTA per token row): h' = T(h + delta) (torch's residual add), then
//     y = T( T(w) * T(h' * rsqrt(mean(h'^2) + eps)) )   (HF LlamaRMSNorm: statistics in
// fp32, normalised value cast to T, then multiplied by the weight in T).
// silu_mul: out = T( T(silu(g)) * u ) (F.silu in fp32 rounded to T, then the product).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (sizeof(T) == 4)
    return v;
  else if constexpr (std::is_same<T, __half>::value)
    return __half2float(v);
  else
    return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f(float v) {
  if constexpr (sizeof(T) == 4)
    return v;
  else if constexpr (std::is_same<T, __half>::value)
    return __float2half_rn(v);
  else
    return __float2bfloat16_rn(v);
}

template <typename T>
__device__ __forceinline__ float round_t(float v) {
  return to_f<T>(from_f<T>(v));
}

constexpr int kNormThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    const T* h, const T* __restrict__ delta, const T* __restrict__ w, float eps, int dim,
    T* h_out, T* __restrict__ y) {  // h_out may be h (in-place residual update)
  __shared__ float red[kNormThreads / 32];
  const int64_t off = static_cast<int64_t>(blockIdx.x) * dim;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < dim; i += kNormThreads) {
    float v = to_f<T>(h[off + i]);
    if (delta != nullptr) {
      v = round_t<T>(v + to_f<T>(delta[off + i]));
      h_out[off + i] = from_f<T>(v);
    }
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(dim) + eps);
  for (int i = threadIdx.x; i < dim; i += kNormThreads) {
    const float v = delta != nullptr ? to_f<T>(h_out[off + i]) : to_f<T>(h[off + i]);
    y[off + i] = from_f<T>(to_f<T>(w[i]) * round_t<T>(v * r));
  }
}

// out[r][i] = silu(g[r * stride + i]) * u[r * stride + i] for r < rows, i < inter.
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t rows,
                                int64_t inter, int64_t stride, T* __restrict__ out) {
  const int64_t n = rows * inter;
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < n;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = j / inter;
    const int64_t i = r * stride + (j - r * inter);
    const float x = to_f<T>(g[i]);
    const float s = round_t<T>(x / (1.0f + expf(-x)));
    out[j] = from_f<T>(s * to_f<T>(u[i]));
  }
}

template <typename T>
static int launch_norm_t(const void* h, const void* delta, const void* w, float eps, int rows,
                         int dim, void* h_out, void* y, cudaStream_t st) {
  add_rmsnorm_kernel<T><<<rows, kNormThreads, 0, st>>>(
      static_cast<const T*>(h), static_cast<const T*>(delta), static_cast<const T*>(w), eps, dim,
      static_cast<T*>(h_out), static_cast<T*>(y));
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

template <typename T>
static int launch_silu_t(const void* g, const void* u, int64_t rows, int64_t inter,
                         int64_t stride, void* out, cudaStream_t st) {
  const int threads = 256;
  int64_t blocks = (rows * inter + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  silu_mul_kernel<T><<<static_cast<unsigned>(blocks), threads, 0, st>>>(
      static_cast<const T*>(g), static_cast<const T*>(u), rows, inter, stride,
      static_cast<T*>(out));
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

}  // namespace dcr

using namespace dcr;

extern "C" {

int dcr_add_rmsnorm(const void* h, const void* delta, const void* weight, int dtype, int rows,
                    int dim, float eps, void* h_out, void* y, void* stream) {
  if (h == nullptr || weight == nullptr || y == nullptr) return DCR_ERR_NULL;
  if (delta != nullptr && h_out == nullptr) return DCR_ERR_NULL;
  if (rows <= 0 || dim <= 0) return DCR_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DCR_DTYPE_BF16: return launch_norm_t<__nv_bfloat16>(h, delta, weight, eps, rows, dim, h_out, y, st);
    case DCR_DTYPE_F16: return launch_norm_t<__half>(h, delta, weight, eps, rows, dim, h_out, y, st);
    case DCR_DTYPE_F32: return launch_norm_t<float>(h, delta, weight, eps, rows, dim, h_out, y, st);
    default: return DCR_ERR_DTYPE;
  }
}

static int silu_any(const void* g, const void* u, int dtype, int64_t rows, int64_t inter,
                    int64_t stride, void* out, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DCR_DTYPE_BF16: return launch_silu_t<__nv_bfloat16>(g, u, rows, inter, stride, out, st);
    case DCR_DTYPE_F16: return launch_silu_t<__half>(g, u, rows, inter, stride, out, st);
    case DCR_DTYPE_F32: return launch_silu_t<float>(g, u, rows, inter, stride, out, st);
    default: return DCR_ERR_DTYPE;
  }
}

int dcr_silu_mul(const void* gate, const void* up, int dtype, int64_t n, void* out, void* stream) {
  if (gate == nullptr || up == nullptr || out == nullptr) return DCR_ERR_NULL;
  if (n <= 0) return DCR_ERR_SHAPE;
  return silu_any(gate, up, dtype, 1, n, n, out, stream);
}

int dcr_silu_mul_packed(const void* gate_up, int dtype, int rows, int inter, void* out,
                        void* stream) {
  if (gate_up == nullptr || out == nullptr) return DCR_ERR_NULL;
  if (rows <= 0 || inter <= 0) return DCR_ERR_SHAPE;
  const size_t eb = dtype == DCR_DTYPE_F32 ? 4 : 2;
  const void* up = static_cast<const char*>(gate_up) + static_cast<size_t>(inter) * eb;
  return silu_any(gate_up, up, dtype, rows, inter, 2 * static_cast<int64_t>(inter), out, stream);
}

}  // extern "C"
