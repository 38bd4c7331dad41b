// dcr_decode_ops.cu — the non-attention kernels of a decode step (sm_100a): residual add +
// RMSNorm, SiLU-gated product, and the skinny linear layer y = x W^T for a few tokens.
//
// These serve the decode model around the attention layer (the reference runs them as HF
// LlamaRMSNorm, LlamaMLP and nn.Linear in torch, dcr_attention/models/llama/compat.py and
// transformers' modeling_llama). A decode step has M = B tokens (1-8), so every linear layer
// is a matrix-vector product per token: it reads each weight once and is HBM-bound; the
// norms and activations are a few kilobytes each and cost their launch. Numerics follow
// torch's composition of the same ops: values rounded to the model dtype where torch
// stores a tensor, fp32 in between.
//
// add_rmsnorm (one CTA per token row): h' = T(h + delta) (torch's residual add), then
//     y = T( T(w) * T(h' * rsqrt(mean(h'^2) + eps)) )   (HF LlamaRMSNorm: statistics in
// fp32, normalised value cast to T, then multiplied by the weight in T).
// silu_mul: out = T( T(silu(g)) * u ) (F.silu in fp32 rounded to T, then the product).
// linear_skinny: y[m, n] = T( sum_k x[m, k] * W[n, k] ) with fp32 accumulation; x staged
// in shared memory, each warp streams R rows of W with 16-byte loads (4 in flight per
// lane), lanes stride over k, then one warp reduction per (token, row).
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

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t n,
                                T* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float x = to_f<T>(g[i]);
    const float s = round_t<T>(x / (1.0f + expf(-x)));
    out[i] = from_f<T>(s * to_f<T>(u[i]));
  }
}

constexpr int kLinWarps = 8;
constexpr int kLinRows = 4;  // rows of W per warp

// y[M][N] = x[M][K] . W[N][K]^T, 16-bit T, K a multiple of 256 (32 lanes x 8 elements).
template <typename T, int M>
__global__ void __launch_bounds__(kLinWarps * 32) linear_skinny_kernel(
    const T* __restrict__ x, const T* __restrict__ W, int N, int K, T* __restrict__ y) {
  extern __shared__ __align__(16) uint8_t smem_lin[];
  T* xs = reinterpret_cast<T*>(smem_lin);  // [M][K]
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  {
    const uint4* src = reinterpret_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(xs);
    for (int i = tid; i < M * K / 8; i += kLinWarps * 32) dst[i] = src[i];
  }
  __syncthreads();
  const int n0 = (blockIdx.x * kLinWarps + warp) * kLinRows;
  if (n0 >= N) return;
  float acc[kLinRows][M];
#pragma unroll
  for (int r = 0; r < kLinRows; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;
  const int chunks = K / 256;  // 8-element chunks per lane per row
  for (int c0 = 0; c0 < chunks; c0 += 4) {
    uint4 wv[kLinRows][4];
#pragma unroll
    for (int r = 0; r < kLinRows; ++r)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int n = n0 + r;
        const int c = c0 + u;
        wv[r][u] = (n < N && c < chunks)
                       ? __ldg(reinterpret_cast<const uint4*>(W + static_cast<int64_t>(n) * K) +
                               c * 32 + lane)
                       : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u;
      if (c >= chunks) break;
      float xf[M][8];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 xv = reinterpret_cast<const uint4*>(xs + m * K)[c * 32 + lane];
        ElemTraits<T>::widen(xv, xf[m]);
      }
#pragma unroll
      for (int r = 0; r < kLinRows; ++r) {
        float wf[8];
        ElemTraits<T>::widen(wv[r][u], wf);
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(wf[e], xf[m][e], acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kLinRows; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[r][m] = v;
    }
  if (lane < kLinRows * M) {
    const int r = lane / M;
    const int m = lane - r * M;
    float v = 0.0f;
#pragma unroll
    for (int rr = 0; rr < kLinRows; ++rr)
#pragma unroll
      for (int mm = 0; mm < M; ++mm)
        if (rr == r && mm == m) v = acc[rr][mm];
    if (n0 + r < N) y[static_cast<int64_t>(m) * N + n0 + r] = from_f<T>(v);
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
static int launch_silu_t(const void* g, const void* u, int64_t n, void* out, cudaStream_t st) {
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  silu_mul_kernel<T><<<static_cast<unsigned>(blocks), threads, 0, st>>>(
      static_cast<const T*>(g), static_cast<const T*>(u), n, static_cast<T*>(out));
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

template <typename T, int M>
static int launch_lin_tm(const void* x, const void* W, int N, int K, void* y, cudaStream_t st) {
  const int smem = M * K * static_cast<int>(sizeof(T));
  const void* fn = reinterpret_cast<const void*>(&linear_skinny_kernel<T, M>);
  if (ensure_smem_attr(fn, smem) != cudaSuccess) return DCR_ERR_CUDA;
  const int rows_per_cta = kLinWarps * kLinRows;
  const int grid = (N + rows_per_cta - 1) / rows_per_cta;
  linear_skinny_kernel<T, M><<<grid, kLinWarps * 32, smem, st>>>(
      static_cast<const T*>(x), static_cast<const T*>(W), N, K, static_cast<T*>(y));
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

template <typename T>
static int launch_lin_t(const void* x, const void* W, int M, int N, int K, void* y,
                        cudaStream_t st) {
  switch (M) {
    case 1: return launch_lin_tm<T, 1>(x, W, N, K, y, st);
    case 2: return launch_lin_tm<T, 2>(x, W, N, K, y, st);
    case 3: return launch_lin_tm<T, 3>(x, W, N, K, y, st);
    case 4: return launch_lin_tm<T, 4>(x, W, N, K, y, st);
    case 5: return launch_lin_tm<T, 5>(x, W, N, K, y, st);
    case 6: return launch_lin_tm<T, 6>(x, W, N, K, y, st);
    case 7: return launch_lin_tm<T, 7>(x, W, N, K, y, st);
    case 8: return launch_lin_tm<T, 8>(x, W, N, K, y, st);
    default: return DCR_ERR_SHAPE;
  }
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

int dcr_silu_mul(const void* gate, const void* up, int dtype, int64_t n, void* out, void* stream) {
  if (gate == nullptr || up == nullptr || out == nullptr) return DCR_ERR_NULL;
  if (n <= 0) return DCR_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DCR_DTYPE_BF16: return launch_silu_t<__nv_bfloat16>(gate, up, n, out, st);
    case DCR_DTYPE_F16: return launch_silu_t<__half>(gate, up, n, out, st);
    case DCR_DTYPE_F32: return launch_silu_t<float>(gate, up, n, out, st);
    default: return DCR_ERR_DTYPE;
  }
}

int dcr_linear_skinny(const void* x, const void* weight, int dtype, int M, int N, int K, void* y,
                      void* stream) {
  if (x == nullptr || weight == nullptr || y == nullptr) return DCR_ERR_NULL;
  if (M < 1 || M > DCR_SKINNY_MAX_M || N <= 0 || K <= 0 || K % 256 != 0) return DCR_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight)) & 15u)
    return DCR_ERR_ALIGN;
  if (static_cast<int64_t>(M) * K * 2 > 200 * 1024) return DCR_ERR_SHAPE;  // x in shared memory
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DCR_DTYPE_BF16: return launch_lin_t<__nv_bfloat16>(x, weight, M, N, K, y, st);
    case DCR_DTYPE_F16: return launch_lin_t<__half>(x, weight, M, N, K, y, st);
    default: return DCR_ERR_DTYPE;
  }
}

}  // extern "C"
