// dcr_rope.cu — decode prologue: RoPE on the step's new query and key rows, the cache
// append of the rotated key and the value, and (projected mode) the projected key row
// and the projected unit query, in one launch.
//
// Replaces, for one decode step, steps 2-3 of the reference's DCRLlamaAttention.forward
// (dcr_attention/models/llama/attention.py:395-421): HF apply_rotary_pos_emb
// (compat.py:63), q' = q*cos + rotate_half(q)*sin with rotate_half(x) = [-x[32:], x[:32]],
// evaluated as torch does it in the model dtype (each product and the sum rounded to the
// dtype: the 16-bit products are exact in fp32, so rounding the fp32 product reproduces
// torch's op), then cache_update (compat.py:208), a torch.cat of the whole cache, replaced
// by writing the new rows at position `pos` of the preallocated caches. In projected mode
// the same launch writes KP = k'.P (the fmaf chain of dcr_cache_append) and
// qp = unit(q').P (the unit query and fmaf chain of the projected Pass 1), so Pass 1 does
// not recompute them.
//
// One CTA per batch row, one warp per head (8 warps looping over the H query and H_kv key
// heads); lane l holds the rotate_half pair (l, l + 32).
#include <type_traits>

#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

constexpr int kRopeWarps = 8;

struct RopeParams {
  const void* q;       // [B, H, D]     (contiguous)
  const void* k;       // [B, H_kv, D]
  const void* v;       // [B, H_kv, D]
  const void* cos;     // [B, D] in the model dtype
  const void* sin;     // [B, D]
  void* q_out;         // [B, H, D] rotated query
  void* k_cache;       // [B, H_kv, N_max, D], strides csb, csh
  void* v_cache;
  int64_t csb, csh;
  int pos;
  void* kp;            // optional [B, H_kv, N_max, R], strides psb, psh
  int64_t psb, psh;
  const float* P;      // [D][R] (with kp or qp)
  float* qp;           // optional [B, H, R] projected unit queries
  float eps;
  int H, H_kv;
  int64_t q_sb, kv_sb;  // elements between the batch rows of q and of k/v
};

template <typename T>
__device__ __forceinline__ float rope_round(float x) {
  if constexpr (sizeof(T) == 4) {
    return x;
  } else if constexpr (std::is_same<T, __half>::value) {
    return __half2float(__float2half_rn(x));
  } else {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
}

template <typename T>
__device__ __forceinline__ float elem(const void* base, int64_t i) {
  if constexpr (sizeof(T) == 4) return static_cast<const float*>(base)[i];
  else if constexpr (std::is_same<T, __half>::value) return __half2float(static_cast<const __half*>(base)[i]);
  else return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
}

template <typename T>
__global__ void __launch_bounds__(kRopeWarps * 32) rope_append_kernel(const RopeParams p) {
  constexpr int kR = DCR_PROJ_RANK;
  __shared__ float P_s[kD * kR];
  __shared__ float row_s[kRopeWarps][kD];
  __shared__ float u_s[kRopeWarps][kD];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int b = blockIdx.x;
  if (p.P != nullptr)
    for (int i = tid; i < kD * kR; i += kRopeWarps * 32) P_s[i] = p.P[i];
  __syncthreads();
  const float c0 = elem<T>(p.cos, static_cast<int64_t>(b) * kD + lane);
  const float c1 = elem<T>(p.cos, static_cast<int64_t>(b) * kD + lane + 32);
  const float s0 = elem<T>(p.sin, static_cast<int64_t>(b) * kD + lane);
  const float s1 = elem<T>(p.sin, static_cast<int64_t>(b) * kD + lane + 32);
  for (int head = warp; head < p.H + p.H_kv; head += kRopeWarps) {
    const bool is_q = head < p.H;
    const int h = is_q ? head : head - p.H;
    const void* src = is_q ? p.q : p.k;
    const int64_t in_row = static_cast<int64_t>(b) * (is_q ? p.q_sb : p.kv_sb) +
                           static_cast<int64_t>(h) * kD;
    const int64_t row = (static_cast<int64_t>(b) * (is_q ? p.H : p.H_kv) + h) * kD;
    const float x0 = elem<T>(src, in_row + lane);
    const float x1 = elem<T>(src, in_row + lane + 32);
    // q*cos + rotate_half(q)*sin, each op rounded to T as torch evaluates it (the _rn
    // intrinsics keep fp32 from contracting the products into the sum)
    const float y0 = rope_round<T>(__fadd_rn(rope_round<T>(__fmul_rn(x0, c0)),
                                             rope_round<T>(__fmul_rn(-x1, s0))));
    const float y1 = rope_round<T>(__fadd_rn(rope_round<T>(__fmul_rn(x1, c1)),
                                             rope_round<T>(__fmul_rn(x0, s1))));
    row_s[warp][lane] = y0;
    row_s[warp][lane + 32] = y1;
    __syncwarp();
    if (is_q) {
      ElemTraits<T>::store(p.q_out, static_cast<int>(row + lane), y0);
      ElemTraits<T>::store(p.q_out, static_cast<int>(row + lane + 32), y1);
      if (p.qp != nullptr) {
        // unit query of the stored (rounded) row, exactly as Pass 1 computes it
        float a0 = row_s[warp][2 * lane], a1 = row_s[warp][2 * lane + 1];
        const float sq0 = a0 * a0;
        float part = fmaf(a1, a1, sq0);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) part = part + __shfl_xor_sync(0xffffffffu, part, off);
        const float norm = fmaxf(sqrtf(part), p.eps);
        u_s[warp][2 * lane] = a0 / norm;
        u_s[warp][2 * lane + 1] = a1 / norm;
        __syncwarp();
        if (lane < kR) {
          float acc = 0.0f;
          for (int d = 0; d < kD; ++d) acc = fmaf(u_s[warp][d], P_s[d * kR + lane], acc);
          p.qp[(static_cast<int64_t>(b) * p.H + h) * kR + lane] = acc;
        }
      }
    } else {
      T* kc = static_cast<T*>(p.k_cache) + b * p.csb + h * p.csh + static_cast<int64_t>(p.pos) * kD;
      T* vc = static_cast<T*>(p.v_cache) + b * p.csb + h * p.csh + static_cast<int64_t>(p.pos) * kD;
      ElemTraits<T>::store(kc, lane, y0);
      ElemTraits<T>::store(kc, lane + 32, y1);
      const int64_t vrow = static_cast<int64_t>(b) * p.kv_sb + static_cast<int64_t>(h) * kD;
      ElemTraits<T>::store(vc, lane, elem<T>(p.v, vrow + lane));
      ElemTraits<T>::store(vc, lane + 32, elem<T>(p.v, vrow + lane + 32));
      if (p.kp != nullptr && lane < kR) {
        // KP of the stored (rounded) key row: the fmaf chain of dcr_cache_append
        float acc = 0.0f;
        for (int d = 0; d < kD; ++d) acc = fmaf(row_s[warp][d], P_s[d * kR + lane], acc);
        T* kpr = static_cast<T*>(p.kp) + b * p.psb + h * p.psh + static_cast<int64_t>(p.pos) * kR;
        ElemTraits<T>::store(kpr, lane, acc);
      }
    }
    __syncwarp();
  }
}

int launch_rope_append(const void* q, const void* k, const void* v, const void* cos,
                       const void* sin, int dtype, int B, int H, int H_kv, void* q_out,
                       void* k_cache, void* v_cache, int64_t csb, int64_t csh, int pos,
                       void* kp, int64_t psb, int64_t psh, const float* P, float* qp,
                       float eps, cudaStream_t st, int64_t q_sb, int64_t kv_sb) {
  RopeParams p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.cos = cos;
  p.sin = sin;
  p.q_out = q_out;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.csb = csb;
  p.csh = csh;
  p.pos = pos;
  p.kp = kp;
  p.psb = psb;
  p.psh = psh;
  p.P = P;
  p.qp = qp;
  p.eps = eps;
  p.H = H;
  p.H_kv = H_kv;
  p.q_sb = q_sb > 0 ? q_sb : static_cast<int64_t>(H) * kD;
  p.kv_sb = kv_sb > 0 ? kv_sb : static_cast<int64_t>(H_kv) * kD;
  switch (dtype) {
    case DCR_DTYPE_BF16: rope_append_kernel<__nv_bfloat16><<<B, kRopeWarps * 32, 0, st>>>(p); break;
    case DCR_DTYPE_F16: rope_append_kernel<__half><<<B, kRopeWarps * 32, 0, st>>>(p); break;
    case DCR_DTYPE_F32: rope_append_kernel<float><<<B, kRopeWarps * 32, 0, st>>>(p); break;
    default: return DCR_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

}  // namespace dcr
