// dcr_attend.cu — Pass 3 (gather + online-softmax attention) for sm_100a.
//
// Replaces the reference's _pass3_fused_attn_kernel
// (dcr_attention/kernel/triton/fused_attn.py:40) and its oracle _gather_kv +
// _fused_softmax_attention (dcr_attention/kernel/qaxis_topk_reference.py:111, :148):
//     z_j = (K[b, h/G, idx_j] . f32(Q[b, h])) / sqrt(D)      (unnormalised Q)
//     O[b, h] = sum_j softmax(z)_j V[b, h/G, idx_j]
// with an fp32 running state (m, l, o) and a single rounding of o / l to the output type.
//
// Design (B200): the reference runs one program per (b, h) over all k_eff rows. Here the
// sorted index list of every (b, h) is cut into S contiguous pieces (split-K, S chosen so
// that B*H*S CTAs fill the 148 SMs once). CTA (b, h_kv, s, j) handles piece s of query
// head j of KV group (b, h_kv); the G heads of one group and piece are launched next to
// each other, so the rows they share are fetched from HBM once and served from L2.
// Each CTA gathers 64-row tiles of K and V with 16-byte cp.async copies (8 lanes per
// 128-byte row, fully coalesced) into a 4-stage ring of 128-byte-swizzled shared-memory
// tiles. Scores use two threads per row (32 dims each, Q held in registers); the P.V
// product uses one thread per (dimension pair, 16-row group). Each CTA writes its partial
// (m, l, o[64]) to the workspace; the last CTA of a (b, h) to finish (atomic ticket,
// no waiting) merges the S partials:
//     M = max_s m_s,  O = sum_s e^{m_s - M} o_s / sum_s e^{m_s - M} l_s.
// Every gathered index is checked against [0, N); a bad one is skipped (zero row, zero
// weight) and raises DCR_ERR_DEVICE_INDEX.
#include <math.h>

#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

constexpr int kP3Threads = 128;
constexpr int kP3Tile = 64;

template <typename T>
struct P3Cfg {
  static constexpr int kRowBytes = RowTraits<T>::kRowBytes;
  static constexpr int kChunks = RowTraits<T>::kChunks;
  static constexpr int kTileBytes = kP3Tile * kRowBytes;  // one of K or V
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = sizeof(T) == 4 ? 3 : 4;
  static constexpr int kSmem = 1024 + kStages * kStageBytes;
};

struct P3Params {
  const void* q;
  const void* k;
  const void* v;
  int64_t ksb, ksh, vsb, vsh;  // element strides
  const int32_t* idx;
  int H, H_kv, G, N, k_eff, S;
  void* o;
  float* part;
  int* counters;
};

template <typename T>
__global__ void __launch_bounds__(kP3Threads, 3) attend_kernel(const P3Params p) {
  using Cfg = P3Cfg<T>;
  constexpr int kChunks = Cfg::kChunks;
  constexpr int kPer = ElemTraits<T>::kPerChunk;
  constexpr int kHalfChunks = kChunks / 2;
  constexpr int kRowsPerPass = kP3Threads / kChunks;  // 16 (16-bit) or 8 (fp32)
  constexpr int kPasses = kP3Tile / kRowsPerPass;     // 4 or 8

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ float P_s[kP3Tile];
  __shared__ float red[kP3Threads / 32];
  __shared__ float o_red[kP3Threads / 32][kD];
  __shared__ float l_red[kP3Threads / 32];
  __shared__ int is_last;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  int id = blockIdx.x;
  const int j = id % p.G;
  id /= p.G;
  const int s = id % p.S;
  const int g = id / p.S;
  const int b = g / p.H_kv;
  const int hk = g - b * p.H_kv;
  const int h = hk * p.G + j;
  const int64_t row = static_cast<int64_t>(b) * p.H + h;

  const int64_t p0 = static_cast<int64_t>(s) * p.k_eff / p.S;
  const int64_t p1 = static_cast<int64_t>(s + 1) * p.k_eff / p.S;
  const int cnt = static_cast<int>(p1 - p0);
  const int ntiles = (cnt + kP3Tile - 1) / kP3Tile;
  const int32_t* idx_row = p.idx + row * p.k_eff + p0;
  const uint8_t* kbase = static_cast<const uint8_t*>(p.k) + (b * p.ksb + hk * p.ksh) * static_cast<int64_t>(sizeof(T));
  const uint8_t* vbase = static_cast<const uint8_t*>(p.v) + (b * p.vsb + hk * p.vsh) * static_cast<int64_t>(sizeof(T));

  // Q half owned by this thread (two threads per row in the score phase).
  const int half = tid & 1;
  float qf[kD / 2];
  {
    const uint8_t* qrow = static_cast<const uint8_t*>(p.q) + row * kD * static_cast<int64_t>(sizeof(T));
    const uint4* q4 = reinterpret_cast<const uint4*>(qrow) + half * kHalfChunks;
#pragma unroll
    for (int c = 0; c < kHalfChunks; ++c) {
      float f[kPer];
      ElemTraits<T>::widen(q4[c], f);
#pragma unroll
      for (int e = 0; e < kPer; ++e) qf[c * kPer + e] = f[e];
    }
  }

  auto issue = [&](int tt) {
    if (tt < ntiles) {
      uint8_t* kt = smem + (tt % Cfg::kStages) * Cfg::kStageBytes;
      uint8_t* vt = kt + Cfg::kTileBytes;
      const int c = tid % kChunks;
#pragma unroll
      for (int i = 0; i < kPasses; ++i) {
        const int r = tid / kChunks + i * kRowsPerPass;
        const int pos = tt * kP3Tile + r;
        uint32_t bytes = 0;
        int64_t n = 0;
        if (pos < cnt) {
          n = idx_row[pos];
          if (n >= 0 && n < p.N) {
            bytes = 16;
          } else {
            if (c == 0) raise_status(DCR_ERR_DEVICE_INDEX);
            n = 0;
          }
        }
        const uint32_t off = swz_offset(r, c, kP3Tile);
        cp_async_16(kt + off, kbase + n * Cfg::kRowBytes + c * 16, bytes);
        cp_async_16(vt + off, vbase + n * Cfg::kRowBytes + c * 16, bytes);
      }
    }
    cp_async_commit();  // always commit so group counting stays uniform
  };

#pragma unroll
  for (int i = 0; i < Cfg::kStages - 1; ++i) issue(i);

  float m_run = -INFINITY;
  float l_part = 0.0f;
  float o0 = 0.0f, o1 = 0.0f;
  const int dp = lane;  // dimension pair 2dp, 2dp+1
  const int rg = warp;  // rows rg*16 .. rg*16+15 in the P.V phase

  for (int tt = 0; tt < ntiles; ++tt) {
    cp_async_wait<Cfg::kStages - 2>();
    __syncthreads();
    issue(tt + Cfg::kStages - 1);

    const uint8_t* kt = smem + (tt % Cfg::kStages) * Cfg::kStageBytes;
    const uint8_t* vt = kt + Cfg::kTileBytes;
    const uint32_t kt_addr = smem_u32(kt);

    // ---- scores: row r = tid / 2, dims [32*half, 32*half + 32) ----
    const int r = tid >> 1;
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
    for (int c = 0; c < kHalfChunks; ++c) {
      float f[kPer];
      ElemTraits<T>::widen(lds128(kt_addr + swz_offset(r, half * kHalfChunks + c, kP3Tile)), f);
#pragma unroll
      for (int e = 0; e < kPer; e += 2) {
        acc0 = fmaf(f[e], qf[c * kPer + e], acc0);
        acc1 = fmaf(f[e + 1], qf[c * kPer + e + 1], acc1);
      }
    }
    float z = acc0 + acc1;
    z += __shfl_xor_sync(0xffffffffu, z, 1);
    z *= 0.125f;  // 1 / sqrt(64), exact
    const bool valid = tt * kP3Tile + r < cnt;
    if (!valid) z = -INFINITY;

    float mt = z;
#pragma unroll
    for (int off = 2; off < 32; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
    if (lane == 0) red[warp] = mt;
    __syncthreads();
    const float m_tile = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float m_new = fmaxf(m_run, m_tile);
    const float alpha = expf(m_run - m_new);
    const float pr = valid ? expf(z - m_new) : 0.0f;
    if (half == 0) P_s[r] = pr;
    l_part = l_part * alpha + (half == 0 ? pr : 0.0f);
    m_run = m_new;
    __syncthreads();

    // ---- P.V: thread (dp, rg) accumulates dims 2dp, 2dp+1 over 16 rows ----
    o0 *= alpha;
    o1 *= alpha;
    const uint32_t vt_addr = smem_u32(vt);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int rr = rg * 16 + i;
      const float pw = P_s[rr];
      if constexpr (sizeof(T) == 4) {
        const uint32_t addr = vt_addr + swz_offset(rr, dp >> 1, kP3Tile) + (dp & 1) * 8;
        float2 v2;
        asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v2.x), "=f"(v2.y) : "r"(addr));
        o0 = fmaf(pw, v2.x, o0);
        o1 = fmaf(pw, v2.y, o1);
      } else {
        const uint32_t addr = vt_addr + swz_offset(rr, dp >> 2, kP3Tile) + (dp & 3) * 4;
        uint32_t w;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w) : "r"(addr));
        const float2 v2 = ElemTraits<T>::widen2(w);
        o0 = fmaf(pw, v2.x, o0);
        o1 = fmaf(pw, v2.y, o1);
      }
    }
  }
  cp_async_wait<0>();

  // ---- CTA reduction: l over threads, o over the 4 row groups ----
  float ls = l_part;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
  if (lane == 0) l_red[warp] = ls;
  o_red[rg][2 * dp] = o0;
  o_red[rg][2 * dp + 1] = o1;
  __syncthreads();
  const float l_cta = (l_red[0] + l_red[1]) + (l_red[2] + l_red[3]);

  if (p.S == 1) {
    if (tid < kD) {
      const float od = (o_red[0][tid] + o_red[1][tid]) + (o_red[2][tid] + o_red[3][tid]);
      ElemTraits<T>::store(p.o, static_cast<int>(row * kD + tid), od / l_cta);
    }
    return;
  }

  float* mine = p.part + (row * p.S + s) * (kD + 2);
  if (tid < kD) mine[2 + tid] = (o_red[0][tid] + o_red[1][tid]) + (o_red[2][tid] + o_red[3][tid]);
  if (tid == 0) {
    mine[0] = m_run;
    mine[1] = l_cta;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(&p.counters[row], 1) == p.S - 1) ? 1 : 0;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (tid < kD) {
    const float* base = p.part + row * p.S * (kD + 2);
    float M = -INFINITY;
    for (int t = 0; t < p.S; ++t) M = fmaxf(M, __ldcg(base + t * (kD + 2)));
    float L = 0.0f, od = 0.0f;
    for (int t = 0; t < p.S; ++t) {
      const float* pt = base + t * (kD + 2);
      const float w = expf(__ldcg(pt) - M);
      L = fmaf(w, __ldcg(pt + 1), L);
      od = fmaf(w, __ldcg(pt + 2 + tid), od);
    }
    ElemTraits<T>::store(p.o, static_cast<int>(row * kD + tid), od / L);
  }
  if (tid == 0) p.counters[row] = 0;
}

int attend_splits(int rows, int k_eff) {
  const int slots = device_sm_count() * 3;  // 3 CTAs per SM
  int S = slots / (rows > 0 ? rows : 1);
  const int max_by_tiles = (k_eff + kP3Tile - 1) / kP3Tile;
  if (S > max_by_tiles) S = max_by_tiles;
  if (S > 64) S = 64;
  if (S < 1) S = 1;
  return S;
}

template <typename T>
static int launch_attend_t(const P3Params& p, int B, cudaStream_t st) {
  constexpr int smem = P3Cfg<T>::kSmem;
  if (ensure_smem_attr(reinterpret_cast<const void*>(&attend_kernel<T>), smem) != cudaSuccess)
    return DCR_ERR_CUDA;
  const int64_t grid = static_cast<int64_t>(B) * p.H_kv * p.S * p.G;
  if (grid > 0x7fffffff) return DCR_ERR_SHAPE;
  attend_kernel<T><<<static_cast<unsigned>(grid), kP3Threads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

int launch_attend(const void* Q, const void* K, const void* V, int dtype, int64_t k_stride_b,
                  int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_h,
                  const int32_t* idx, int B, int H, int H_kv, int N, int k_eff, void* O,
                  int splits, float* partials, int* counters, cudaStream_t st) {
  P3Params p;
  p.q = Q;
  p.k = K;
  p.v = V;
  p.ksb = k_stride_b;
  p.ksh = k_stride_h;
  p.vsb = v_stride_b;
  p.vsh = v_stride_h;
  p.idx = idx;
  p.H = H;
  p.H_kv = H_kv;
  p.G = H / H_kv;
  p.N = N;
  p.k_eff = k_eff;
  p.S = splits;
  p.o = O;
  p.part = partials;
  p.counters = counters;
  switch (dtype) {
    case DCR_DTYPE_BF16: return launch_attend_t<__nv_bfloat16>(p, B, st);
    case DCR_DTYPE_F16: return launch_attend_t<__half>(p, B, st);
    case DCR_DTYPE_F32: return launch_attend_t<float>(p, B, st);
    default: return DCR_ERR_DTYPE;
  }
}

}  // namespace dcr
