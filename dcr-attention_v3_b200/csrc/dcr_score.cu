// dcr_score.cu — unit query and Pass 1 (projection scores) for sm_100a.
//
// Pass 1 replaces the reference's _pass1_projection_kernel
// (dcr_attention/kernel/triton/topk_axis_pass1.py:29) and its oracle
// _compute_projection_scores (dcr_attention/kernel/qaxis_topk_reference.py:58):
//     score[b, h, n] = bf16_rne( sum_d f32(K[b, h / G, n, d]) * u[b, h, d] ).
// The unit query replaces _compute_u_Q (qaxis_topk_reference.py:42):
//     u = f32(q) / max(||f32(q)||_2, eps).
//
// Design (B200): the pass is a pure HBM stream of the K cache (128 B per row for 16-bit
// caches) with G = H / H_kv query heads scored per row. A persistent grid of
// 3 CTAs per SM (for 16-bit caches and G = 4; the count follows the shared-memory size)
// walks contiguous ranges of 256-row tiles; one thread per CTA issues 4-D TMA tile loads
// (128-byte swizzle) into a 2-stage shared-memory ring completed by mbarriers. Every
// thread scores two rows of each tile (r and r + 128) with packed fp32 FMAs
// (fma.rn.f32x2) that advance two heads of one row per instruction: the unit
// queries sit in shared memory transposed, u_t[d][head], so one 16-byte load feeds two
// head pairs. (For G = 1 the pair is two rows of one head and u is stored as {u, u}.)
// Each lane of the packed FMA is an IEEE fma, so the fp32 dot product of every
// (row, head) is still one chain of fused multiply-adds over d = 0..63 from 0, and a CPU
// restatement with fmaf in that order reproduces every score bit for bit.
// A tile's scores are staged in shared memory and written out during the next tile with
// one 16-byte store per thread. The fused decode path stores the 16-bit order keys of
// the scores (see bf16_order_key) instead of their bf16 bits, so Pass 2 reads keys.
//
// The unit query is computed by one warp per query row: lane l squares elements 2l and
// 2l+1 (x0*x0 rounded, then fmaf(x1, x1, .)), the 32 partial sums are combined by an
// xor butterfly (offsets 16, 8, 4, 2, 1), then u = x / max(sqrtf(sum), eps) with IEEE
// sqrt and division.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

// ---------------------------------------------------------------------------------------
// Unit query
// ---------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load_pair(const void* row, int lane, float& x0, float& x1) {
  if constexpr (sizeof(T) == 4) {
    const float2 v = reinterpret_cast<const float2*>(row)[lane];
    x0 = v.x;
    x1 = v.y;
  } else {
    const uint32_t w = reinterpret_cast<const uint32_t*>(row)[lane];
    const float2 v = ElemTraits<T>::widen2(w);
    x0 = v.x;
    x1 = v.y;
  }
}

// One warp: u[d] = q_row[d] / max(||q_row||, eps) for d = 0..63, written as
// u_out[d * stride]. All lanes of the warp must call.
template <typename T>
__device__ __forceinline__ void unit_query_warp(const void* q_row, float eps, float* u_out,
                                                int stride = 1) {
  const int lane = threadIdx.x & 31;
  float x0, x1;
  load_pair<T>(q_row, lane, x0, x1);
  const float sq0 = x0 * x0;
  float part = fmaf(x1, x1, sq0);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) part = part + __shfl_xor_sync(0xffffffffu, part, off);
  const float norm = fmaxf(sqrtf(part), eps);
  u_out[(2 * lane) * stride] = x0 / norm;
  u_out[(2 * lane + 1) * stride] = x1 / norm;
}

template <typename T>
__global__ void __launch_bounds__(128) unit_query_kernel(const void* __restrict__ q, int rows,
                                                         float eps, float* __restrict__ u) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (warp >= rows) return;
  const char* q_row = static_cast<const char*>(q) + static_cast<size_t>(warp) * kD * sizeof(T);
  unit_query_warp<T>(q_row, eps, u + static_cast<size_t>(warp) * kD);
}

int launch_unit_query(const void* Q, int dtype, int rows, float eps, float* u, cudaStream_t st) {
  const int threads = 128;
  const int blocks = (rows * 32 + threads - 1) / threads;
  switch (dtype) {
    case DCR_DTYPE_BF16:
      unit_query_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(Q, rows, eps, u);
      break;
    case DCR_DTYPE_F16:
      unit_query_kernel<__half><<<blocks, threads, 0, st>>>(Q, rows, eps, u);
      break;
    default:
      unit_query_kernel<float><<<blocks, threads, 0, st>>>(Q, rows, eps, u);
      break;
  }
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

// ---------------------------------------------------------------------------------------
// Pass 1
// ---------------------------------------------------------------------------------------
// Launch shape of Pass 1 (compile-time; overridable for tuning sweeps).
#ifndef DCR_P1_THREADS
#define DCR_P1_THREADS 128
#endif
#ifndef DCR_P1_RPT
#define DCR_P1_RPT 2
#endif
#ifndef DCR_P1_STAGES
#define DCR_P1_STAGES 2
#endif
constexpr int kP1Threads = DCR_P1_THREADS;

template <typename T>
struct P1Cfg {
  static constexpr int kRPT = DCR_P1_RPT;               // rows per thread per tile
  static constexpr int kTileRows = kP1Threads * kRPT;   // <= 256 (TMA box limit)
  static constexpr int kStageBytes = kTileRows * RowTraits<T>::kRowBytes;
  static constexpr int kStages = sizeof(T) == 4 ? 2 : DCR_P1_STAGES;
  static constexpr int kBoxCols = 128 / ElemTraits<T>::kBytes;            // 64 or 32
  static_assert(kTileRows <= 256, "TMA box height is at most 256 rows");
};

__host__ __device__ constexpr int p1_u_bytes(int G) { return G * kD * 4; }  // u_t[d][G]

template <typename T, int G>
__host__ __device__ constexpr int p1_smem_bytes() {
  // tiles + unit queries + double-buffered score staging [2][G][tile] u16 + mbarriers
  return 1024 + P1Cfg<T>::kStages * P1Cfg<T>::kStageBytes + p1_u_bytes(G) +
         2 * G * P1Cfg<T>::kTileRows * 2 + P1Cfg<T>::kStages * 8;
}

// Resident CTAs per SM allowed by shared memory (228 KB per SM, 1 KB reserved per CTA).
template <typename T, int G>
__host__ __device__ constexpr int p1_ctas_per_sm() {
  return (233472 / (p1_smem_bytes<T, G>() + 1024)) < 1
             ? 1
             : ((233472 / (p1_smem_bytes<T, G>() + 1024)) > 4
                    ? 4
                    : (233472 / (p1_smem_bytes<T, G>() + 1024)));
}

struct P1Params {
  const float* u;  // [rows_q, 64] fp32 or nullptr (then computed from q)
  const void* q;   // [rows_q, 64] in the cache dtype
  float eps;
  uint16_t* scores;
  int64_t s_stride;
  int keys_out;    // store order keys instead of bf16 bits
  int vec_store;   // score rows are 16-byte aligned (16-byte stores)
  int N;
  int H_kv;
  int tiles_per_group;
  int total_tiles;
};

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// Order key of a bf16 score without branches, equal to bf16_order_key for all 65536
// patterns: -0 sorts as +0, every NaN on top.
__device__ __forceinline__ uint32_t bf16_order_key_lean(uint32_t b) {
  const uint32_t m = b & 0x7fffu;
  const uint32_t neg = (b >> 15) & (m != 0u ? 1u : 0u);
  const uint32_t key = neg ? (m ^ 0x7fffu) : (m | 0x8000u);
  return m > 0x7f80u ? 0xffffu : key;
}

// kKeys: store order keys (the decode steps) instead of bf16 bits (p.keys_out).
template <typename T, int G, bool kKeys>
__global__ void __launch_bounds__(kP1Threads, (p1_ctas_per_sm<T, G>()))
    score_kernel(const __grid_constant__ CUtensorMap kmap, const P1Params p) {
  using Cfg = P1Cfg<T>;
  constexpr int kChunks = RowTraits<T>::kChunks;
  constexpr int kPer = ElemTraits<T>::kPerChunk;
  constexpr int kStages = Cfg::kStages;
  constexpr int kTR = Cfg::kTileRows;
  constexpr int kRPT = Cfg::kRPT;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  float* u_s = reinterpret_cast<float*>(smem + kStages * Cfg::kStageBytes);  // u_t[d][G]
  uint16_t* stage_sc = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(u_s) + p1_u_bytes(G));
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_sc + 2 * G * kTR);

  const int tid = threadIdx.x;
  const int t_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.total_tiles / gridDim.x);
  const int t_end =
      static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.total_tiles / gridDim.x);
  const int my_tiles = t_end - t_begin;
  if (my_tiles <= 0) return;

  if (tid == 0) {
    tma_prefetch_desc(&kmap);
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto tile_of = [&](int it, int& g, int& n0) {
    const int t = t_begin + it;
    g = t / p.tiles_per_group;
    n0 = (t - g * p.tiles_per_group) * kTR;
  };
  auto issue = [&](int it) {
    int g, n0;
    tile_of(it, g, n0);
    const int s = it % kStages;
    const int b = g / p.H_kv;
    const int hk = g - b * p.H_kv;
    uint8_t* dst = tiles + s * Cfg::kStageBytes;
    mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
#pragma unroll
    for (int sub = 0; sub < RowTraits<T>::kSubTiles; ++sub)
      tma_load_4d(dst + sub * kTR * 128, &kmap, &full[s], sub * Cfg::kBoxCols, n0, hk, b);
  };
  // Writes the staged scores of tile `it` (buffer it & 1) to global memory: each pass of
  // the loop stores 8 consecutive scores of one head row per thread.
  auto flush = [&](int it) {
    int g, n0;
    tile_of(it, g, n0);
    const uint16_t* src = stage_sc + (it & 1) * G * kTR;
    for (int i = tid; i < G * kTR / 8; i += kP1Threads) {
      const int j = i / (kTR / 8);
      const int r = (i - j * (kTR / 8)) * 8;
      const int n = n0 + r;
      uint16_t* dst = p.scores + (static_cast<int64_t>(g) * G + j) * p.s_stride + n;
      const uint4 v = *reinterpret_cast<const uint4*>(src + j * kTR + r);
      if (p.vec_store && n + 8 <= p.N) {
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (n + q < p.N) dst[q] = e[q];
      }
    }
  };

  if (tid == 0) {
    const int pre = my_tiles < kStages ? my_tiles : kStages;
    for (int it = 0; it < pre; ++it) issue(it);
  }

  int cur_group = -1;
  for (int it = 0; it < my_tiles; ++it) {
    int g, n0;
    tile_of(it, g, n0);
    const int s = it % kStages;

    if (g != cur_group) {  // uniform across the CTA
      __syncthreads();     // earlier readers of u_s are done
      const int warp = tid >> 5;
      for (int j = warp; j < G; j += kP1Threads / 32) {
        if (p.u != nullptr) {
          const float* src = p.u + (static_cast<size_t>(g) * G + j) * kD;
          for (int d = tid & 31; d < kD; d += 32) u_s[d * G + j] = src[d];
        } else {
          const char* q_row = static_cast<const char*>(p.q) +
                              (static_cast<size_t>(g) * G + j) * kD * sizeof(T);
          unit_query_warp<T>(q_row, p.eps, u_s + j, G);
        }
      }
      __syncthreads();
      cur_group = g;
    }

    if (it > 0) flush(it - 1);  // scores of the previous tile, staged before the barrier

    const bool ok = mbar_wait_bounded(&full[s], static_cast<uint32_t>((it / kStages) & 1));
    const uint32_t tile_addr = smem_u32(tiles + s * Cfg::kStageBytes);
    float res[kRPT][G];  // [row][head]

    if constexpr (G == 1) {
      // one query head: a plain fmaf chain per row
      float acc[kRPT];
#pragma unroll
      for (int i = 0; i < kRPT; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const float4* ud = reinterpret_cast<const float4*>(u_s + c * kPer);
        float uv[kPer];
#pragma unroll
        for (int q4 = 0; q4 < kPer / 4; ++q4) {
          const float4 t4 = ud[q4];
          uv[4 * q4] = t4.x;
          uv[4 * q4 + 1] = t4.y;
          uv[4 * q4 + 2] = t4.z;
          uv[4 * q4 + 3] = t4.w;
        }
#pragma unroll
        for (int i = 0; i < kRPT; ++i) {
          float f[kPer];
          ElemTraits<T>::widen(lds128(tile_addr + swz_offset(tid + i * kP1Threads, c, kTR)), f);
#pragma unroll
          for (int e = 0; e < kPer; ++e) acc[i] = fmaf(f[e], uv[e], acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < kRPT; ++i) res[i][0] = acc[i];
    } else {
      // pair = (head 2m, head 2m+1) of one row, advanced by one packed FMA
      constexpr int kPairs = G / 2;
      float2 acc[kRPT][kPairs];
#pragma unroll
      for (int i = 0; i < kRPT; ++i)
#pragma unroll
        for (int m = 0; m < kPairs; ++m) acc[i][m] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        float f[kRPT][kPer];
#pragma unroll
        for (int i = 0; i < kRPT; ++i)
          ElemTraits<T>::widen(lds128(tile_addr + swz_offset(tid + i * kP1Threads, c, kTR)), f[i]);
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const float* ud = u_s + (c * kPer + e) * G;
          float uv[G];
          if constexpr (G == 2) {
            const float2 t2 = *reinterpret_cast<const float2*>(ud);
            uv[0] = t2.x;
            uv[1] = t2.y;
          } else {
#pragma unroll
            for (int q4 = 0; q4 < G / 4; ++q4) {
              const float4 t4 = reinterpret_cast<const float4*>(ud)[q4];
              uv[4 * q4 + 0] = t4.x;
              uv[4 * q4 + 1] = t4.y;
              uv[4 * q4 + 2] = t4.z;
              uv[4 * q4 + 3] = t4.w;
            }
          }
#pragma unroll
          for (int m = 0; m < kPairs; ++m) {
            const float2 um = make_float2(uv[2 * m], uv[2 * m + 1]);
#pragma unroll
            for (int i = 0; i < kRPT; ++i)
              acc[i][m] = ffma2(make_float2(f[i][e], f[i][e]), um, acc[i][m]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kRPT; ++i)
#pragma unroll
        for (int m = 0; m < kPairs; ++m) {
          res[i][2 * m] = acc[i][m].x;
          res[i][2 * m + 1] = acc[i][m].y;
        }
    }

    uint16_t* sc = stage_sc + (it & 1) * G * kTR;
#pragma unroll
    for (int i = 0; i < kRPT; ++i)
#pragma unroll
      for (int j = 0; j < G; ++j) {
        uint32_t bits = f32_to_bf16_bits(res[i][j]);
        if constexpr (kKeys) bits = bf16_order_key_lean(bits);
        sc[j * kTR + tid + i * kP1Threads] = static_cast<uint16_t>(bits);
      }

    if (__syncthreads_or(!ok)) break;  // stage s read; staged scores complete
    if (tid == 0 && it + kStages < my_tiles) {
      fence_proxy_async_smem();
      issue(it + kStages);
    }
    if (it == my_tiles - 1) flush(it);
  }
}

// ---------------------------------------------------------------------------------------
// Host side: tensor map + launch
// ---------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

template <typename T, int G>
static int launch_score_t(const void* K, int64_t ksb, int64_t ksh, const P1Params& p, int B,
                          int H_kv, cudaStream_t st) {
  using Cfg = P1Cfg<T>;
  EncodeTiledFn encode = get_encode_fn();
  if (!encode) return DCR_ERR_CUDA;
  CUtensorMapDataType dt = sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                          : (std::is_same<T, __half>::value
                                                 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(p.N),
                              static_cast<cuuint64_t>(H_kv), static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kD * sizeof(T)),
                                 static_cast<cuuint64_t>(ksh * sizeof(T)),
                                 static_cast<cuuint64_t>(ksb * sizeof(T))};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(Cfg::kBoxCols),
                             static_cast<cuuint32_t>(Cfg::kTileRows), 1u, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUtensorMap map;
  CUresult r = encode(&map, dt, 4, const_cast<void*>(K), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return DCR_ERR_CUDA;

  constexpr int smem = p1_smem_bytes<T, G>();
  const void* fn = p.keys_out ? reinterpret_cast<const void*>(&score_kernel<T, G, true>)
                              : reinterpret_cast<const void*>(&score_kernel<T, G, false>);
  if (ensure_smem_attr(fn, smem) != cudaSuccess) return DCR_ERR_CUDA;
  const int max_ctas = device_sm_count() * p1_ctas_per_sm<T, G>();
  const int grid = p.total_tiles < max_ctas ? p.total_tiles : max_ctas;
  if (p.keys_out)
    score_kernel<T, G, true><<<grid, kP1Threads, smem, st>>>(map, p);
  else
    score_kernel<T, G, false><<<grid, kP1Threads, smem, st>>>(map, p);
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

template <typename T>
static int launch_score_g(const void* K, int64_t ksb, int64_t ksh, const P1Params& p, int B,
                          int H_kv, int G, cudaStream_t st) {
  switch (G) {
    case 1: return launch_score_t<T, 1>(K, ksb, ksh, p, B, H_kv, st);
    case 2: return launch_score_t<T, 2>(K, ksb, ksh, p, B, H_kv, st);
    case 4: return launch_score_t<T, 4>(K, ksb, ksh, p, B, H_kv, st);
    case 8: return launch_score_t<T, 8>(K, ksb, ksh, p, B, H_kv, st);
    default: return DCR_ERR_SHAPE;
  }
}

int launch_score(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h,
                 const float* u, const void* Q, float eps, int B, int H, int H_kv, int N,
                 uint16_t* scores, int64_t s_stride_row, int keys_out, cudaStream_t st) {
  P1Params p;
  p.keys_out = keys_out;
  p.vec_store = ((reinterpret_cast<uintptr_t>(scores) & 15u) == 0 && (s_stride_row & 7) == 0) ? 1 : 0;
  p.u = u;
  p.q = Q;
  p.eps = eps;
  p.scores = scores;
  p.s_stride = s_stride_row;
  p.N = N;
  p.H_kv = H_kv;
  const int G = H / H_kv;
  const int tile_rows = P1Cfg<__nv_bfloat16>::kTileRows;  // same for every dtype
  p.tiles_per_group = (N + tile_rows - 1) / tile_rows;
  const int64_t total = static_cast<int64_t>(p.tiles_per_group) * B * H_kv;
  if (total > 0x7fffffff) return DCR_ERR_SHAPE;
  p.total_tiles = static_cast<int>(total);
  switch (dtype) {
    case DCR_DTYPE_BF16:
      return launch_score_g<__nv_bfloat16>(K, k_stride_b, k_stride_h, p, B, H_kv, G, st);
    case DCR_DTYPE_F16:
      return launch_score_g<__half>(K, k_stride_b, k_stride_h, p, B, H_kv, G, st);
    case DCR_DTYPE_F32:
      return launch_score_g<float>(K, k_stride_b, k_stride_h, p, B, H_kv, G, st);
    default:
      return DCR_ERR_DTYPE;
  }
}

}  // namespace dcr
