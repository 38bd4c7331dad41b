// dcr_project.cu — projected-score mode: keys projected to rank R (= 16) when they are
// appended to the cache, and Pass 1 computed from the projected keys.
//
// The reference's Pass 1 (_pass1_projection_kernel, dcr_attention/kernel/triton/
// topk_axis_pass1.py:29) reads every 64-dim key row (128 B in 16-bit caches) to score it
// against the unit query u. In projected mode the cache also holds KP = K . P (P a fixed
// 64 x R fp32 matrix, R = 16), written once per token by the append kernel below, and the
// scores are s = bf16(KP . (u . P)): 32 B per key row instead of 128 B, a quarter of
// Pass 1's HBM traffic. Selection (Pass 2) and attention (Pass 3, on the full K and V)
// are unchanged. The reference has no such mode; the arithmetic below is pinned against
// the CPU restatement in oracle/dcr_oracle.c (oracle_project_keys,
// oracle_query_projection, oracle_scores_projected), whose fmaf chains it follows:
//   KP[n, j] = round_T(sum_{d=0..63} K[n, d] * P[d, j])      (fmaf chain in d)
//   qp[h, j] = sum_{d=0..63} u[h, d] * P[d, j]                (fmaf chain in d)
//   s[h, n]  = bf16_rne(e + o), e = sum over even j, o = sum over odd j of
//              KP[n, j] * qp[h, j]                              (two fmaf chains in j)
// The two chains are the two lanes of packed FMAs (fma.rn.f32x2, the same rounding as
// fmaf per lane) over the element pairs (j, j + 1) that the widening of a row produces.
//
// Append kernel: a CTA of 256 threads takes 16 rows; 16 threads per row copy its K and V
// chunks (16-byte loads and stores) and then compute its R projected elements from the
// row staged in shared memory (P staged there too). Score kernel: a CTA takes 512
// positions of one (b, h_kv) row group; the G unit queries and their projections are
// computed in the CTA prologue; each thread then streams 4 consecutive KP rows (4 x 32 B
// contiguous, 16-byte loads) and stores 4 consecutive keys per head (8-byte stores).
#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

constexpr int kProjR = DCR_PROJ_RANK;
constexpr int kApThreads = 256;
constexpr int kApRows = kApThreads / kProjR;  // 16 rows per CTA

struct AppendParams {
  const void* k_new;   // [B, H_kv, n_new, D] with strides nsb, nsh (rows contiguous)
  const void* v_new;
  int64_t nsb, nsh;
  void* k_cache;       // [B, H_kv, N_max, D] with strides csb, csh (may be null: no copy)
  void* v_cache;
  int64_t csb, csh;
  void* kp;            // [B, H_kv, N_max, R] with strides psb, psh (may be null)
  int64_t psb, psh;
  const float* P;      // [D][R]
  int H_kv, n_new, pos;
  int64_t rows;        // B * H_kv * n_new
};

template <typename T>
__global__ void __launch_bounds__(kApThreads) append_kernel(const AppendParams p) {
  constexpr int kChunks = RowTraits<T>::kChunks;  // 16-byte chunks per row (8 or 16)
  constexpr int kPer = ElemTraits<T>::kPerChunk;
  __shared__ float P_s[kD * kProjR];
  __shared__ float k_s[kApRows][kD + 1];
  const int tid = threadIdx.x;
  if (p.kp != nullptr)
    for (int i = tid; i < kD * kProjR; i += kApThreads) P_s[i] = p.P[i];
  const int r_local = tid / kProjR;  // row of this thread within the CTA
  const int j = tid % kProjR;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kApRows + r_local;
  const bool live = r < p.rows;
  int64_t b = 0, hk = 0, n = 0;
  if (live) {
    n = r % p.n_new;
    const int64_t g = r / p.n_new;
    hk = g % p.H_kv;
    b = g / p.H_kv;
  }
  const uint8_t* ksrc = static_cast<const uint8_t*>(p.k_new) + (b * p.nsb + hk * p.nsh + n * kD) * sizeof(T);
  const uint8_t* vsrc = static_cast<const uint8_t*>(p.v_new) + (b * p.nsb + hk * p.nsh + n * kD) * sizeof(T);
  const int64_t crow = b * p.csb + hk * p.csh + (p.pos + n) * kD;
  // copy: the row's 2 * kChunks chunks over its 16 threads
  if (live && p.k_cache != nullptr) {
    for (int c = j; c < 2 * kChunks; c += kProjR) {
      const bool is_v = c >= kChunks;
      const int cc = is_v ? c - kChunks : c;
      const uint4 w = reinterpret_cast<const uint4*>(is_v ? vsrc : ksrc)[cc];
      uint8_t* dst = static_cast<uint8_t*>(is_v ? p.v_cache : p.k_cache) + crow * sizeof(T);
      reinterpret_cast<uint4*>(dst)[cc] = w;
    }
  }
  if (p.kp == nullptr) return;
  // stage the K row as fp32 (16 threads, kChunks chunks)
  if (live) {
    for (int c = j; c < kChunks; c += kProjR) {
      float f[kPer];
      ElemTraits<T>::widen(reinterpret_cast<const uint4*>(ksrc)[c], f);
#pragma unroll
      for (int e = 0; e < kPer; ++e) k_s[r_local][c * kPer + e] = f[e];
    }
  }
  __syncthreads();
  if (!live) return;
  float acc = 0.0f;
#pragma unroll 16
  for (int d = 0; d < kD; ++d) acc = fmaf(k_s[r_local][d], P_s[d * kProjR + j], acc);
  const int64_t prow = b * p.psb + hk * p.psh + (p.pos + n) * kProjR;
  ElemTraits<T>::store(static_cast<T*>(p.kp) + prow, j, acc);
}

// ---- projected Pass 1 ------------------------------------------------------------------
constexpr int kSpThreads = 128;
constexpr int kSpRpt = 4;                              // rows per thread
constexpr int kSpRows = kSpThreads * kSpRpt;           // positions per CTA

struct ProjScoreParams {
  const void* kp;      // [B, H_kv, N, R], strides psb, psh (rows of R contiguous)
  int64_t psb, psh;
  const void* q;       // [B, H, D]
  const float* P;      // [D][R]
  const float* qp;     // optional [B*H][R]: the projected unit queries (else computed here)
  float eps;
  int H_kv, N, tiles;  // tiles = ceil(N / kSpRows) per (b, h_kv)
  int cpg;             // CTAs per (b, h_kv): CTA c of a group takes tiles c, c + cpg, ...
  uint16_t* out;       // [B*H, stride]
  int64_t stride;
  int keys_out;
};

template <typename T, int G>
__global__ void __launch_bounds__(kSpThreads) score_proj_kernel(const ProjScoreParams p) {
  constexpr int kRowChunks = kProjR * sizeof(T) / 16;  // 16-byte chunks per KP row: 2 or 4
  __shared__ float u_s[G][kD];
  __shared__ float qp_s[G][kProjR];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int g = blockIdx.x / p.cpg;   // (b, h_kv)
  const int c0 = blockIdx.x % p.cpg;
  const int b = g / p.H_kv, hk = g % p.H_kv;
  const T* base = static_cast<const T*>(p.kp) + b * p.psb + hk * p.psh;
  // The KP rows of tile `tile` this thread scores (zero past the end of the row).
  auto load_tile = [&](int tile, uint4 (&raw)[kSpRpt][kRowChunks]) {
    const int64_t n0 = static_cast<int64_t>(tile) * kSpRows + static_cast<int64_t>(tid) * kSpRpt;
#pragma unroll
    for (int rr = 0; rr < kSpRpt; ++rr) {
      const uint4* src = reinterpret_cast<const uint4*>(base + (n0 + rr) * kProjR);
#pragma unroll
      for (int c = 0; c < kRowChunks; ++c)
        raw[rr][c] = (tile < p.tiles && n0 + rr < p.N) ? __ldcs(src + c) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // the first tile's loads are in flight while the queries are prepared
  uint4 raw[kSpRpt][kRowChunks];
  load_tile(c0, raw);

  // unit queries of the G heads (one warp each; unit_query_warp of dcr_score.cu, the same
  // arithmetic as Pass 1), then their projections
  if (p.qp != nullptr) {
    for (int i = tid; i < G * kProjR; i += kSpThreads)
      qp_s[i / kProjR][i % kProjR] = __ldg(p.qp + static_cast<int64_t>(g) * G * kProjR + i);
  } else {
    for (int h = warp; h < G; h += kSpThreads / 32) {
      const char* q_row =
          static_cast<const char*>(p.q) + (static_cast<size_t>(g) * G + h) * kD * sizeof(T);
      unit_query_warp<T>(q_row, p.eps, &u_s[h][0]);
    }
    __syncthreads();
    for (int i = tid; i < G * kProjR; i += kSpThreads) {
      const int h = i / kProjR, jj = i % kProjR;
      float acc = 0.0f;
#pragma unroll 16
      for (int d = 0; d < kD; ++d) acc = fmaf(u_s[h][d], __ldg(p.P + d * kProjR + jj), acc);
      qp_s[h][jj] = acc;
    }
  }
  __syncthreads();
  float2 qp[G][kProjR / 2];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int m = 0; m < kProjR / 2; ++m) qp[h][m] = make_float2(qp_s[h][2 * m], qp_s[h][2 * m + 1]);

  for (int tile = c0; tile < p.tiles; tile += p.cpg) {
    const int64_t n0 = static_cast<int64_t>(tile) * kSpRows + static_cast<int64_t>(tid) * kSpRpt;
    uint4 nxt[kSpRpt][kRowChunks];
    load_tile(tile + p.cpg, nxt);  // next tile in flight during this one's arithmetic
    uint16_t key[G][kSpRpt];
#pragma unroll
    for (int rr = 0; rr < kSpRpt; ++rr) {
      float2 kr[kProjR / 2];  // element pairs (2m, 2m + 1)
#pragma unroll
      for (int c = 0; c < kRowChunks; ++c) {
        const uint32_t w[4] = {raw[rr][c].x, raw[rr][c].y, raw[rr][c].z, raw[rr][c].w};
        if constexpr (sizeof(T) == 4) {
          kr[2 * c] = make_float2(__uint_as_float(w[0]), __uint_as_float(w[1]));
          kr[2 * c + 1] = make_float2(__uint_as_float(w[2]), __uint_as_float(w[3]));
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) kr[4 * c + i] = ElemTraits<T>::widen2(w[i]);
        }
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int m = 0; m < kProjR / 2; ++m) acc = ffma2(kr[m], qp[h][m], acc);
        const uint16_t bits = f32_to_bf16_bits(acc.x + acc.y);
        key[h][rr] = p.keys_out ? static_cast<uint16_t>(bf16_order_key(bits)) : bits;
      }
    }
    if (n0 < p.N) {
#pragma unroll
      for (int h = 0; h < G; ++h) {
        uint16_t* dst = p.out + (static_cast<int64_t>(g) * G + h) * p.stride + n0;
        if (n0 + kSpRpt <= p.N && (p.stride & 3) == 0) {
          uint2 w;
          w.x = static_cast<uint32_t>(key[h][0]) | (static_cast<uint32_t>(key[h][1]) << 16);
          w.y = static_cast<uint32_t>(key[h][2]) | (static_cast<uint32_t>(key[h][3]) << 16);
          *reinterpret_cast<uint2*>(dst) = w;
        } else {
#pragma unroll
          for (int rr = 0; rr < kSpRpt; ++rr)
            if (n0 + rr < p.N) dst[rr] = key[h][rr];
        }
      }
    }
#pragma unroll
    for (int rr = 0; rr < kSpRpt; ++rr)
#pragma unroll
      for (int c = 0; c < kRowChunks; ++c) raw[rr][c] = nxt[rr][c];
  }
}

template <typename T>
static int launch_append_t(const AppendParams& p, cudaStream_t st) {
  const int64_t blocks = (p.rows + kApRows - 1) / kApRows;
  if (blocks > 0x7fffffff) return DCR_ERR_SHAPE;
  if (blocks == 0) return DCR_OK;
  append_kernel<T><<<static_cast<unsigned>(blocks), kApThreads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

int launch_append(const void* k_new, const void* v_new, int64_t nsb, int64_t nsh, void* k_cache,
                  void* v_cache, int64_t csb, int64_t csh, void* kp, int64_t psb, int64_t psh,
                  const float* P, int B, int H_kv, int n_new, int pos, int dtype,
                  cudaStream_t st) {
  AppendParams p;
  p.k_new = k_new;
  p.v_new = v_new;
  p.nsb = nsb;
  p.nsh = nsh;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.csb = csb;
  p.csh = csh;
  p.kp = kp;
  p.psb = psb;
  p.psh = psh;
  p.P = P;
  p.H_kv = H_kv;
  p.n_new = n_new;
  p.pos = pos;
  p.rows = static_cast<int64_t>(B) * H_kv * n_new;
  switch (dtype) {
    case DCR_DTYPE_BF16: return launch_append_t<__nv_bfloat16>(p, st);
    case DCR_DTYPE_F16: return launch_append_t<__half>(p, st);
    case DCR_DTYPE_F32: return launch_append_t<float>(p, st);
    default: return DCR_ERR_DTYPE;
  }
}

// Resident CTAs per SM of one instantiation (registers decide it: 102 for the 16-bit G = 4
// kernel, which rounds to 4 CTAs of 128 threads per SM).
template <typename T, int G>
static int score_proj_ctas_per_sm() {
  static int n = 0;
  if (n == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, score_proj_kernel<T, G>, kSpThreads, 0) !=
            cudaSuccess ||
        v < 1)
      v = 1;
    n = v;
  }
  return n;
}

template <typename T, int G>
static int launch_score_proj_tg(ProjScoreParams p, int B, cudaStream_t st) {
  // One wave spread over the (b, h_kv) groups, each CTA looping over its group's tiles (the
  // unit queries and projections are computed once per CTA). The CTAs per group are the
  // fewest that keep the longest CTA at ceil(tiles / (slots per group)) tiles, so a group's
  // CTAs take equal shares and the grid never spills into a second wave (sized for 5 CTAs
  // per SM where registers allow 4, the hero grid ran 768 CTAs on 592 slots).
  const int64_t groups = static_cast<int64_t>(B) * p.H_kv;
  const int64_t slots = static_cast<int64_t>(device_sm_count()) * score_proj_ctas_per_sm<T, G>();
  int64_t cpg = slots / groups;
  if (cpg > p.tiles) cpg = p.tiles;
  if (cpg < 1) cpg = 1;
  const int64_t per_cta = (p.tiles + cpg - 1) / cpg;
  cpg = (p.tiles + per_cta - 1) / per_cta;
  p.cpg = static_cast<int>(cpg);
  const int64_t blocks = groups * cpg;
  if (blocks > 0x7fffffff) return DCR_ERR_SHAPE;
  score_proj_kernel<T, G><<<static_cast<unsigned>(blocks), kSpThreads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

template <typename T>
static int launch_score_proj_t(ProjScoreParams p, int B, int G, cudaStream_t st) {
  switch (G) {
    case 1: return launch_score_proj_tg<T, 1>(p, B, st);
    case 2: return launch_score_proj_tg<T, 2>(p, B, st);
    case 4: return launch_score_proj_tg<T, 4>(p, B, st);
    case 8: return launch_score_proj_tg<T, 8>(p, B, st);
    default: return DCR_ERR_SHAPE;
  }
}

int launch_score_projected(const void* KP, int dtype, int64_t p_stride_b, int64_t p_stride_h,
                           const void* Q, const float* P, const float* qp, float eps, int B,
                           int H, int H_kv, int N, uint16_t* scores, int64_t s_stride,
                           int keys_out, cudaStream_t st) {
  ProjScoreParams p;
  p.qp = qp;
  p.kp = KP;
  p.psb = p_stride_b;
  p.psh = p_stride_h;
  p.q = Q;
  p.P = P;
  p.eps = eps;
  p.H_kv = H_kv;
  p.N = N;
  p.tiles = (N + kSpRows - 1) / kSpRows;
  p.out = scores;
  p.stride = s_stride;
  p.keys_out = keys_out;
  const int G = H / H_kv;
  switch (dtype) {
    case DCR_DTYPE_BF16: return launch_score_proj_t<__nv_bfloat16>(p, B, G, st);
    case DCR_DTYPE_F16: return launch_score_proj_t<__half>(p, B, G, st);
    case DCR_DTYPE_F32: return launch_score_proj_t<float>(p, B, G, st);
    default: return DCR_ERR_DTYPE;
  }
}

}  // namespace dcr
