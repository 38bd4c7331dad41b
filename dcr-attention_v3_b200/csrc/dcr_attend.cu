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
// 128-byte row, fully coalesced) into a 3-stage ring of 128-byte-swizzled shared-memory
// tiles (4 CTAs per SM); the indices of a tile are loaded two iterations before its
// copies are issued.
// Warp w owns rows 16w..16w+15 of every tile and keeps its own online-softmax state
// (in base 2, with the 1/sqrt(D) scale and log2(e) folded into the scores; the running
// maximum is only refreshed when a warp vote sees a score more than 2^8 above it):
// scores use two lanes per row (32 dims each, Q held in registers) and the P.V product
// one lane per dimension pair, so a tile needs no block barrier besides the stage
// hand-over. The 4 warp states are merged at the end. Each CTA writes its partial
// (m, l, o[64]) to the workspace; the last CTA of a (b, h) to finish (atomic ticket,
// no waiting) merges the S partials:
//     M = max_s m_s,  O = sum_s 2^{m_s - M} o_s / sum_s 2^{m_s - M} l_s.
// Every gathered index is checked against [0, N); a bad one is skipped (zero row, zero
// weight) and raises DCR_ERR_DEVICE_INDEX.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include "dcr_common.cuh"
#include "dcr_internal.h"
#include "dcr_peer.cuh"

namespace dcr {

constexpr int kP3Threads = 128;
constexpr int kP3Tile = 64;
#ifndef DCR_P3_CTAS_PER_SM
#define DCR_P3_CTAS_PER_SM 4
#endif

template <typename T>
struct P3Cfg {
  static constexpr int kRowBytes = RowTraits<T>::kRowBytes;
  static constexpr int kChunks = RowTraits<T>::kChunks;
  static constexpr int kTileBytes = kP3Tile * kRowBytes;  // one of K or V
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = 3;
  static constexpr int kMinBlocks = sizeof(T) == 4 ? 2 : DCR_P3_CTAS_PER_SM;  // CTAs per SM
  static constexpr int kSmem = 1024 + kStages * kStageBytes;
};

struct P3Params {
  const void* q;
  const void* k;
  const void* v;
  int64_t ksb, ksh, vsb, vsh;  // element strides
  const int32_t* idx;       // [rows][k_eff]: row r's list starts at r * k_eff
  const int32_t* counts;    // optional [rows]: row r uses its first counts[r] entries
  int H, H_kv, G, N, k_eff, S;
  void* o;                  // [rows][D] output (when state == nullptr)
  float* state;             // optional [rows][D + 2]: (m, l, o) instead of O
  float* part;
  int* counters;
  PeerView pv;              // pv.world > 0 (with state): publish each row's state into
                            // the ranks' exchange buffers instead (exchange 2)
  int64_t rows_per_head;    // TMA gather: cache rows of (b, h_kv) start at
                            // (b * H_kv + h_kv) * rows_per_head in the 2-D tensor maps
};

// Writes a row's (m, l, o) to the state output, or in peer mode publishes it into slot
// `rank` of every rank's exchange buffer as epoch-tagged words. Called by all threads of
// the CTA; threads 0..D-1 hold o, thread 0 holds m and l.
__device__ __forceinline__ void write_state_row(const P3Params& p, int64_t row, float m, float l,
                                                float o) {
  const int tid = threadIdx.x;
  if (p.pv.world > 0) {
    const uint32_t epoch = step_epoch(p.pv);
    for (int i = 0; i < p.pv.world; ++i) {  // own slot first, then the next ranks in turn
      const int q = peer_order(p.pv, i);
      uint64_t* dst = p.pv.st(q, p.pv.rank, row);
      if (tid < kD) ll_put(dst + 2 + tid, __float_as_uint(o), epoch);
      if (tid == 0) {
        ll_put(dst, __float_as_uint(m), epoch);
        ll_put(dst + 1, __float_as_uint(l), epoch);
      }
    }
    return;
  }
  float* st = p.state + row * (kD + 2);
  if (tid < kD) st[2 + tid] = o;
  if (tid == 0) {
    st[0] = m;
    st[1] = l;
  }
}

template <typename T, bool kTma>
__global__ void __launch_bounds__(kP3Threads, P3Cfg<T>::kMinBlocks)
    attend_kernel(const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const P3Params p) {
  using Cfg = P3Cfg<T>;
  constexpr int kChunks = Cfg::kChunks;
  constexpr int kPer = ElemTraits<T>::kPerChunk;
  constexpr int kHalfChunks = kChunks / 2;
  constexpr int kRowsPerPass = kP3Threads / kChunks;  // 16 (16-bit) or 8 (fp32)
  constexpr int kPasses = kP3Tile / kRowsPerPass;     // 4 or 8
  constexpr int kWarps = kP3Threads / 32;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ float2 P_s[kP3Tile];  // {p, p}: one packed operand of the P.V FMA
  __shared__ float o_red[kWarps][kD];
  __shared__ float m_red[kWarps];
  __shared__ float l_red[kWarps];
  __shared__ int is_last;
  __shared__ alignas(8) uint64_t full_bar[Cfg::kStages];  // TMA: one per stage

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

  int row_k = p.k_eff;
  if (p.counts != nullptr) row_k = min(max(__ldg(p.counts + row), 0), p.k_eff);
  const int64_t p0 = static_cast<int64_t>(s) * row_k / p.S;
  const int64_t p1 = static_cast<int64_t>(s + 1) * row_k / p.S;
  const int cnt = static_cast<int>(p1 - p0);
  const int ntiles = (cnt + kP3Tile - 1) / kP3Tile;
  const int32_t* idx_row = p.idx + row * p.k_eff + p0;
  const uint8_t* kbase = static_cast<const uint8_t*>(p.k) + (b * p.ksb + hk * p.ksh) * static_cast<int64_t>(sizeof(T));
  const uint8_t* vbase = static_cast<const uint8_t*>(p.v) + (b * p.vsb + hk * p.vsh) * static_cast<int64_t>(sizeof(T));

  // Q half owned by this thread (two lanes per row in the score phase).
  const int half = lane & 1;
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

  // Gather assignment: thread copies chunk `cchunk` of rows rbase + i * kRowsPerPass.
  const int cchunk = tid % kChunks;
  const int rbase = tid / kChunks;
  const int64_t tma_row0 = (static_cast<int64_t>(b) * p.H_kv + hk) * p.rows_per_head;
  if constexpr (kTma) {
    if (tid == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
#pragma unroll
      for (int i = 0; i < Cfg::kStages; ++i) mbar_init(&full_bar[i], 1);
      fence_mbar_init();
    }
    __syncthreads();
  }

  // Indices of the rows this thread copies in tile tt (-1: past the end of the list).
  // TMA: lane l < 16 of warp 0 gathers rows 4l .. 4l + 3 of the tile.
  auto load_idx = [&](int tt, int32_t (&n)[kPasses]) {
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
      const int pos = kTma ? tt * kP3Tile + 4 * lane + i : tt * kP3Tile + rbase + i * kRowsPerPass;
      const bool mine = !kTma || (warp == 0 && lane < kP3Tile / 4 && i < 4);
      n[i] = (mine && pos < cnt) ? __ldg(idx_row + pos) : -1;
    }
  };
  auto issue = [&](int tt, const int32_t (&n)[kPasses]) {
    if constexpr (kTma) {
      if (tt < ntiles && warp == 0) {
        const int stage = tt % Cfg::kStages;
        uint8_t* kt = smem + stage * Cfg::kStageBytes;
        uint8_t* vt = kt + Cfg::kTileBytes;
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
        __syncwarp();
        if (lane < kP3Tile / 4) {
          int r[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            int nn = n[i];
            if (nn < 0 || nn >= p.N) {
              // past the list: any valid row (masked by `valid`); a bad index: row 0 of
              // the head, reported
              if (nn >= 0 || tt * kP3Tile + 4 * lane + i < cnt) raise_status(DCR_ERR_DEVICE_INDEX);
              nn = 0;
            }
            r[i] = static_cast<int>(tma_row0 + nn);
          }
          tma_gather4(kt + 4 * lane * Cfg::kRowBytes, &kmap, &full_bar[stage], 0, r[0], r[1], r[2], r[3]);
          tma_gather4(vt + 4 * lane * Cfg::kRowBytes, &vmap, &full_bar[stage], 0, r[0], r[1], r[2], r[3]);
        }
      }
      return;
    }
    if (tt < ntiles) {
      uint8_t* kt = smem + (tt % Cfg::kStages) * Cfg::kStageBytes;
      uint8_t* vt = kt + Cfg::kTileBytes;
#pragma unroll
      for (int i = 0; i < kPasses; ++i) {
        const int r = rbase + i * kRowsPerPass;
        int64_t nn = n[i];
        uint32_t bytes = 16;
        if (nn < 0 || nn >= p.N) {
          if (nn >= 0 || tt * kP3Tile + r < cnt) {
            if (cchunk == 0) raise_status(DCR_ERR_DEVICE_INDEX);
          }
          nn = 0;
          bytes = 0;  // zero-fill, read nothing
        }
        const uint32_t off = swz_offset(r, cchunk, kP3Tile);
        cp_async_16(kt + off, kbase + nn * Cfg::kRowBytes + cchunk * 16, bytes);
        cp_async_16(vt + off, vbase + nn * Cfg::kRowBytes + cchunk * 16, bytes);
      }
    }
    cp_async_commit();  // always commit so group counting stays uniform
  };

  {
    int32_t n0[kPasses];
#pragma unroll
    for (int i = 0; i < Cfg::kStages - 1; ++i) {
      load_idx(i, n0);
      issue(i, n0);
    }
  }
  // Index prefetch two iterations deep: n_next is issued this iteration, n_after next.
  int32_t n_next[kPasses], n_after[kPasses];
  load_idx(Cfg::kStages - 1, n_next);
  load_idx(Cfg::kStages, n_after);

  // Per-warp online-softmax state: warp w owns rows 16w .. 16w+15 of every tile.
  float m_w = -INFINITY;
  float l_part = 0.0f;       // lanes with half == 0 accumulate their row's weights
  float2 oe = make_float2(0.0f, 0.0f);  // dims 2*lane, 2*lane+1 (even rows)
  float2 oo = make_float2(0.0f, 0.0f);  // (odd rows)
  const int r_own = warp * 16 + (lane >> 1);

  for (int tt = 0; tt < ntiles; ++tt) {
    if constexpr (kTma) {
      mbar_wait_bounded(&full_bar[tt % Cfg::kStages], (tt / Cfg::kStages) & 1u);
    } else {
      cp_async_wait<Cfg::kStages - 2>();
    }
    __syncthreads();  // tile tt visible to all; stage (tt-1) free for reuse
    issue(tt + Cfg::kStages - 1, n_next);
#pragma unroll
    for (int i = 0; i < kPasses; ++i) n_next[i] = n_after[i];
    load_idx(tt + Cfg::kStages + 1, n_after);

    const uint8_t* kt = smem + (tt % Cfg::kStages) * Cfg::kStageBytes;
    const uint8_t* vt = kt + Cfg::kTileBytes;
    const uint32_t kt_addr = smem_u32(kt);
    const uint32_t vt_addr = smem_u32(vt);

    // ---- scores of the warp's 16 rows: dims [32*half, 32*half + 32) per lane; two
    // chains (even and odd dims) advanced by one packed FMA ----
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < kHalfChunks; ++c) {
      float f[kPer];
      ElemTraits<T>::widen(lds128(kt_addr + swz_offset(r_own, half * kHalfChunks + c, kP3Tile)), f);
#pragma unroll
      for (int e = 0; e < kPer; e += 2)
        acc = ffma2(make_float2(f[e], f[e + 1]),
                    make_float2(qf[c * kPer + e], qf[c * kPer + e + 1]), acc);
    }
    // z in log2 units: dot * (1/sqrt(64)) * log2(e); p = 2^(z - m) with m the warp's
    // reference point (its running maximum, kept unless a score exceeds it by 2^8).
    float z = acc.x + acc.y;
    z += __shfl_xor_sync(0xffffffffu, z, 1);
    z *= 0.125f * 1.4426950408889634f;
    const bool valid = tt * kP3Tile + r_own < cnt;
    float alpha = 1.0f;
    if (__any_sync(0xffffffffu, valid && !(z <= m_w + 8.0f))) {
      float mt = valid ? z : -INFINITY;
#pragma unroll
      for (int off = 2; off < 32; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m_w, mt);
      alpha = (m_w == -INFINITY) ? 0.0f : exp2f(m_w - m_new);
      m_w = m_new;
    }
    const float pr = valid ? exp2f(z - m_w) : 0.0f;
    if (half == 0) P_s[r_own] = make_float2(pr, pr);
    l_part = l_part * alpha + (half == 0 ? pr : 0.0f);
    __syncwarp();

    // ---- P.V over the warp's rows: lane owns dims 2*lane, 2*lane+1; even and odd rows
    // accumulate separately (shorter dependent chains) and are added after the loop ----
    oe.x *= alpha;
    oe.y *= alpha;
    oo.x *= alpha;
    oo.y *= alpha;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int rr = warp * 16 + i;
      const float2 pw = P_s[rr];
      float2 v2;
      if constexpr (sizeof(T) == 4) {
        const uint32_t addr = vt_addr + swz_offset(rr, lane >> 1, kP3Tile) + (lane & 1) * 8;
        asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v2.x), "=f"(v2.y) : "r"(addr));
      } else {
        const uint32_t addr = vt_addr + swz_offset(rr, lane >> 2, kP3Tile) + (lane & 3) * 4;
        uint32_t w;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w) : "r"(addr));
        v2 = ElemTraits<T>::widen2(w);
      }
      if (i & 1)
        oo = ffma2(pw, v2, oo);
      else
        oe = ffma2(pw, v2, oe);
    }
  }
  const float o0 = oe.x + oo.x;
  const float o1 = oe.y + oo.y;
  if constexpr (!kTma) cp_async_wait<0>();

  // ---- merge the 4 warps' (m, l, o) ----
  float ls = l_part;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
  if (lane == 0) {
    m_red[warp] = m_w;
    l_red[warp] = ls;
  }
  o_red[warp][2 * lane] = o0;
  o_red[warp][2 * lane + 1] = o1;
  __syncthreads();
  float M = m_red[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) M = fmaxf(M, m_red[w]);
  float sc[kWarps];
  float l_cta = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    sc[w] = (m_red[w] == -INFINITY) ? 0.0f : exp2f(m_red[w] - M);
    l_cta = fmaf(sc[w], l_red[w], l_cta);
  }
  float od = 0.0f;
  if (tid < kD) {
#pragma unroll
    for (int w = 0; w < kWarps; ++w) od = fmaf(sc[w], o_red[w][tid], od);
  }

  if (p.S == 1) {
    if (p.state != nullptr) {
      write_state_row(p, row, M, l_cta, od);
    } else if (tid < kD) {
      ElemTraits<T>::store(p.o, static_cast<int>(row * kD + tid), od / l_cta);
    }
    return;
  }

  float* mine = p.part + (row * p.S + s) * (kD + 2);
  if (tid < kD) mine[2 + tid] = od;
  if (tid == 0) {
    mine[0] = M;
    mine[1] = l_cta;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(&p.counters[row], 1) == p.S - 1) ? 1 : 0;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  float Mg = -INFINITY, L = 0.0f, o = 0.0f;
  if (tid < kD) {
    const float* base = p.part + row * p.S * (kD + 2);
    for (int t = 0; t < p.S; ++t) Mg = fmaxf(Mg, __ldcg(base + t * (kD + 2)));
    for (int t = 0; t < p.S; ++t) {
      const float* pt = base + t * (kD + 2);
      const float mt = __ldcg(pt);
      const float w = (mt == -INFINITY) ? 0.0f : exp2f(mt - Mg);
      L = fmaf(w, __ldcg(pt + 1), L);
      o = fmaf(w, __ldcg(pt + 2 + tid), o);
    }
  }
  if (p.state != nullptr) {
    write_state_row(p, row, Mg, L, o);
  } else if (tid < kD) {
    ElemTraits<T>::store(p.o, static_cast<int>(row * kD + tid), o / L);
  }
  if (tid == 0) p.counters[row] = 0;
}

int attend_splits(int rows, int k_eff) {
  const int slots = device_sm_count() * DCR_P3_CTAS_PER_SM;  // resident CTAs (16-bit caches)
  int S = slots / (rows > 0 ? rows : 1);
  const int max_by_tiles = (k_eff + kP3Tile - 1) / kP3Tile;
  if (S > max_by_tiles) S = max_by_tiles;
  if (S > 64) S = 64;
  if (S < 1) S = 1;
  return S;
}

// TMA gathers need one row index space per cache: rows of (b, h_kv) at a fixed pitch
// (batch stride = H_kv x head stride, head stride a whole number of rows, K and V alike),
// 16-bit elements (a 128-byte row is one swizzle span) and int32 row indices. They are
// opt-in (DCR_ATTEND_GATHER=tma in the environment): at the hero shape the 16-byte
// cp.async path is faster (35 us against 45 us per launch), the TMA unit's rate for
// 128-byte rows being lower than the load units' for the same bytes.
static bool tma_gather_allowed() {
  static const bool allowed = [] {
    const char* e = getenv("DCR_ATTEND_GATHER");
    return e != nullptr && strcmp(e, "tma") == 0;
  }();
  return allowed;
}

template <typename T>
static bool encode_row_map(CUtensorMap* map, const void* base, int64_t rows) {
  EncodeTiledFn encode = get_encode_fn();
  if (!encode) return false;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD * sizeof(T))};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kD), 1u};  // gather4: one row high
  const cuuint32_t estr[2] = {1u, 1u};
  return encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
static int launch_attend_t(P3Params p, int B, cudaStream_t st) {
  const int64_t grid = static_cast<int64_t>(B) * p.H_kv * p.S * p.G;
  if (grid > 0x7fffffff) return DCR_ERR_SHAPE;
  CUtensorMap kmap, vmap;
  memset(&kmap, 0, sizeof(kmap));
  memset(&vmap, 0, sizeof(vmap));
  bool tma = false;
  if constexpr (sizeof(T) == 2) {
    const int64_t rph = p.ksh / kD;
    const int64_t rows = static_cast<int64_t>(B) * p.H_kv * rph;
    tma = tma_gather_allowed() && p.ksh % kD == 0 && p.ksh == p.vsh && p.ksb == p.vsb &&
          (B == 1 || p.ksb == p.H_kv * p.ksh) && rows > 0 && rows <= 0x7fffffffLL &&
          encode_row_map<T>(&kmap, p.k, rows) && encode_row_map<T>(&vmap, p.v, rows);
    p.rows_per_head = rph;
    if (tma) {
      constexpr int smem = P3Cfg<T>::kSmem;
      if (ensure_smem_attr(reinterpret_cast<const void*>(&attend_kernel<T, true>), smem) !=
          cudaSuccess)
        return DCR_ERR_CUDA;
      attend_kernel<T, true><<<static_cast<unsigned>(grid), kP3Threads, smem, st>>>(kmap, vmap, p);
      return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
    }
  }
  constexpr int smem = P3Cfg<T>::kSmem;
  if (ensure_smem_attr(reinterpret_cast<const void*>(&attend_kernel<T, false>), smem) !=
      cudaSuccess)
    return DCR_ERR_CUDA;
  attend_kernel<T, false><<<static_cast<unsigned>(grid), kP3Threads, smem, st>>>(kmap, vmap, p);
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

int launch_attend(const void* Q, const void* K, const void* V, int dtype, int64_t k_stride_b,
                  int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_h,
                  const int32_t* idx, const int32_t* counts, int B, int H, int H_kv, int N,
                  int k_eff, void* O, float* state, int splits, float* partials, int* counters,
                  const PeerView* pv, cudaStream_t st) {
  P3Params p;
  p.q = Q;
  p.k = K;
  p.v = V;
  p.ksb = k_stride_b;
  p.ksh = k_stride_h;
  p.vsb = v_stride_b;
  p.vsh = v_stride_h;
  p.idx = idx;
  p.counts = counts;
  p.H = H;
  p.H_kv = H_kv;
  p.G = H / H_kv;
  p.N = N;
  p.k_eff = k_eff;
  p.S = splits;
  p.o = O;
  p.state = state;
  p.pv.world = 0;
  if (pv != nullptr) p.pv = *pv;
  p.rows_per_head = 0;
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
