// dcr_attend_union.cu — Pass 3 over the union of a KV group's selections, on tensor cores
// (16-bit caches).
//
// The per-head Pass 3 (dcr_attend.cu) gathers each (b, h) row's k_eff selected K and V rows
// separately; the G query heads of one KV head select overlapping rows (at c = 0.15 and
// G = 4 the union is ~78% of the per-head total), so L2 and the SMs move every shared row up
// to G times. Here a CTA takes one (b, h_kv) group and one range of positions, builds the
// union of the G heads' selections inside the range — from the selection bitmaps Pass 2
// writes in the decode step (G words per thread), or, where Pass 2 wrote index lists, by
// searching each head's ascending list — and gathers each union row once. All G heads are
// scored against every union row and the rows a head did not select are masked: masked
// dense work, which on CUDA cores cost 3x the arithmetic of the selected pairs, is cheap
// on the tensor cores.
//
// Per 64-row tile, warp w takes union rows [16w, 16w + 16):
//   S = Q K^T   mma.sync m16n8k16 (rows: the G heads, zero-padded to 16; fp32 accumulation
//               of exact 16-bit products), scaled by 1/8 and log2(e), masked to -inf;
//   online softmax per head in base 2 (per-warp running max and sum, merged at the end);
//   O += P V    mma.sync m16n8k16 with P split into two 16-bit parts (hi = rn(p),
//               lo = rn(p - hi)), so the weights keep ~16 significant bits: the hi parts
//               are A rows 0..7 and the lo parts rows 8..15 of one MMA, whose two output
//               halves are added when the partial is written.
// A masked row has weight exactly 0; if a V row in a warp's tile holds a non-finite value
// (0 x inf would reach heads that did not select the row), that warp computes the tile's
// P.V with scalar fp32 FMAs over each head's own rows instead.
//
// The CTAs of a group each write (m, l, o) per head into the workspace partials, laid out
// group-major ([group][split][head][66]) so that a group's partials are one block; the last
// CTA (atomic ticket per group, reset by Pass 2 of the next step) merges them into O.
//
// The kernel is launched as a programmatic dependent of Pass 2: its CTAs can start while
// Pass 2's last CTAs drain, load Q, and wait (griddepcontrol.wait) before reading Pass 2's
// results.
#include "dcr_common.cuh"
#include "dcr_internal.h"
#include "dcr_peer.cuh"

namespace dcr {

// Programmatic dependent launch of this kernel behind Pass 2 (compile-time; 0 disables it
// for comparisons).
#ifndef DCR_UNION_PDL
#define DCR_UNION_PDL 1
#endif

constexpr int kUnThreads = 128;
constexpr int kUnWarps = kUnThreads / 32;
constexpr int kUnTile = 64;      // union rows per tile, 16 per warp
constexpr int kUnStages = 3;
constexpr int kUnMaxG = 8;
constexpr int kUnTileBytes = kUnTile * 128;  // one of K or V (16-bit rows of 128 B)
constexpr int kUnStageBytes = 2 * kUnTileBytes;

struct UnionParams {
  const void* q;
  const void* k;
  const void* v;
  int64_t ksb, ksh, vsb, vsh;  // element strides
  const int32_t* idx;          // [rows][k_eff], every row ascending (when bits is null)
  const uint32_t* bits;        // optional [rows][bits_stride] selection bitmaps from Pass 2
  int64_t bits_stride;
  int H, H_kv, G, N, k_eff;
  int S, span;                 // ranges per group and positions per range
  int S_cap;                   // partial slots per group (the workspace's split capacity)
  void* o;                     // [rows][64] (when state is null)
  float* state;                // optional [rows][66]: unnormalised (m, l, o) instead of O,
  PeerView pv;                 // or, with pv.world > 0, published into the ranks' exchange
                               // buffers (the sequence-sharded step's state exchange)
  float* part;                 // [groups][S_cap][G][66]
  int* counters;               // [B * H_kv] tickets
};

template <typename T>
struct UnionMma;

template <>
struct UnionMma<__half> {
  __device__ __forceinline__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  // (x, y) rounded to 16 bits, and the remainders rounded again
  __device__ __forceinline__ static void split(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
  static constexpr uint32_t kExpMask = 0x7c007c00u;  // all-ones exponent: inf or NaN
  static constexpr uint32_t kExpInc = 0x04000400u;
};

template <>
struct UnionMma<__nv_bfloat16> {
  __device__ __forceinline__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static void split(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
  static constexpr uint32_t kExpMask = 0x7f807f80u;
  static constexpr uint32_t kExpInc = 0x00800080u;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Union list entry: 12-bit offset of the position inside the range (span <= 4096) in the low
// bits, the G-bit head mask above it; 16 bits wide when G <= 4, else 32.
template <typename E>
__device__ __forceinline__ E un_entry(int off, uint32_t heads) {
  return static_cast<E>(static_cast<uint32_t>(off) | (heads << 12));
}

// Dynamic shared memory: the ring (3 stages of 64 K rows and 64 V rows), then the list. The
// per-head bitmaps of the range are built inside the ring, which is free until the gathers.
__host__ __device__ constexpr int union_smem_bytes(int span, int entry_bytes) {
  return 128 + kUnStages * kUnStageBytes + span * entry_bytes;
}

// One 64-row tile of the ring for warp `warp`, which takes tile rows [16 warp, 16 warp + 16):
// S = Q K^T on the tensor cores, the scores masked to the rows this lane's head row
// selected (sel(r) for tile row r), online softmax in base 2, O += P V. m_run, l_part and o
// are the warp's running state (see the kernels).
template <typename T, typename Sel>
__device__ __forceinline__ void union_tile(uint32_t kt, uint32_t vt, const uint32_t (&aq)[4][2],
                                           const Sel& sel, float& m_run, float& l_part,
                                           float (&o)[8][4]) {
  using Mma = UnionMma<T>;
  constexpr float kScale = 0.125f * 1.4426950408889634f;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int q4 = lane & 3;
  const int wrow = 16 * warp;  // this warp's first row in the tile

  // S = Q K^T for the warp's 16 rows (two n-tiles of 8)
  float sacc[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
#pragma unroll
    for (int kp = 0; kp < 2; ++kp) {
      // matrices: rows wrow + 8j + (lane & 7), chunks 4kp + (lane >> 3)
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kt + swz_offset(wrow + 8 * j + (lane & 7), 4 * kp + (lane >> 3), kUnTile), b0, b1,
              b2, b3);
      const uint32_t a0[4] = {aq[2 * kp][0], 0u, aq[2 * kp][1], 0u};
      const uint32_t a1[4] = {aq[2 * kp + 1][0], 0u, aq[2 * kp + 1][1], 0u};
      Mma::mma(sacc[j], a0, b0, b1);
      Mma::mma(sacc[j], a1, b2, b3);
    }
  }

  // mask, online softmax (per head row; the row's 16 values sit in the 4 lanes of a quad)
  float z[2][2];
  bool valid[2][2];
  float tmax = -INFINITY;
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      valid[j][e] = sel(wrow + 8 * j + 2 * q4 + e);
      z[j][e] = sacc[j][e] * kScale;
      if (valid[j][e]) tmax = fmaxf(tmax, z[j][e]);
    }
  tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
  tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
  const float m_new = fmaxf(m_run, tmax);
  float alpha = 1.0f;
  if (m_new != -INFINITY) {
    alpha = exp2f(m_run - m_new);  // 0 while m_run is -inf
    m_run = m_new;
  }
  float pw[2][2];
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) pw[j][e] = valid[j][e] ? exp2f(z[j][e] - m_run) : 0.0f;
  l_part = l_part * alpha + (pw[0][0] + pw[0][1]) + (pw[1][0] + pw[1][1]);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    o[nt][0] *= alpha;
    o[nt][1] *= alpha;
    o[nt][2] *= alpha;
    o[nt][3] *= alpha;
  }

  // V fragments of the warp's 16 rows (k) for the 8 dim tiles (n), transposed loads
  uint32_t bv[8][2];
#pragma unroll
  for (int d4 = 0; d4 < 4; ++d4)
    ldsm_x4_t(vt + swz_offset(wrow + 8 * ((lane >> 3) & 1) + (lane & 7), 2 * d4 + (lane >> 4),
                              kUnTile),
              bv[2 * d4][0], bv[2 * d4][1], bv[2 * d4 + 1][0], bv[2 * d4 + 1][1]);
  uint32_t nonfin = 0u;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    nonfin |= (bv[nt][0] & Mma::kExpMask) + Mma::kExpInc;
    nonfin |= (bv[nt][1] & Mma::kExpMask) + Mma::kExpInc;
  }
  if (!__any_sync(0xffffffffu, (nonfin & 0x80008000u) != 0u)) {
    // O += P V with P = hi + lo in one MMA: A rows 0..7 hold the heads' hi parts and rows
    // 8..15 their lo parts, so o[.][0..1] accumulate hi . V and o[.][2..3] lo . V (summed
    // when the partial is written)
    uint32_t a[4];
    Mma::split(pw[0][0], pw[0][1], a[0], a[1]);
    Mma::split(pw[1][0], pw[1][1], a[2], a[3]);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) Mma::mma(o[nt], a, bv[nt][0], bv[nt][1]);
  } else {
    // a non-finite V value in the warp's rows: each head accumulates only its own rows
#pragma unroll 1
    for (int kr = 0; kr < 16; ++kr) {
      const int j = kr >> 3, c = kr & 7;
      const int src = (lane & ~3) | (c >> 1);
      const float w0 = __shfl_sync(0xffffffffu, j ? pw[1][0] : pw[0][0], src);
      const float w1 = __shfl_sync(0xffffffffu, j ? pw[1][1] : pw[0][1], src);
      const float w = (c & 1) ? w1 : w0;
      if (!sel(wrow + kr)) continue;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const uint32_t addr = vt + swz_offset(wrow + kr, nt, kUnTile) + 4 * q4;
        uint32_t vv;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(vv) : "r"(addr));
        const float2 f = ElemTraits<T>::widen2(vv);
        o[nt][0] = fmaf(w, f.x, o[nt][0]);
        o[nt][1] = fmaf(w, f.y, o[nt][1]);
      }
    }
  }
}

// Merges the 4 warps' running (m, l, o) of every head row into one partial per head,
// [G][66] = (m, l, o[64]) at dst. Called by all threads once the ring is free (it stages the
// warps' states there).
__device__ __forceinline__ void union_store_partial(uint8_t* ring, int G, float m_run,
                                                    float l_part, const float (&o)[8][4],
                                                    float* dst) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int hr = lane >> 2;
  const int q4 = lane & 3;
  const bool head_ok = hr < G;
  float* o_red = reinterpret_cast<float*>(ring);                 // [warp][G][64]
  float* m_red = o_red + kUnWarps * kUnMaxG * kD;                // [warp][G]
  float* l_red = m_red + kUnWarps * kUnMaxG;                     // [warp][G]
  float lsum = l_part;
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
  if (head_ok) {
    float* orow = o_red + (warp * kUnMaxG + hr) * kD;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {  // the hi and lo accumulators of union_tile
      orow[8 * nt + 2 * q4] = o[nt][0] + o[nt][2];
      orow[8 * nt + 2 * q4 + 1] = o[nt][1] + o[nt][3];
    }
    if (q4 == 0) {
      m_red[warp * kUnMaxG + hr] = m_run;
      l_red[warp * kUnMaxG + hr] = lsum;
    }
  }
  __syncthreads();
  for (int i = tid; i < G * (kD + 2); i += kUnThreads) {
    const int h = i / (kD + 2), c = i - h * (kD + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kUnWarps; ++w) M = fmaxf(M, m_red[w * kUnMaxG + h]);
    float acc = 0.0f;
    if (c == 0) {
      acc = M;
    } else {
#pragma unroll
      for (int w = 0; w < kUnWarps; ++w) {
        const float mw = m_red[w * kUnMaxG + h];
        const float sc = mw == -INFINITY ? 0.0f : exp2f(mw - M);
        acc += sc * (c == 1 ? l_red[w * kUnMaxG + h] : o_red[(w * kUnMaxG + h) * kD + c - 2]);
      }
    }
    dst[h * (kD + 2) + c] = acc;
  }
}

// The group's last CTA: folds the group's nparts partials ([nparts][G][66] floats at gpart)
// of every head into the outputs of rows row0 .. row0 + G - 1: O (o_out), or the
// unnormalised state (state), or, with pv.world > 0, the state published into the ranks'
// exchange buffers. Called by all threads; the ring is free.
template <typename T>
__device__ __forceinline__ void union_merge(uint8_t* ring, const float* gpart, int nparts, int G,
                                            int64_t row0, void* o_out, float* state,
                                            const PeerView* pv) {
  const int tid = threadIdx.x;
  // The group's partials are one block ([nparts][G][66] floats). They are staged in the ring
  // in chunks of up to `cap` splits (16-byte loads, up to 12 per thread in flight), and every
  // output folds a chunk into its running (M, L, o) online: item = (head, pair of dims), `tpi`
  // adjacent lanes per item, each taking every tpi-th split of the chunk, combined by
  // shuffles at the end.
  const int qs = G * (kD + 2);  // floats between consecutive splits of one head
  const int cap = kUnStages * kUnStageBytes / 4 / qs;
  float* sp = reinterpret_cast<float*>(ring);
  const int items = G * (kD / 2);
  const int tpi = items >= kUnThreads ? 1 : kUnThreads / items;  // G = 1, 2, 4, 8: 4, 2, 1, 1
  const int rounds = (items * tpi + kUnThreads - 1) / kUnThreads;  // 2 for G = 8, else 1
  float Mr[2] = {-INFINITY, -INFINITY}, Lr[2] = {0.0f, 0.0f};
  float2 Ar[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
  for (int q0 = 0; q0 < nparts; q0 += cap) {
    const int cnt = min(cap, nparts - q0);
    const int nfl = cnt * qs;
    const float* src = gpart + static_cast<int64_t>(q0) * qs;
    if (q0 > 0) __syncthreads();  // the previous chunk is consumed
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {  // 264-byte splits: not always
      const float4* src4 = reinterpret_cast<const float4*>(src);
      float4* dst4 = reinterpret_cast<float4*>(sp);
      const int n4 = nfl / 4;
      for (int i0 = 0; i0 < n4; i0 += 12 * kUnThreads) {
        float4 v[12];
#pragma unroll
        for (int u = 0; u < 12; ++u) {
          const int i = i0 + u * kUnThreads + tid;
          if (i < n4) v[u] = __ldcg(src4 + i);
        }
#pragma unroll
        for (int u = 0; u < 12; ++u) {
          const int i = i0 + u * kUnThreads + tid;
          if (i < n4) dst4[i] = v[u];
        }
      }
      done = n4 * 4;
    }
    for (int i0 = done; i0 < nfl; i0 += 8 * kUnThreads) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kUnThreads + tid;
        if (i < nfl) v[u] = __ldcg(src + i);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kUnThreads + tid;
        if (i < nfl) sp[i] = v[u];
      }
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      if (rr >= rounds) break;
      const int item = (rr * kUnThreads + tid) / tpi;
      if (item >= items) continue;
      const int part = (rr * kUnThreads + tid) - item * tpi;
      const int h = item / (kD / 2), dp = item - h * (kD / 2);
      const float* pr = sp + h * (kD + 2);
      // the head's maximum over the chunk (the same splits for every lane of the head)
      float Mc = -INFINITY;
#pragma unroll 4
      for (int q = 0; q < cnt; ++q) Mc = fmaxf(Mc, pr[q * qs]);
      const float Mn = fmaxf(Mr[rr], Mc);
      if (Mn == -INFINITY) continue;  // nothing selected so far
      const float a = Mr[rr] == -INFINITY ? 0.0f : exp2f(Mr[rr] - Mn);
      float L = Lr[rr] * a;
      float2 A = make_float2(Ar[rr].x * a, Ar[rr].y * a);
#pragma unroll 4
      for (int q = part; q < cnt; q += tpi) {
        const float mq = pr[q * qs];
        const float sc = mq == -INFINITY ? 0.0f : exp2f(mq - Mn);
        const float2 ov = *reinterpret_cast<const float2*>(pr + q * qs + 2 + 2 * dp);
        L = fmaf(sc, pr[q * qs + 1], L);
        A.x = fmaf(sc, ov.x, A.x);
        A.y = fmaf(sc, ov.y, A.y);
      }
      Mr[rr] = Mn;
      Lr[rr] = L;
      Ar[rr] = A;
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    if (rr >= rounds) break;
    const int item = (rr * kUnThreads + tid) / tpi;
    const int part = (rr * kUnThreads + tid) - item * tpi;
    float L = Lr[rr];
    float2 A = Ar[rr];
    for (int o2 = 1; o2 < tpi; o2 <<= 1) {  // lanes of an item share Mr: plain sums
      L += __shfl_xor_sync(0xffffffffu, L, o2);
      A.x += __shfl_xor_sync(0xffffffffu, A.x, o2);
      A.y += __shfl_xor_sync(0xffffffffu, A.y, o2);
    }
    if (item < items && part == 0) {
      const int h = item / (kD / 2), dp = item - h * (kD / 2);
      if (state == nullptr) {
        ElemTraits<T>::store(o_out, static_cast<int>((row0 + h) * kD + 2 * dp), A.x / L);
        ElemTraits<T>::store(o_out, static_cast<int>((row0 + h) * kD + 2 * dp + 1), A.y / L);
      } else if (pv != nullptr && pv->world > 0) {  // epoch-tagged words into slot `rank`
        const uint32_t epoch = step_epoch(*pv);            // of every rank
        for (int i = 0; i < pv->world; ++i) {  // own slot first, then the next ranks
          const int q = peer_order(*pv, i);
          uint64_t* dst = pv->st(q, pv->rank, row0 + h);
          ll_put(dst + 2 + 2 * dp, __float_as_uint(A.x), epoch);
          ll_put(dst + 3 + 2 * dp, __float_as_uint(A.y), epoch);
          if (dp == 0) {
            ll_put(dst, __float_as_uint(Mr[rr]), epoch);
            ll_put(dst + 1, __float_as_uint(L), epoch);
          }
        }
      } else {
        float* st = state + (row0 + h) * (kD + 2);
        st[2 + 2 * dp] = A.x;
        st[3 + 2 * dp] = A.y;
        if (dp == 0) {
          st[0] = Mr[rr];
          st[1] = L;
        }
      }
    }
  }
}

template <typename T, typename E>
__global__ void __launch_bounds__(kUnThreads, 4) attend_union_kernel(const UnionParams p) {
  extern __shared__ uint8_t un_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(un_raw) + 127) & ~static_cast<uintptr_t>(127));
  E* list = reinterpret_cast<E*>(ring + kUnStages * kUnStageBytes);  // [span]
  uint32_t* hbits = reinterpret_cast<uint32_t*>(ring);               // [G][span / 32]
  __shared__ uint32_t wpre[kUnWarps];
  __shared__ int n_union_s;
  __shared__ int is_last;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int G = p.G;
  const int S_g = p.S;
  const int span = p.span;
  const int g = blockIdx.x / S_g;  // (b, h_kv)
  const int s = blockIdx.x - g * S_g;
  const int b = g / p.H_kv;
  const int hk = g - b * p.H_kv;
  const int lo = min(p.N, s * span);
  const int hi = min(p.N, lo + span);
  const int nwords = (hi - lo + 31) >> 5;
  const int wstride = span >> 5;  // words per head in hbits
  const int64_t row0 = static_cast<int64_t>(b) * p.H + static_cast<int64_t>(hk) * G;  // head 0

  // ---- Q as the A operand: row r = lane / 4 is head r (rows >= G and 8..15 are zero);
  // loaded first, so that its latency overlaps the list building below ----
  const int hr = lane >> 2;  // head row of this lane's accumulators (c0, c1)
  const int q4 = lane & 3;
  const bool head_ok = hr < G;
  uint32_t aq[4][2];  // A rows 8..15 (the other two registers of a fragment) are zero
  {
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        static_cast<const uint8_t*>(p.q) + (row0 + (head_ok ? hr : 0)) * 128);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      aq[kk][0] = head_ok ? __ldg(qrow + 8 * kk + q4) : 0u;      // dims 16kk + 2q4, +1
      aq[kk][1] = head_ok ? __ldg(qrow + 8 * kk + 4 + q4) : 0u;  // dims 16kk + 8 + 2q4, +1
    }
  }

#if DCR_UNION_PDL
  // launched early behind Pass 2 (programmatic dependent launch): wait for its results
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif

  // ---- the union of the G heads' selections inside [lo, hi): word tid of each head -------
  // Up to 64 words per range, two threads share a word (16 bits each) so that the list is
  // emitted by twice as many threads; thread t takes word t >> sh, bits [16 (t & 1), +16).
  const int sh = nwords <= kUnThreads / 2 ? 1 : 0;
  const int wi = tid >> sh;
  const uint32_t part_mask = sh ? (0xffffu << (16 * (tid & 1))) : 0xffffffffu;
  uint32_t hw[kUnMaxG];
#pragma unroll
  for (int h = 0; h < kUnMaxG; ++h) hw[h] = 0u;
  if (p.bits != nullptr) {  // Pass 2's bitmaps: G loads per thread, all in flight
    if (wi < nwords) {
#pragma unroll
      for (int h = 0; h < kUnMaxG; ++h)
        if (h < G) hw[h] = __ldg(p.bits + (row0 + h) * p.bits_stride + (lo >> 5) + wi);
    }
  } else {  // search each head's ascending index list for the range
  for (int i = tid; i < G * wstride; i += kUnThreads) hbits[i] = 0u;
  __syncthreads();
  for (int h = warp; h < G; h += kUnWarps) {
    const int32_t* ix = p.idx + (row0 + h) * p.k_eff;
    // first entry >= lo and first entry >= hi (the list is ascending): two 32-ary searches
    // in lockstep, each round one load per lane per bound (3 rounds for 4916 entries)
    int l0[2] = {0, 0}, l1[2] = {p.k_eff, p.k_eff};
    const int key[2] = {lo, hi};
    while (l0[0] < l1[0] || l0[1] < l1[1]) {  // warp-uniform
      int per[2], a[2];
      bool below[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        per[e] = (l1[e] - l0[e] + 31) / 32;
        a[e] = l0[e] + lane * per[e];
        below[e] = l0[e] < l1[e] && a[e] < l1[e];
      }
      int v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) v[e] = below[e] ? __ldg(ix + a[e]) : 0;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t m = __ballot_sync(0xffffffffu, below[e] && v[e] < key[e]);
        if (l0[e] >= l1[e]) continue;
        if (m == 0u) {  // ix[l0] >= key: the answer is l0
          l1[e] = l0[e];
        } else {        // ix[l0 + sl * per] < key <= ix[l0 + (sl + 1) * per] (or the end)
          const int sl = 31 - __clz(m);
          const int nl1 = min(l1[e], l0[e] + (sl + 1) * per[e]);
          l0[e] = l0[e] + sl * per[e] + 1;
          l1[e] = nl1;
        }
      }
    }
    // the entries in [lo, hi): 8 loads per lane in flight before their atomics
    for (int base = l0[0]; base < l0[1]; base += 32 * 8) {
      int v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + lane + 32 * u;
        v[u] = i < l0[1] ? __ldg(ix + i) : -1;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int n = v[u] - lo;
        if (v[u] >= 0 && n >= 0 && n < hi - lo)
          atomicOr(&hbits[h * wstride + (n >> 5)], 1u << (n & 31));
      }
    }
  }
  __syncthreads();
  if (wi < nwords) {
#pragma unroll
    for (int h = 0; h < kUnMaxG; ++h)
      if (h < G) hw[h] = hbits[h * wstride + wi];
  }
  __syncthreads();  // every thread has its words before the ring is reused
  }
  // this thread's share of its word (span <= 4096 positions)
  uint32_t uw = 0u;
#pragma unroll
  for (int h = 0; h < kUnMaxG; ++h) uw |= hw[h];
  uw &= part_mask;
  {
    const uint32_t c = __popc(uw);
    const uint32_t incl = warp_incl_scan(c);
    if (lane == 31) wpre[warp] = incl;
    __syncthreads();
    uint32_t before = 0;
    for (int w = 0; w < warp; ++w) before += wpre[w];
    if (tid == kUnThreads - 1) n_union_s = static_cast<int>(before + incl);
    uint32_t off = before + incl - c;
    uint32_t m = uw;
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1;
      uint32_t heads = 0;
#pragma unroll
      for (int h = 0; h < kUnMaxG; ++h) heads |= ((hw[h] >> bit) & 1u) << h;
      list[off++] = un_entry<E>(wi * 32 + bit, heads);
    }
  }
  __syncthreads();  // list complete; the ring is free for the gathers
  const int n_union = n_union_s;
  const int ntiles = (n_union + kUnTile - 1) / kUnTile;

  // ---- gathers: thread copies chunk tid % 8 of rows tid / 8 + 16 i (i < 4), K and V -----
  const uint8_t* kbase = static_cast<const uint8_t*>(p.k) + (b * p.ksb + hk * p.ksh) * 2;
  const uint8_t* vbase = static_cast<const uint8_t*>(p.v) + (b * p.vsb + hk * p.vsh) * 2;
  const int cchunk = tid & 7;
  const int rbase = tid >> 3;
  auto issue = [&](int tt) {
    if (tt < ntiles) {
      uint8_t* kt = ring + (tt % kUnStages) * kUnStageBytes;
      uint8_t* vt = kt + kUnTileBytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = rbase + 16 * i;
        const int t = tt * kUnTile + r;
        int64_t n = 0;
        uint32_t bytes = 0;  // past the list: zero-fill, read nothing
        if (t < n_union) {
          n = lo + static_cast<int>(static_cast<uint32_t>(list[t]) & 0xfffu);
          bytes = 16;
        }
        const uint32_t off = swz_offset(r, cchunk, kUnTile);
        cp_async_16(kt + off, kbase + n * 128 + cchunk * 16, bytes);
        cp_async_16(vt + off, vbase + n * 128 + cchunk * 16, bytes);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < kUnStages - 1; ++i) issue(i);

  float m_run = -INFINITY;  // this head row's running maximum (log2 units)
  float l_part = 0.0f;      // this lane's share of the row's sum
  float o[8][4];            // O: dim tile nt, c0/c1 = (head hr, dims 8nt + 2q4, +1)
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;

  for (int tt = 0; tt < ntiles; ++tt) {
    cp_async_wait<kUnStages - 2>();
    __syncthreads();  // tile tt visible to all; stage (tt - 1) free for reuse
    issue(tt + kUnStages - 1);
    const uint32_t kt = smem_u32(ring + (tt % kUnStages) * kUnStageBytes);
    const uint32_t vt = kt + kUnTileBytes;
    auto sel = [&](int r) {
      const int t = tt * kUnTile + r;
      return head_ok && t < n_union && ((static_cast<uint32_t>(list[t]) >> (12 + hr)) & 1u);
    };

    union_tile<T>(kt, vt, aq, sel, m_run, l_part, o);
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is free: reuse it for the warps' merge

  // ---- merge the 4 warps' (m, l, o) per head, then publish this range's partial ----------
  union_store_partial(ring, G, m_run, l_part, o,
                      p.part + (static_cast<int64_t>(g) * p.S_cap + s) * G * (kD + 2));

  const int nparts = S_g;  // partials the group's last CTA merges

  // ---- the group's last CTA merges the S partials of each head into O -------------------
  // The barrier orders every thread's partial stores before thread 0's ticket, an
  // acquire-release atomic: its release publishes the CTA's partial (cumulative through the
  // barrier) and, in the last CTA, its acquire makes every other CTA's partial visible to
  // the loads that follow the next barrier. No separate fences.
  __syncthreads();
  if (tid == 0) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(old)
                 : "l"(p.counters + g)
                 : "memory");
    is_last = old == S_g - 1;
  }
  __syncthreads();
  if (!is_last) return;
  union_merge<T>(ring, p.part + static_cast<int64_t>(g) * p.S_cap * G * (kD + 2), nparts, G,
                 row0, p.o, p.state, &p.pv);
  if (tid == 0) p.counters[g] = 0;
}

constexpr int kUnSpanMin = 256;

int union_max_splits(int N) {
  const int min_s = (N + kUnSpanMax - 1) / kUnSpanMax;
  return min_s > 64 ? min_s : 64;
}

// Splits per (b, h_kv) group for `per_sm` resident CTAs per SM, and positions per split (a
// multiple of 32, at most kUnSpanMax).
static void union_split(int N, int groups, int per_sm, int& S, int& span) {
  const int slots = device_sm_count() * per_sm;
  S = slots / (groups > 0 ? groups : 1);
  if (S < 1) S = 1;
  const int min_s = (N + kUnSpanMax - 1) / kUnSpanMax;
  if (S < min_s) S = min_s;
  if (S > union_max_splits(N)) S = union_max_splits(N);  // what the workspace partials hold
  // at least kUnSpanMin positions per range: below that a CTA's fixed costs (list, partial,
  // ticket) outweigh its gathers
  const int max_s = (N + kUnSpanMin - 1) / kUnSpanMin;
  if (S > max_s && max_s >= min_s) S = max_s;
  span = ((N + S - 1) / S + 31) / 32 * 32;
  if (span > kUnSpanMax) span = kUnSpanMax;
  S = (N + span - 1) / span;
}

template <typename T, typename E>
static int launch_union_t(UnionParams p, int groups, int part_splits, cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&attend_union_kernel<T, E>);
  p.S_cap = part_splits;
  if (ensure_smem_attr(fn, union_smem_bytes(kUnSpanMax, sizeof(E))) != cudaSuccess)
    return DCR_ERR_CUDA;
  // size the split for 4 CTAs per SM, then for what the resulting shared memory allows
  union_split(p.N, groups, 4, p.S, p.span);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attend_union_kernel<T, E>, kUnThreads,
                                                    union_smem_bytes(p.span, sizeof(E))) !=
      cudaSuccess)
    return DCR_ERR_CUDA;
  if (per_sm < 1) return DCR_ERR_SHAPE;
  if (per_sm < 4) union_split(p.N, groups, per_sm, p.S, p.span);
  if (p.S > part_splits) return DCR_ERR_SHAPE;
  const int64_t grid = static_cast<int64_t>(groups) * p.S;
  if (grid <= 0 || grid > 0x7fffffff) return DCR_ERR_SHAPE;
  // launched as a programmatic dependent of the preceding kernel (Pass 2)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kUnThreads);
  cfg.dynamicSmemBytes = union_smem_bytes(p.span, sizeof(E));
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = DCR_UNION_PDL ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attend_union_kernel<T, E>, p) == cudaSuccess ? DCR_OK
                                                                               : DCR_ERR_CUDA;
}

// The decode steps use the union Pass 3 for 16-bit caches; DCR_ATTEND_UNION=0 in the
// environment selects the per-head kernel instead (read once per process).
bool union_enabled() {
  static const bool on = [] {
    const char* e = getenv("DCR_ATTEND_UNION");
    return !(e != nullptr && strcmp(e, "0") == 0);
  }();
  return on;
}

bool union_supported(int dtype, int H, int H_kv) {
  if (dtype != DCR_DTYPE_BF16 && dtype != DCR_DTYPE_F16) return false;
  if (H_kv <= 0 || H % H_kv != 0) return false;
  const int G = H / H_kv;
  return G >= 1 && G <= kUnMaxG;
}

int launch_attend_union(const void* Q, const void* K, const void* V, int dtype, int64_t ksb,
                        int64_t ksh, int64_t vsb, int64_t vsh, const int32_t* idx,
                        const uint32_t* bits, int64_t bits_stride, int B, int H, int H_kv, int N,
                        int k_eff, void* O, float* partials, int part_splits, int* counters,
                        cudaStream_t st, float* state, const PeerView* pv) {
  if (!union_supported(dtype, H, H_kv)) return DCR_ERR_SHAPE;
  UnionParams p;
  p.state = state;
  p.pv.world = 0;
  if (pv != nullptr && state != nullptr) p.pv = *pv;
  p.q = Q;
  p.k = K;
  p.v = V;
  p.ksb = ksb;
  p.ksh = ksh;
  p.vsb = vsb;
  p.vsh = vsh;
  p.idx = idx;
  p.bits = bits;
  p.bits_stride = bits_stride;
  p.H = H;
  p.H_kv = H_kv;
  p.G = H / H_kv;
  p.N = N;
  p.k_eff = k_eff;
  p.o = O;
  p.part = partials;
  p.counters = counters;
  const int groups = B * H_kv;
  const bool narrow = p.G <= 4;  // 16-bit list entries
  if (dtype == DCR_DTYPE_F16)
    return narrow ? launch_union_t<__half, uint16_t>(p, groups, part_splits, st)
                  : launch_union_t<__half, uint32_t>(p, groups, part_splits, st);
  return narrow ? launch_union_t<__nv_bfloat16, uint16_t>(p, groups, part_splits, st)
                : launch_union_t<__nv_bfloat16, uint32_t>(p, groups, part_splits, st);
}

}  // namespace dcr
