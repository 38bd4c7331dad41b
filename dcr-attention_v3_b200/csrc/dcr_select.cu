// dcr_select.cu — Pass 2 (exact top-K selection) for sm_100a.
//
// Replaces topk_pass2_select (dcr_attention/kernel/triton/topk_axis_pass2.py:16) and its
// oracle _select_topk_indices (dcr_attention/kernel/qaxis_topk_reference.py:91): a stable
// descending argsort of f32(score), the first k_eff positions, re-sorted ascending.
// Stability means: among equal scores the lower index is taken first. Sorting is not
// needed to produce that set in ascending order:
//
//   1. Map each bf16 score to an order-preserving 16-bit key (-0 -> +0, NaN -> top).
//   2. Radix-select the k-th largest key T: a 4096-bin histogram of key >> 4, then a
//      16-bin histogram of key & 15 inside the chosen high bin.
//   3. need = k_eff - #{key > T}. Emit, in index order, every position with key > T and
//      the first `need` positions with key == T. The output is the reference's set,
//      already ascending.
//
// One CTA of 1024 threads owns one (b, h) row. When the row fits (N <= 96K scores, rows
// 16-byte aligned) one thread brings it into shared memory with a single bulk copy
// (cp.async.bulk, completion on an mbarrier); otherwise the passes read it from global
// memory (L2). The row is processed in chunks of 32768 positions:
//   A. histogram of key >> 4 (4096 bins, shared-memory atomics); a block-wide suffix
//      scan finds the high bin BH holding the k-th largest key;
//   B. a 16-bin histogram of key & 15 over the keys in BH gives T and #{key > T};
//   D. per chunk, thread t owns 32 consecutive positions: it counts its keys > T and
//      == T, one block-wide exclusive scan of the packed counts gives every thread its
//      output offset and its rank among the equal keys, and the thread writes its
//      selected positions in order.
#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

constexpr int kP2Threads = 1024;
constexpr int kP2Warps = kP2Threads / 32;
constexpr int kHiBins = 4096;
constexpr int kP2SmemKeys = 96 * 1024;                  // scores staged in shared memory
constexpr int kP2DynSmem = kP2SmemKeys * 2 + 16;        // + the bulk-copy mbarrier

struct P2Params {
  const uint16_t* scores;
  int64_t stride;
  int N;
  int k;
  int32_t* idx;
  int* row_counters;  // Pass 3 split-K tickets reset here (may be null)
  int vec;            // rows are 16-byte aligned: 8 keys per uint4 load
  int staged;         // the row is bulk-copied into shared memory first
  int keys_in;        // rows already hold order keys (Pass 1 keys_out), not bf16 bits
};

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Branch-free order key of a raw bf16 score (same map as bf16_order_key): -0 and +0
// share key 0x8000, every NaN gets 0xffff.
__device__ __forceinline__ uint32_t order_key_fast(uint32_t x) {
  x &= 0xffffu;
  const uint32_t mag = x & 0x7fffu;
  x = mag ? x : 0u;
  const uint32_t key = x ^ (((x >> 15) * 0x7fffu) | 0x8000u);
  return mag > 0x7f80u ? 0xffffu : key;
}

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  return x;
}

// The row as 16-bit order keys, 8 per 16-byte vector. STAGED: the keys live in shared
// memory (converted in place by pass A). Otherwise they are read from global memory and
// converted on every pass; positions >= N read as key 0, which ranks below every real
// score (the smallest real key, -inf's, is 0x007f), so they are never selected.
template <bool STAGED>
struct KeyRow {
  const uint16_t* g;  // global row (raw bf16 bits, or keys if keys_in)
  uint16_t* s;        // shared row (keys)
  int N;
  int vec;
  int keys_in;
  __device__ __forceinline__ uint32_t key_of(uint32_t raw) const {
    return keys_in ? (raw & 0xffffu) : order_key_fast(raw);
  }
  __device__ __forceinline__ void load(int v, uint32_t (&key)[8]) const {
    if constexpr (STAGED) {
      const uint4 w = reinterpret_cast<const uint4*>(s)[v];
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        key[2 * i] = ww[i] & 0xffffu;
        key[2 * i + 1] = ww[i] >> 16;
      }
    } else {
      const int base = v * 8;
      if (vec && base + 8 <= N) {
        const uint4 w = *reinterpret_cast<const uint4*>(g + base);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          key[2 * i] = key_of(ww[i]);
          key[2 * i + 1] = key_of(ww[i] >> 16);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) key[e] = (base + e < N) ? key_of(g[base + e]) : 0u;
      }
    }
  }
};

template <bool STAGED>
__global__ void __launch_bounds__(kP2Threads, 1) select_kernel(const P2Params p) {
  constexpr int kVPT = 4;                                // vectors per thread per chunk
  constexpr int kChunkVec = kP2Threads * kVPT;           // 4096 vectors = 32768 keys
  __shared__ uint32_t hist[kHiBins];
  __shared__ uint32_t hist2[16];
  __shared__ uint32_t scan_buf[kP2Threads];
  __shared__ uint32_t wsum[kP2Warps];
  __shared__ int s_bh, s_above, s_T, s_need;
  __shared__ uint32_t s_chunk_tot;
  extern __shared__ __align__(16) uint8_t p2_dyn[];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int row = blockIdx.x;
  const int N = p.N;
  const int k = p.k;
  const int nvec = (N + 7) >> 3;
  int32_t* out = p.idx + static_cast<int64_t>(row) * p.k;

  KeyRow<STAGED> kr;
  kr.g = p.scores + static_cast<int64_t>(row) * p.stride;
  kr.s = reinterpret_cast<uint16_t*>(p2_dyn);
  kr.N = N;
  kr.vec = p.vec;
  kr.keys_in = p.keys_in;

  uint64_t* bar = reinterpret_cast<uint64_t*>(p2_dyn + kP2SmemKeys * 2);
  if (STAGED && tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    const uint32_t bytes = static_cast<uint32_t>(nvec) * 16u;
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load(p2_dyn, kr.g, bytes, bar);
  }
  if (p.row_counters != nullptr && tid == 0) p.row_counters[row] = 0;
  for (int i = tid; i < kHiBins; i += kP2Threads) hist[i] = 0;
  if (tid < 16) hist2[tid] = 0;
  __syncthreads();

  // Exclusive prefix sum of x over the CTA (thread order); returns the total in *tot.
  auto block_excl_scan = [&](uint32_t x, uint32_t* tot) -> uint32_t {
    const uint32_t incl = warp_incl_scan(x);
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const uint32_t ws = wsum[lane];
      const uint32_t wi = warp_incl_scan(ws);
      wsum[lane] = wi - ws;
      if (lane == 31) s_chunk_tot = wi;
    }
    __syncthreads();
    const uint32_t r = incl - x + wsum[warp];
    *tot = s_chunk_tot;
    __syncthreads();  // wsum / s_chunk_tot may be reused by the next scan
    return r;
  };

  // ---- pass A: (convert to keys in place and) histogram the high 12 bits ---------------
  if constexpr (STAGED) {
    mbar_wait_bounded(bar, 0);
    uint4* sv = reinterpret_cast<uint4*>(kr.s);
    for (int v = tid; v < nvec; v += kP2Threads) {
      uint4 w = sv[v];
      uint32_t ww[4] = {w.x, w.y, w.z, w.w};
      const int base = v * 8;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t k0 = p.keys_in ? (ww[i] & 0xffffu) : order_key_fast(ww[i]);
        uint32_t k1 = p.keys_in ? (ww[i] >> 16) : order_key_fast(ww[i] >> 16);
        if (base + 2 * i >= N) k0 = 0u;
        if (base + 2 * i + 1 >= N) k1 = 0u;
        atomicAdd(&hist[k0 >> 4], 1u);
        atomicAdd(&hist[k1 >> 4], 1u);
        ww[i] = k0 | (k1 << 16);
      }
      sv[v] = make_uint4(ww[0], ww[1], ww[2], ww[3]);
    }
  } else {
    for (int v = tid; v < nvec; v += kP2Threads) {
      uint32_t key[8];
      kr.load(v, key);
#pragma unroll
      for (int e = 0; e < 8; ++e) atomicAdd(&hist[key[e] >> 4], 1u);
    }
  }
  __syncthreads();

  // ---- find the high bin BH: #{hi > BH} < k <= #{hi >= BH} --------------------------
  // Thread t owns bins 4t..4t+3. Suffix sum = exclusive prefix sum over positions
  // rt = 1023 - tid: thread tid's count is placed at position rt, the buffer is
  // prefix-scanned in position order, and thread tid reads its result back from rt.
  {
    uint32_t h4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h4[i] = hist[4 * tid + i];
    const int rt = kP2Threads - 1 - tid;
    scan_buf[rt] = h4[0] + h4[1] + h4[2] + h4[3];
    __syncthreads();
    uint32_t tot;
    const uint32_t ex = block_excl_scan(scan_buf[tid], &tot);
    scan_buf[tid] = ex;
    __syncthreads();
    uint32_t above = scan_buf[rt];  // #{keys in bins above 4*tid+3}
#pragma unroll
    for (int i = 3; i >= 0; --i) {
      const uint32_t c = h4[i];
      if (above < static_cast<uint32_t>(k) && static_cast<uint32_t>(k) <= above + c) {
        s_bh = 4 * tid + i;
        s_above = static_cast<int>(above);
      }
      above += c;
    }
  }
  __syncthreads();
  const uint32_t bh = static_cast<uint32_t>(s_bh);

  // ---- pass B: 16-bin histogram of the low nibble of the keys in BH --------------------
  for (int v = tid; v < nvec; v += kP2Threads) {
    uint32_t key[8];
    kr.load(v, key);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if ((key[e] >> 4) == bh) atomicAdd(&hist2[key[e] & 15u], 1u);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t above = static_cast<uint32_t>(s_above);  // #{key >> 4 > BH} < k
    int lo = 0;
    for (int nib = 15; nib >= 0; --nib) {
      const uint32_t c = hist2[nib];
      if (static_cast<uint32_t>(k) <= above + c) {
        lo = nib;
        break;
      }
      above += c;
    }
    s_T = static_cast<int>((bh << 4) | static_cast<uint32_t>(lo));
    s_need = k - static_cast<int>(above);  // above == #{key > T}
  }
  __syncthreads();

  // ---- pass D: ordered emission, one 32768-position chunk at a time -------------------
  const uint32_t T = static_cast<uint32_t>(s_T);
  const int need = s_need;
  int E = 0;  // keys == T before the current chunk
  int P = 0;  // positions emitted before the current chunk
  for (int c0 = 0; c0 < nvec; c0 += kChunkVec) {
    const int v0 = c0 + tid * kVPT;
    uint32_t key[kVPT][8];
    uint32_t ngt = 0, neq = 0;
#pragma unroll
    for (int j = 0; j < kVPT; ++j) {
      if (v0 + j < nvec) {
        kr.load(v0 + j, key[j]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) key[j][e] = 0u;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ngt += key[j][e] > T ? 1u : 0u;
        neq += key[j][e] == T ? 1u : 0u;
      }
    }
    uint32_t tot;
    const uint32_t ex = block_excl_scan(ngt | (neq << 16), &tot);
    const int eq_before = E + static_cast<int>(ex >> 16);
    // P counts the ties taken before this chunk (min(E, need)); add the ones taken in
    // this chunk before this thread.
    int pos = P + static_cast<int>(ex & 0xffffu) + (min(eq_before, need) - min(E, need));
    int eq_rank = eq_before;
#pragma unroll
    for (int j = 0; j < kVPT; ++j) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t kk = key[j][e];
        bool sel = kk > T;
        if (kk == T) {
          sel = eq_rank < need;
          ++eq_rank;
        }
        if (sel) {
          if (pos < k) out[pos] = (v0 + j) * 8 + e;
          else raise_status(DCR_ERR_DEVICE_INDEX);
          ++pos;
        }
      }
    }
    const int chunk_eq = static_cast<int>(tot >> 16);
    const int chunk_gt = static_cast<int>(tot & 0xffffu);
    P += chunk_gt + (min(E + chunk_eq, need) - min(E, need));
    E += chunk_eq;
  }
}

int launch_select(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                  int keys_in, int32_t* idx, int* row_counters, cudaStream_t st) {
  P2Params p;
  p.keys_in = keys_in;
  p.scores = scores;
  p.stride = s_stride_row;
  p.N = N;
  p.k = k_eff;
  p.idx = idx;
  p.row_counters = row_counters;
  p.vec = ((reinterpret_cast<uintptr_t>(scores) & 15u) == 0 && (s_stride_row & 7) == 0) ? 1 : 0;
  p.staged = (p.vec && N <= kP2SmemKeys) ? 1 : 0;
  if (p.staged) {
    if (ensure_smem_attr(reinterpret_cast<const void*>(&select_kernel<true>), kP2DynSmem) !=
        cudaSuccess)
      return DCR_ERR_CUDA;
    select_kernel<true><<<rows, kP2Threads, kP2DynSmem, st>>>(p);
  } else {
    select_kernel<false><<<rows, kP2Threads, 0, st>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

}  // namespace dcr
