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
// One CTA of 1024 threads owns one (b, h) row. The row is read from L2/L1 three times
// (pass A histogram, pass B low-nibble histogram + per-warp counts, pass D emission).
// Warp w owns a contiguous segment of the row in passes B and D, so the per-warp counts
// of pass B give every warp its exclusive output offset, and the warp-level emission in
// pass D uses ballot/scan prefix sums only.
#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

constexpr int kP2Threads = 1024;
constexpr int kP2Warps = kP2Threads / 32;
constexpr int kHiBins = 4096;

struct P2Params {
  const uint16_t* scores;
  int64_t stride;
  int N;
  int k;
  int32_t* idx;
  int* row_counters;  // Pass 3 split-K tickets reset here (may be null)
  int vec;            // rows are 16-byte aligned: 8 keys per uint4 load
};

// Loads the 8 keys of vector v (positions 8v .. 8v+7); invalid positions (>= N) get
// valid-bit 0.
__device__ __forceinline__ void load_keys8(const uint16_t* row, int v, int N, int vec,
                                           uint32_t (&key)[8], uint32_t& valid) {
  const int base = v * 8;
  if (vec && base + 8 <= N) {
    const uint4 w = *reinterpret_cast<const uint4*>(row + base);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      key[2 * i] = bf16_order_key(ww[i] & 0xffffu);
      key[2 * i + 1] = bf16_order_key(ww[i] >> 16);
    }
    valid = 0xffu;
  } else {
    valid = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (base + e < N) {
        key[e] = bf16_order_key(row[base + e]);
        valid |= 1u << e;
      } else {
        key[e] = 0;
      }
    }
  }
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

__global__ void __launch_bounds__(kP2Threads, 1) select_kernel(const P2Params p) {
  __shared__ uint32_t hist[kHiBins];
  __shared__ uint32_t whist[kP2Warps][16];
  __shared__ uint32_t wgt_hi[kP2Warps];
  __shared__ uint32_t wsum[kP2Warps];
  __shared__ uint32_t w_gt_excl[kP2Warps];
  __shared__ uint32_t w_eq_excl[kP2Warps];
  __shared__ int s_bh, s_above, s_T, s_need;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int row = blockIdx.x;
  const uint16_t* src = p.scores + static_cast<int64_t>(row) * p.stride;
  int32_t* out = p.idx + static_cast<int64_t>(row) * p.k;
  const int N = p.N;
  const int k = p.k;
  const int nvec = (N + 7) >> 3;

  if (p.row_counters != nullptr && tid == 0) p.row_counters[row] = 0;
  for (int i = tid; i < kHiBins; i += kP2Threads) hist[i] = 0;
  if (tid < kP2Warps * 16) (&whist[0][0])[tid] = 0;
  __syncthreads();

  // ---- pass A: histogram of the high 12 bits ------------------------------------------
  for (int v = tid; v < nvec; v += kP2Threads) {
    uint32_t key[8], valid;
    load_keys8(src, v, N, p.vec, key, valid);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (valid & (1u << e)) atomicAdd(&hist[key[e] >> 4], 1u);
  }
  __syncthreads();

  // ---- find the high bin BH: #{hi > BH} < k <= #{hi >= BH} --------------------------
  // Thread t owns bins 4t..4t+3; an exclusive suffix sum over threads gives #{hi > 4t+3}.
  {
    uint32_t h4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h4[i] = hist[4 * tid + i];
    const uint32_t local = h4[0] + h4[1] + h4[2] + h4[3];
    // Suffix sum = exclusive prefix sum over positions rt = 1023 - tid: thread tid's count
    // is placed at position rt, the buffer is prefix-scanned in position order, and
    // thread tid reads its result back from position rt.
    const int rt = kP2Threads - 1 - tid;
    __shared__ uint32_t scan_buf[kP2Threads];
    scan_buf[rt] = local;
    __syncthreads();
    const uint32_t x = scan_buf[tid];  // value of the thread with rt == tid
    const uint32_t incl = warp_incl_scan(x);
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const uint32_t ws = wsum[lane];
      const uint32_t wi = warp_incl_scan(ws);
      wsum[lane] = wi - ws;  // exclusive prefix of warp totals
    }
    __syncthreads();
    scan_buf[tid] = incl - x + wsum[warp];  // exclusive prefix at position tid (rt order)
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

  // ---- pass B: per-warp #{hi > BH} and low-nibble histogram of hi == BH --------------
  const int vpw = (nvec + kP2Warps - 1) / kP2Warps;  // vectors per warp segment
  const int seg0 = warp * vpw;
  const int seg1 = min(nvec, seg0 + vpw);
  {
    uint32_t gt = 0;
    for (int v = seg0 + lane; v < seg1; v += 32) {
      uint32_t key[8], valid;
      load_keys8(src, v, N, p.vec, key, valid);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (!(valid & (1u << e))) continue;
        const uint32_t hi = key[e] >> 4;
        if (hi > bh) ++gt;
        else if (hi == bh) atomicAdd(&whist[warp][key[e] & 15u], 1u);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) gt += __shfl_xor_sync(0xffffffffu, gt, off);
    if (lane == 0) wgt_hi[warp] = gt;
  }
  __syncthreads();

  // ---- threshold T, need, per-warp exclusive offsets ---------------------------------
  if (warp == 0) {
    // lanes 0..15 total the low-nibble histogram
    // Lanes 0..15 total the low-nibble histogram of the high bin; every lane then walks
    // the 16 totals from the top nibble down to the one where the count reaches k.
    uint32_t tot = 0;
    if (lane < 16)
      for (int w = 0; w < kP2Warps; ++w) tot += whist[w][lane];
    uint32_t t16[16];
#pragma unroll
    for (int nib = 0; nib < 16; ++nib) t16[nib] = __shfl_sync(0xffffffffu, tot, nib);
    uint32_t above = static_cast<uint32_t>(s_above);  // #{key >> 4 > BH} < k
    uint32_t gt_T = above;
    int lo = 0;
    bool found = false;
#pragma unroll
    for (int nib = 15; nib >= 0; --nib) {
      const uint32_t c = t16[nib];
      if (!found && static_cast<uint32_t>(k) <= above + c) {
        lo = nib;
        gt_T = above;  // #{key > T}
        found = true;
      }
      above += c;
    }
    const int need = k - static_cast<int>(gt_T);
    // per-warp counts (lane = warp index)
    uint32_t wg = wgt_hi[lane];
    for (int nib = lo + 1; nib < 16; ++nib) wg += whist[lane][nib];
    const uint32_t we = whist[lane][lo];
    const uint32_t wg_incl = warp_incl_scan(wg);
    const uint32_t we_incl = warp_incl_scan(we);
    w_gt_excl[lane] = wg_incl - wg;
    w_eq_excl[lane] = we_incl - we;
    if (lane == 0) {
      s_T = static_cast<int>((bh << 4) | static_cast<uint32_t>(lo));
      s_need = need;
    }
  }
  __syncthreads();

  // ---- pass D: ordered emission -------------------------------------------------------
  {
    const uint32_t T = static_cast<uint32_t>(s_T);
    const int need = s_need;
    int E = static_cast<int>(w_eq_excl[warp]);  // equal keys before this lane's step
    int P = static_cast<int>(w_gt_excl[warp]) + min(static_cast<int>(w_eq_excl[warp]), need);
    for (int vb = seg0; vb < seg1; vb += 32) {
      const int v = vb + lane;
      uint32_t gtm = 0, eqm = 0;
      if (v < seg1) {
        uint32_t key[8], valid;
        load_keys8(src, v, N, p.vec, key, valid);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (!(valid & (1u << e))) continue;
          if (key[e] > T) gtm |= 1u << e;
          else if (key[e] == T) eqm |= 1u << e;
        }
      }
      const int ne = __popc(eqm);
      const int eq_incl = static_cast<int>(warp_incl_scan(static_cast<uint32_t>(ne)));
      const int eq_before = E + eq_incl - ne;
      int take = need - eq_before;
      take = take < 0 ? 0 : (take > ne ? ne : take);
      uint32_t selm = gtm;
      uint32_t rem = eqm;
      for (int i = 0; i < take; ++i) {
        const uint32_t bit = rem & (0u - rem);
        selm |= bit;
        rem ^= bit;
      }
      const int ns = __popc(selm);
      const int s_incl = static_cast<int>(warp_incl_scan(static_cast<uint32_t>(ns)));
      int pos = P + s_incl - ns;
      while (selm) {
        const int e = __ffs(selm) - 1;
        selm &= selm - 1;
        if (pos < k) out[pos] = v * 8 + e;
        else raise_status(DCR_ERR_DEVICE_INDEX);
        ++pos;
      }
      E += __shfl_sync(0xffffffffu, eq_incl, 31);
      P += __shfl_sync(0xffffffffu, s_incl, 31);
    }
  }
}

int launch_select(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                  int32_t* idx, int* row_counters, cudaStream_t st) {
  P2Params p;
  p.scores = scores;
  p.stride = s_stride_row;
  p.N = N;
  p.k = k_eff;
  p.idx = idx;
  p.row_counters = row_counters;
  p.vec = ((reinterpret_cast<uintptr_t>(scores) & 15u) == 0 && (s_stride_row & 7) == 0) ? 1 : 0;
  select_kernel<<<rows, kP2Threads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

}  // namespace dcr
