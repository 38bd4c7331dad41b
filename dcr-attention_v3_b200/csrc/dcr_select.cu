// dcr_select.cu — Pass 2 (exact top-K selection) for sm_100a.
//
// Replaces topk_pass2_select (dcr_attention/kernel/triton/topk_axis_pass2.py:16) and its
// oracle _select_topk_indices (dcr_attention/kernel/qaxis_topk_reference.py:91): a stable
// descending argsort of f32(score), the first k_eff positions, re-sorted ascending.
// Stability means: among equal scores the lower index is taken first. Sorting is not
// needed to produce that set in ascending order:
//
//   1. Map each bf16 score to an order-preserving 16-bit key (-0 -> +0, NaN -> top).
//   2. Radix-select the k-th largest key T in two levels: a 4096-bin histogram of
//      key >> 4 gives the high 12 bits BH of T, then a 16-bin histogram of the low 4 bits
//      of the keys in BH gives T.
//   3. need = k_eff - #{key > T}. Emit, in index order, every position with key > T and
//      the first `need` positions with key == T. The output is the reference's set,
//      already ascending.
//
// Design (B200): a row is processed by one CTA of 512 threads, or, for long rows or few
// rows, by a thread-block cluster of C CTAs (C = 1..8) that splits it into contiguous
// segments. Each thread keeps a contiguous run of up to 64 keys in registers (loaded
// once from L2, where Pass 1 just wrote them). Histograms are built with shared-memory
// atomics and, in a cluster, added into CTA 0 through distributed shared memory; CTA 0
// scans its 4096 bins block-wide and one warp scans the 16 low bins. The 12-bit first
// level matters for decode scores: their keys crowd into a few exponents, so a 256-bin
// first level leaves a quarter of the row in the threshold bin and every warp then issues
// every second-level atomic; with 4096 bins the threshold bin holds a few percent of the
// row and most warps skip most second-level atomics outright (a warp-uniform vote per key).
// The per-CTA counts of keys > T and == T are exchanged
// through CTA 0, and a block-wide exclusive scan of the packed per-thread counts gives
// every thread its output offset and its rank among the equal keys. Threads emit their
// selected positions from bit masks.
#include <cooperative_groups.h>

#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace cg = cooperative_groups;

#ifndef DCR_UNION_PDL
#define DCR_UNION_PDL 1
#endif

namespace dcr {

#ifndef DCR_P2_WIDE
#define DCR_P2_WIDE 1
#endif
constexpr int kP2Threads = 512;
constexpr int kP2Warps = kP2Threads / 32;
constexpr int kP2MaxCluster = 8;
constexpr int kP2Bins1 = 4096;  // first level: key >> 4
constexpr int kP2Bins2 = 16;    // second level: key & 15

struct P2Params {
  const uint16_t* scores;
  int64_t stride;
  int N;
  int k;
  int32_t* idx;
  int* row_counters;      // Pass 3 split-K tickets reset here (may be null)
  int vec;                // rows are 16-byte aligned: 8 keys per uint4 load
  int keys_in;            // rows already hold order keys (Pass 1 keys_out), not bf16 bits
  int seg_vec;            // vectors (8 positions) per CTA segment
  uint32_t* bits;         // optional bitmap output instead of idx (whole-word layouts only)
  int64_t bits_stride;    // words per bitmap row
};

// Branch-free order key of a raw bf16 score (same map as bf16_order_key): -0 and +0
// share key 0x8000, every NaN gets 0xffff.
__device__ __forceinline__ uint32_t order_key_fast(uint32_t x) {
  x &= 0xffffu;
  const uint32_t mag = x & 0x7fffu;
  x = mag ? x : 0u;
  const uint32_t key = x ^ (((x >> 15) * 0x7fffu) | 0x8000u);
  return mag > 0x7f80u ? 0xffffu : key;
}

// VPT: vectors (8 positions each) per thread, 1..8.
template <int VPT, int TPB>
__global__ void __launch_bounds__(TPB, 1) select_kernel(const P2Params p) {
  constexpr int kWarpsB = TPB / 32;
  constexpr int kKeys = VPT * 8;
  constexpr int kWords = (kKeys + 31) / 32;
  constexpr int kBpt = kP2Bins1 / TPB;  // first-level bins per thread in the search
  __shared__ uint32_t hist_hi[kP2Bins1];
  __shared__ uint32_t hist_lo[kP2Bins2];
  __shared__ uint32_t wsum[kWarpsB];
  __shared__ uint32_t scan_tot;
  __shared__ uint32_t cta_gt[kP2MaxCluster];
  __shared__ uint32_t cta_eq[kP2MaxCluster];
  __shared__ int s_bh;
  __shared__ uint32_t s_above;

  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int crank = static_cast<int>(cluster.block_rank());
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int row = blockIdx.x / C;
  const int N = p.N;
  const int k = p.k;
  const int nvec = (N + 7) >> 3;
  const uint16_t* src = p.scores + static_cast<int64_t>(row) * p.stride;

  // CTA 0's copies (its own shared memory when the row has one CTA)
  const bool clustered = C > 1;
  uint32_t* hist_hi0 = clustered ? cluster.map_shared_rank(hist_hi, 0) : hist_hi;
  uint32_t* hist_lo0 = clustered ? cluster.map_shared_rank(hist_lo, 0) : hist_lo;
  uint32_t* gt0 = cluster.map_shared_rank(cta_gt, 0);
  uint32_t* eq0 = cluster.map_shared_rank(cta_eq, 0);
  int* bh0 = clustered ? cluster.map_shared_rank(&s_bh, 0) : &s_bh;
  uint32_t* above0 = clustered ? cluster.map_shared_rank(&s_above, 0) : &s_above;

  // A one-CTA row needs only a block barrier between the phases.
  auto row_sync = [&]() {
    if (clustered)
      cluster.sync();
    else
      __syncthreads();
  };

#if DCR_UNION_PDL
  // let the union Pass 3 launch now; it waits for this grid before reading its results
  asm volatile("griddepcontrol.launch_dependents;");
#endif
  if (crank == 0 && tid == 0 && p.row_counters != nullptr) p.row_counters[row] = 0;
  if (tid == 0) {
    s_bh = 0;
    s_above = 0;
  }
#pragma unroll
  for (int i = 0; i < kBpt; ++i) hist_hi[tid + i * TPB] = 0;
  if (tid < kP2Bins2) hist_lo[tid] = 0;

  // ---- keys of this thread: positions [v0 * 8, (v0 + VPT) * 8), 0 past the segment ----
  // Key 0 ranks below every real score (the smallest real key, -inf's, is 0x007f), so
  // padding is never selected.
  const int v_begin = crank * p.seg_vec;
  const int v_end = min(nvec, v_begin + p.seg_vec);
  const int v0 = v_begin + tid * VPT;
  uint32_t key[kKeys];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = v0 + j;
    const int base = v * 8;
    if (v < v_end && p.vec && base + 8 <= N) {
      const uint4 w = *reinterpret_cast<const uint4*>(src + base);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        key[8 * j + 2 * i] = p.keys_in ? (ww[i] & 0xffffu) : order_key_fast(ww[i]);
        key[8 * j + 2 * i + 1] = p.keys_in ? (ww[i] >> 16) : order_key_fast(ww[i] >> 16);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uint32_t kk = 0u;
        if (v < v_end && base + e < N) {
          const uint32_t raw = src[base + e];
          kk = p.keys_in ? raw : order_key_fast(raw);
        }
        key[8 * j + e] = kk;
      }
    }
  }
  row_sync();  // histograms initialised everywhere before anyone adds into CTA 0's

  // ---- level 1: histogram of the high 12 bits, added into CTA 0 -----------------------
#pragma unroll
  for (int e = 0; e < kKeys; ++e)
    if (key[e] != 0u) atomicAdd(&hist_hi[key[e] >> 4], 1u);
  if (C > 1) {
    __syncthreads();
    if (crank != 0) {
#pragma unroll
      for (int i = 0; i < kBpt; ++i) {
        const uint32_t c = hist_hi[tid + i * TPB];
        if (c) atomicAdd(hist_hi0 + tid + i * TPB, c);
      }
    }
  }
  row_sync();
  if (crank == 0) {
    // block-wide search from the top: thread t holds bins [kBpt g, kBpt g + kBpt) with
    // g = TPB - 1 - t, so thread 0 holds the highest bins
    const int g = TPB - 1 - tid;
    uint32_t c[kBpt], tot = 0;
#pragma unroll
    for (int i = 0; i < kBpt; ++i) {
      c[i] = hist_hi[kBpt * g + i];
      tot += c[i];
    }
    const uint32_t incl = warp_incl_scan(tot);
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const uint32_t ws = lane < kWarpsB ? wsum[lane] : 0u;
      const uint32_t wi = warp_incl_scan(ws);
      if (lane < kWarpsB) wsum[lane] = wi - ws;
    }
    __syncthreads();
    uint32_t a = incl - tot + wsum[warp];  // keys in the bins above this thread's
#pragma unroll
    for (int i = kBpt - 1; i >= 0; --i) {
      if (a < static_cast<uint32_t>(k) && static_cast<uint32_t>(k) <= a + c[i]) {
        s_bh = kBpt * g + i;
        s_above = a;
      }
      a += c[i];
    }
  }
  row_sync();
  const uint32_t bh = static_cast<uint32_t>(*bh0);

  // ---- level 2: low 4 bits of the keys in BH (a warp skips a key no lane has in BH) ---
#pragma unroll
  for (int e = 0; e < kKeys; ++e) {
    const bool in_bh = (key[e] >> 4) == bh && key[e] != 0u;
    if (__any_sync(0xffffffffu, in_bh)) {
      if (in_bh) atomicAdd(&hist_lo[key[e] & 15u], 1u);
    }
  }
  if (C > 1) {
    __syncthreads();
    if (crank != 0 && tid < kP2Bins2 && hist_lo[tid]) atomicAdd(hist_lo0 + tid, hist_lo[tid]);
  }
  row_sync();

  // T and need: every CTA's warp 0 scans CTA 0's low-byte histogram
  __shared__ uint32_t s_T;
  __shared__ int s_need;
  if (warp == 0) {
    // lane l < 16 holds low bin 15 - l (lane 0 the highest)
    const uint32_t above = *above0;
    const uint32_t kk = static_cast<uint32_t>(k) - above;
    const uint32_t c = lane < kP2Bins2 ? hist_lo0[kP2Bins2 - 1 - lane] : 0u;
    const uint32_t incl = warp_incl_scan(c);
    const bool hit = lane < kP2Bins2 && incl - c < kk && kk <= incl;
    const uint32_t m = __ballot_sync(0xffffffffu, hit);
    if (m != 0u && lane == __ffs(m) - 1) {
      s_T = (bh << 4) | static_cast<uint32_t>(kP2Bins2 - 1 - lane);
      s_need = k - static_cast<int>(above + (incl - c));  // minus #{key > T}
    } else if (m == 0u && lane == 0) {  // inconsistent counts: select nothing, report
      s_T = 0x10000u;
      s_need = 0;
      raise_status(DCR_ERR_DEVICE_INDEX);
    }
  }
  __syncthreads();
  const uint32_t T = s_T;
  const int need = s_need;

  // ---- per-thread masks and counts ----------------------------------------------------
  uint32_t gtm[kWords], eqm[kWords];
#pragma unroll
  for (int w = 0; w < kWords; ++w) gtm[w] = eqm[w] = 0u;
#pragma unroll
  for (int e = 0; e < kKeys; ++e) {
    gtm[e >> 5] |= (key[e] > T ? 1u : 0u) << (e & 31);
    eqm[e >> 5] |= (key[e] == T ? 1u : 0u) << (e & 31);
  }
  uint32_t ngt = 0, neq = 0;
#pragma unroll
  for (int w = 0; w < kWords; ++w) {
    ngt += __popc(gtm[w]);
    neq += __popc(eqm[w]);
  }

  // block exclusive scan of the packed counts (gt in the low 16 bits, eq in the high)
  const uint32_t packed = ngt | (neq << 16);
  const uint32_t incl = warp_incl_scan(packed);
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t ws = lane < kWarpsB ? wsum[lane] : 0u;
    const uint32_t wi = warp_incl_scan(ws);
    if (lane < kWarpsB) wsum[lane] = wi - ws;
    if (lane == kWarpsB - 1) scan_tot = wi;
  }
  __syncthreads();
  const uint32_t ex = incl - packed + wsum[warp];

  // ---- exchange the per-CTA totals through CTA 0 -------------------------------------
  uint32_t gt_before = 0, eq_before_cta = 0;
  if (C > 1) {
    if (tid == 0) {
      gt0[crank] = scan_tot & 0xffffu;
      eq0[crank] = scan_tot >> 16;
    }
    row_sync();
    for (int c = 0; c < crank; ++c) {
      gt_before += gt0[c];
      eq_before_cta += eq0[c];
    }
  }

  // ---- emission ----------------------------------------------------------------------
  const int eq_before = static_cast<int>(eq_before_cta + (ex >> 16));
  int pos = static_cast<int>(gt_before + (ex & 0xffffu)) + min(eq_before, need);
  int take = need - eq_before;  // ties this thread may take, lowest positions first
  const int base = v0 * 8;
  if (p.bits != nullptr) {
    // Segments start on whole words. With VPT % 4 == 0 a thread's positions are whole words
    // (base a multiple of 32), and a word is written by the thread whose positions start it,
    // if it starts inside the segment. With 8 or 16 positions per thread, the 4 or 2
    // adjacent lanes that share a word OR their bits together and the first one writes it.
    // With 40, a thread's bits start 0, 8, 16 or 24 bits into a word and reach into the
    // next: the CTA ORs them into its words in shared memory (the first-level histogram's,
    // free by now) and writes them out.
    uint32_t* brow = p.bits + static_cast<int64_t>(row) * p.bits_stride;
    uint32_t selw[kWords];
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
      uint32_t sel = gtm[w];
      const uint32_t eq = eqm[w];
      const int neq_w = __popc(eq);
      if (take >= neq_w) {
        sel |= eq;
        take -= neq_w;
      } else if (take > 0) {
        uint32_t rem = eq;
        for (int i = 0; i < take; ++i) rem &= rem - 1;
        sel |= eq & ~rem;
        take = 0;
      }
      selw[w] = sel;
    }
    if constexpr (kKeys == 40) {
      constexpr int kCtaWords = TPB * kKeys / 32;  // the CTA's words (its positions / 32)
      static_assert(kCtaWords <= kP2Bins1, "staged in the first-level histogram");
      for (int i = tid; i < kCtaWords; i += TPB) hist_hi[i] = 0u;
      __syncthreads();
      const int rel = base - v_begin * 8;  // 40 tid: bits 0, 8, 16 or 24 into word rel / 32
      const uint64_t placed =
          (static_cast<uint64_t>(selw[0]) | (static_cast<uint64_t>(selw[1] & 0xffu) << 32))
          << (rel & 31);
      if (static_cast<uint32_t>(placed)) atomicOr(&hist_hi[rel >> 5], static_cast<uint32_t>(placed));
      if (static_cast<uint32_t>(placed >> 32))
        atomicOr(&hist_hi[(rel >> 5) + 1], static_cast<uint32_t>(placed >> 32));
      __syncthreads();
      const int w0 = v_begin >> 2;  // the segment's first word (segments start on words)
      const int end = min(N, v_end * 8);
      for (int i = tid; i < kCtaWords; i += TPB)
        if ((w0 + i) * 32 < end) brow[w0 + i] = hist_hi[i];
    } else {
#pragma unroll
      for (int w = 0; w < kWords; ++w) {
        if constexpr (kKeys < 32) {
          uint32_t word = selw[w] << (base & 31);
#pragma unroll
          for (int o = 1; o < 32 / kKeys; o <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
          if ((base & 31) == 0 && base < v_end * 8 && base < N) brow[base >> 5] = word;
        } else {
          const int start = base + 32 * w;
          if (start < v_end * 8 && start < N) brow[start >> 5] = selw[w];
        }
      }
    }
    if (C > 1) cluster.sync();
    return;
  }
  int32_t* out = p.idx + static_cast<int64_t>(row) * k;
#pragma unroll
  for (int w = 0; w < kWords; ++w) {
    uint32_t sel = gtm[w];
    const uint32_t eq = eqm[w];
    const int neq_w = __popc(eq);
    if (take >= neq_w) {
      sel |= eq;
      take -= neq_w;
    } else if (take > 0) {
      uint32_t rem = eq;
      for (int i = 0; i < take; ++i) rem &= rem - 1;  // drop the lowest `take` bits
      sel |= eq & ~rem;
      take = 0;
    }
    while (sel) {
      const int b = __ffs(sel) - 1;
      sel &= sel - 1;
      if (pos < k) out[pos] = base + 32 * w + b;
      else raise_status(DCR_ERR_DEVICE_INDEX);
      ++pos;
    }
  }
  if (C > 1) cluster.sync();  // CTA 0's shared memory stays alive until all reads are done
}

template <int VPT, int TPB>
static int launch_select_t(const P2Params& p, int rows, int C, cudaStream_t st) {
  return launch_cluster(select_kernel<VPT, TPB>, dim3(static_cast<unsigned>(rows * C)),
                        dim3(TPB), 0, st, C, p) == cudaSuccess
             ? DCR_OK
             : DCR_ERR_CUDA;
}

int launch_select(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                  int keys_in, int32_t* idx, int* row_counters, cudaStream_t st, uint32_t* bits,
                  int64_t bits_stride, int* bits_written, uint8_t* scratch) {
  if (bits_written != nullptr) *bits_written = 0;
  if (scratch != nullptr && select_stream_path(rows, N)) {
    const int e = launch_select_stream(scores, s_stride_row, rows, N, k_eff, keys_in, idx,
                                       row_counters, scratch, bits, bits_stride, st);
    if (e == DCR_OK && bits != nullptr && bits_written != nullptr) *bits_written = 1;
    return e;
  }
  // the bitmap goes out only where every thread's keys are whole aligned words
  auto with_bits = [&](P2Params& q, int vpt, int C) {
    if (bits != nullptr && (vpt == 1 || vpt == 2 || vpt == 5 || vpt % 4 == 0) &&
        (C == 1 || q.seg_vec % 4 == 0)) {
      q.bits = bits;
      q.bits_stride = bits_stride;
      if (bits_written != nullptr) *bits_written = 1;
    }
  };
  P2Params p;
  p.bits = nullptr;
  p.bits_stride = 0;
  p.scores = scores;
  p.stride = s_stride_row;
  p.N = N;
  p.k = k_eff;
  p.idx = idx;
  p.row_counters = row_counters;
  p.keys_in = keys_in;
  p.vec = ((reinterpret_cast<uintptr_t>(scores) & 15u) == 0 && (s_stride_row & 7) == 0) ? 1 : 0;
  const int nvec = (N + 7) / 8;
  // Cluster size: split a row only when the rows alone leave SMs idle or a row is longer
  // than 32K positions (at most 64 keys per thread).
  const int64_t sms = device_sm_count();
  int C = 1;
  while (C < kP2MaxCluster && static_cast<int64_t>(rows) * (2 * C) <= sms) C *= 2;
  while (C < kP2MaxCluster && nvec > C * kP2Threads * 8) C *= 2;
  if (nvec > C * kP2Threads * 8) {
    // past 262144 positions: 1024-thread CTAs with 40 keys per thread, up to 327680
    int C2 = 1;
    while (C2 < kP2MaxCluster && nvec > C2 * 1024 * 5) C2 *= 2;
    if (nvec > C2 * 1024 * 5) return DCR_ERR_SHAPE;  // more than 327680 positions per row
    p.seg_vec = (nvec + C2 - 1) / C2;
    if ((p.seg_vec + 3) / 4 * 4 <= 1024 * 5) p.seg_vec = (p.seg_vec + 3) / 4 * 4;  // on words
    with_bits(p, 5, C2);
    return launch_select_t<5, 1024>(p, rows, C2, st);  // 40 keys per thread
  }
  p.seg_vec = (nvec + C - 1) / C;
  // clustered rows: segments start on whole bitmap words (4 vectors), where that still fits
  if (C > 1 && (p.seg_vec + 3) / 4 * 4 <= kP2Threads * 8) p.seg_vec = (p.seg_vec + 3) / 4 * 4;
#if DCR_P2_WIDE
  // One CTA per row: 1024 threads with half the keys each (up to 32 per thread, which fit
  // the 64 registers a 1024-thread CTA allows), also when the rows take several waves (256
  // rows of 32768: 23.6 against 26.8 us with 512 threads).
  if (C == 1 && p.seg_vec > kP2Threads * 4 && p.seg_vec <= 1024 * 4) {
    with_bits(p, 4, C);
    return launch_select_t<4, 1024>(p, rows, C, st);
  }
  // Just past 32768 positions a two-CTA cluster per row would need two waves for 128
  // rows: one 1024-thread CTA with 40 keys per thread covers up to 40960 positions (in
  // waves when the rows are more than the SMs).
  if (nvec > 1024 * 4 && nvec <= 1024 * 5 && C <= 2) {
    p.seg_vec = nvec;
    with_bits(p, 5, 1);
    return launch_select_t<5, 1024>(p, rows, 1, st);
  }
#endif
  const int vpt = (p.seg_vec + kP2Threads - 1) / kP2Threads;
  if (vpt <= 1) {
    with_bits(p, 1, C);
    return launch_select_t<1, kP2Threads>(p, rows, C, st);
  }
  if (vpt <= 2) {
    with_bits(p, 2, C);
    return launch_select_t<2, kP2Threads>(p, rows, C, st);
  }
  if (vpt <= 4) {
    with_bits(p, 4, C);
    return launch_select_t<4, kP2Threads>(p, rows, C, st);
  }
  with_bits(p, 8, C);
  return launch_select_t<8, kP2Threads>(p, rows, C, st);
}

}  // namespace dcr
