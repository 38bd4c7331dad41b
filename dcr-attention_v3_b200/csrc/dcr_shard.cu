// dcr_shard.cu — sequence-sharded decode: the exact global top-K over KV-cache chunks held
// by several GPUs, and the cross-GPU (m, l, o) combine.
//
// The reference's decode path runs on one GPU; this file has no counterpart there. The
// set it selects is the reference's (_select_topk_indices,
// dcr_attention/kernel/qaxis_topk_reference.py:91: stable descending argsort of the
// scores over the whole context, first k_eff) taken over the concatenation of the ranks'
// chunks in rank order, and the attention is _fused_softmax_attention (:148) over that
// set, computed piecewise by rank and merged exactly.
//
// Rank r holds positions [off_r, off_r + N_r) of every (b, h_kv) cache, off_r increasing
// with r. One decode step is four phases separated by three collectives that the caller
// runs (NCCL over NVLink in dcr_b200.sharded):
//   1. dcr_shard_score: Pass 1 over the local chunk (16-bit order keys into the
//      workspace) and, per row, a 256-bin histogram of the keys' high byte.
//                                                      -> all-reduce (sum) of [rows][256]
//   2. dcr_shard_refine: from the global high-byte histogram, the bin BH that holds the
//      k-th largest key; a 256-bin histogram of the low byte of the local keys in BH.
//                                                      -> all-gather into [world][rows][256]
//   3. dcr_shard_attend: the summed low-byte histograms give T (the k-th largest key) and
//      need = k_eff - #{key > T} over all ranks. Keys equal to T are taken in position
//      order, and lower ranks hold lower positions, so rank r takes
//          quota_r = clamp(need - #{key == T on ranks < r}, 0, #{key == T on rank r}).
//      The rank lists its positions with key > T and its first quota_r positions with
//      key == T, ascending, and runs Pass 3 over them, writing the unnormalised state
//      (m, l, o[64]) of every row instead of O.       -> all-gather into [world][rows][66]
//   4. dcr_shard_combine: O = sum_r 2^{m_r - M} o_r / sum_r 2^{m_r - M} l_r, M = max_r m_r.
//
// Phase kernels (B200): a CTA of 256 threads takes an 8192-position chunk of one row, 32
// contiguous keys per thread read as four 16-byte loads (the keys were just written by
// Pass 1 and are served from L2). Histograms use shared-memory atomics and add their
// non-zero bins into the row's global histogram. Listing the selection takes two
// launches: per-chunk counts of (key > T, key == T), then each chunk's output offset
// from the counts of the chunks before it and a block-wide scan inside the chunk.
#include "dcr_common.cuh"
#include "dcr_internal.h"
#include "dcr_peer.cuh"

namespace dcr {

constexpr int kShThreads = 256;
constexpr int kShWarps = kShThreads / 32;
constexpr int kShKeys = 32;                     // contiguous keys per thread
constexpr int kShChunk = kShThreads * kShKeys;  // positions per CTA
constexpr int kShStateFloats = kD + 2;          // (m, l, o[64])

struct ShardParams {
  const uint16_t* keys;       // order keys (Pass 1 keys_out), rows n_pad apart
  int64_t stride;
  int rows, N, k, chunks, cap, world, rank;
  const int32_t* hist_hi;     // [rows][256] summed over ranks (phase 2)
  const int32_t* hist_lo_all; // [world][rows][256] (phase 3)
  int32_t* hist_out;          // [rows][256] this rank's histogram (phases 1, 2)
  int32_t* row_state;         // [rows][4]: BH, #{key above bin BH}, T, quota
  uint32_t* chunk_cnt;        // [rows][chunks]: #{key > T} | #{key == T} << 16
  int32_t* idx;               // [rows][cap] selected local positions, ascending
  int32_t* count;             // [rows] number of selected local positions
  int* counters;              // Pass 3 split-K tickets, reset by phase 3
  PeerView v;                 // v.world > 0: exchange through the peers' buffers instead of
                              // hist_hi / hist_out / hist_lo_all
  uint32_t* bits;             // optional (fused selection): [rows][bits_stride] bitmaps of the
  int64_t bits_stride;        // selected local positions, written besides idx
  int emit_idx;               // 0: bitmaps only (the union Pass 3 reads nothing else)
  int32_t* mode;              // [1]: 1 if the last selection wrote bitmaps only, else 0
};

// The 32 keys of this thread in chunk `chunk` of row `row`; 0 past the end of the row
// (no real score maps to key 0: the lowest real key is that of -inf, 0x007f).
__device__ __forceinline__ void shard_load_keys(const ShardParams& p, int64_t row, int chunk,
                                                uint32_t (&key)[kShKeys]) {
  const uint16_t* src = p.keys + row * p.stride;
  const int64_t base = static_cast<int64_t>(chunk) * kShChunk +
                       static_cast<int64_t>(threadIdx.x) * kShKeys;
  if (base + kShKeys <= p.N) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src + base);
#pragma unroll
    for (int j = 0; j < kShKeys / 8; ++j) {
      const uint4 w = __ldcg(s4 + j);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        key[8 * j + 2 * i] = ww[i] & 0xffffu;
        key[8 * j + 2 * i + 1] = ww[i] >> 16;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < kShKeys; ++e) key[e] = (base + e < p.N) ? src[base + e] : 0u;
  }
}

// Phase 1 (kLevel 0): histogram of key >> 8. Phase 2 (kLevel 1): find BH in the global
// high-byte histogram, then histogram key & 0xff over the keys in BH.
// Peer mode: the row's histogram accumulates in this rank's accumulator; the last CTA of
// the row publishes it into slot `rank` of every rank's buffer as epoch-tagged words
// (exchange kLevel) and clears the accumulator. Phase 2 first reads every rank's
// high-byte row (waiting for each word's epoch) and sums them.
template <int kLevel>
__global__ void __launch_bounds__(kShThreads) shard_hist_kernel(const ShardParams p) {
  __shared__ uint32_t h[256];
  __shared__ uint32_t hsum[256];
  __shared__ uint32_t s_bh;
  __shared__ int s_last;
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x / p.chunks;
  const int chunk = blockIdx.x % p.chunks;
  const bool peer = p.v.world > 0;
  const uint32_t epoch = peer ? step_epoch(p.v) : 0u;
  h[tid] = 0u;
  if (kLevel == 1) {
    const uint32_t* hist_hi = reinterpret_cast<const uint32_t*>(p.hist_hi + row * 256);
    if (peer) {
      uint64_t w[kMaxPeers];
      ll_gather(p.v, p.v.hh(p.v.rank, 0, row) + tid, static_cast<int64_t>(p.v.rows) * 256, epoch,
                32, w);
      uint32_t sum = 0;
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r < p.v.world) sum += static_cast<uint32_t>(w[r]);
      hsum[tid] = sum;
      __syncthreads();
      hist_hi = hsum;
    }
    if (tid < 32) {
      int bin;
      uint32_t above;
      warp_find_bin(hist_hi, static_cast<uint32_t>(p.k), bin, above);
      if (tid == 0) {
        if (bin < 0) {  // fewer than k keys over all ranks
          raise_status(DCR_ERR_DEVICE_SHARD);
          bin = 0;
          above = 0;
        }
        s_bh = static_cast<uint32_t>(bin);
        if (chunk == 0) {
          p.row_state[row * 4 + 0] = bin;
          p.row_state[row * 4 + 1] = static_cast<int32_t>(above);
        }
      }
    }
  }
  uint32_t key[kShKeys];
  shard_load_keys(p, row, chunk, key);
  __syncthreads();
  if (kLevel == 0) {
#pragma unroll
    for (int e = 0; e < kShKeys; ++e)
      if (key[e] != 0u) atomicAdd(&h[key[e] >> 8], 1u);
  } else {
    const uint32_t bh = s_bh;
#pragma unroll
    for (int e = 0; e < kShKeys; ++e)
      if (key[e] != 0u && (key[e] >> 8) == bh) atomicAdd(&h[key[e] & 0xffu], 1u);
  }
  __syncthreads();
  const uint32_t c = h[tid];
  int32_t* dst = peer ? p.v.acc(kLevel, row) : p.hist_out + row * 256;
  if (c) atomicAdd(reinterpret_cast<unsigned int*>(dst + tid), c);
  if (!peer) return;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = (atomicAdd(p.v.ticket(kLevel, row), 1u) == static_cast<uint32_t>(p.chunks - 1));
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  const uint32_t val = static_cast<uint32_t>(__ldcg(dst + tid));
  dst[tid] = 0;  // every chunk CTA of the row has added: clear for the next step
  for (int i = 0; i < p.v.world; ++i) {
    const int q = peer_order(p.v, i);
    ll_put((kLevel ? p.v.hl(q, p.v.rank, row) : p.v.hh(q, p.v.rank, row)) + tid, val, epoch);
  }
  if (tid == 0) *p.v.ticket(kLevel, row) = 0u;
}

// Phase 3a: T and this rank's tie quota from the gathered low-byte histograms; per-chunk
// counts of keys > T and == T.
__global__ void __launch_bounds__(kShThreads) shard_count_kernel(const ShardParams p) {
  __shared__ uint32_t h[256];
  __shared__ uint32_t h_below[256];
  __shared__ uint32_t h_mine[256];
  __shared__ uint32_t s_T;
  __shared__ uint32_t red[kShWarps];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t row = blockIdx.x / p.chunks;
  const int chunk = blockIdx.x % p.chunks;
  const uint32_t bh = static_cast<uint32_t>(p.row_state[row * 4 + 0]);
  const uint32_t above = static_cast<uint32_t>(p.row_state[row * 4 + 1]);
  const bool peer = p.v.world > 0;
  const uint32_t epoch = peer ? step_epoch(p.v) : 0u;
  // rank r's low-byte count of bin b: its published word (peer mode) or hist_lo_all
  auto lo = [&](int r, int b) -> uint32_t {
    if (peer) return ll_get(p.v, p.v.hl(p.v.rank, r, row) + b, epoch);
    return static_cast<uint32_t>(
        __ldcg(p.hist_lo_all + (static_cast<int64_t>(r) * p.rows + row) * 256 + b));
  };
  // bin tid's count summed over the ranks, over the ranks below this one, and this rank's
  uint32_t tot = 0, below = 0, mine = 0;
  if (peer) {
    uint64_t w[kMaxPeers];
    ll_gather(p.v, p.v.hl(p.v.rank, 0, row) + tid, static_cast<int64_t>(p.v.rows) * 256, epoch,
              32, w);
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r >= p.v.world) break;
      const uint32_t c = static_cast<uint32_t>(w[r]);
      if (r < p.rank) below += c;
      if (r == p.rank) mine = c;
      tot += c;
    }
  } else {
    for (int r = 0; r < p.world; ++r) {
      const uint32_t c = lo(r, tid);
      if (r < p.rank) below += c;
      if (r == p.rank) mine = c;
      tot += c;
    }
  }
  h[tid] = tot;
  h_below[tid] = below;
  h_mine[tid] = mine;
  uint32_t key[kShKeys];
  shard_load_keys(p, row, chunk, key);
  __syncthreads();
  if (warp == 0) {
    int bl;
    uint32_t above_lo;
    warp_find_bin(h, static_cast<uint32_t>(p.k) - above, bl, above_lo);
    if (lane == 0) {
      if (bl < 0) {
        raise_status(DCR_ERR_DEVICE_SHARD);
        bl = 0;
        above_lo = 0;
      }
      const uint32_t T = (bh << 8) | static_cast<uint32_t>(bl);
      const int need = p.k - static_cast<int>(above + above_lo);
      const int eq_lower = static_cast<int>(h_below[bl]);
      const int eq_mine = static_cast<int>(h_mine[bl]);
      const int quota = max(0, min(need - eq_lower, eq_mine));
      s_T = T;
      if (chunk == 0) {
        p.row_state[row * 4 + 2] = static_cast<int32_t>(T);
        p.row_state[row * 4 + 3] = quota;
      }
    }
  }
  __syncthreads();
  const uint32_t T = s_T;
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < kShKeys; ++e) packed += (key[e] > T) ? 1u : ((key[e] == T) ? 0x10000u : 0u);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) packed += __shfl_xor_sync(0xffffffffu, packed, off);
  if (lane == 0) red[warp] = packed;
  __syncthreads();
  if (tid == 0) {
    uint32_t s = 0;
#pragma unroll
    for (int w = 0; w < kShWarps; ++w) s += red[w];
    p.chunk_cnt[row * p.chunks + chunk] = s;
  }
}

// Phase 3b: list the selected local positions of the chunk, ascending.
__global__ void __launch_bounds__(kShThreads) shard_emit_kernel(const ShardParams p) {
  __shared__ uint32_t wsum[kShWarps];
  __shared__ uint32_t s_gt_before, s_eq_before, s_gt_all;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t row = blockIdx.x / p.chunks;
  const int chunk = blockIdx.x % p.chunks;
  const uint32_t T = static_cast<uint32_t>(p.row_state[row * 4 + 2]);
  const uint32_t quota = static_cast<uint32_t>(p.row_state[row * 4 + 3]);
  if (blockIdx.x == 0 && tid == 0) *p.mode = 0;  // index lists
  if (warp == 0) {
    uint32_t gb = 0, eb = 0, ga = 0;
    for (int c = lane; c < p.chunks; c += 32) {
      const uint32_t v = p.chunk_cnt[row * p.chunks + c];
      ga += v & 0xffffu;
      if (c < chunk) {
        gb += v & 0xffffu;
        eb += v >> 16;
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      gb += __shfl_xor_sync(0xffffffffu, gb, off);
      eb += __shfl_xor_sync(0xffffffffu, eb, off);
      ga += __shfl_xor_sync(0xffffffffu, ga, off);
    }
    if (lane == 0) {
      s_gt_before = gb;
      s_eq_before = eb;
      s_gt_all = ga;
    }
  }
  uint32_t key[kShKeys];
  shard_load_keys(p, row, chunk, key);
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < kShKeys; ++e) packed += (key[e] > T) ? 1u : ((key[e] == T) ? 0x10000u : 0u);
  const uint32_t incl = warp_incl_scan(packed);
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t ws = lane < kShWarps ? wsum[lane] : 0u;
    const uint32_t wi = warp_incl_scan(ws);
    if (lane < kShWarps) wsum[lane] = wi - ws;
  }
  __syncthreads();
  const uint32_t ex = incl - packed + wsum[warp];
  uint32_t eq_rank = s_eq_before + (ex >> 16);  // ties on this rank before this thread's keys
  int64_t pos = static_cast<int64_t>(s_gt_before) + (ex & 0xffffu) + min(eq_rank, quota);
  int32_t* out = p.idx + row * p.cap;
  const int base = chunk * kShChunk + tid * kShKeys;
#pragma unroll
  for (int e = 0; e < kShKeys; ++e) {
    bool take = key[e] > T;
    if (key[e] == T) {
      take = eq_rank < quota;
      ++eq_rank;
    }
    if (take) {
      if (pos < p.cap) {
        out[pos] = base + e;
      } else {
        raise_status(DCR_ERR_DEVICE_SHARD);
      }
      ++pos;
    }
  }
  if (chunk == 0 && tid == 0) {
    p.count[row] = static_cast<int32_t>(min(s_gt_all + quota, static_cast<uint32_t>(p.cap)));
    p.counters[row] = 0;
  }
}

// Phase 4: merge the ranks' (m, l, o) states of a row into O. Peer mode: read every
// rank's state words of the row from this rank's slots (waiting for their epoch), and
// let the last CTA advance the epoch (the step is complete on this rank).
template <typename T>
__global__ void __launch_bounds__(kD) shard_combine_kernel(const float* states, int world,
                                                           int rows, void* O, const PeerView v) {
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const uint32_t epoch = v.world > 0 ? step_epoch(v) : 0u;
  float M = -INFINITY, L = 0.0f, o = 0.0f;
  if (v.world > 0) {
    // every rank's (m, l, o[tid]) of this row: all 3 x world words requested at once, then
    // the late ones polled
    uint64_t wm[kMaxPeers], wl[kMaxPeers], wo[kMaxPeers];
    const int64_t stride = static_cast<int64_t>(v.rows) * kShStateFloats;
    const uint64_t* base = v.st(v.rank, 0, row);
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      wm[r] = r < v.world ? ll_load(base + r * stride) : 0ull;
      wl[r] = r < v.world ? ll_load(base + 1 + r * stride) : 0ull;
      wo[r] = r < v.world ? ll_load(base + 2 + tid + r * stride) : 0ull;
    }
    ll_gather_late(v, base, stride, epoch, wm);
    ll_gather_late(v, base + 1, stride, epoch, wl);
    ll_gather_late(v, base + 2 + tid, stride, epoch, wo);
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < v.world) M = fmaxf(M, __uint_as_float(static_cast<uint32_t>(wm[r])));
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r >= v.world) break;
      const float m = __uint_as_float(static_cast<uint32_t>(wm[r]));
      const float w = (m == -INFINITY) ? 0.0f : exp2f(m - M);
      L = fmaf(w, __uint_as_float(static_cast<uint32_t>(wl[r])), L);
      o = fmaf(w, __uint_as_float(static_cast<uint32_t>(wo[r])), o);
    }
  } else {
    for (int r = 0; r < world; ++r)
      M = fmaxf(M, __ldcg(states + (static_cast<int64_t>(r) * rows + row) * kShStateFloats));
    for (int r = 0; r < world; ++r) {
      const float* st = states + (static_cast<int64_t>(r) * rows + row) * kShStateFloats;
      const float m = __ldcg(st);
      const float w = (m == -INFINITY) ? 0.0f : exp2f(m - M);
      L = fmaf(w, __ldcg(st + 1), L);
      o = fmaf(w, __ldcg(st + 2 + tid), o);
    }
  }
  ElemTraits<T>::store(O, static_cast<int>(row * kD + tid), o / L);
  if (v.world > 0) {
    __syncthreads();
    if (tid == 0 && atomicAdd(v.cticket(), 1u) == static_cast<uint32_t>(rows - 1)) {
      *v.cticket() = 0u;
      __threadfence();
      atomicExch(v.epoch(), epoch);
    }
  }
}

// Fused selection of the peer-exchange step (kernels above, phases 1-3b, in one launch):
// one 512-thread CTA per row holds the row's keys in registers (up to 64 per thread)
// through both histogram exchanges, which use packed words (every rank's chunk is at
// most 32768 positions, so counts fit 16 bits). The CTA publishes its row's high-byte histogram into
// slot `rank` of every rank's buffer (exchange 0), reads every rank's row as its words
// arrive, finds BH, publishes the low-byte histogram of its keys in BH (exchange 1),
// reads, finds T and its tie quota, and emits its positions as Pass 2 does. Each row
// waits only for the same row of the other ranks, never for another CTA of its own GPU;
// the kernel runs only when all its rows fit in one wave (every rank alike), so no row
// waits behind a row that the other GPU has not started.
constexpr int kFsThreads = 512;  // CTA size for chunks up to 8192 positions (else 1024)

// Publishes this row's 256-bin histogram h (exchange x, packed words) into slot `rank` of
// every rank's buffer and sums every rank's row into out. Block-wide; ends with a barrier.
// lower (optional): per bin, the counts of the ranks below this one (the tie quota's input).
__device__ __forceinline__ void exchange_row_packed(const PeerView& v, int x, int64_t row,
                                                    const uint32_t* h, uint32_t* out,
                                                    uint32_t epoch, uint32_t* lower = nullptr) {
  const int tid = threadIdx.x;
  if (tid < kPackedWords) {
    const int b = 3 * tid;
    const uint32_t c0 = h[b], c1 = b + 1 < 256 ? h[b + 1] : 0u, c2 = b + 2 < 256 ? h[b + 2] : 0u;
    for (int i = 0; i < v.world; ++i) {
      const int q = peer_order(v, i);
      ll_put_packed((x ? v.hl(q, v.rank, row) : v.hh(q, v.rank, row)) + tid, c0, c1, c2, epoch);
    }
    uint64_t w[kMaxPeers];
    ll_gather(v, (x ? v.hl(v.rank, 0, row) : v.hh(v.rank, 0, row)) + tid,
              static_cast<int64_t>(v.rows) * 256, epoch, 48, w);
    uint32_t s0 = 0, s1 = 0, s2 = 0, l0 = 0, l1 = 0, l2 = 0;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r >= v.world) break;
      if (r == v.rank) {
        l0 = s0;
        l1 = s1;
        l2 = s2;
      }
      s0 += static_cast<uint32_t>(w[r] & 0xffffu);
      s1 += static_cast<uint32_t>((w[r] >> 16) & 0xffffu);
      s2 += static_cast<uint32_t>((w[r] >> 32) & 0xffffu);
    }
    out[b] = s0;
    if (b + 1 < 256) out[b + 1] = s1;
    if (b + 2 < 256) out[b + 2] = s2;
    if (lower != nullptr) {
      lower[b] = l0;
      if (b + 1 < 256) lower[b + 1] = l1;
      if (b + 2 < 256) lower[b + 2] = l2;
    }
  }
  __syncthreads();
}

template <int VPT, int TPB>
__global__ void __launch_bounds__(TPB, 1) shard_select_fused_kernel(const ShardParams p) {
  constexpr int kKeys = VPT * 8;
  constexpr int kWords = (kKeys + 31) / 32;
  constexpr int kWarpsB = TPB / 32;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t hsum[256];
  __shared__ uint32_t hlow[256];  // low-byte counts of the ranks below this one
  __shared__ uint32_t wsum[kWarpsB];
  __shared__ uint32_t s_bh, s_above, s_T, s_quota, s_tot;
  const PeerView& v = p.v;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const int rank = v.rank;
  const uint32_t epoch = step_epoch(v);
  if (tid < 256) hist[tid] = 0u;

  // keys of this thread: positions [v0 * 8, (v0 + VPT) * 8); 0 past the row
  const uint16_t* src = p.keys + row * p.stride;
  const int v0 = tid * VPT;
  uint32_t key[kKeys];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int base = (v0 + j) * 8;
    if (base + 8 <= p.N) {
      const uint4 w = __ldcg(reinterpret_cast<const uint4*>(src + base));
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        key[8 * j + 2 * i] = ww[i] & 0xffffu;
        key[8 * j + 2 * i + 1] = ww[i] >> 16;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) key[8 * j + e] = (base + e < p.N) ? src[base + e] : 0u;
    }
  }
  __syncthreads();

  // ---- exchange 0: high-byte histograms ----
#pragma unroll
  for (int e = 0; e < kKeys; ++e)
    if (key[e] != 0u) atomicAdd(&hist[key[e] >> 8], 1u);
  __syncthreads();
  exchange_row_packed(v, 0, row, hist, hsum, epoch);
  if (tid < 256) hist[tid] = 0u;
  __syncthreads();
  if (warp == 0) {
    int bin;
    uint32_t above;
    warp_find_bin(hsum, static_cast<uint32_t>(p.k), bin, above);
    if (lane == 0) {
      if (bin < 0) {
        raise_status(DCR_ERR_DEVICE_SHARD);
        bin = 0;
        above = 0;
      }
      s_bh = static_cast<uint32_t>(bin);
      s_above = above;
      p.row_state[row * 4 + 0] = bin;
      p.row_state[row * 4 + 1] = static_cast<int32_t>(above);
    }
  }
  __syncthreads();

  // ---- exchange 1: low-byte histograms of the keys in BH ----
  const uint32_t bh = s_bh;
#pragma unroll
  for (int e = 0; e < kKeys; ++e)
    if ((key[e] >> 8) == bh && key[e] != 0u) atomicAdd(&hist[key[e] & 0xffu], 1u);
  __syncthreads();
  exchange_row_packed(v, 1, row, hist, hsum, epoch, hlow);
  __syncthreads();
  if (warp == 0) {
    int bl;
    uint32_t above_lo;
    warp_find_bin(hsum, static_cast<uint32_t>(p.k) - s_above, bl, above_lo);
    if (lane == 0) {
      if (bl < 0) {
        raise_status(DCR_ERR_DEVICE_SHARD);
        bl = 0;
        above_lo = 0;
      }
      const uint32_t T = (bh << 8) | static_cast<uint32_t>(bl);
      const int need = p.k - static_cast<int>(s_above + above_lo);
      const int eq_lower = static_cast<int>(hlow[bl]);  // ranks below this one
      const int eq_mine = static_cast<int>(hist[bl]);
      s_T = T;
      s_quota = static_cast<uint32_t>(max(0, min(need - eq_lower, eq_mine)));
      p.row_state[row * 4 + 2] = static_cast<int32_t>(T);
      p.row_state[row * 4 + 3] = static_cast<int32_t>(s_quota);
    }
  }
  __syncthreads();
  const uint32_t T = s_T;
  const int quota = static_cast<int>(s_quota);

  // ---- masks, block scan, ordered emission (as Pass 2) ----
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
  const uint32_t packed = ngt | (neq << 16);
  const uint32_t incl = warp_incl_scan(packed);
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t ws = lane < kWarpsB ? wsum[lane] : 0u;
    const uint32_t wi = warp_incl_scan(ws);
    if (lane < kWarpsB) wsum[lane] = wi - ws;
    if (lane == kWarpsB - 1) s_tot = wi;
  }
  __syncthreads();
  const uint32_t ex = incl - packed + wsum[warp];
  const int eq_before = static_cast<int>(ex >> 16);
  int pos = static_cast<int>(ex & 0xffffu) + min(eq_before, quota);
  int take = quota - eq_before;
  int32_t* out = p.idx + row * p.cap;
  const int base = v0 * 8;
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
    // whole words (VPT a multiple of 4: positions base + 32 w start a word)
    if (p.bits != nullptr && base + 32 * w < p.N)
      p.bits[row * p.bits_stride + ((base + 32 * w) >> 5)] = sel;
    if (!p.emit_idx) continue;
    while (sel) {
      const int bb = __ffs(sel) - 1;
      sel &= sel - 1;
      if (pos < p.cap) out[pos] = base + 32 * w + bb;
      else raise_status(DCR_ERR_DEVICE_SHARD);
      ++pos;
    }
  }
  if (tid == 0) {
    p.count[row] = min(static_cast<int>(s_tot & 0xffffu) + quota, p.cap);
    p.counters[row] = 0;
    if (row == 0) *p.mode = p.emit_idx ? 0 : 1;
  }
}

size_t align_up_256(size_t x) { return (x + 255) / 256 * 256; }

ShardLayout shard_layout(int rows, int N_local, int k_eff) {
  ShardLayout w;
  w.cap = k_eff < N_local ? k_eff : N_local;
  w.splits = attend_splits(rows, w.cap);
  w.n_pad = (static_cast<int64_t>(N_local) + 7) / 8 * 8;
  w.chunks = static_cast<int>((static_cast<int64_t>(N_local) + kShChunk - 1) / kShChunk);
  size_t off = 0;
  w.counters = off;
  off = align_up_256(off + sizeof(int) * static_cast<size_t>(rows));
  w.partials = off;
  w.part_splits = w.splits;
  if (union_enabled() && union_max_splits(N_local) > w.part_splits)
    w.part_splits = union_max_splits(N_local);
  off = align_up_256(off + sizeof(float) * static_cast<size_t>(rows) * w.part_splits * (kD + 2));
  w.scores = off;
  off = align_up_256(off + sizeof(uint16_t) * static_cast<size_t>(rows) * w.n_pad);
  w.idx = off;
  off = align_up_256(off + sizeof(int32_t) * static_cast<size_t>(rows) * w.cap);
  w.count = off;
  off = align_up_256(off + sizeof(int32_t) * static_cast<size_t>(rows));
  w.row_state = off;
  off = align_up_256(off + sizeof(int32_t) * 4 * static_cast<size_t>(rows));
  w.chunk_cnt = off;
  off = align_up_256(off + sizeof(uint32_t) * static_cast<size_t>(rows) * w.chunks);
  w.bits = off;
  w.bits_stride = (static_cast<int64_t>(N_local) + 31) / 32;
  off = align_up_256(off + sizeof(uint32_t) * static_cast<size_t>(rows) * w.bits_stride);
  w.mode = off;
  off = align_up_256(off + sizeof(int32_t));
  w.total = off;
  return w;
}

static ShardParams shard_params(const ShardLayout& w, uint8_t* ws, int rows, int N_local,
                                int k_eff) {
  ShardParams p = {};
  p.v.world = 0;
  p.keys = reinterpret_cast<const uint16_t*>(ws + w.scores);
  p.stride = w.n_pad;
  p.rows = rows;
  p.N = N_local;
  p.k = k_eff;
  p.chunks = w.chunks;
  p.cap = w.cap;
  p.row_state = reinterpret_cast<int32_t*>(ws + w.row_state);
  p.chunk_cnt = reinterpret_cast<uint32_t*>(ws + w.chunk_cnt);
  p.idx = reinterpret_cast<int32_t*>(ws + w.idx);
  p.count = reinterpret_cast<int32_t*>(ws + w.count);
  p.counters = reinterpret_cast<int*>(ws + w.counters);
  p.bits = nullptr;
  p.bits_stride = w.bits_stride;
  p.emit_idx = 1;
  p.mode = reinterpret_cast<int32_t*>(ws + w.mode);
  return p;
}

static int check_launch() { return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA; }

int launch_shard_hist(const ShardLayout& w, uint8_t* ws, int rows, int N_local, int k_eff,
                      int level, const int32_t* hist_hi_sum, int32_t* hist_out,
                      const PeerView* pv, cudaStream_t st) {
  ShardParams p = shard_params(w, ws, rows, N_local, k_eff);
  p.hist_hi = hist_hi_sum;
  p.hist_out = hist_out;
  if (pv != nullptr) {
    p.v = *pv;
  } else if (cudaMemsetAsync(hist_out, 0, sizeof(int32_t) * 256 * static_cast<size_t>(rows),
                             st) != cudaSuccess) {
    return DCR_ERR_CUDA;
  }
  const int64_t grid = static_cast<int64_t>(rows) * w.chunks;
  if (grid > 0x7fffffff) return DCR_ERR_SHAPE;
  if (level == 0)
    shard_hist_kernel<0><<<static_cast<unsigned>(grid), kShThreads, 0, st>>>(p);
  else
    shard_hist_kernel<1><<<static_cast<unsigned>(grid), kShThreads, 0, st>>>(p);
  return check_launch();
}

int launch_shard_select(const ShardLayout& w, uint8_t* ws, int rows, int N_local, int k_eff,
                        const int32_t* hist_lo_all, int world, int rank, const PeerView* pv,
                        cudaStream_t st) {
  ShardParams p = shard_params(w, ws, rows, N_local, k_eff);
  p.hist_lo_all = hist_lo_all;
  if (pv != nullptr) p.v = *pv;
  p.world = world;
  p.rank = rank;
  const int64_t grid = static_cast<int64_t>(rows) * w.chunks;
  if (grid > 0x7fffffff) return DCR_ERR_SHAPE;
  shard_count_kernel<<<static_cast<unsigned>(grid), kShThreads, 0, st>>>(p);
  int e = check_launch();
  if (e) return e;
  shard_emit_kernel<<<static_cast<unsigned>(grid), kShThreads, 0, st>>>(p);
  return check_launch();
}

template <int VPT, int TPB>
static int launch_fused_t(const ShardParams& p, cudaStream_t st, bool* launched) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, shard_select_fused_kernel<VPT, TPB>,
                                                    TPB, 0) != cudaSuccess)
    return DCR_ERR_CUDA;
  // Every row's CTA waits on the same row of the other ranks, so all rows must be resident
  // at once; otherwise the caller runs the phase kernels (rows and the launch shape are the
  // same on every rank, so every rank decides alike).
  if (static_cast<int64_t>(per_sm) * device_sm_count() < p.rows) return DCR_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows));
  cfg.blockDim = dim3(TPB);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  if (cudaLaunchKernelEx(&cfg, shard_select_fused_kernel<VPT, TPB>, p) != cudaSuccess)
    return DCR_ERR_CUDA;
  *launched = true;
  return DCR_OK;
}

int launch_shard_select_fused(const ShardLayout& w, uint8_t* ws, int rows, int N_local,
                              int n_local_max, int k_eff, const PeerView* pv, cudaStream_t st,
                              bool* launched, bool* bits_written, bool bits_only) {
  *launched = false;
  if (bits_written != nullptr) *bits_written = false;
  // every rank takes the same path: decided from the longest chunk of all ranks
  if (pv == nullptr || n_local_max > kFsThreads * 64 || N_local > n_local_max) return DCR_OK;
  const int nvec = (N_local + 7) / 8;
  ShardParams p = shard_params(w, ws, rows, N_local, k_eff);
  p.v = *pv;
  p.world = pv->world;
  p.rank = pv->rank;
  // Past 8192 positions, when every row has its own SM: 1024-thread CTAs with at most 32
  // keys per thread (Pass 2's launch shape there); otherwise 512 threads with up to 64.
  // The shape follows n_local_max and rows, the same on every rank.
  const int nvec_max = (n_local_max + 7) / 8;
  // With 4 or 8 vectors per thread a thread's keys are whole 32-bit words, so the bitmaps
  // go out too.
  auto with_bits = [&](int e) {
    if (bits_written != nullptr) *bits_written = e == DCR_OK && *launched;
    return e;
  };
  if (bits_written != nullptr) p.bits = reinterpret_cast<uint32_t*>(ws + w.bits);
  // where the bitmaps go out and the caller reads nothing else, no index lists are written
  const int emit_idx_bits = (bits_written != nullptr && bits_only) ? 0 : 1;
  if (nvec_max > 512 * 2 && rows <= device_sm_count()) {
    const int vpt = (nvec + 1023) / 1024;
    if (vpt <= 2) {
      p.bits = nullptr;
      return launch_fused_t<2, 1024>(p, st, launched);
    }
    p.emit_idx = emit_idx_bits;
    return with_bits(launch_fused_t<4, 1024>(p, st, launched));
  }
  const int vpt = (nvec + kFsThreads - 1) / kFsThreads;
  if (vpt <= 2) {
    p.bits = nullptr;
    return vpt <= 1 ? launch_fused_t<1, kFsThreads>(p, st, launched)
                    : launch_fused_t<2, kFsThreads>(p, st, launched);
  }
  p.emit_idx = emit_idx_bits;
  if (vpt <= 4) return with_bits(launch_fused_t<4, kFsThreads>(p, st, launched));
  return with_bits(launch_fused_t<8, kFsThreads>(p, st, launched));
}

// The selection of the last step as ascending index lists and counts: copied, or, where the
// step wrote bitmaps only, rebuilt from them (one CTA per row, a block scan per 256 words).
__global__ void __launch_bounds__(kShThreads) shard_selection_out_kernel(const ShardParams p,
                                                                        int32_t* idx_out,
                                                                        int32_t* count_out) {
  __shared__ uint32_t wsum[kShWarps];
  __shared__ uint32_t s_carry;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t row = blockIdx.x;
  int32_t* out = idx_out + row * p.cap;
  if (*p.mode == 0) {
    for (int i = tid; i < p.cap; i += kShThreads) out[i] = p.idx[row * p.cap + i];
    if (tid == 0) count_out[row] = p.count[row];
    return;
  }
  if (tid == 0) s_carry = 0;
  __syncthreads();
  const uint32_t* brow = p.bits + row * p.bits_stride;
  for (int64_t w0 = 0; w0 < p.bits_stride; w0 += kShThreads) {
    const int64_t wi = w0 + tid;
    uint32_t word = wi < p.bits_stride ? brow[wi] : 0u;
    const uint32_t c = static_cast<uint32_t>(__popc(word));
    const uint32_t incl = warp_incl_scan(c);
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    uint32_t pos = s_carry + incl - c;
    for (int w = 0; w < warp; ++w) pos += wsum[w];
    uint32_t tot = 0;
    for (int w = 0; w < kShWarps; ++w) tot += wsum[w];
    while (word) {
      const int b = __ffs(word) - 1;
      word &= word - 1;
      if (static_cast<int>(pos) < p.cap) out[pos] = static_cast<int32_t>(wi * 32 + b);
      ++pos;
    }
    __syncthreads();
    if (tid == 0) s_carry += tot;
    __syncthreads();
  }
  if (tid == 0) count_out[row] = min(static_cast<int>(s_carry), p.cap);
}

int launch_shard_selection_out(const ShardLayout& w, const uint8_t* ws, int rows, int N_local,
                               int k_eff, int32_t* idx_out, int32_t* count_out, cudaStream_t st) {
  ShardParams p = shard_params(w, const_cast<uint8_t*>(ws), rows, N_local, k_eff);
  p.bits = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(ws) + w.bits);
  shard_selection_out_kernel<<<static_cast<unsigned>(rows), kShThreads, 0, st>>>(p, idx_out,
                                                                               count_out);
  return check_launch();
}

int launch_shard_combine(const float* states, int world, int rows, int dtype, void* O,
                         const PeerView* pv, cudaStream_t st) {
  PeerView v = {};
  if (pv != nullptr) v = *pv;
  switch (dtype) {
    case DCR_DTYPE_BF16:
      shard_combine_kernel<__nv_bfloat16><<<rows, kD, 0, st>>>(states, world, rows, O, v);
      break;
    case DCR_DTYPE_F16:
      shard_combine_kernel<__half><<<rows, kD, 0, st>>>(states, world, rows, O, v);
      break;
    case DCR_DTYPE_F32:
      shard_combine_kernel<float><<<rows, kD, 0, st>>>(states, world, rows, O, v);
      break;
    default: return DCR_ERR_DTYPE;
  }
  return check_launch();
}

}  // namespace dcr
