// dcr_select_stream.cu — Pass 2 for large selections: the same exact top-K as dcr_select.cu
// (replaces topk_pass2_select, dcr_attention/kernel/triton/topk_axis_pass2.py:16, and its
// oracle _select_topk_indices, dcr_attention/kernel/qaxis_topk_reference.py:91), organised
// for throughput instead of latency.
//
// The one-CTA-per-row kernel of dcr_select.cu keeps a row's keys in registers through a
// chain of dependent phases; it is fastest while every row (or row cluster) has an SM of its
// own. Past that (B x H x N beyond one wave: config-4 rows of 262144 positions, B = 16 at
// 32K-128K) its waves run one after another and the chain's latency is paid per wave. Here
// the row is cut into chunks of 8192 positions (256 threads x 32 keys, one bitmap word per
// thread) and the selection runs as five short kernels, each a grid over every chunk of
// every row (or over the rows), so any number of waves overlaps:
//
//   A  hist     per chunk: 4096-bin histogram of key >> 4 in shared memory, added into the
//               row's global histogram (non-zero bins only);
//   B  bin      per row: the bin BH holding the k-th largest key, #keys above it;
//   C  refine   per chunk: #keys above BH and the 16-bin histogram of key & 15 in BH;
//   D  thresh   per row: T = BH << 4 | L, need = k - #{key > T}; every chunk's count of
//               keys > T and == T before it (exclusive prefix over the row's chunks);
//   E  emit     per chunk: every position with key > T and the first `need` positions with
//               key == T of the row, in index order, as a bitmap word per thread or as
//               the ascending index list.
//
// The selected set is the one dcr_select.cu produces (the same keys, the same threshold
// and the same lowest-position rule for ties), so both paths are bit-identical. The row
// histogram is cleared by a memset in the step before A.
#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

constexpr int kSsThreads = 256;
constexpr int kSsKeys = 32;                      // keys per thread: one bitmap word
constexpr int kSsChunk = kSsThreads * kSsKeys;   // 8192 positions per chunk
constexpr int kSsBins1 = 4096;                   // key >> 4
constexpr int kSsBins2 = 16;                     // key & 15
constexpr int kSsChunkWords = 1 + kSsBins2;      // per chunk: #above BH, 16 low bins

struct SsParams {
  const uint16_t* scores;  // [rows][stride]
  int64_t stride;
  int N, k, nchunks;
  int keys_in;             // rows hold order keys (else raw bf16 scores)
  int vec;                 // rows 16-byte aligned
  uint32_t* hist;          // [rows][4096], zero on entry to A
  int4* rowinfo;           // [rows]: BH, #above BH, T, need
  uint32_t* chunk;         // [rows][nchunks][17]
  int2* chunk_pre;         // [rows][nchunks]: #key > T and #key == T in earlier chunks
  int32_t* idx;            // [rows][k] (when bits is null)
  int* row_counters;       // Pass 3 split-K tickets reset in B (may be null)
  uint32_t* bits;          // [rows][bits_stride] (optional)
  int64_t bits_stride;
};

// The five kernels run as a chain of programmatic dependent launches: each lets the next
// one launch at its start, and each waits for the previous one (griddepcontrol.wait: that
// grid complete and its writes visible) only before it reads that grid's results, so the
// next kernel's CTAs load Pass 1's keys while the previous one drains.
__device__ __forceinline__ void ss_let_next_launch() {
#if DCR_UNION_PDL
  asm volatile("griddepcontrol.launch_dependents;");
#endif
}
__device__ __forceinline__ void ss_wait_prev() {
#if DCR_UNION_PDL
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

// The 32 keys of this thread, positions [base, base + 32); 0 (below every real key) past N.
__device__ __forceinline__ void ss_load(const SsParams& p, const uint16_t* src, int base,
                                        uint32_t (&key)[kSsKeys]) {
  if (p.vec && base + kSsKeys <= p.N) {
    const uint4* v = reinterpret_cast<const uint4*>(src + base);
#pragma unroll
    for (int j = 0; j < kSsKeys / 8; ++j) {
      const uint4 w = v[j];
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        key[8 * j + 2 * i] = ww[i] & 0xffffu;
        key[8 * j + 2 * i + 1] = ww[i] >> 16;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < kSsKeys; ++e) key[e] = base + e < p.N ? static_cast<uint32_t>(src[base + e]) : 0u;
  }
  if (!p.keys_in) {
#pragma unroll
    for (int e = 0; e < kSsKeys; ++e)
      if (base + e < p.N) key[e] = order_key_fast(key[e]);
  }
}

// A and C need no position order: thread t of the chunk's CTA takes vectors t, t + 256,
// t + 512 and t + 768 (8 keys each), so every load instruction of a warp reads 512
// contiguous bytes. Key 8 i + e sits at position chunk0 + 8 (256 i + t) + e.
__device__ __forceinline__ int ss_pos(int chunk0, int i, int e) {
  return chunk0 + 8 * (kSsThreads * i + static_cast<int>(threadIdx.x)) + e;
}

__device__ __forceinline__ void ss_load_spread(const SsParams& p, const uint16_t* src,
                                               int chunk0, uint32_t (&key)[kSsKeys]) {
#pragma unroll
  for (int i = 0; i < kSsKeys / 8; ++i) {
    const int pos0 = ss_pos(chunk0, i, 0);
    if (p.vec && pos0 + 8 <= p.N) {
      const uint4 w = *reinterpret_cast<const uint4*>(src + pos0);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        key[8 * i + 2 * q] = ww[q] & 0xffffu;
        key[8 * i + 2 * q + 1] = ww[q] >> 16;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        key[8 * i + e] = pos0 + e < p.N ? static_cast<uint32_t>(src[pos0 + e]) : 0u;
    }
    if (!p.keys_in) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (pos0 + e < p.N) key[8 * i + e] = order_key_fast(key[8 * i + e]);
    }
  }
}

// A: the chunk's first-level histogram, added into the row's.
__global__ void __launch_bounds__(kSsThreads) ss_hist_kernel(const SsParams p) {
  __shared__ uint32_t h[kSsBins1];
  ss_let_next_launch();
  const int tid = threadIdx.x;
  const int row = blockIdx.x / p.nchunks;
  const int c = blockIdx.x - row * p.nchunks;
  const uint16_t* src = p.scores + static_cast<int64_t>(row) * p.stride;
  uint32_t key[kSsKeys];
  ss_load(p, src, c * kSsChunk + tid * kSsKeys, key);  // in flight while h is cleared
#pragma unroll
  for (int i = 0; i < kSsBins1 / kSsThreads; ++i) h[tid + i * kSsThreads] = 0u;
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kSsKeys; ++e)
    if (key[e] != 0u) atomicAdd(&h[key[e] >> 4], 1u);
  __syncthreads();
  uint32_t* hrow = p.hist + static_cast<int64_t>(row) * kSsBins1;
#pragma unroll
  for (int i = 0; i < kSsBins1 / kSsThreads; ++i) {
    const uint32_t v = h[tid + i * kSsThreads];
    if (v) atomicAdd(hrow + tid + i * kSsThreads, v);
  }
}

// B: per row, the bin BH with #{bins above} < k <= #{bins above} + count(BH).
__global__ void __launch_bounds__(kSsThreads) ss_bin_kernel(const SsParams p) {
  constexpr int kBpt = kSsBins1 / kSsThreads;  // 16 bins per thread
  constexpr int kWarps = kSsThreads / 32;
  __shared__ uint32_t wsum[kWarps];
  __shared__ int s_found;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int row = blockIdx.x;
  ss_let_next_launch();
  ss_wait_prev();  // A's row histograms
  if (tid == 0) {
    s_found = 0;
    if (p.row_counters != nullptr) p.row_counters[row] = 0;
  }
  // thread t holds bins [kBpt g, kBpt g + kBpt) with g = 255 - t: thread 0 the highest
  const int g = kSsThreads - 1 - tid;
  const uint4* hv = reinterpret_cast<const uint4*>(p.hist + static_cast<int64_t>(row) * kSsBins1 + kBpt * g);
  uint32_t cnt[kBpt], tot = 0;
#pragma unroll
  for (int j = 0; j < kBpt / 4; ++j) {
    const uint4 w = hv[j];
    cnt[4 * j] = w.x;
    cnt[4 * j + 1] = w.y;
    cnt[4 * j + 2] = w.z;
    cnt[4 * j + 3] = w.w;
  }
#pragma unroll
  for (int i = 0; i < kBpt; ++i) tot += cnt[i];
  const uint32_t incl = warp_incl_scan(tot);
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  uint32_t before = 0;
  for (int w = 0; w < warp; ++w) before += wsum[w];
  uint32_t a = before + incl - tot;  // keys in the bins above this thread's
  const uint32_t k = static_cast<uint32_t>(p.k);
  int hit = -1;
  uint32_t hit_above = 0;
#pragma unroll
  for (int i = kBpt - 1; i >= 0; --i) {
    if (a < k && k <= a + cnt[i]) {
      hit = kBpt * g + i;
      hit_above = a;
    }
    a += cnt[i];
  }
  if (hit >= 0) {
    p.rowinfo[row] = make_int4(hit, static_cast<int>(hit_above), 0, 0);
    s_found = 1;
  }
  __syncthreads();
  if (tid == 0 && !s_found) {  // inconsistent counts: select nothing, report
    p.rowinfo[row] = make_int4(-1, 0, 0, 0);
    raise_status(DCR_ERR_DEVICE_INDEX);
  }
}

// C: per chunk, #keys above BH and the low-4-bit histogram of the keys in BH.
__global__ void __launch_bounds__(kSsThreads) ss_refine_kernel(const SsParams p) {
  constexpr int kWarps = kSsThreads / 32;
  __shared__ uint32_t h[kSsBins2];
  __shared__ uint32_t wsum[kWarps];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int row = blockIdx.x / p.nchunks;
  const int c = blockIdx.x - row * p.nchunks;
  const int chunk0 = c * kSsChunk;
  const uint16_t* src = p.scores + static_cast<int64_t>(row) * p.stride;
  ss_let_next_launch();
  uint32_t key[kSsKeys];
  ss_load_spread(p, src, chunk0, key);  // Pass 1's keys: before the wait
  if (tid < kSsBins2) h[tid] = 0u;
  ss_wait_prev();  // B's bins
  // BH's keys are [lo16, lo16 + 15]; with no bin (-1) lo16 = 0xfffffff0 and no key is in
  // or above it. Padding (key 0) is never in BH: a real BH is at least 0x007f >> 4.
  const uint32_t lo16 = static_cast<uint32_t>(p.rowinfo[row].x) << 4;
  const uint32_t hi16 = lo16 | 15u;
  __syncthreads();
  uint32_t above = 0, cand = 0;
#pragma unroll
  for (int e = 0; e < kSsKeys; ++e) {
    if (key[e] > hi16) ++above;
    if (key[e] - lo16 < 16u) cand |= 1u << e;
  }
  // BH holds a few percent of the keys: each is added from its stored key, read again
  while (cand) {
    const int e = __ffs(cand) - 1;
    cand &= cand - 1;
    const int pos = ss_pos(chunk0, e >> 3, e & 7);
    uint32_t x = src[pos];
    if (!p.keys_in) x = order_key_fast(x);
    atomicAdd(&h[x & 15u], 1u);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) above += __shfl_xor_sync(0xffffffffu, above, o);
  if (lane == 0) wsum[warp] = above;
  __syncthreads();
  uint32_t* out = p.chunk + (static_cast<int64_t>(row) * p.nchunks + c) * kSsChunkWords;
  if (tid == 0) {
    uint32_t t = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += wsum[w];
    out[0] = t;
  }
  if (tid < kSsBins2) out[1 + tid] = h[tid];
}

// D: per row (one warp), the threshold key T, need, and every chunk's prefix counts.
__global__ void __launch_bounds__(kSsThreads) ss_thresh_kernel(const SsParams p, int rows) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kSsThreads / 32) + (threadIdx.x >> 5);
  ss_let_next_launch();
  if (row >= rows) return;
  ss_wait_prev();  // C's chunk counts
  const int4 ri = p.rowinfo[row];
  const uint32_t* crow = p.chunk + static_cast<int64_t>(row) * p.nchunks * kSsChunkWords;
  // the row's low-bin histogram: lane l sums chunks l, l + 32, ...
  uint32_t h[kSsBins2];
#pragma unroll
  for (int b = 0; b < kSsBins2; ++b) h[b] = 0u;
  for (int c = lane; c < p.nchunks; c += 32) {
#pragma unroll
    for (int b = 0; b < kSsBins2; ++b) h[b] += crow[c * kSsChunkWords + 1 + b];
  }
#pragma unroll
  for (int b = 0; b < kSsBins2; ++b)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) h[b] += __shfl_xor_sync(0xffffffffu, h[b], o);
  // L: the low bin where the k-th largest key sits (every lane computes the same)
  const uint32_t kk = static_cast<uint32_t>(p.k) - static_cast<uint32_t>(ri.y);
  int L = -1;
  uint32_t cum = 0, cum_at_L = 0;
#pragma unroll
  for (int b = kSsBins2 - 1; b >= 0; --b) {
    if (L < 0 && cum < kk && kk <= cum + h[b]) {
      L = b;
      cum_at_L = cum;
    }
    cum += h[b];
  }
  uint32_t T;
  int need;
  if (ri.x < 0 || L < 0) {  // inconsistent counts: select nothing, report
    T = 0x10000u;
    need = 0;
    L = kSsBins2;  // every low bin counts as "above" nothing below
    if (lane == 0) raise_status(DCR_ERR_DEVICE_INDEX);
  } else {
    T = (static_cast<uint32_t>(ri.x) << 4) | static_cast<uint32_t>(L);
    need = static_cast<int>(kk - cum_at_L);
  }
  if (lane == 0) p.rowinfo[row] = make_int4(ri.x, ri.y, static_cast<int>(T), need);
  // chunk prefixes: #key > T = #above BH + #low bins above L; #key == T = low bin L
  const bool valid = T != 0x10000u;
  int2* pre = p.chunk_pre + static_cast<int64_t>(row) * p.nchunks;
  uint32_t carry_gt = 0, carry_eq = 0;
  for (int c0 = 0; c0 < p.nchunks; c0 += 32) {
    const int c = c0 + lane;
    uint32_t gt = 0, eq = 0;
    if (c < p.nchunks && valid) {
      const uint32_t* cc = crow + c * kSsChunkWords;
      gt = cc[0];
      for (int b = L + 1; b < kSsBins2; ++b) gt += cc[1 + b];
      eq = cc[1 + L];
    }
    const uint32_t ig = warp_incl_scan(gt);
    const uint32_t ie = warp_incl_scan(eq);
    if (c < p.nchunks)
      pre[c] = make_int2(static_cast<int>(carry_gt + ig - gt), static_cast<int>(carry_eq + ie - eq));
    carry_gt += __shfl_sync(0xffffffffu, ig, 31);
    carry_eq += __shfl_sync(0xffffffffu, ie, 31);
  }
}

// E: per chunk, the selected positions in index order.
__global__ void __launch_bounds__(kSsThreads) ss_emit_kernel(const SsParams p) {
  constexpr int kWarps = kSsThreads / 32;
  __shared__ uint32_t wsum[kWarps];
#if DCR_UNION_PDL
  // let the union Pass 3 launch now; it waits for this grid before reading its results
  asm volatile("griddepcontrol.launch_dependents;");
#endif
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int row = blockIdx.x / p.nchunks;
  const int c = blockIdx.x - row * p.nchunks;
  const uint16_t* src = p.scores + static_cast<int64_t>(row) * p.stride;
  const int base = c * kSsChunk + tid * kSsKeys;
  uint32_t key[kSsKeys];
  ss_load(p, src, base, key);  // Pass 1's keys: before the wait
  ss_wait_prev();              // D's thresholds and chunk prefixes
  const int4 ri = p.rowinfo[row];
  const int2 pre = p.chunk_pre[static_cast<int64_t>(row) * p.nchunks + c];
  const uint32_t T = static_cast<uint32_t>(ri.z);
  const int need = ri.w;
  uint32_t gtm = 0u, eqm = 0u;
#pragma unroll
  for (int e = 0; e < kSsKeys; ++e) {
    if (key[e] > T) gtm |= 1u << e;
    if (key[e] == T) eqm |= 1u << e;
  }
  // block exclusive scan of (#gt | #eq << 16): at most 8192 of each per chunk
  const uint32_t packed = static_cast<uint32_t>(__popc(gtm)) | (static_cast<uint32_t>(__popc(eqm)) << 16);
  const uint32_t incl = warp_incl_scan(packed);
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  uint32_t ex = incl - packed;
  for (int w = 0; w < warp; ++w) ex += wsum[w];
  const int eq_before = pre.y + static_cast<int>(ex >> 16);
  int take = need - eq_before;  // ties this thread may take, lowest positions first
  uint32_t sel = gtm;
  const int neq = __popc(eqm);
  if (take >= neq) {
    sel |= eqm;
  } else if (take > 0) {
    uint32_t rem = eqm;
    for (int i = 0; i < take; ++i) rem &= rem - 1;  // drop the lowest `take` bits
    sel |= eqm & ~rem;
  }
  if (p.bits != nullptr) {
    if (base < p.N) p.bits[static_cast<int64_t>(row) * p.bits_stride + (base >> 5)] = sel;
    return;
  }
  int pos = pre.x + static_cast<int>(ex & 0xffffu) + min(eq_before, need);
  int32_t* out = p.idx + static_cast<int64_t>(row) * p.k;
  while (sel) {
    const int b = __ffs(sel) - 1;
    sel &= sel - 1;
    if (pos < p.k) out[pos] = base + b;
    else raise_status(DCR_ERR_DEVICE_INDEX);
    ++pos;
  }
}

// Taken where the one-CTA-per-row kernel would need more than one wave on a 148-SM B200:
// more keys than 148 rows of 32768. The layout reserves the scratch from the same rule, so
// the decision needs no device.
bool select_stream_path(int rows, int N) {
  // Rows of up to 40960 positions take one CTA each (keys in registers): in waves they still
  // beat the chunked kernels (256 rows of 32768: 26.7 against 36.6 us). Longer rows need
  // clusters, whose waves lose to the chunked kernels past one wave of rows.
  return N > 40960 && static_cast<int64_t>(rows) * N > static_cast<int64_t>(148) * 32768;
}

size_t select_stream_bytes(int rows, int N) {
  if (!select_stream_path(rows, N)) return 0;
  const int64_t nchunks = (static_cast<int64_t>(N) + kSsChunk - 1) / kSsChunk;
  size_t b = sizeof(uint32_t) * static_cast<size_t>(rows) * kSsBins1;              // hist
  b += sizeof(int4) * static_cast<size_t>(rows);                                   // rowinfo
  b += sizeof(uint32_t) * static_cast<size_t>(rows) * nchunks * kSsChunkWords;     // chunk
  b += sizeof(int2) * static_cast<size_t>(rows) * nchunks;                         // chunk_pre
  return (b + 255) / 256 * 256 + 4 * 256;  // each part 256-byte aligned
}

int launch_select_stream(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                         int keys_in, int32_t* idx, int* row_counters, uint8_t* scratch,
                         uint32_t* bits, int64_t bits_stride, cudaStream_t st) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  SsParams p;
  p.scores = scores;
  p.stride = s_stride_row;
  p.N = N;
  p.k = k_eff;
  p.nchunks = (N + kSsChunk - 1) / kSsChunk;
  p.keys_in = keys_in;
  p.vec = ((reinterpret_cast<uintptr_t>(scores) & 15u) == 0 && (s_stride_row & 7) == 0) ? 1 : 0;
  size_t off = 0;
  p.hist = reinterpret_cast<uint32_t*>(scratch + off);
  off = al(off + sizeof(uint32_t) * static_cast<size_t>(rows) * kSsBins1);
  p.rowinfo = reinterpret_cast<int4*>(scratch + off);
  off = al(off + sizeof(int4) * static_cast<size_t>(rows));
  p.chunk = reinterpret_cast<uint32_t*>(scratch + off);
  off = al(off + sizeof(uint32_t) * static_cast<size_t>(rows) * p.nchunks * kSsChunkWords);
  p.chunk_pre = reinterpret_cast<int2*>(scratch + off);
  p.idx = idx;
  p.row_counters = row_counters;
  p.bits = bits;
  p.bits_stride = bits_stride;
  const int64_t grid = static_cast<int64_t>(rows) * p.nchunks;
  if (grid > 0x7fffffff) return DCR_ERR_SHAPE;
  if (cudaMemsetAsync(p.hist, 0, sizeof(uint32_t) * static_cast<size_t>(rows) * kSsBins1, st) !=
      cudaSuccess)
    return DCR_ERR_CUDA;
  const unsigned g = static_cast<unsigned>(grid);
  const unsigned rows_grid = static_cast<unsigned>(rows);
  const unsigned thr_grid = static_cast<unsigned>((rows + kSsThreads / 32 - 1) / (kSsThreads / 32));
  ss_hist_kernel<<<g, kSsThreads, 0, st>>>(p);
  // B..E: programmatic dependents of the kernel before them
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = DCR_UNION_PDL ? 1 : 0;
  auto cfg = [&](unsigned grid) {
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(grid);
    c.blockDim = dim3(kSsThreads);
    c.stream = st;
    c.attrs = attr;
    c.numAttrs = 1;
    return c;
  };
  cudaLaunchConfig_t cb = cfg(rows_grid), cc = cfg(g), cd = cfg(thr_grid), ce = cfg(g);
  if (cudaLaunchKernelEx(&cb, ss_bin_kernel, p) != cudaSuccess ||
      cudaLaunchKernelEx(&cc, ss_refine_kernel, p) != cudaSuccess ||
      cudaLaunchKernelEx(&cd, ss_thresh_kernel, p, rows) != cudaSuccess ||
      cudaLaunchKernelEx(&ce, ss_emit_kernel, p) != cudaSuccess)
    return DCR_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

}  // namespace dcr
