// dcr_internal.h — launch helpers shared by the translation units of libdcr_b200.
// Every launcher validates nothing (the C-ABI layer in dcr_capi.cu does) and returns a
// dcr_status code (DCR_ERR_CUDA when a launch fails).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "dcr_b200.h"

namespace dcr {

struct PeerView;  // dcr_peer.cuh

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Records a timing event on stream s. Inside a stream capture the record becomes an
// external event-record node of the graph, so every replay of the graph stamps the event
// (a plain record there only orders the capture and is never timed).
inline int record_mark(void* event, cudaStream_t s) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) return DCR_ERR_CUDA;
  const cudaError_t e =
      cap == cudaStreamCaptureStatusActive
          ? cudaEventRecordWithFlags(static_cast<cudaEvent_t>(event), s, cudaEventRecordExternal)
          : cudaEventRecord(static_cast<cudaEvent_t>(event), s);
  return e == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

// Sets the dynamic shared-memory limit of a kernel once per (kernel, device).
cudaError_t ensure_smem_attr(const void* func, int bytes);

// Launches a kernel as a grid of 1-D thread-block clusters of `cluster` CTAs.
template <typename Kernel, typename... Args>
cudaError_t launch_cluster(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                           int cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Split-K factor used by Pass 3 for this shape (1 = no split, no workspace partials).
int attend_splits(int rows, int k_eff);

// Union Pass 3 (dcr_attend_union.cu): positions per CTA range at most kUnSpanMax; the
// workspace partials hold union_max_splits(N) splits per row.
constexpr int kUnSpanMax = 4096;
int union_max_splits(int N);
bool union_supported(int dtype, int H, int H_kv);
bool union_enabled();
int launch_attend_union(const void* Q, const void* K, const void* V, int dtype, int64_t ksb,
                        int64_t ksh, int64_t vsb, int64_t vsh, const int32_t* idx,
                        const uint32_t* bits, int64_t bits_stride, int B, int H, int H_kv, int N,
                        int k_eff, void* O, float* partials, int part_splits, int* counters,
                        cudaStream_t st, float* state = nullptr,
                        const struct PeerView* pv = nullptr);

// Workspace layout shared by dcr_decode / dcr_select_indices / dcr_attend.
struct WorkspaceLayout {
  size_t counters;  // int32 [rows]
  size_t partials;  // fp32 [rows * splits * (D + 2)]
  size_t scores;    // uint16 [rows * n_pad]
  size_t idx;       // int32 [rows * k_eff]
  size_t bits;      // uint32 [rows * bits_stride] selection bitmaps (union Pass 3 only)
  int64_t bits_stride;
  size_t sel;       // the chunked Pass 2's scratch (select_stream_bytes; 0 bytes if unused)
  size_t sel_bytes;
  size_t total;
  int splits;
  int part_splits;  // splits the partials hold (>= splits; the union Pass 3 may use more)
  int64_t n_pad;
};
WorkspaceLayout workspace_layout(int rows, int N, int k_eff);

int launch_unit_query(const void* Q, int dtype, int rows, float eps, float* u, cudaStream_t st);

// keys_out != 0: store 16-bit order keys (bf16_order_key) instead of bf16 score bits.
int launch_score(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h,
                 const float* u, const void* Q, float eps, int B, int H, int H_kv, int N,
                 uint16_t* scores, int64_t s_stride_row, int keys_out, cudaStream_t st);

// keys_in != 0: the rows hold order keys (from launch_score with keys_out) not bf16 bits.
// bits (optional): when the threads' positions tile the row in whole 32-bit words (8, 16
// or a multiple of 32 positions per thread, segments starting on words), the selection is
// written as a bitmap [rows][bits_stride] words (bit n of word n / 32) instead of the index
// lists, and *bits_written is set to 1; otherwise idx is written and it is 0.
// scratch (optional, select_stream_bytes(rows, N) bytes): where select_stream_path(rows, N)
// holds, the selection runs as the chunked kernels of dcr_select_stream.cu (bit-identical
// output, always as bitmaps when bits is given); without it, the one-CTA-per-row kernel.
int launch_select(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                  int keys_in, int32_t* idx, int* row_counters, cudaStream_t st,
                  uint32_t* bits = nullptr, int64_t bits_stride = 0, int* bits_written = nullptr,
                  uint8_t* scratch = nullptr);
bool select_stream_path(int rows, int N);
size_t select_stream_bytes(int rows, int N);
int launch_select_stream(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                         int keys_in, int32_t* idx, int* row_counters, uint8_t* scratch,
                         uint32_t* bits, int64_t bits_stride, cudaStream_t st);

// counts (optional): row r attends to the first counts[r] of its k_eff index slots.
// state (optional): write the unnormalised (m, l, o[D]) per row (m in base-2 units of
// the scaled scores) instead of O.
int launch_attend(const void* Q, const void* K, const void* V, int dtype, int64_t k_stride_b,
                  int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_h,
                  const int32_t* idx, const int32_t* counts, int B, int H, int H_kv, int N,
                  int k_eff, void* O, float* state, int splits, float* partials, int* counters,
                  const struct PeerView* pv, cudaStream_t st);

// Workspace layout of the sequence-sharded step (dcr_shard_*): a dcr_decode layout for
// the local chunk plus the selection's bookkeeping.
struct ShardLayout {
  size_t counters;   // int32 [rows] Pass 3 split-K tickets
  size_t partials;   // fp32 [rows * splits * (D + 2)]
  size_t scores;     // uint16 [rows * n_pad] order keys of the local chunk
  size_t idx;        // int32 [rows * cap] selected local positions
  size_t count;      // int32 [rows]
  size_t row_state;  // int32 [rows * 4]
  size_t chunk_cnt;  // uint32 [rows * chunks]
  size_t bits;       // uint32 [rows * bits_stride] selection bitmaps (fused selection)
  int64_t bits_stride;
  size_t mode;       // int32: 1 if the last selection wrote bitmaps only, else 0
  size_t total;
  int splits, cap, chunks;
  int part_splits;   // splits the partials hold (the union Pass 3 may use more)
  int64_t n_pad;
};
ShardLayout shard_layout(int rows, int N_local, int k_eff);

// level 0: high-byte histogram of the local keys; level 1: low-byte histogram of the keys
// in the bin that hist_hi_sum (summed over ranks) puts the k-th largest key in.
// pv (optional, all launchers below): exchange with the peers' buffers inside the kernels
// instead of through the caller's collectives.
int launch_shard_hist(const ShardLayout& w, uint8_t* ws, int rows, int N_local, int k_eff,
                      int level, const int32_t* hist_hi_sum, int32_t* hist_out,
                      const struct PeerView* pv, cudaStream_t st);
// This rank's selected positions (ascending) and counts from all ranks' low-byte histograms.
int launch_shard_select(const ShardLayout& w, uint8_t* ws, int rows, int N_local, int k_eff,
                        const int32_t* hist_lo_all, int world, int rank,
                        const struct PeerView* pv, cudaStream_t st);
int launch_shard_combine(const float* states, int world, int rows, int dtype, void* O,
                         const struct PeerView* pv, cudaStream_t st);
// Peer mode: phases 1-3b in one cooperative launch when every rank's chunk fits one CTA
// per row (n_local_max, the longest chunk of all ranks, <= 32768: every rank decides
// alike); *launched tells whether it ran. DCR_ERR_SHAPE if the rows cannot all be
// resident (every rank, same GPUs, fails alike).
// *bits_written: the selection was also written as bitmaps (w.bits; every thread's
// positions are whole 32-bit words), which the union Pass 3 reads.
// bits_only: where the bitmaps are written, skip the index lists (the caller's union
// Pass 3 reads the bitmaps only; launch_shard_selection_out rebuilds the lists on request).
int launch_shard_select_fused(const ShardLayout& w, uint8_t* ws, int rows, int N_local,
                              int n_local_max, int k_eff, const struct PeerView* pv,
                              cudaStream_t st, bool* launched, bool* bits_written = nullptr,
                              bool bits_only = false);
// The last step's selection as index lists [rows][cap] and counts [rows].
int launch_shard_selection_out(const ShardLayout& w, const uint8_t* ws, int rows, int N_local,
                               int k_eff, int32_t* idx_out, int32_t* count_out, cudaStream_t st);

// Projected-score mode (dcr_project.cu). Append: copies n_new rows of K and V into the
// caches at position pos (k_cache may be null: no copy) and writes their projection
// KP = K . P (kp may be null). Score: Pass 1 from KP [B, H_kv, N, R] and P [D][R].
int launch_append(const void* k_new, const void* v_new, int64_t nsb, int64_t nsh, void* k_cache,
                  void* v_cache, int64_t csb, int64_t csh, void* kp, int64_t psb, int64_t psh,
                  const float* P, int B, int H_kv, int n_new, int pos, int dtype,
                  cudaStream_t st);
// qp (optional): the projected unit queries [B*H][R] (from the decode prologue).
int launch_score_projected(const void* KP, int dtype, int64_t p_stride_b, int64_t p_stride_h,
                           const void* Q, const float* P, const float* qp, float eps, int B,
                           int H, int H_kv, int N, uint16_t* scores, int64_t s_stride,
                           int keys_out, cudaStream_t st);
// Decode prologue (dcr_rope.cu): RoPE of the step's q and k rows, cache append at pos,
// and (optional) KP of the new key row and the projected unit queries qp. q_sb / kv_sb:
// elements between the batch rows of q and of k, v (0: contiguous [B, H or H_kv, D]).
int launch_rope_append(const void* q, const void* k, const void* v, const void* cos,
                       const void* sin, int dtype, int B, int H, int H_kv, void* q_out,
                       void* k_cache, void* v_cache, int64_t csb, int64_t csh, int pos,
                       void* kp, int64_t psb, int64_t psh, const float* P, float* qp,
                       float eps, cudaStream_t st,
                       int64_t q_sb = 0, int64_t kv_sb = 0);

}  // namespace dcr
