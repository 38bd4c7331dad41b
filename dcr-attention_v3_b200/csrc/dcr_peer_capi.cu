// dcr_peer_capi.cu — extern "C" entry points of the peer-memory exchange (dcr_xchg_*) and
// the one-call sequence-sharded step that uses it (dcr_shard_decode_peer).
//
// The reference has no multi-GPU decode; these have no counterpart there. Setup
// allocates (once per decoder, never per step): the exchange buffer is a cudaMalloc'd
// block, so that its CUDA IPC handle names exactly that block.
#include <cuda_runtime.h>

#include <string.h>

#include "dcr_b200.h"
#include "dcr_internal.h"
#include "dcr_peer.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == DCR_IPC_HANDLE_BYTES, "IPC handle size");

using namespace dcr;

extern "C" {

size_t dcr_xchg_bytes(int B, int H, int world) {
  if (B <= 0 || H <= 0 || world < 1 || world > kMaxPeers) return 0;
  if (static_cast<int64_t>(B) * H * kD > 0x7fffffffLL) return 0;
  return static_cast<size_t>(xchg_layout(B * H, world).total);
}

int dcr_xchg_create(int B, int H, int world, void** buf_out, void* ipc_handle_out) {
  if (buf_out == nullptr || ipc_handle_out == nullptr) return DCR_ERR_NULL;
  const size_t bytes = dcr_xchg_bytes(B, H, world);
  if (bytes == 0) return DCR_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return DCR_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return DCR_ERR_CUDA;
  }
  memcpy(ipc_handle_out, &h, sizeof(h));
  *buf_out = p;
  return DCR_OK;
}

int dcr_xchg_open(const void* ipc_handles, int world, int rank, void* buf, void** peers_out) {
  if (ipc_handles == nullptr || buf == nullptr || peers_out == nullptr) return DCR_ERR_NULL;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world) return DCR_ERR_SHAPE;
  for (int p = 0; p < world; ++p) peers_out[p] = nullptr;
  peers_out[rank] = buf;
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(ipc_handles) + static_cast<size_t>(p) * sizeof(h),
           sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      for (int q = 0; q < p; ++q)
        if (q != rank && peers_out[q] != nullptr) cudaIpcCloseMemHandle(peers_out[q]);
      for (int q = 0; q < world; ++q) peers_out[q] = nullptr;
      cudaGetLastError();
      return DCR_ERR_CUDA;
    }
    peers_out[p] = ptr;
  }
  return DCR_OK;
}

int dcr_xchg_close(void* const* peers, int world, int rank) {
  if (peers == nullptr) return DCR_ERR_NULL;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world) return DCR_ERR_SHAPE;
  int st = DCR_OK;
  for (int p = 0; p < world; ++p)
    if (p != rank && peers[p] != nullptr && cudaIpcCloseMemHandle(peers[p]) != cudaSuccess)
      st = DCR_ERR_CUDA;
  return st;
}

int dcr_xchg_destroy(void* buf) {
  if (buf == nullptr) return DCR_ERR_NULL;
  return cudaFree(buf) == cudaSuccess ? DCR_OK : DCR_ERR_CUDA;
}

int dcr_xchg_reset(void* buf, int B, int H, int world, void* stream) {
  if (buf == nullptr) return DCR_ERR_NULL;
  const size_t bytes = dcr_xchg_bytes(B, H, world);
  if (bytes == 0) return DCR_ERR_SHAPE;
  return cudaMemsetAsync(buf, 0, bytes, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? DCR_OK
             : DCR_ERR_CUDA;
}

static int shard_decode_peer_impl(const void* Q, const void* K, const void* V, int dtype,
                                  int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                                  int64_t v_stride_h, int B, int H, int H_kv, int N_local, int D,
                                  int k_eff, float eps, void* const* peers, int world, int rank,
                                  int n_local_max, void* O, void* workspace,
                                  size_t workspace_bytes, void* stream, void* const* events) {
  int st = check_heads(B, H, H_kv, N_local, D);
  if (st) return st;
  if ((st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N_local))) return st;
  if ((st = check_cache(V, dtype, v_stride_b, v_stride_h, B, H_kv, N_local))) return st;
  if (Q == nullptr || O == nullptr || peers == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q) || !aligned16(O)) return DCR_ERR_ALIGN;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world) return DCR_ERR_SHAPE;
  if (n_local_max < N_local) return DCR_ERR_SHAPE;
  for (int p = 0; p < world; ++p)
    if (peers[p] == nullptr) return DCR_ERR_NULL;
  if (k_eff <= 0) return DCR_ERR_K_RANGE;
  const int rows = B * H;
  const ShardLayout w = shard_layout(rows, N_local, k_eff);
  if (workspace == nullptr || workspace_bytes < w.total) return DCR_ERR_WORKSPACE;
  if (!aligned16(workspace)) return DCR_ERR_ALIGN;
  PeerView v = {};
  for (int p = 0; p < world; ++p) v.base[p] = static_cast<uint8_t*>(peers[p]);
  v.world = world;
  v.rank = rank;
  v.rows = rows;
  v.lay = xchg_layout(rows, world);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto mark = [&](int i) -> int {
    if (events == nullptr) return DCR_OK;
    return record_mark(events[i], s);
  };
  if ((st = mark(0))) return st;
  if ((st = launch_score(K, dtype, k_stride_b, k_stride_h, nullptr, Q, eps, B, H, H_kv, N_local,
                         reinterpret_cast<uint16_t*>(ws + w.scores), w.n_pad, 1, s)))
    return st;
  if ((st = mark(1))) return st;
  bool fused = false, bits = false;
  const bool use_union = union_enabled() && union_supported(dtype, H, H_kv);
  if ((st = launch_shard_select_fused(w, ws, rows, N_local, n_local_max, k_eff, &v, s, &fused,
                                      &bits, use_union)))
    return st;
  if (fused) {
    if ((st = mark(2)) || (st = mark(3))) return st;
  } else {
    if ((st = launch_shard_hist(w, ws, rows, N_local, k_eff, 0, nullptr, nullptr, &v, s)))
      return st;
    if ((st = mark(2))) return st;
    if ((st = launch_shard_hist(w, ws, rows, N_local, k_eff, 1, nullptr, nullptr, &v, s)))
      return st;
    if ((st = mark(3))) return st;
    if ((st = launch_shard_select(w, ws, rows, N_local, k_eff, nullptr, world, rank, &v, s)))
      return st;
  }
  if ((st = mark(4))) return st;
  // Pass 3 publishes its states into the exchange buffers; the pointer only selects the
  // state output
  float* own_state = reinterpret_cast<float*>(v.base[rank] + v.lay.st);
  if (fused && bits && use_union) {
    // the union Pass 3 over the fused selection's bitmaps
    if ((st = launch_attend_union(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h,
                                  reinterpret_cast<const int32_t*>(ws + w.idx),
                                  reinterpret_cast<const uint32_t*>(ws + w.bits), w.bits_stride,
                                  B, H, H_kv, N_local, w.cap, nullptr,
                                  reinterpret_cast<float*>(ws + w.partials), w.part_splits,
                                  reinterpret_cast<int*>(ws + w.counters), s, own_state, &v)))
      return st;
  } else if ((st = launch_attend(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h,
                          reinterpret_cast<const int32_t*>(ws + w.idx),
                          reinterpret_cast<const int32_t*>(ws + w.count), B, H, H_kv, N_local,
                          w.cap, nullptr, own_state, w.splits,
                          reinterpret_cast<float*>(ws + w.partials),
                          reinterpret_cast<int*>(ws + w.counters), &v, s)))
    return st;
  if ((st = mark(5))) return st;
  if ((st = launch_shard_combine(nullptr, world, rows, dtype, O, &v, s))) return st;
  return mark(6);
}

int dcr_shard_decode_peer(const void* Q, const void* K, const void* V, int dtype,
                          int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                          int64_t v_stride_h, int B, int H, int H_kv, int N_local, int D,
                          int k_eff, float eps, void* const* peers, int world, int rank,
                          int n_local_max, void* O, void* workspace, size_t workspace_bytes,
                          void* stream) {
  return shard_decode_peer_impl(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h,
                                B, H, H_kv, N_local, D, k_eff, eps, peers, world, rank,
                                n_local_max, O, workspace, workspace_bytes, stream, nullptr);
}

int dcr_shard_decode_peer_timed(const void* Q, const void* K, const void* V, int dtype,
                                int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                                int64_t v_stride_h, int B, int H, int H_kv, int N_local, int D,
                                int k_eff, float eps, void* const* peers, int world, int rank,
                                int n_local_max, void* O, void* workspace,
                                size_t workspace_bytes, void* stream, void* const* events) {
  if (events == nullptr) return DCR_ERR_NULL;
  for (int i = 0; i < 7; ++i)
    if (events[i] == nullptr) return DCR_ERR_NULL;
  return shard_decode_peer_impl(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h,
                                B, H, H_kv, N_local, D, k_eff, eps, peers, world, rank,
                                n_local_max, O, workspace, workspace_bytes, stream, events);
}

}  // extern "C"
