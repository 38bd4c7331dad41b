// dcr_capi.cu — extern "C" entry points of libdcr_b200 (declared in include/dcr_b200.h).
//
// This layer validates arguments the way the reference's Python wrappers do
// (dcr_attention/kernel/triton/topk_axis.py:37-44, topk_axis_pass1.py:114-130,
// topk_axis_pass2.py:30-36, fused_attn.py:170-193), lays out the caller's workspace and
// enqueues the kernels on the caller's stream. It allocates nothing and never
// synchronises (except dcr_read_device_status, a diagnostic).
#include <cuda_runtime.h>

#include <math.h>
#include <mutex>
#include <map>
#include <set>
#include <utility>

#include "dcr_b200.h"
#include "dcr_common.cuh"
#include "dcr_internal.h"

namespace dcr {

int device_sm_count() {
  static int cache[128] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

cudaError_t ensure_smem_attr(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> limit;  // the largest size set so far
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = limit.find({func, dev});
  if (it != limit.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) limit[{func, dev}] = bytes;
  return e;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

WorkspaceLayout workspace_layout(int rows, int N, int k_eff) {
  WorkspaceLayout w;
  w.splits = attend_splits(rows, k_eff);
  w.part_splits = w.splits;
  if (union_enabled() && union_max_splits(N) > w.part_splits) w.part_splits = union_max_splits(N);
  w.n_pad = (static_cast<int64_t>(N) + 7) / 8 * 8;
  size_t off = 0;
  w.counters = off;
  off = align_up(off + sizeof(int) * static_cast<size_t>(rows), 256);
  w.partials = off;
  off = align_up(off + sizeof(float) * static_cast<size_t>(rows) * w.part_splits * (kD + 2), 256);
  w.scores = off;
  off = align_up(off + sizeof(uint16_t) * static_cast<size_t>(rows) * w.n_pad, 256);
  w.idx = off;
  off = align_up(off + sizeof(int32_t) * static_cast<size_t>(rows) * k_eff, 256);
  w.bits = off;
  w.bits_stride = 0;
  if (union_enabled()) {
    w.bits_stride = (static_cast<int64_t>(N) + 31) / 32;
    off = align_up(off + sizeof(uint32_t) * static_cast<size_t>(rows) * w.bits_stride, 256);
  }
  w.sel = off;
  w.sel_bytes = select_stream_bytes(rows, N);
  off = align_up(off + w.sel_bytes, 256);
  w.total = off;
  return w;
}

}  // namespace dcr

using namespace dcr;

namespace {

size_t dtype_bytes(int dtype) {
  switch (dtype) {
    case DCR_DTYPE_BF16:
    case DCR_DTYPE_F16: return 2;
    case DCR_DTYPE_F32: return 4;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_heads(int B, int H, int H_kv, int N, int D) {
  if (B <= 0 || H <= 0 || H_kv <= 0 || N <= 0) return DCR_ERR_SHAPE;
  if (D != kD) return DCR_ERR_SHAPE;
  if (H % H_kv != 0) return DCR_ERR_SHAPE;
  const int G = H / H_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return DCR_ERR_SHAPE;
  if (static_cast<int64_t>(B) * H * kD > 0x7fffffffLL) return DCR_ERR_SHAPE;
  return DCR_OK;
}

// The stride of a size-1 dimension never enters an address; replace it by the natural one
// so that tensor-map encoding (which checks every stride) accepts views with odd strides
// there (torch gives size-1 dims arbitrary strides).
void normalize_strides(int64_t& sb, int64_t& sh, int B, int H_kv, int N) {
  if (H_kv == 1) sh = static_cast<int64_t>(N) * kD;
  if (B == 1) sb = sh * H_kv;
}

int check_cache(const void* C, int dtype, int64_t& sb, int64_t& sh, int B, int H_kv, int N) {
  if (C == nullptr) return DCR_ERR_NULL;
  normalize_strides(sb, sh, B, H_kv, N);
  const size_t eb = dtype_bytes(dtype);
  if (eb == 0) return DCR_ERR_DTYPE;
  if (!aligned16(C)) return DCR_ERR_ALIGN;
  if (sb < 0 || sh < 0) return DCR_ERR_SHAPE;
  if ((sb * static_cast<int64_t>(eb)) % 16 != 0 || (sh * static_cast<int64_t>(eb)) % 16 != 0)
    return DCR_ERR_ALIGN;
  // rows of one head must not overlap the next head / batch entry
  if (H_kv > 1 && sh < static_cast<int64_t>(N) * kD) return DCR_ERR_SHAPE;
  if (B > 1 && sb < static_cast<int64_t>(N) * kD) return DCR_ERR_SHAPE;
  return DCR_OK;
}

int check_k(int k_eff, int N) { return (k_eff > 0 && k_eff < N) ? DCR_OK : DCR_ERR_K_RANGE; }

}  // namespace

extern "C" {

int dcr_version(void) { return DCR_ABI_VERSION; }

const char* dcr_status_string(int status) {
  switch (status) {
    case DCR_OK: return "ok";
    case DCR_ERR_NULL: return "a required pointer is NULL";
    case DCR_ERR_SHAPE: return "unsupported shape or stride (D must be 64, H/H_kv in {1,2,4,8})";
    case DCR_ERR_K_RANGE: return "k_eff must be in (0, N); caller must dispatch to SDPA";
    case DCR_ERR_DTYPE: return "unknown dtype code";
    case DCR_ERR_ALIGN: return "pointer or stride is not 16-byte aligned";
    case DCR_ERR_WORKSPACE: return "workspace is NULL or smaller than dcr_workspace_bytes()";
    case DCR_ERR_CUDA: return "a CUDA runtime call failed";
    case DCR_ERR_DEVICE_TIMEOUT: return "device: a bounded wait expired";
    case DCR_ERR_NOALLOC_LIMIT:
      return "shape needs more scratch than dcr_decode_noalloc's 16 MiB array; use dcr_decode";
    case DCR_ERR_DEVICE_INDEX: return "device: an index outside [0, N) was skipped";
    case DCR_ERR_DEVICE_SHARD:
      return "device: sharded selection saw inconsistent global histograms (k_eff >= total N?)";
    default: return "unknown status";
  }
}

int dcr_adaptive_k_window(int k_window_min, int n_kv, double coverage_floor) {
  // adaptive_k_window, dcr_attention/models/llama/adaptive.py:85-105
  if (n_kv <= 0) return -1;
  if (!(coverage_floor >= 0.0 && coverage_floor <= 1.0)) return -1;
  const long long floor_value = static_cast<long long>(static_cast<double>(n_kv) * coverage_floor);
  long long k = floor_value > k_window_min ? floor_value : k_window_min;
  if (k > n_kv) k = n_kv;
  if (k % 2 == 1) k = (k + 1 < n_kv) ? k + 1 : n_kv;
  return static_cast<int>(k);
}

size_t dcr_workspace_bytes(int B, int H, int H_kv, int N, int D, int k_eff) {
  if (check_heads(B, H, H_kv, N, D) != DCR_OK || k_eff <= 0) return 0;
  return workspace_layout(B * H, N, k_eff).total;
}

int dcr_unit_query(const void* Q, int dtype, int B, int H, int D, float eps, float* u_out,
                   void* stream) {
  if (Q == nullptr || u_out == nullptr) return DCR_ERR_NULL;
  if (dtype_bytes(dtype) == 0) return DCR_ERR_DTYPE;
  if (B <= 0 || H <= 0 || D != kD) return DCR_ERR_SHAPE;
  if (!aligned16(Q) || !aligned16(u_out)) return DCR_ERR_ALIGN;
  return launch_unit_query(Q, dtype, B * H, eps, u_out, static_cast<cudaStream_t>(stream));
}

int dcr_score(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h, const float* u,
              const void* Q, float eps, int B, int H, int H_kv, int N, int D, uint16_t* scores,
              int64_t s_stride_row, void* stream) {
  int st = check_heads(B, H, H_kv, N, D);
  if (st) return st;
  st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N);
  if (st) return st;
  if (scores == nullptr) return DCR_ERR_NULL;
  if (u == nullptr && Q == nullptr) return DCR_ERR_NULL;
  if (u != nullptr && !aligned16(u)) return DCR_ERR_ALIGN;
  if (u == nullptr && !aligned16(Q)) return DCR_ERR_ALIGN;
  if (s_stride_row < N) return DCR_ERR_SHAPE;
  return launch_score(K, dtype, k_stride_b, k_stride_h, u, Q, eps, B, H, H_kv, N, scores,
                      s_stride_row, 0, static_cast<cudaStream_t>(stream));
}

int dcr_select(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
               int32_t* idx_out, void* stream) {
  if (scores == nullptr || idx_out == nullptr) return DCR_ERR_NULL;
  if (rows <= 0 || N <= 0 || s_stride_row < N) return DCR_ERR_SHAPE;
  int st = check_k(k_eff, N);
  if (st) return st;
  return launch_select(scores, s_stride_row, rows, N, k_eff, 0, idx_out, nullptr,
                       static_cast<cudaStream_t>(stream));
}

size_t dcr_select_workspace_bytes(int rows, int N) {
  if (rows <= 0 || N <= 0) return 0;
  return select_stream_bytes(rows, N);
}

int dcr_select_ws(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                  int32_t* idx_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (scores == nullptr || idx_out == nullptr) return DCR_ERR_NULL;
  if (rows <= 0 || N <= 0 || s_stride_row < N) return DCR_ERR_SHAPE;
  int st = check_k(k_eff, N);
  if (st) return st;
  const size_t need = select_stream_bytes(rows, N);
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes < need) return DCR_ERR_WORKSPACE;
    if (!aligned16(workspace)) return DCR_ERR_ALIGN;
  }
  return launch_select(scores, s_stride_row, rows, N, k_eff, 0, idx_out, nullptr,
                       static_cast<cudaStream_t>(stream), nullptr, 0, nullptr,
                       need > 0 ? static_cast<uint8_t*>(workspace) : nullptr);
}

int dcr_attend(const void* Q, const void* K, const void* V, int dtype, int64_t k_stride_b,
               int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_h, const int32_t* idx,
               int B, int H, int H_kv, int N, int D, int k_eff, void* O, void* workspace,
               size_t workspace_bytes, void* stream) {
  int st = check_heads(B, H, H_kv, N, D);
  if (st) return st;
  if ((st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N))) return st;
  if ((st = check_cache(V, dtype, v_stride_b, v_stride_h, B, H_kv, N))) return st;
  if (Q == nullptr || O == nullptr || idx == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q) || !aligned16(O)) return DCR_ERR_ALIGN;
  if ((st = check_k(k_eff, N))) return st;
  const int rows = B * H;
  const WorkspaceLayout w = workspace_layout(rows, N, k_eff);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partials = nullptr;
  int* counters = nullptr;
  if (w.splits > 1) {
    if (workspace == nullptr || workspace_bytes < w.total) return DCR_ERR_WORKSPACE;
    if (!aligned16(workspace)) return DCR_ERR_ALIGN;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    partials = reinterpret_cast<float*>(ws + w.partials);
    counters = reinterpret_cast<int*>(ws + w.counters);
    if (cudaMemsetAsync(counters, 0, sizeof(int) * rows, s) != cudaSuccess) return DCR_ERR_CUDA;
  }
  return launch_attend(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, idx,
                       nullptr, B, H, H_kv, N, k_eff, O, nullptr, w.splits, partials, counters,
                       nullptr, s);
}

int dcr_select_indices(const void* Q, const void* K, int dtype, int64_t k_stride_b,
                       int64_t k_stride_h, int B, int H, int H_kv, int N, int D, int k_eff,
                       float eps, int32_t* idx_out, void* workspace, size_t workspace_bytes,
                       void* stream) {
  int st = check_heads(B, H, H_kv, N, D);
  if (st) return st;
  if ((st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N))) return st;
  if (Q == nullptr || idx_out == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q)) return DCR_ERR_ALIGN;
  if ((st = check_k(k_eff, N))) return st;
  const int rows = B * H;
  const WorkspaceLayout w = workspace_layout(rows, N, k_eff);
  if (workspace == nullptr || workspace_bytes < w.total) return DCR_ERR_WORKSPACE;
  if (!aligned16(workspace)) return DCR_ERR_ALIGN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* scores = reinterpret_cast<uint16_t*>(ws + w.scores);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = launch_score(K, dtype, k_stride_b, k_stride_h, nullptr, Q, eps, B, H, H_kv, N, scores,
                         w.n_pad, 1, s)))
    return st;
  return launch_select(scores, w.n_pad, rows, N, k_eff, 1, idx_out, nullptr, s, nullptr, 0,
                       nullptr, w.sel_bytes ? ws + w.sel : nullptr);
}

// Projected-score inputs of a decode step (null kp: the exact Pass 1 on K).
struct ProjArgs {
  const void* kp;
  int64_t psb, psh;
  const float* P;
  const float* qp;  // optional projected unit queries
};

static int check_proj(const void* KP, int dtype, int64_t& psb, int64_t& psh, int B, int H_kv,
                      int N, const float* P, int R) {
  if (KP == nullptr || P == nullptr) return DCR_ERR_NULL;
  if (R != DCR_PROJ_RANK) return DCR_ERR_SHAPE;
  const size_t eb = dtype_bytes(dtype);
  if (eb == 0) return DCR_ERR_DTYPE;
  if (H_kv == 1) psh = static_cast<int64_t>(N) * R;
  if (B == 1) psb = psh * H_kv;
  if (!aligned16(KP) || (reinterpret_cast<uintptr_t>(P) & 3u) != 0) return DCR_ERR_ALIGN;
  if (psb < 0 || psh < 0) return DCR_ERR_SHAPE;
  if ((psb * static_cast<int64_t>(eb)) % 16 != 0 || (psh * static_cast<int64_t>(eb)) % 16 != 0)
    return DCR_ERR_ALIGN;
  if (H_kv > 1 && psh < static_cast<int64_t>(N) * R) return DCR_ERR_SHAPE;
  if (B > 1 && psb < static_cast<int64_t>(N) * R) return DCR_ERR_SHAPE;
  return DCR_OK;
}

static int decode_impl(const void* Q, const void* K, const void* V, int dtype,
                       int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                       int64_t v_stride_h, int B, int H, int H_kv, int N, int D, int k_eff,
                       float eps, void* O, void* workspace, size_t workspace_bytes,
                       void* stream, void* const* events, const ProjArgs* proj = nullptr,
                       int passes = 3) {
  int st = check_heads(B, H, H_kv, N, D);
  if (st) return st;
  if ((st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N))) return st;
  if ((st = check_cache(V, dtype, v_stride_b, v_stride_h, B, H_kv, N))) return st;
  if (Q == nullptr || O == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q) || !aligned16(O)) return DCR_ERR_ALIGN;
  if ((st = check_k(k_eff, N))) return st;
  const int rows = B * H;
  const WorkspaceLayout w = workspace_layout(rows, N, k_eff);
  if (workspace == nullptr || workspace_bytes < w.total) return DCR_ERR_WORKSPACE;
  if (!aligned16(workspace)) return DCR_ERR_ALIGN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* scores = reinterpret_cast<uint16_t*>(ws + w.scores);
  int32_t* idx = reinterpret_cast<int32_t*>(ws + w.idx);
  int* counters = reinterpret_cast<int*>(ws + w.counters);
  float* partials = reinterpret_cast<float*>(ws + w.partials);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto mark = [&](int i) -> int {
    if (events == nullptr) return DCR_OK;
    return record_mark(events[i], s);
  };
  if ((st = mark(0))) return st;
  // Pass 1 stores order keys, which Pass 2 reads directly.
  if (proj != nullptr)
    st = launch_score_projected(proj->kp, dtype, proj->psb, proj->psh, Q, proj->P, proj->qp,
                                eps, B, H, H_kv, N, scores, w.n_pad, 1, s);
  else
    st = launch_score(K, dtype, k_stride_b, k_stride_h, nullptr, Q, eps, B, H, H_kv, N, scores,
                      w.n_pad, 1, s);
  if (st) return st;
  if ((st = mark(1))) return st;
  if (passes < 2) return DCR_OK;
  // Pass 2 also resets the Pass 3 split-K tickets of its row.
  // With the union Pass 3, Pass 2 writes selection bitmaps where its layout allows.
  const bool use_union = union_enabled() && union_supported(dtype, H, H_kv);
  uint32_t* bits = reinterpret_cast<uint32_t*>(ws + w.bits);
  int bits_written = 0;
  if ((st = launch_select(scores, w.n_pad, rows, N, k_eff, 1, idx, counters, s,
                          use_union ? bits : nullptr, w.bits_stride, &bits_written,
                          w.sel_bytes ? ws + w.sel : nullptr)))
    return st;
  if ((st = mark(2))) return st;
  if (passes < 3) return DCR_OK;
  if (use_union) {
    if ((st = launch_attend_union(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h,
                                  idx, bits_written ? bits : nullptr, w.bits_stride, B, H, H_kv,
                                  N, k_eff, O, partials, w.part_splits, counters, s)))
      return st;
    return mark(3);
  }
  if ((st = launch_attend(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, idx,
                          nullptr, B, H, H_kv, N, k_eff, O, nullptr, w.splits, partials,
                          counters, nullptr, s)))
    return st;
  return mark(3);
}

int dcr_decode(const void* Q, const void* K, const void* V, int dtype, int64_t k_stride_b,
               int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_h, int B, int H,
               int H_kv, int N, int D, int k_eff, float eps, void* O, void* workspace,
               size_t workspace_bytes, void* stream) {
  return decode_impl(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, B, H, H_kv,
                     N, D, k_eff, eps, O, workspace, workspace_bytes, stream, nullptr);
}

int dcr_decode_timed(const void* Q, const void* K, const void* V, int dtype, int64_t k_stride_b,
                     int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_h, int B, int H,
                     int H_kv, int N, int D, int k_eff, float eps, void* O, void* workspace,
                     size_t workspace_bytes, void* stream, void* const* events) {
  if (events == nullptr) return DCR_ERR_NULL;
  for (int i = 0; i < 4; ++i)
    if (events[i] == nullptr) return DCR_ERR_NULL;
  return decode_impl(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, B, H, H_kv,
                     N, D, k_eff, eps, O, workspace, workspace_bytes, stream, events);
}

int dcr_decode_prefix(const void* Q, const void* K, const void* V, int dtype,
                      int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                      int64_t v_stride_h, int B, int H, int H_kv, int N, int D, int k_eff,
                      float eps, void* O, void* workspace, size_t workspace_bytes, void* stream,
                      int passes) {
  if (passes < 1 || passes > 3) return DCR_ERR_SHAPE;
  return decode_impl(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, B, H, H_kv,
                     N, D, k_eff, eps, O, workspace, workspace_bytes, stream, nullptr, nullptr,
                     passes);
}

// ---- projected-score mode --------------------------------------------------------------

int dcr_project_keys(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h, int B,
                     int H_kv, int N, int D, const float* P, int R, void* KP,
                     int64_t p_stride_b, int64_t p_stride_h, void* stream) {
  if (B <= 0 || H_kv <= 0 || N <= 0 || D != kD) return DCR_ERR_SHAPE;
  int st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N);
  if (st) return st;
  if ((st = check_proj(KP, dtype, p_stride_b, p_stride_h, B, H_kv, N, P, R))) return st;
  return launch_append(K, K, k_stride_b, k_stride_h, nullptr, nullptr, 0, 0, KP, p_stride_b,
                       p_stride_h, P, B, H_kv, N, 0, dtype, static_cast<cudaStream_t>(stream));
}

int dcr_cache_append(const void* K_new, const void* V_new, int dtype, int64_t new_stride_b,
                     int64_t new_stride_h, int B, int H_kv, int n_new, int D, void* K_cache,
                     void* V_cache, int64_t c_stride_b, int64_t c_stride_h, int pos, int N_max,
                     const float* P, int R, void* KP_cache, int64_t p_stride_b,
                     int64_t p_stride_h, void* stream) {
  if (B <= 0 || H_kv <= 0 || n_new <= 0 || N_max <= 0 || D != kD) return DCR_ERR_SHAPE;
  if (pos < 0 || static_cast<int64_t>(pos) + n_new > N_max) return DCR_ERR_SHAPE;
  int64_t vsb = new_stride_b, vsh = new_stride_h, cvb = c_stride_b, cvh = c_stride_h;
  int st = check_cache(K_new, dtype, new_stride_b, new_stride_h, B, H_kv, n_new);
  if (st) return st;
  if ((st = check_cache(V_new, dtype, vsb, vsh, B, H_kv, n_new))) return st;
  if ((st = check_cache(K_cache, dtype, c_stride_b, c_stride_h, B, H_kv, N_max))) return st;
  if ((st = check_cache(V_cache, dtype, cvb, cvh, B, H_kv, N_max))) return st;
  if (KP_cache != nullptr || P != nullptr)
    if ((st = check_proj(KP_cache, dtype, p_stride_b, p_stride_h, B, H_kv, N_max, P, R)))
      return st;
  return launch_append(K_new, V_new, new_stride_b, new_stride_h, K_cache, V_cache, c_stride_b,
                       c_stride_h, KP_cache, p_stride_b, p_stride_h, P, B, H_kv, n_new, pos,
                       dtype, static_cast<cudaStream_t>(stream));
}

int dcr_score_projected(const void* KP, int dtype, int64_t p_stride_b, int64_t p_stride_h,
                        const void* Q, float eps, const float* P, int R, const float* qp, int B,
                        int H, int H_kv, int N, int D, uint16_t* scores, int64_t s_stride_row,
                        void* stream) {
  int st = check_heads(B, H, H_kv, N, D);
  if (st) return st;
  if ((st = check_proj(KP, dtype, p_stride_b, p_stride_h, B, H_kv, N, P, R))) return st;
  if (Q == nullptr || scores == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q)) return DCR_ERR_ALIGN;
  if (s_stride_row < N) return DCR_ERR_SHAPE;
  return launch_score_projected(KP, dtype, p_stride_b, p_stride_h, Q, P, qp, eps, B, H, H_kv,
                                N, scores, s_stride_row, 0, static_cast<cudaStream_t>(stream));
}

int dcr_select_indices_projected(const void* Q, const void* KP, int dtype, int64_t p_stride_b,
                                 int64_t p_stride_h, const float* P, int R, const float* qp,
                                 int B, int H, int H_kv, int N, int D, int k_eff, float eps,
                                 int32_t* idx_out, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  int st = check_heads(B, H, H_kv, N, D);
  if (st) return st;
  if ((st = check_proj(KP, dtype, p_stride_b, p_stride_h, B, H_kv, N, P, R))) return st;
  if (Q == nullptr || idx_out == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q)) return DCR_ERR_ALIGN;
  if ((st = check_k(k_eff, N))) return st;
  const int rows = B * H;
  const WorkspaceLayout w = workspace_layout(rows, N, k_eff);
  if (workspace == nullptr || workspace_bytes < w.total) return DCR_ERR_WORKSPACE;
  if (!aligned16(workspace)) return DCR_ERR_ALIGN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* scores = reinterpret_cast<uint16_t*>(ws + w.scores);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = launch_score_projected(KP, dtype, p_stride_b, p_stride_h, Q, P, qp, eps, B, H,
                                   H_kv, N, scores, w.n_pad, 1, s)))
    return st;
  return launch_select(scores, w.n_pad, rows, N, k_eff, 1, idx_out, nullptr, s, nullptr, 0,
                       nullptr, w.sel_bytes ? ws + w.sel : nullptr);
}

int dcr_decode_projected(const void* Q, const void* K, const void* V, const void* KP, int dtype,
                         int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                         int64_t v_stride_h, int64_t p_stride_b, int64_t p_stride_h,
                         const float* P, int R, const float* qp, int B, int H, int H_kv, int N,
                         int D, int k_eff, float eps, void* O, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (B <= 0 || H_kv <= 0 || N <= 0) return DCR_ERR_SHAPE;
  const int st = check_proj(KP, dtype, p_stride_b, p_stride_h, B, H_kv, N, P, R);
  if (st) return st;
  const ProjArgs proj = {KP, p_stride_b, p_stride_h, P, qp};
  return decode_impl(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h, B, H, H_kv,
                     N, D, k_eff, eps, O, workspace, workspace_bytes, stream, nullptr, &proj);
}

int dcr_decode_prologue_strided(const void* q, const void* k, const void* v, int64_t in_sb_q,
                                int64_t in_sb_kv, const void* cos, const void* sin, int dtype,
                                int B, int H, int H_kv, int D, void* q_out, void* K_cache,
                                void* V_cache, int64_t c_stride_b, int64_t c_stride_h, int pos,
                                int N_max, const float* P, int R, void* KP_cache,
                                int64_t p_stride_b, int64_t p_stride_h, float* qp_out, float eps,
                                void* stream) {
  if (B <= 0 || H <= 0 || H_kv <= 0 || N_max <= 0 || D != kD || H % H_kv != 0)
    return DCR_ERR_SHAPE;
  if (in_sb_q < 0 || in_sb_kv < 0 || (in_sb_q > 0 && in_sb_q < static_cast<int64_t>(H) * kD) ||
      (in_sb_kv > 0 && in_sb_kv < static_cast<int64_t>(H_kv) * kD))
    return DCR_ERR_SHAPE;
  if (pos < 0 || pos >= N_max) return DCR_ERR_SHAPE;
  if (q == nullptr || k == nullptr || v == nullptr || cos == nullptr || sin == nullptr ||
      q_out == nullptr)
    return DCR_ERR_NULL;
  if (dtype_bytes(dtype) == 0) return DCR_ERR_DTYPE;
  int64_t cvb = c_stride_b, cvh = c_stride_h;
  int st = check_cache(K_cache, dtype, c_stride_b, c_stride_h, B, H_kv, N_max);
  if (st) return st;
  if ((st = check_cache(V_cache, dtype, cvb, cvh, B, H_kv, N_max))) return st;
  if ((KP_cache != nullptr || qp_out != nullptr) && (P == nullptr || R != DCR_PROJ_RANK))
    return P == nullptr ? DCR_ERR_NULL : DCR_ERR_SHAPE;
  if (KP_cache != nullptr &&
      (st = check_proj(KP_cache, dtype, p_stride_b, p_stride_h, B, H_kv, N_max, P, R)))
    return st;
  return launch_rope_append(q, k, v, cos, sin, dtype, B, H, H_kv, q_out, K_cache, V_cache,
                            c_stride_b, c_stride_h, pos, KP_cache, p_stride_b, p_stride_h, P,
                            qp_out, eps, static_cast<cudaStream_t>(stream), in_sb_q, in_sb_kv);
}

int dcr_decode_prologue(const void* q, const void* k, const void* v, const void* cos,
                        const void* sin, int dtype, int B, int H, int H_kv, int D, void* q_out,
                        void* K_cache, void* V_cache, int64_t c_stride_b, int64_t c_stride_h,
                        int pos, int N_max, const float* P, int R, void* KP_cache,
                        int64_t p_stride_b, int64_t p_stride_h, float* qp_out, float eps,
                        void* stream) {
  return dcr_decode_prologue_strided(q, k, v, 0, 0, cos, sin, dtype, B, H, H_kv, D, q_out,
                                     K_cache, V_cache, c_stride_b, c_stride_h, pos, N_max, P, R,
                                     KP_cache, p_stride_b, p_stride_h, qp_out, eps, stream);
}

// ---- sequence-sharded decode ----------------------------------------------------------

size_t dcr_shard_workspace_bytes(int B, int H, int H_kv, int N_local, int D, int k_eff) {
  if (check_heads(B, H, H_kv, N_local, D) != DCR_OK || k_eff <= 0) return 0;
  return shard_layout(B * H, N_local, k_eff).total;
}

static int shard_ws(int B, int H, int N_local, int k_eff, void* workspace,
                    size_t workspace_bytes, ShardLayout& w) {
  if (k_eff <= 0) return DCR_ERR_K_RANGE;
  w = shard_layout(B * H, N_local, k_eff);
  if (workspace == nullptr || workspace_bytes < w.total) return DCR_ERR_WORKSPACE;
  if (!aligned16(workspace)) return DCR_ERR_ALIGN;
  return DCR_OK;
}

static bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

int dcr_shard_score(const void* Q, const void* K, int dtype, int64_t k_stride_b,
                    int64_t k_stride_h, int B, int H, int H_kv, int N_local, int D, int k_eff,
                    float eps, int32_t* hist_hi, void* workspace, size_t workspace_bytes,
                    void* stream) {
  int st = check_heads(B, H, H_kv, N_local, D);
  if (st) return st;
  if ((st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N_local))) return st;
  if (Q == nullptr || hist_hi == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q) || !aligned4(hist_hi)) return DCR_ERR_ALIGN;
  ShardLayout w;
  if ((st = shard_ws(B, H, N_local, k_eff, workspace, workspace_bytes, w))) return st;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = launch_score(K, dtype, k_stride_b, k_stride_h, nullptr, Q, eps, B, H, H_kv, N_local,
                         reinterpret_cast<uint16_t*>(ws + w.scores), w.n_pad, 1, s)))
    return st;
  return launch_shard_hist(w, ws, B * H, N_local, k_eff, 0, nullptr, hist_hi, nullptr, s);
}

int dcr_shard_refine(int B, int H, int H_kv, int N_local, int D, int k_eff,
                     const int32_t* hist_hi_sum, int32_t* hist_lo, void* workspace,
                     size_t workspace_bytes, void* stream) {
  int st = check_heads(B, H, H_kv, N_local, D);
  if (st) return st;
  if (hist_hi_sum == nullptr || hist_lo == nullptr) return DCR_ERR_NULL;
  if (!aligned4(hist_hi_sum) || !aligned4(hist_lo)) return DCR_ERR_ALIGN;
  ShardLayout w;
  if ((st = shard_ws(B, H, N_local, k_eff, workspace, workspace_bytes, w))) return st;
  return launch_shard_hist(w, static_cast<uint8_t*>(workspace), B * H, N_local, k_eff, 1,
                           hist_hi_sum, hist_lo, nullptr, static_cast<cudaStream_t>(stream));
}

int dcr_shard_attend(const void* Q, const void* K, const void* V, int dtype, int64_t k_stride_b,
                     int64_t k_stride_h, int64_t v_stride_b, int64_t v_stride_h, int B, int H,
                     int H_kv, int N_local, int D, int k_eff, const int32_t* hist_lo_all,
                     int world, int rank, float* state, void* workspace,
                     size_t workspace_bytes, void* stream) {
  int st = check_heads(B, H, H_kv, N_local, D);
  if (st) return st;
  if ((st = check_cache(K, dtype, k_stride_b, k_stride_h, B, H_kv, N_local))) return st;
  if ((st = check_cache(V, dtype, v_stride_b, v_stride_h, B, H_kv, N_local))) return st;
  if (Q == nullptr || hist_lo_all == nullptr || state == nullptr) return DCR_ERR_NULL;
  if (!aligned16(Q) || !aligned4(hist_lo_all) || !aligned4(state)) return DCR_ERR_ALIGN;
  if (world <= 0 || rank < 0 || rank >= world) return DCR_ERR_SHAPE;
  ShardLayout w;
  if ((st = shard_ws(B, H, N_local, k_eff, workspace, workspace_bytes, w))) return st;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rows = B * H;
  // the selection also resets the Pass 3 tickets
  if ((st = launch_shard_select(w, ws, rows, N_local, k_eff, hist_lo_all, world, rank, nullptr,
                                s)))
    return st;
  return launch_attend(Q, K, V, dtype, k_stride_b, k_stride_h, v_stride_b, v_stride_h,
                       reinterpret_cast<const int32_t*>(ws + w.idx),
                       reinterpret_cast<const int32_t*>(ws + w.count), B, H, H_kv, N_local,
                       w.cap, nullptr, state, w.splits, reinterpret_cast<float*>(ws + w.partials),
                       reinterpret_cast<int*>(ws + w.counters), nullptr, s);
}

int dcr_shard_combine(const float* states, int world, int B, int H, int D, int dtype, void* O,
                      void* stream) {
  if (states == nullptr || O == nullptr) return DCR_ERR_NULL;
  if (B <= 0 || H <= 0 || D != kD || world <= 0) return DCR_ERR_SHAPE;
  if (static_cast<int64_t>(B) * H * kD > 0x7fffffffLL) return DCR_ERR_SHAPE;
  if (dtype_bytes(dtype) == 0) return DCR_ERR_DTYPE;
  if (!aligned4(states) || !aligned16(O)) return DCR_ERR_ALIGN;
  return launch_shard_combine(states, world, B * H, dtype, O, nullptr,
                              static_cast<cudaStream_t>(stream));
}

int dcr_shard_selection(const void* workspace, size_t workspace_bytes, int B, int H, int H_kv,
                        int N_local, int D, int k_eff, int32_t* idx_out, int32_t* count_out,
                        void* stream) {
  int st = check_heads(B, H, H_kv, N_local, D);
  if (st) return st;
  if (idx_out == nullptr || count_out == nullptr) return DCR_ERR_NULL;
  ShardLayout w;
  if ((st = shard_ws(B, H, N_local, k_eff, const_cast<void*>(workspace), workspace_bytes, w)))
    return st;
  const uint8_t* ws = static_cast<const uint8_t*>(workspace);
  return launch_shard_selection_out(w, ws, B * H, N_local, k_eff, idx_out, count_out,
                                    static_cast<cudaStream_t>(stream));
}

int dcr_binary_version(int* version_out) {
  if (version_out == nullptr) return DCR_ERR_NULL;
  cudaFuncAttributes a{};
  if (cudaFuncGetAttributes(&a, reinterpret_cast<const void*>(&dcr::unit_query_kernel<__half>)) !=
      cudaSuccess)
    return DCR_ERR_CUDA;
  *version_out = a.binaryVersion;
  return DCR_OK;
}

int dcr_read_device_status(int* status_out, int clear) {
  if (status_out == nullptr) return DCR_ERR_NULL;
  if (cudaDeviceSynchronize() != cudaSuccess) return DCR_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, dcr::g_device_status, sizeof(int)) != cudaSuccess)
    return DCR_ERR_CUDA;
  *status_out = v;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(dcr::g_device_status, &zero, sizeof(int)) != cudaSuccess)
      return DCR_ERR_CUDA;
  }
  return DCR_OK;
}

}  // extern "C"
