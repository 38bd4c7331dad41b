/*
 * dcr_b200.h — C ABI of the B200 (sm_100a) sparse top-K decode-attention library
 * (libdcr_b200.so).
 *
 * This is the drop-in boundary for DCR-Attention's per-step sparse decode attention.
 * Each entry point replaces one function of the reference's Python kernel API; the
 * comment above each declaration names the function it replaces (file:line within the
 * Seqev/dcr-attention_v3 project).
 *
 * Conventions shared by every entry point
 * ---------------------------------------
 *  - All tensor arguments are DEVICE pointers owned by the caller. Inputs are only read.
 *    Outputs are written in place; nothing is allocated by the library (except the
 *    exchange buffer of dcr_xchg_create, at setup).
 *  - Shapes follow the reference: Q and O are [B, H, D]; the KV caches are
 *    [B, H_kv, N, D]; scores are [B*H, N]; indices are [B*H, k_eff] int32.
 *    Query head h reads KV head h / (H / H_kv) (GQA).
 *  - D must be 64 (DCR_HEAD_DIM) and H / H_kv must be 1, 2, 4 or 8.
 *  - Cache rows must be contiguous (stride D along N, 1 along D). The batch and head
 *    strides (in elements) are free, so a cache allocated for N_max >= N positions can
 *    be passed directly. Every cache pointer and stride must be 16-byte aligned.
 *  - dtype is one of dcr_dtype; Q, K and V share it. O is written in the same dtype.
 *    Scores are always bfloat16 (raw bits, uint16), as in the reference.
 *  - `stream` is a cudaStream_t cast to void* (NULL = legacy default stream). Calls are
 *    asynchronous and stream ordered; nothing synchronises. Kernels never spin without a
 *    bound; a wait that expires, or an index outside [0, N), sets a sticky device status
 *    that dcr_read_device_status() returns.
 *  - Return value: 0 (DCR_OK) or a dcr_status code. A non-zero code means nothing was
 *    launched.
 */
#ifndef DCR_B200_H_
#define DCR_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DCR_HEAD_DIM 64
#define DCR_ABI_VERSION 1
/* Size of the library-owned scratch array used by dcr_decode_noalloc (16 MiB). */
#define DCR_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
/* Rank of the key projection of the projected-score mode (dcr_*_projected). */
#define DCR_PROJ_RANK 16
/* Size of a CUDA IPC handle of an exchange buffer (dcr_xchg_create). */
#define DCR_IPC_HANDLE_BYTES 64
/* Most ranks one peer exchange connects. */
#define DCR_MAX_PEERS 8

typedef enum dcr_dtype {
  DCR_DTYPE_BF16 = 0,
  DCR_DTYPE_F16 = 1,
  DCR_DTYPE_F32 = 2
} dcr_dtype;

typedef enum dcr_status {
  DCR_OK = 0,
  DCR_ERR_NULL = 1,             /* a required pointer is NULL                         */
  DCR_ERR_SHAPE = 2,            /* B, H, H_kv, N, D or a stride out of range          */
  DCR_ERR_K_RANGE = 3,          /* k_eff not in (0, N): caller must dispatch to SDPA  */
  DCR_ERR_DTYPE = 4,            /* unknown dtype code                                 */
  DCR_ERR_ALIGN = 5,            /* pointer or stride not 16-byte aligned              */
  DCR_ERR_WORKSPACE = 6,        /* workspace pointer NULL or smaller than required    */
  DCR_ERR_CUDA = 7,             /* a CUDA runtime call failed                         */
  DCR_ERR_DEVICE_TIMEOUT = 8,   /* device status: a bounded wait expired              */
  DCR_ERR_NOALLOC_LIMIT = 9,    /* shape needs more than DCR_NOALLOC_SCRATCH_BYTES    */
  DCR_ERR_DEVICE_INDEX = 16,    /* device status: an index outside [0, N) was skipped */
  DCR_ERR_DEVICE_SHARD = 32     /* device status: sharded selection found the global
                                   histograms inconsistent (fewer than k_eff keys over
                                   all ranks, or a rank's list overflowed its slots)  */
} dcr_status;

/* Library ABI version (DCR_ABI_VERSION). */
int dcr_version(void);

/* Human-readable text for a dcr_status code (static storage). */
const char* dcr_status_string(int status);

/* k_eff = min(N, max(k_min, floor(N * c))), rounded up to even and capped at N.
 * Replaces adaptive_k_window, dcr_attention/models/llama/adaptive.py:39.
 * Returns -1 when n_kv <= 0 or c is outside [0, 1]. */
int dcr_adaptive_k_window(int k_window_min, int n_kv, double coverage_floor);

/* Bytes of workspace dcr_decode / dcr_select_indices / dcr_attend need for this shape
 * (a superset for all three). Returns 0 for an invalid shape. */
size_t dcr_workspace_bytes(int B, int H, int H_kv, int N, int D, int k_eff);

/* u = f32(Q) / max(||f32(Q)||_2, eps), fp32 [B, H, D].
 * Replaces _compute_u_Q, dcr_attention/kernel/qaxis_topk_reference.py:42
 * (called by topk_qaxis_select, dcr_attention/kernel/triton/topk_axis.py:47). */
int dcr_unit_query(const void* Q, int dtype, int B, int H, int D, float eps,
                   float* u_out, void* stream);

/* Pass 1: scores[b*H + h, n] = bf16_rne(sum_d f32(K[b, h/G, n, d]) * u[b, h, d]).
 * The fp32 sum runs d = 0..63 as a chain of fused multiply-adds.
 * If u is NULL the unit query is computed from Q (same dtype as K) with eps.
 * Replaces topk_pass1_projection, dcr_attention/kernel/triton/topk_axis_pass1.py:104
 * (kernel _pass1_projection_kernel, topk_axis_pass1.py:29). */
int dcr_score(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h,
              const float* u, const void* Q, float eps,
              int B, int H, int H_kv, int N, int D,
              uint16_t* scores, int64_t s_stride_row, void* stream);

/* Pass 2: per row, the k_eff indices of the largest bf16 scores (ties: lower index
 * first), written in ascending index order as int32. -0 equals +0; NaN ranks highest.
 * Replaces topk_pass2_select, dcr_attention/kernel/triton/topk_axis_pass2.py:16. */
int dcr_select(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
               int32_t* idx_out, void* stream);

/* Bytes of device workspace dcr_select_ws needs for rows x N: 0 where the one-CTA-per-row
 * selection of dcr_select runs anyway (rows x N up to 148 x 32768), else the scratch of
 * the chunked selection (row histograms and per-chunk counts). */
size_t dcr_select_workspace_bytes(int rows, int N);

/* dcr_select with a workspace (16-byte aligned, dcr_select_workspace_bytes bytes; it need
 * not be zeroed): past one wave of rows the selection runs as chunked grid-wide kernels,
 * bit-identical to dcr_select. The same replacement of topk_pass2_select
 * (topk_axis_pass2.py:16) for large B x H x N. */
int dcr_select_ws(const uint16_t* scores, int64_t s_stride_row, int rows, int N, int k_eff,
                  int32_t* idx_out, void* workspace, size_t workspace_bytes, void* stream);

/* Pass 3: O[b, h] = softmax((K[b, h/G, idx] . f32(Q[b, h])) / sqrt(D)) @ V[b, h/G, idx],
 * fp32 online softmax, one rounding to the output dtype. idx is [B*H, k_eff] int32.
 * Replaces fused_topk_attention, dcr_attention/kernel/triton/fused_attn.py:158
 * (kernel _pass3_fused_attn_kernel, fused_attn.py:40). */
int dcr_attend(const void* Q, const void* K, const void* V, int dtype,
               int64_t k_stride_b, int64_t k_stride_h,
               int64_t v_stride_b, int64_t v_stride_h,
               const int32_t* idx, int B, int H, int H_kv, int N, int D, int k_eff,
               void* O, void* workspace, size_t workspace_bytes, void* stream);

/* Pass 1 + Pass 2: u_Q, scores and the top-K indices [B*H, k_eff] int32 ascending.
 * Replaces topk_qaxis_select, dcr_attention/kernel/triton/topk_axis.py:20. */
int dcr_select_indices(const void* Q, const void* K, int dtype,
                       int64_t k_stride_b, int64_t k_stride_h,
                       int B, int H, int H_kv, int N, int D, int k_eff, float eps,
                       int32_t* idx_out, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Full decode step (Pass 1 + 2 + 3): O [B, H, D] from Q, K, V and k_eff.
 * Replaces topk_qaxis_attention, dcr_attention/kernel/triton/topk_axis.py:58
 * (and its oracle topk_qaxis_attention_reference,
 *  dcr_attention/kernel/qaxis_topk_reference.py:200). */
int dcr_decode(const void* Q, const void* K, const void* V, int dtype,
               int64_t k_stride_b, int64_t k_stride_h,
               int64_t v_stride_b, int64_t v_stride_h,
               int B, int H, int H_kv, int N, int D, int k_eff, float eps,
               void* O, void* workspace, size_t workspace_bytes, void* stream);

/* dcr_decode without a caller workspace, for callers that cannot allocate device memory
 * where they run a decode step (an engine plugin whose enqueue must not allocate because
 * the engine owns all device memory, a serving loop that cannot take cudaMalloc's
 * implicit synchronisation).
 * No counterpart in the reference: its Python path allocates through torch on every call.
 * Scratch is a 16 MiB (DCR_NOALLOC_SCRATCH_BYTES) __device__ array inside the library,
 * held by every GPU that loads the library until exit; shapes whose dcr_workspace_bytes
 * exceed it return DCR_ERR_NOALLOC_LIMIT and launch nothing. All calls on a device share
 * the array: calls that overlap on the GPU race, calls ordered on one stream do not.
 * The first call on a device looks up the array's address and sets kernel attributes
 * (the driver may load the module then): make it a warm-up at initialisation, outside
 * the no-allocation region and before any stream capture begins. Later calls allocate
 * nothing. */
int dcr_decode_noalloc(const void* Q, const void* K, const void* V, int dtype,
                       int64_t k_stride_b, int64_t k_stride_h,
                       int64_t v_stride_b, int64_t v_stride_h,
                       int B, int H, int H_kv, int N, int D, int k_eff, float eps,
                       void* O, void* stream);

/* dcr_decode with four caller-created CUDA events (cudaEvent_t cast to void*) recorded on
 * the stream before Pass 1, between the passes and after Pass 3, for per-pass timing of
 * exactly the kernels dcr_decode launches. Diagnostic: the reference has no counterpart. */
int dcr_decode_timed(const void* Q, const void* K, const void* V, int dtype,
                     int64_t k_stride_b, int64_t k_stride_h,
                     int64_t v_stride_b, int64_t v_stride_h,
                     int B, int H, int H_kv, int N, int D, int k_eff, float eps,
                     void* O, void* workspace, size_t workspace_bytes, void* stream,
                     void* const* events);

/* The first `passes` (1, 2 or 3) passes of dcr_decode, launched exactly as dcr_decode
 * launches them (Pass 2 writes the selection in the form the decode step's Pass 3 reads),
 * for timing each pass as its marginal cost inside the step. Diagnostic: the reference has
 * no counterpart. */
int dcr_decode_prefix(const void* Q, const void* K, const void* V, int dtype,
                      int64_t k_stride_b, int64_t k_stride_h,
                      int64_t v_stride_b, int64_t v_stride_h,
                      int B, int H, int H_kv, int N, int D, int k_eff, float eps,
                      void* O, void* workspace, size_t workspace_bytes, void* stream,
                      int passes);

/* ---------------------------------------------------------------------------------
 * Projected-score mode. No counterpart in the reference (its Pass 1 always reads the
 * 64-dim keys): the cache also holds KP = K . P, the keys projected by a fixed
 * DCR_HEAD_DIM x DCR_PROJ_RANK fp32 matrix P (row-major, P[d * R + j]), stored in the
 * cache dtype as [B, H_kv, N, R] with contiguous rows of R elements. Pass 1 then scores
 * bf16(KP . (u . P)), reading R instead of D elements per key; Pass 2 and Pass 3 are
 * those of dcr_decode. The reference's DynamicCache.update (dcr_attention/models/llama/
 * compat.py:208-254), a torch.cat of the whole cache per step, becomes dcr_cache_append
 * into preallocated caches. R must be DCR_PROJ_RANK; P must be 4-byte aligned.
 * --------------------------------------------------------------------------------- */

/* KP [B, H_kv, N, R] of the N rows of an existing K cache (prefill). */
int dcr_project_keys(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h,
                     int B, int H_kv, int N, int D, const float* P, int R, void* KP,
                     int64_t p_stride_b, int64_t p_stride_h, void* stream);

/* Writes n_new rows of K_new and V_new ([B, H_kv, n_new, D], one pair of strides for
 * both) into K_cache and V_cache ([B, H_kv, N_max, D], one pair of strides) at positions
 * [pos, pos + n_new), and, if KP_cache and P are given, their projections into KP_cache
 * at the same positions. pos + n_new must not exceed N_max. */
int dcr_cache_append(const void* K_new, const void* V_new, int dtype,
                     int64_t new_stride_b, int64_t new_stride_h, int B, int H_kv, int n_new,
                     int D, void* K_cache, void* V_cache, int64_t c_stride_b,
                     int64_t c_stride_h, int pos, int N_max, const float* P, int R,
                     void* KP_cache, int64_t p_stride_b, int64_t p_stride_h, void* stream);

/* Pass 1 of the projected mode: bf16 score bits [B*H, N] (row stride s_stride_row).
 * qp (optional, else NULL): the projected unit queries [B*H][R] fp32 that
 * dcr_decode_prologue wrote; without it Pass 1 computes them from Q and P. */
int dcr_score_projected(const void* KP, int dtype, int64_t p_stride_b, int64_t p_stride_h,
                        const void* Q, float eps, const float* P, int R, const float* qp,
                        int B, int H, int H_kv, int N, int D, uint16_t* scores,
                        int64_t s_stride_row, void* stream);

/* Pass 1 (projected) + Pass 2: indices [B*H, k_eff] int32 ascending. Workspace as
 * dcr_workspace_bytes. */
int dcr_select_indices_projected(const void* Q, const void* KP, int dtype, int64_t p_stride_b,
                                 int64_t p_stride_h, const float* P, int R, const float* qp,
                                 int B, int H, int H_kv, int N, int D, int k_eff, float eps,
                                 int32_t* idx_out, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* Full decode step with projected Pass 1: O [B, H, D]. Workspace as dcr_workspace_bytes. */
int dcr_decode_projected(const void* Q, const void* K, const void* V, const void* KP, int dtype,
                         int64_t k_stride_b, int64_t k_stride_h,
                         int64_t v_stride_b, int64_t v_stride_h,
                         int64_t p_stride_b, int64_t p_stride_h, const float* P, int R,
                         const float* qp, int B, int H, int H_kv, int N, int D, int k_eff,
                         float eps, void* O, void* workspace, size_t workspace_bytes,
                         void* stream);

/* Decode prologue of one step, in one launch: RoPE of the step's projected q [B, H, D] and
 * k [B, H_kv, D] rows with the model's position embeddings cos, sin [B, D] (HF
 * apply_rotary_pos_emb, dcr_attention/models/llama/compat.py:63, evaluated op by op in
 * the dtype like torch), the rotated query into q_out [B, H, D], the rotated key and v
 * [B, H_kv, D] into K_cache / V_cache at position pos (replacing cache_update's torch.cat,
 * compat.py:208); optionally (P given) the key's projection into KP_cache at pos and the
 * projected unit queries into qp_out [B*H][R] fp32 for dcr_decode_projected. q, k, v are
 * contiguous. */
int dcr_decode_prologue(const void* q, const void* k, const void* v, const void* cos,
                        const void* sin, int dtype, int B, int H, int H_kv, int D, void* q_out,
                        void* K_cache, void* V_cache, int64_t c_stride_b, int64_t c_stride_h,
                        int pos, int N_max, const float* P, int R, void* KP_cache,
                        int64_t p_stride_b, int64_t p_stride_h, float* qp_out, float eps,
                        void* stream);

/* The same with q, k and v rows read at in_stride_b_q / in_stride_b_kv elements between
 * batch rows (0: contiguous), e.g. slices of one [B][(H + 2 H_kv) D] output of a GEMM over
 * the concatenated q/k/v weights. q_out stays contiguous [B, H, D]. */
int dcr_decode_prologue_strided(const void* q, const void* k, const void* v,
                                int64_t in_stride_b_q, int64_t in_stride_b_kv, const void* cos,
                                const void* sin, int dtype, int B, int H, int H_kv, int D,
                                void* q_out, void* K_cache, void* V_cache, int64_t c_stride_b,
                                int64_t c_stride_h, int pos, int N_max, const float* P, int R,
                                void* KP_cache, int64_t p_stride_b, int64_t p_stride_h,
                                float* qp_out, float eps, void* stream);

/* ---------------------------------------------------------------------------------
 * Sequence-sharded decode over several GPUs (exact global top-K).
 *
 * No counterpart in the reference: its decode path runs on one GPU. The result is that
 * of dcr_decode over the whole context: the selected set is the reference's
 * (_select_topk_indices, dcr_attention/kernel/qaxis_topk_reference.py:91) taken over the
 * concatenation of the ranks' chunks, and O is _fused_softmax_attention (:148) over it.
 *
 * Rank r of `world` holds positions [off_r, off_r + N_local) of every (b, h_kv) cache
 * row, off_r increasing with r; N_local may differ between ranks. Every rank holds the
 * whole Q. k_eff is the GLOBAL k (0 < k_eff < sum of N_local). One step is:
 *   dcr_shard_score   -> caller all-reduces (sum) hist_hi   int32 [B*H][256]
 *   dcr_shard_refine  -> caller all-gathers  hist_lo  into  int32 [world][B*H][256]
 *   dcr_shard_attend  -> caller all-gathers  state    into  fp32  [world][B*H][D + 2]
 *   dcr_shard_combine -> O [B, H, D]
 * with the same workspace (dcr_shard_workspace_bytes) on all four calls. The workspace
 * carries state between the calls; do not reuse it for another step in between.
 * --------------------------------------------------------------------------------- */
size_t dcr_shard_workspace_bytes(int B, int H, int H_kv, int N_local, int D, int k_eff);

/* Phase 1: Pass 1 over the local chunk and the per-row histogram of the score keys'
 * high byte (hist_hi, overwritten). */
int dcr_shard_score(const void* Q, const void* K, int dtype, int64_t k_stride_b,
                    int64_t k_stride_h, int B, int H, int H_kv, int N_local, int D,
                    int k_eff, float eps, int32_t* hist_hi, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Phase 2: given hist_hi summed over all ranks, the per-row histogram of the low byte of
 * the local keys in the threshold's high-byte bin (hist_lo, overwritten). */
int dcr_shard_refine(int B, int H, int H_kv, int N_local, int D, int k_eff,
                     const int32_t* hist_hi_sum, int32_t* hist_lo, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Phase 3: from all ranks' hist_lo (rank-major), this rank's share of the global top-K
 * (ascending local positions) and the attention over it, written as the unnormalised
 * fp32 state (m, l, o[D]) of every row (m in base-2 units of the scaled scores; a row
 * with nothing selected on this rank gets m = -inf, l = 0, o = 0). */
int dcr_shard_attend(const void* Q, const void* K, const void* V, int dtype,
                     int64_t k_stride_b, int64_t k_stride_h,
                     int64_t v_stride_b, int64_t v_stride_h,
                     int B, int H, int H_kv, int N_local, int D, int k_eff,
                     const int32_t* hist_lo_all, int world, int rank, float* state,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Phase 4: O [B, H, D] (dtype) from all ranks' states (rank-major). */
int dcr_shard_combine(const float* states, int world, int B, int H, int D, int dtype, void* O,
                      void* stream);

/* Copies this rank's selection of the last dcr_shard_attend on `workspace`: idx_out
 * int32 [B*H][min(k_eff, N_local)] (ascending local positions; row r's first
 * count_out[r] entries are valid) and count_out int32 [B*H]. Diagnostic. */
int dcr_shard_selection(const void* workspace, size_t workspace_bytes, int B, int H, int H_kv,
                        int N_local, int D, int k_eff, int32_t* idx_out, int32_t* count_out,
                        void* stream);

/* ---------------------------------------------------------------------------------
 * The same sequence-sharded step with the exchanges done inside the kernels, through
 * the ranks' exchange buffers over NVLink (CUDA IPC peer memory, plain loads and stores,
 * no multicast), instead of three collectives between phases. No counterpart in the
 * reference.
 *
 * Setup, once per (B, H, world) and rank, all ranks of one node (world <= 8):
 *   dcr_xchg_create  -> this rank's buffer (cudaMalloc'd, zeroed) and its IPC handle
 *   (share the handles: all-gather of DCR_IPC_HANDLE_BYTES bytes per rank)
 *   dcr_xchg_open    -> peers[world]: every rank's buffer mapped into this process
 * Step (every rank, in the same order, one call each):
 *   dcr_shard_decode_peer -> O [B, H, D]
 * Teardown after a barrier: dcr_xchg_close, then dcr_xchg_destroy.
 * Kernels wait for peers with a bound (2 s): if a peer does not arrive, the wait sets the
 * device status DCR_ERR_DEVICE_TIMEOUT and the rank's abort word (later waits return at
 * once), and O of that step is invalid. dcr_xchg_reset (on every rank, between steps,
 * after a barrier) clears the buffer to start again.
 * --------------------------------------------------------------------------------- */
size_t dcr_xchg_bytes(int B, int H, int world);
int dcr_xchg_create(int B, int H, int world, void** buf_out, void* ipc_handle_out);
int dcr_xchg_open(const void* ipc_handles, int world, int rank, void* buf, void** peers_out);
int dcr_xchg_close(void* const* peers, int world, int rank);
int dcr_xchg_destroy(void* buf);
int dcr_xchg_reset(void* buf, int B, int H, int world, void* stream);

/* One sequence-sharded decode step of this rank (arguments as dcr_shard_attend, with the
 * workspace of dcr_shard_workspace_bytes); returns O [B, H, D] on every rank.
 * n_local_max is the longest N_local of all ranks (the same value on every rank, and
 * constant for one exchange buffer: reset the buffers on every rank after changing it);
 * it selects the step's kernels and exchange format alike on every rank. */
int dcr_shard_decode_peer(const void* Q, const void* K, const void* V, int dtype,
                          int64_t k_stride_b, int64_t k_stride_h,
                          int64_t v_stride_b, int64_t v_stride_h,
                          int B, int H, int H_kv, int N_local, int D, int k_eff, float eps,
                          void* const* peers, int world, int rank, int n_local_max, void* O,
                          void* workspace, size_t workspace_bytes, void* stream);

/* dcr_shard_decode_peer with seven caller-created CUDA events recorded on the stream
 * around its kernels (before Pass 1, after Pass 1, after each histogram, after the
 * selection, after Pass 3, after the combine). Diagnostic. */
int dcr_shard_decode_peer_timed(const void* Q, const void* K, const void* V, int dtype,
                                int64_t k_stride_b, int64_t k_stride_h,
                                int64_t v_stride_b, int64_t v_stride_h,
                                int B, int H, int H_kv, int N_local, int D, int k_eff,
                                float eps, void* const* peers, int world, int rank,
                                int n_local_max, void* O, void* workspace,
                                size_t workspace_bytes, void* stream, void* const* events);

/* Synchronises the current device and returns (in *status_out) the OR of the device
 * status bits (DCR_ERR_DEVICE_*) set since the last clear; clears them if clear != 0.
 * Diagnostic: the reference has no counterpart (its kernels have no device status). */
int dcr_read_device_status(int* status_out, int clear);

/* Writes the compute capability the library's device code was built for, as the CUDA
 * runtime reports it for the current device (cudaFuncGetAttributes().binaryVersion:
 * 100 for sm_100a). Diagnostic: the reference has no counterpart. */
int dcr_binary_version(int* version_out);

/* ---- native step runner (dcr_runner.cu) ------------------------------------------
 * One decode step over fixed caches — the H2D copy of the step's query from pinned
 * staging, the three passes (dcr_decode, or dcr_decode_projected when KP and P are given)
 * and the D2H copy of O — captured once as a CUDA graph on a runner-owned stream, with
 * runner-owned device buffers, pinned staging and workspace. Replaces the per-step Python
 * calls of the reference's hook (dcr_attention/models/llama/attention.py:805-813) for a
 * serving loop; the graph bakes in the cache pointers, N and k_eff (one runner per length
 * bucket). Create on the device that holds the caches (the current device). */
int dcr_runner_create(const void* K, const void* V, const void* KP, const float* P, int dtype,
                      int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                      int64_t v_stride_h, int64_t p_stride_b, int64_t p_stride_h, int B, int H,
                      int H_kv, int N, int D, int k_eff, float eps, void** runner_out);
/* Copies q_host [B, H, D] (host memory, the caches' dtype) into the staging, replays the
 * step, waits for it and copies O [B, H, D] to o_host. Either pointer may be the runner's
 * own pinned buffer (dcr_runner_query_buffer / dcr_runner_output_buffer): no copy then. */
int dcr_runner_step(void* runner, const void* q_host, void* o_host);
void* dcr_runner_query_buffer(void* runner);
void* dcr_runner_output_buffer(void* runner);
int dcr_runner_destroy(void* runner);

/* ---- the rest of a decode step (dcr_decode_ops.cu) -----------------------------------
 * Kernels for the layers around the attention in a decode model (HF LlamaRMSNorm, the
 * residual adds, LlamaMLP's SiLU-gated product), with torch's rounding of the same op
 * sequence. All pointers are device pointers, row-major and
 * contiguous; dtype is a dcr_dtype. */

/* h_out = h + delta (rounded to dtype; delta may be NULL: no add, h_out unused; h_out may
 * equal h), then y = weight * dtype(h_out * rsqrt(mean(h_out^2) + eps)) per row of `dim`.
 * Replaces the residual add and LlamaRMSNorm.forward (transformers modeling_llama). */
int dcr_add_rmsnorm(const void* h, const void* delta, const void* weight, int dtype, int rows,
                    int dim, float eps, void* h_out, void* y, void* stream);

/* out = dtype(dtype(silu(gate)) * up) elementwise over n values (LlamaMLP's act_fn(gate) * up). */
int dcr_silu_mul(const void* gate, const void* up, int dtype, int64_t n, void* out,
                 void* stream);

/* The same from one [rows][2 * inter] tensor holding gate then up in each row (the output
 * of one GEMM over the concatenated gate and up weights): out [rows][inter]. */
int dcr_silu_mul_packed(const void* gate_up, int dtype, int rows, int inter, void* out,
                        void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* DCR_B200_H_ */
