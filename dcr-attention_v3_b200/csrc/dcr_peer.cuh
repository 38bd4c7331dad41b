// dcr_peer.cuh — the peer-memory exchange of the sequence-sharded step (NVLink, no NCCL).
//
// Every rank owns one exchange buffer (cudaMalloc'd by dcr_xchg_create, shared with the
// other ranks of the node through CUDA IPC). All ranks use the same layout:
//   hh [world][rows][256] int32   slot s: rank s's high-byte histograms
//   hl [world][rows][256] int32   slot s: rank s's low-byte histograms
//   st [world][rows][D+2] fp32    slot s: rank s's attention states (m, l, o)
//   flags [3][world] uint32       flags[x][s] = epoch once all of rank s's rows of exchange x
//                                 (0 hh, 1 hl, 2 st) have landed in this buffer
//   ctl: epoch (steps completed), abort, combine ticket, exchange tickets [3];
//        row tickets tickets0/1 [rows]
// A rank accumulates its own row into its own slot; the CTA that completes a row copies it
// into slot `rank` of every peer's buffer with plain stores over NVLink (no multicast) and
// counts itself on the exchange's ticket (GPU-scope fence and atomic). The CTA completing
// the last row fences once at system scope and releases flag x on every peer: one system
// fence per exchange, the data stores of all rows ordered before it through the ticket.
// Consumers wait, with a bounded poll, until every peer's flag reaches this step's epoch
// and then read the slots from their own buffer. Each step runs the three exchanges once, in order, so
// a slot is never rewritten before every rank has read it (a rank's next push of a slot
// only follows the peers' pushes that prove they are past the read).
#pragma once

#include <stdint.h>

#include "dcr_common.cuh"

namespace dcr {

constexpr int kMaxPeers = 8;
constexpr int kStateFloats = kD + 2;

struct XchgLayout {
  int64_t hh, hl, st, flags, epoch, abort, cticket, xtickets, tickets0, tickets1, total;
};

__host__ __device__ inline int64_t xchg_align(int64_t x) { return (x + 255) / 256 * 256; }

__host__ __device__ inline XchgLayout xchg_layout(int rows, int world) {
  XchgLayout l;
  int64_t off = 0;
  const int64_t wr = static_cast<int64_t>(world) * rows;
  l.hh = off;
  off = xchg_align(off + wr * 256 * 4);
  l.hl = off;
  off = xchg_align(off + wr * 256 * 4);
  l.st = off;
  off = xchg_align(off + wr * kStateFloats * 4);
  l.flags = off;
  off = xchg_align(off + 3 * static_cast<int64_t>(world) * 4);
  l.epoch = off;
  l.abort = off + 4;
  l.cticket = off + 8;
  l.xtickets = off + 16;
  off = xchg_align(off + 32);
  l.tickets0 = off;
  off = xchg_align(off + static_cast<int64_t>(rows) * 4);
  l.tickets1 = off;
  off = xchg_align(off + static_cast<int64_t>(rows) * 4);
  l.total = off;
  return l;
}

// The exchange buffers of all ranks as seen from this rank (base[rank] is its own).
struct PeerView {
  uint8_t* base[kMaxPeers];
  int world;  // 0: no peer exchange (the caller runs collectives between the phases)
  int rank;
  int rows;
  XchgLayout lay;

  __device__ int32_t* hh(int owner, int src, int64_t row) const {
    return reinterpret_cast<int32_t*>(base[owner] + lay.hh) + (static_cast<int64_t>(src) * rows + row) * 256;
  }
  __device__ int32_t* hl(int owner, int src, int64_t row) const {
    return reinterpret_cast<int32_t*>(base[owner] + lay.hl) + (static_cast<int64_t>(src) * rows + row) * 256;
  }
  __device__ float* st(int owner, int src, int64_t row) const {
    return reinterpret_cast<float*>(base[owner] + lay.st) +
           (static_cast<int64_t>(src) * rows + row) * kStateFloats;
  }
  __device__ uint32_t* flag(int owner, int x, int src) const {
    return reinterpret_cast<uint32_t*>(base[owner] + lay.flags) + x * world + src;
  }
  __device__ uint32_t* xticket(int x) const {
    return reinterpret_cast<uint32_t*>(base[rank] + lay.xtickets) + x;
  }
  __device__ uint32_t* epoch() const { return reinterpret_cast<uint32_t*>(base[rank] + lay.epoch); }
  __device__ uint32_t* abort_word() const {
    return reinterpret_cast<uint32_t*>(base[rank] + lay.abort);
  }
  __device__ uint32_t* cticket() const {
    return reinterpret_cast<uint32_t*>(base[rank] + lay.cticket);
  }
  __device__ uint32_t* ticket(int which, int64_t row) const {
    return reinterpret_cast<uint32_t*>(base[rank] + (which ? lay.tickets1 : lay.tickets0)) + row;
  }
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// This step's epoch (1 + the steps completed on this rank; every rank agrees).
__device__ __forceinline__ uint32_t step_epoch(const PeerView& v) {
  return ld_volatile_u32(v.epoch()) + 1u;
}

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// One warp: waits until every peer's flag x reaches `epoch` (lane s polls rank s with
// acquire loads; the caller's block barrier then orders the CTA's reads of the slots after
// them). The wait is bounded: after limit_ns, or once another wait on this rank gave up
// (abort word), it raises DCR_ERR_DEVICE_TIMEOUT, sets the abort word and returns; the
// data read afterwards is then stale, which the status reports.
__device__ __forceinline__ void wait_peers(const PeerView& v, int x, uint32_t epoch,
                                           uint64_t limit_ns = 2000000000ull) {
  const int lane = threadIdx.x & 31;
  if (lane < v.world && lane != v.rank) {
    const uint32_t* f = v.flag(v.rank, x, lane);
    if (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
      const uint64_t t0 = global_timer_ns();
      uint32_t spins = 0;
      while (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
        if (((++spins) & 63u) == 0u) {
          if (ld_volatile_u32(v.abort_word()) != 0u) break;
          if (global_timer_ns() - t0 > limit_ns) {
            raise_status(DCR_ERR_DEVICE_TIMEOUT);
            atomicExch(v.abort_word(), 1u);
            break;
          }
        }
        __nanosleep(32);
      }
    }
    fence_acq_rel_sys();
  }
  __syncwarp();
}

// Called by every thread of a CTA that has just stored one of `rows` rows of exchange x
// into the peers' slots. A block barrier orders the CTA's stores before thread 0, which
// counts the row on the exchange ticket; the CTA that counts the last row fences at
// system scope and releases flag x on every peer.
__device__ __forceinline__ void row_pushed(const PeerView& v, int x, int rows, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(v.xticket(x), 1u) == static_cast<uint32_t>(rows - 1)) {
      *v.xticket(x) = 0u;
      fence_acq_rel_sys();
      for (int p = 0; p < v.world; ++p)
        if (p != v.rank) st_release_sys(v.flag(p, x, v.rank), epoch);
    }
  }
}

}  // namespace dcr
