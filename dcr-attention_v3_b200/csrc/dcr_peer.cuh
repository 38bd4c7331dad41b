// dcr_peer.cuh — the peer-memory exchange of the sequence-sharded step (NVLink, no NCCL).
//
// Every rank owns one exchange buffer (cudaMalloc'd by dcr_xchg_create, shared with the
// other ranks of the node through CUDA IPC). All ranks use the same layout:
//   hh [world][rows][256] u64     slot s: rank s's high-byte histograms
//   hl [world][rows][256] u64     slot s: rank s's low-byte histograms
//   st [world][rows][D+2] u64     slot s: rank s's attention states (m, l, o) as fp32 bits
//   acc_hh, acc_hl [rows][256]    this rank's histograms while chunk CTAs accumulate them
//   ctl: epoch (steps completed), abort, combine ticket; row tickets tickets0/1 [rows]
// Every exchanged value travels in one 64-bit word together with the step's epoch
// (value | epoch << 32), written with a single 64-bit store into slot `rank` of every
// rank's buffer (its own included) — plain stores over NVLink, no multicast. A reader
// polls the words of its slots until they carry this step's epoch: the value and its
// epoch arrive together (a naturally aligned 64-bit access is single-copy atomic), so no
// fence or separate flag is needed, and each row waits only for its own data. Epochs
// start at 1 (a zeroed buffer matches no step). A slot is never rewritten before every
// rank has read it: each step runs the three exchanges once, in order, and a rank's next
// write of a slot always follows reads of its own that need the peers to be past theirs.
#pragma once

#include <stdint.h>

#include "dcr_common.cuh"

namespace dcr {

constexpr int kMaxPeers = 8;
constexpr int kStateFloats = kD + 2;

struct XchgLayout {
  int64_t hh, hl, st, acc_hh, acc_hl, epoch, abort, cticket, tickets0, tickets1, total;
};

__host__ __device__ inline int64_t xchg_align(int64_t x) { return (x + 255) / 256 * 256; }

__host__ __device__ inline XchgLayout xchg_layout(int rows, int world) {
  XchgLayout l;
  int64_t off = 0;
  const int64_t wr = static_cast<int64_t>(world) * rows;
  l.hh = off;
  off = xchg_align(off + wr * 256 * 8);
  l.hl = off;
  off = xchg_align(off + wr * 256 * 8);
  l.st = off;
  off = xchg_align(off + wr * kStateFloats * 8);
  l.acc_hh = off;
  off = xchg_align(off + static_cast<int64_t>(rows) * 256 * 4);
  l.acc_hl = off;
  off = xchg_align(off + static_cast<int64_t>(rows) * 256 * 4);
  l.epoch = off;
  l.abort = off + 4;
  l.cticket = off + 8;
  off = xchg_align(off + 16);
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

  __device__ uint64_t* hh(int owner, int src, int64_t row) const {
    return reinterpret_cast<uint64_t*>(base[owner] + lay.hh) + (static_cast<int64_t>(src) * rows + row) * 256;
  }
  __device__ uint64_t* hl(int owner, int src, int64_t row) const {
    return reinterpret_cast<uint64_t*>(base[owner] + lay.hl) + (static_cast<int64_t>(src) * rows + row) * 256;
  }
  __device__ uint64_t* st(int owner, int src, int64_t row) const {
    return reinterpret_cast<uint64_t*>(base[owner] + lay.st) +
           (static_cast<int64_t>(src) * rows + row) * kStateFloats;
  }
  __device__ int32_t* acc(int level, int64_t row) const {
    return reinterpret_cast<int32_t*>(base[rank] + (level ? lay.acc_hl : lay.acc_hh)) + row * 256;
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

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// The i-th destination of a push to every rank: this rank's own slot first, then the ranks
// after it in turn, so that the ranks' pushes do not all reach the same GPU at once.
__device__ __forceinline__ int peer_order(const PeerView& v, int i) {
  const int q = v.rank + i;
  return q < v.world ? q : q - v.world;
}

// This step's epoch (1 + the steps completed on this rank; every rank agrees).
__device__ __forceinline__ uint32_t step_epoch(const PeerView& v) {
  return ld_volatile_u32(v.epoch()) + 1u;
}

// Writes `value` tagged with `epoch` (one 64-bit store, visible at system scope).
__device__ __forceinline__ void ll_put(uint64_t* p, uint32_t value, uint32_t epoch) {
  const uint64_t w = (static_cast<uint64_t>(epoch) << 32) | value;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ll_load(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Waits until the word at p carries `epoch` and returns its value. The wait is bounded:
// after limit_ns, or once another wait on this rank gave up (abort word), it raises
// DCR_ERR_DEVICE_TIMEOUT, sets the abort word and returns the stale value, which the
// status reports.
__device__ __forceinline__ uint32_t ll_get(const PeerView& v, const uint64_t* p, uint32_t epoch,
                                           uint64_t limit_ns = 2000000000ull) {
  uint64_t w = ll_load(p);
  if (static_cast<uint32_t>(w >> 32) == epoch) return static_cast<uint32_t>(w);
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    __nanosleep(32);
    w = ll_load(p);
    if (static_cast<uint32_t>(w >> 32) == epoch) break;
    if (((++spins) & 63u) == 0u) {
      if (ld_volatile_u32(v.abort_word()) != 0u) break;
      if (global_timer_ns() - t0 > limit_ns) {
        raise_status(DCR_ERR_DEVICE_TIMEOUT);
        atomicExch(v.abort_word(), 1u);
        break;
      }
    }
  }
  return static_cast<uint32_t>(w);
}

// Packed histogram rows (the fused selection, whose counts fit 16 bits): word j carries
// bins 3j, 3j+1, 3j+2 in bits 0-15, 16-31, 32-47 and a 16-bit tag of the step's epoch in
// bits 48-63 (a slot is rewritten every step, so 16 bits tell this step's words from the
// last step's; the tag is never 0, which a zeroed word carries). 86 words per row.
constexpr int kPackedWords = (256 + 2) / 3;

__device__ __forceinline__ uint32_t epoch_tag16(uint32_t epoch) { return epoch % 65535u + 1u; }

__device__ __forceinline__ void ll_put_packed(uint64_t* p, uint32_t b0, uint32_t b1, uint32_t b2,
                                              uint32_t epoch) {
  const uint64_t w = (static_cast<uint64_t>(epoch_tag16(epoch)) << 48) |
                     (static_cast<uint64_t>(b2 & 0xffffu) << 32) |
                     (static_cast<uint64_t>(b1 & 0xffffu) << 16) | (b0 & 0xffffu);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// Waits (bounded, as ll_get) until the word at p carries `epoch` in its top 16 bits and
// returns the word.
__device__ __forceinline__ uint64_t ll_get_packed(const PeerView& v, const uint64_t* p,
                                                  uint32_t epoch,
                                                  uint64_t limit_ns = 2000000000ull) {
  const uint32_t tag = epoch_tag16(epoch);
  uint64_t w = ll_load(p);
  if (static_cast<uint32_t>(w >> 48) == tag) return w;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    __nanosleep(32);
    w = ll_load(p);
    if (static_cast<uint32_t>(w >> 48) == tag) break;
    if (((++spins) & 63u) == 0u) {
      if (ld_volatile_u32(v.abort_word()) != 0u) break;
      if (global_timer_ns() - t0 > limit_ns) {
        raise_status(DCR_ERR_DEVICE_TIMEOUT);
        atomicExch(v.abort_word(), 1u);
        break;
      }
    }
  }
  return w;
}

// Reads word base[r * stride] of every rank r < world into w[r], waiting (bounded, as
// ll_get) for each word's tag: the words are loaded together first, so a read costs one
// round trip, not one per rank. tag_shift: 32 (full epoch) or 48 (packed 16-bit tag).
// The polling half of ll_gather, for words already loaded once into w (full 32-bit tags):
// re-reads only those that do not carry this step's epoch yet.
__device__ __forceinline__ void ll_gather_late(const PeerView& v, const uint64_t* base,
                                               int64_t stride, uint32_t epoch,
                                               uint64_t (&w)[kMaxPeers]);

__device__ __forceinline__ void ll_gather(const PeerView& v, const uint64_t* base,
                                          int64_t stride, uint32_t epoch, int tag_shift,
                                          uint64_t (&w)[kMaxPeers]) {
  const uint32_t tag = tag_shift == 48 ? epoch_tag16(epoch) : epoch;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) w[r] = r < v.world ? ll_load(base + r * stride) : 0ull;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) {
    if (r >= v.world || static_cast<uint32_t>(w[r] >> tag_shift) == tag) continue;
    const uint64_t t0 = global_timer_ns();
    uint32_t spins = 0;
    while (true) {
      __nanosleep(32);
      w[r] = ll_load(base + r * stride);
      if (static_cast<uint32_t>(w[r] >> tag_shift) == tag) break;
      if (((++spins) & 63u) == 0u) {
        if (ld_volatile_u32(v.abort_word()) != 0u) break;
        if (global_timer_ns() - t0 > 2000000000ull) {
          raise_status(DCR_ERR_DEVICE_TIMEOUT);
          atomicExch(v.abort_word(), 1u);
          break;
        }
      }
    }
  }
}

__device__ __forceinline__ void ll_gather_late(const PeerView& v, const uint64_t* base,
                                               int64_t stride, uint32_t epoch,
                                               uint64_t (&w)[kMaxPeers]) {
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) {
    if (r >= v.world || static_cast<uint32_t>(w[r] >> 32) == epoch) continue;
    const uint64_t t0 = global_timer_ns();
    uint32_t spins = 0;
    while (true) {
      __nanosleep(32);
      w[r] = ll_load(base + r * stride);
      if (static_cast<uint32_t>(w[r] >> 32) == epoch) break;
      if (((++spins) & 63u) == 0u) {
        if (ld_volatile_u32(v.abort_word()) != 0u) break;
        if (global_timer_ns() - t0 > 2000000000ull) {
          raise_status(DCR_ERR_DEVICE_TIMEOUT);
          atomicExch(v.abort_word(), 1u);
          break;
        }
      }
    }
  }
}

}  // namespace dcr
