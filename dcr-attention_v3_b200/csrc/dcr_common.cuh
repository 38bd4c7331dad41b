// dcr_common.cuh — device helpers shared by the sm_100a kernels of libdcr_b200.
//
// Row layout: a cache row is D = 64 elements, i.e. 128 B for bf16/fp16 and 256 B for
// fp32, handled as 16-byte chunks. Tiles of rows are staged in shared memory with the
// 128-byte swizzle that the TMA unit applies for CU_TENSOR_MAP_SWIZZLE_128B: the chunk
// c (0..7) of row r of a 128-byte-wide sub-tile lives at chunk position c ^ (r & 7).
// Thread-per-row readers then hit 8 distinct chunk positions in every quarter-warp
// phase, which is conflict free. fp32 rows are two 128-byte sub-tiles (columns 0..31 and
// 32..63) stored one after the other.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dcr_b200.h"

namespace dcr {

constexpr int kD = DCR_HEAD_DIM;

// Sticky device status (OR of DCR_ERR_DEVICE_* bits), one word per device. The library
// is built as one translation unit (dcr_b200_lib.cu), so this is its only definition.
__device__ int g_device_status = 0;

__device__ __forceinline__ void raise_status(int bits) { atomicOr(&g_device_status, bits); }

// ---------------------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------------------
template <typename T>
struct ElemTraits;

template <>
struct ElemTraits<__nv_bfloat16> {
  static constexpr int kBytes = 2;
  static constexpr int kPerChunk = 8;  // elements per 16-byte chunk
  // Exact widening of the 8 bf16 values of a chunk, in element order.
  __device__ __forceinline__ static void widen(const uint4& c, float (&f)[8]) {
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static float2 widen2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  __device__ __forceinline__ static float widen1(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
  }
  __device__ __forceinline__ static void store(void* p, int i, float v) {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
};

template <>
struct ElemTraits<__half> {
  static constexpr int kBytes = 2;
  static constexpr int kPerChunk = 8;
  __device__ __forceinline__ static void widen(const uint4& c, float (&f)[8]) {
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 v = __half22float2(h);
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
  __device__ __forceinline__ static float2 widen2(uint32_t w) {
    __half2 h = *reinterpret_cast<const __half2*>(&w);
    return __half22float2(h);
  }
  __device__ __forceinline__ static float widen1(uint16_t b) {
    return __half2float(__ushort_as_half(b));
  }
  __device__ __forceinline__ static void store(void* p, int i, float v) {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  }
};

template <>
struct ElemTraits<float> {
  static constexpr int kBytes = 4;
  static constexpr int kPerChunk = 4;
  __device__ __forceinline__ static void widen(const uint4& c, float (&f)[4]) {
    f[0] = __uint_as_float(c.x);
    f[1] = __uint_as_float(c.y);
    f[2] = __uint_as_float(c.z);
    f[3] = __uint_as_float(c.w);
  }
  __device__ __forceinline__ static void store(void* p, int i, float v) {
    static_cast<float*>(p)[i] = v;
  }
};

// Bytes of one cache row and 16-byte chunks per row.
template <typename T>
struct RowTraits {
  static constexpr int kRowBytes = kD * ElemTraits<T>::kBytes;  // 128 or 256
  static constexpr int kChunks = kRowBytes / 16;                 // 8 or 16
  static constexpr int kSubTiles = kRowBytes / 128;              // 1 or 2
};

// Byte offset of logical chunk c of row r inside a swizzled tile of R rows.
__device__ __forceinline__ uint32_t swz_offset(int r, int c, int R) {
  const int sub = c >> 3;
  const int cc = c & 7;
  return static_cast<uint32_t>(sub * R * 128 + r * 128 + ((cc ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and raises the device status) if the
// phase has not completed after `limit_ns` nanoseconds of global time.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (((++spins) & 255u) == 0u && global_timer_ns() - t0 > limit_ns) {
      raise_status(DCR_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// 3-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// TMA gather of 4 rows (tile::gather4; the 2-D tensor map's box is one row high): rows
// r0..r3, columns [x, x + box width), written one after another at smem_dst (with the
// map's swizzle); completes on an mbarrier. No multicast.
__device__ __forceinline__ void tma_gather4(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int x, int r0, int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(r0), "r"(r1),
      "r"(r2), "r"(r3)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 16-byte asynchronous global->shared copy; src_bytes = 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)),
               "l"(gsrc), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Two IEEE fused multiply-adds in one instruction: {a.x*b.x + c.x, a.y*b.y + c.y}.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// bf16 round-to-nearest-even of an fp32 value, as raw bits.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Order-preserving 16-bit key of a bf16 score: larger score -> larger key.
// -0 is mapped to +0 (they compare equal in the reference's fp32 argsort) and every NaN
// to the top key (torch's descending sort places NaN first).
__device__ __forceinline__ uint32_t bf16_order_key(uint32_t b) {
  b &= 0xffffu;
  if ((b & 0x7fffu) > 0x7f80u) return 0xffffu;
  if (b == 0x8000u) b = 0u;
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

// Inclusive warp scan (sum) of x over lanes 0..lane.
__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  return x;
}

// One warp finds, in a 256-bin histogram h, the bin B with #{above B} < k <= #{above B-1}
// (counting from the top) and returns B and above = #{keys in bins above B}.
__device__ __forceinline__ void warp_find_bin(const uint32_t* h, uint32_t k, int& bin,
                                              uint32_t& above) {
  const int lane = threadIdx.x & 31;
  uint32_t c[8];
  uint32_t tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = h[8 * lane + i];
    tot += c[i];
  }
  // inclusive suffix sum over lanes: sum of tot over lanes >= lane
  uint32_t suf = tot;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_down_sync(0xffffffffu, suf, off);
    if (lane + off < 32) suf += y;
  }
  uint32_t a = suf - tot;  // keys in bins above this lane's 8 bins
  int found = -1;
  uint32_t found_above = 0;
#pragma unroll
  for (int i = 7; i >= 0; --i) {
    if (found < 0 && a < k && k <= a + c[i]) {
      found = 8 * lane + i;
      found_above = a;
    }
    a += c[i];
  }
  const unsigned m = __ballot_sync(0xffffffffu, found >= 0);
  const int src = m ? (__ffs(m) - 1) : 0;
  bin = __shfl_sync(0xffffffffu, found, src);
  above = __shfl_sync(0xffffffffu, found_above, src);
}

}  // namespace dcr
