// Warp-level bitonic networks over 64 64-bit keys held two a lane (lane l holds elements
// 2l and 2l + 1), descending. Shared by the row pass and the fused LM head.
#pragma once

#include <stdint.h>

namespace tabby {

// Bitonic sort of 64 values held two per lane (lane l holds elements 2l, 2l+1), descending.
__device__ __forceinline__ void warp_sort64_desc(uint64_t &v0, uint64_t &v1) {
  const int lane = threadIdx.x & 31;
  const int j0 = 2 * lane, j1 = j0 + 1;
#pragma unroll
  for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      uint64_t p0, p1;
      if (stride == 1) {
        p0 = v1;
        p1 = v0;
      } else {
        p0 = __shfl_xor_sync(0xffffffffu, v0, stride >> 1);
        p1 = __shfl_xor_sync(0xffffffffu, v1, stride >> 1);
      }
      const bool lower0 = (j0 & stride) == 0, desc0 = (j0 & size) == 0;
      const bool lower1 = (j1 & stride) == 0, desc1 = (j1 & size) == 0;
      v0 = (lower0 == desc0) ? (v0 > p0 ? v0 : p0) : (v0 < p0 ? v0 : p0);
      v1 = (lower1 == desc1) ? (v1 > p1 ? v1 : p1) : (v1 < p1 ? v1 : p1);
    }
  }
}


// Merges the sorted 64-list (w0, w1) into the sorted 64-list (v0, v1) (both descending,
// lane l holding elements 2l and 2l+1), keeping the 64 largest, sorted. The elementwise
// max of one list and the other reversed holds exactly the 64 largest of both and is
// bitonic; a bitonic merge sorts it.
__device__ __forceinline__ void warp_merge64_desc(uint64_t &v0, uint64_t &v1, uint64_t w0,
                                                  uint64_t w1) {
  const int lane = threadIdx.x & 31;
  const uint64_t r0 = __shfl_sync(0xffffffffu, w1, 31 - lane);
  const uint64_t r1 = __shfl_sync(0xffffffffu, w0, 31 - lane);
  v0 = v0 > r0 ? v0 : r0;
  v1 = v1 > r1 ? v1 : r1;
#pragma unroll
  for (int stride = 32; stride >= 2; stride >>= 1) {
    const uint64_t p0 = __shfl_xor_sync(0xffffffffu, v0, stride >> 1);
    const uint64_t p1 = __shfl_xor_sync(0xffffffffu, v1, stride >> 1);
    const bool lower = ((2 * lane) & stride) == 0;
    v0 = lower ? (v0 > p0 ? v0 : p0) : (v0 < p0 ? v0 : p0);
    v1 = lower ? (v1 > p1 ? v1 : p1) : (v1 < p1 ? v1 : p1);
  }
  const uint64_t hi = v0 > v1 ? v0 : v1;
  v1 = v0 > v1 ? v1 : v0;
  v0 = hi;
}


}  // namespace tabby
