// plan.cuh -- the register-path kernel's unit plan, for the grouped FFN's
// planner (grouped.cu). The decode planner (route.cu) computes the same plan
// for its one-chunk segments from its own segment scan.
#pragma once

#include <stdint.h>

#include "wisp_b200.h"

namespace wb {

// Units of the register-path kernel: `per_seg` row blocks per chunk of `cols`
// rows, for every segment of 1..max_rows rows, times a K split: when fewer
// than `target` units would exist, each is cut into up to `max_ksplit`
// K ranges (at most `nk`, one stage each at least), whose partial sums the
// down epilogue adds atomically. units[nseg + 1] receives the split.
static __device__ void plan_units(const WispSegment* segs, int nseg, int per_seg,
                           int cols, int max_rows, int max_ksplit, int nk, int target,
                           int32_t* __restrict__ units) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int base = 0; base < nseg; base += blockDim.x) {
    const int s = base + threadIdx.x;
    int n = 0;
    if (s < nseg) {
      const int rows = segs[s].rows;
      n = (rows > 0 && rows <= max_rows) ? per_seg * ((rows + cols - 1) / cols) : 0;
    }
    int v = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (lane == 31) warp_tot[w] = v;
    __syncthreads();
    if (w == 0) {
      int tv = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, tv, o);
        if (lane >= o) tv += y;
      }
      warp_tot[lane] = tv;
    }
    __syncthreads();
    const int incl = v + (w > 0 ? warp_tot[w - 1] : 0) + carry;
    if (s < nseg) units[s] = incl - n;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
  __syncthreads();
  const int total = carry;
  int ks = 1;
  if (total > 0 && total < target) ks = min(min(max_ksplit, nk), (target + total - 1) / total);
  if (ks < 1) ks = 1;
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) units[i] *= ks;
  if (threadIdx.x == 0) {
    units[nseg] = total * ks;
    units[nseg + 1] = ks;
  }
}

}  // namespace wb
