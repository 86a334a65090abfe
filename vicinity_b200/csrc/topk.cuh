// Warp-level top-k selection over unique 64-bit keys (see common.cuh).
//
// A warp holds the best 32*R keys sorted ascending, element r*32 + lane in
// register v[r] of that lane.  Candidates arrive 32 at a time (one per lane);
// a ballot against the current worst kept key skips rounds that cannot
// change the result, which after the first few rounds is nearly all of them.
// An admitted round is sorted with a 32-wide bitonic network and merged row
// by row: merging a sorted row into the sorted rows keeps the invariant that
// every element of row r is below every element of row r+1.
#pragma once

#include "common.cuh"

namespace vg {

// Sort one key per lane ascending across the warp (bitonic network).
__device__ __forceinline__ uint64_t warp_sort32(uint64_t x) {
  const int lane = lane_id();
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      uint64_t y = shfl_xor64(x, stride);
      bool ascending = (lane & size) == 0 || size == 32;
      bool lower = (lane & stride) == 0;
      x = (lower == ascending) ? (x < y ? x : y) : (x < y ? y : x);
    }
  }
  return x;
}

// Sort a bitonic sequence held one key per lane ascending.
__device__ __forceinline__ uint64_t warp_bitonic_merge32(uint64_t x) {
  const int lane = lane_id();
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) {
    uint64_t y = shfl_xor64(x, stride);
    bool lower = (lane & stride) == 0;
    x = lower ? (x < y ? x : y) : (x < y ? y : x);
  }
  return x;
}

template <int R>
struct WarpTopK {
  uint64_t v[R];

  __device__ __forceinline__ void init() {
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = kEmptyKey;
  }

  // Largest key kept (the admission threshold), identical in all lanes.
  __device__ __forceinline__ uint64_t worst() const { return shfl64(v[R - 1], 31); }

  // Merge a row that is already sorted ascending across the warp.
  __device__ __forceinline__ void merge_sorted_row(uint64_t c) {
    const int lane = lane_id();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint64_t crev = shfl64(c, 31 - lane);
      uint64_t lo = v[r] < crev ? v[r] : crev;
      uint64_t hi = v[r] < crev ? crev : v[r];
      v[r] = warp_bitonic_merge32(lo);
      if (r + 1 < R) c = warp_bitonic_merge32(hi);
    }
  }

  // Offer one key per lane (kEmptyKey for none).
  __device__ __forceinline__ void add(uint64_t key) {
    uint64_t thr = worst();
    bool want = key < thr;
    if (!__any_sync(VG_FULL_MASK, want)) return;
    uint64_t c = warp_sort32(want ? key : kEmptyKey);
    merge_sorted_row(c);
  }

  // Element i (0 <= i < 32*R) of the sorted list, read by every lane.
  __device__ __forceinline__ uint64_t get(int i) const {
    uint64_t out = kEmptyKey;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint64_t x = shfl64(v[r], i & 31);
      if ((i >> 5) == r) out = x;
    }
    return out;
  }
};

}  // namespace vg
