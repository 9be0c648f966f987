// The prompt pass's sort of (token, rank) pairs by expert on the device, for a pass with no host sync: the order of
// drama3/offload.py:141-145 (a stable sort by expert id: within an expert, pairs in (token, rank) order; pairs whose
// id is outside [0, E) sort last, as one more group) and the groups the grouped kernels read, in one launch of one
// block, where the reference reads the per-expert counts back to the host and builds the groups there.
//
// A counting sort: per-key counts by shared-memory atomics, an exclusive scan of the counts (each key's first row),
// then the pairs in chunks of 1024 in index order. Inside a chunk a pair's place among the equal keys before it is
// its rank among its warp's equal keys (__match_any_sync) plus the counts of that key in the chunk's earlier warps
// (a per-key scan over the 32 warps' counts), so the order within a key is the index order, as a stable sort gives.
#pragma once

#include "common.cuh"

namespace d3 {

constexpr int PLAN_THREADS = 1024;
constexpr int PLAN_WARPS = PLAN_THREADS / 32;
constexpr int PLAN_MAX_E = 256;                // experts; one more key holds the out-of-range ids
constexpr int PLAN_STRIDE = PLAN_MAX_E + 1;    // odd row stride of the per-warp count table (conflict-free columns)

// ids [P] int64 -> order [P] int64 (the pairs in key order), pos [P] int64 (its inverse), groups [E + 1][5] int32
// (expert, slot, 0, first, rows) with key E the out-of-range ids (rows 0 when drop_invalid). One block of
// PLAN_THREADS; E <= PLAN_MAX_E.
__global__ void __launch_bounds__(PLAN_THREADS) prefill_plan_kernel(const int64_t* __restrict__ ids, int P, int E,
                                                                    int drop_invalid, int64_t* __restrict__ order,
                                                                    int64_t* __restrict__ pos,
                                                                    int* __restrict__ groups) {
  __shared__ int count[PLAN_MAX_E + 1];
  __shared__ int base[PLAN_MAX_E + 1];
  __shared__ int chunk_total[PLAN_MAX_E + 1];
  __shared__ int warp_sum[PLAN_WARPS];
  __shared__ int wcount[PLAN_WARPS * PLAN_STRIDE];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int keys = E + 1;
  auto key_of = [&](int i) {
    const int64_t v = ids[i];
    return (v >= 0 && v < E) ? (int)v : E;
  };
  for (int e = tid; e < keys; e += PLAN_THREADS) count[e] = 0;
  __syncthreads();
  for (int i = tid; i < P; i += PLAN_THREADS) atomicAdd(&count[key_of(i)], 1);
  __syncthreads();
  // exclusive scan of the counts (keys <= 257 < PLAN_THREADS: one value a thread)
  {
    const int c = tid < keys ? count[tid] : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sum[lane], wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += v;
      }
      warp_sum[lane] = wi - w;
    }
    __syncthreads();
    if (tid < keys) {
      const int first = warp_sum[warp] + incl - c;
      base[tid] = first;
      int* gr = groups + 5 * tid;
      gr[0] = tid;
      gr[1] = tid;
      gr[2] = 0;
      gr[3] = first;
      gr[4] = (tid == E && drop_invalid) ? 0 : c;
    }
  }
  for (int c0 = 0; c0 < P; c0 += PLAN_THREADS) {
    for (int j = tid; j < PLAN_WARPS * keys; j += PLAN_THREADS) wcount[(j / keys) * PLAN_STRIDE + j % keys] = 0;
    __syncthreads();  // also orders the previous chunk's base update before this chunk's reads
    const int i = c0 + tid;
    const bool valid = i < P;
    const int k = valid ? key_of(i) : keys;  // past the end: a key of its own, never counted
    const unsigned peers = __match_any_sync(0xffffffffu, k);
    const int before = __popc(peers & ((1u << lane) - 1u));
    if (valid && before == 0) wcount[warp * PLAN_STRIDE + k] = __popc(peers);
    __syncthreads();
    // per key, the exclusive scan of its counts over the warps: warp w scans keys w, w + 32, ... (lane = warp index)
    for (int e = warp; e < keys; e += PLAN_WARPS) {
      const int v = wcount[lane * PLAN_STRIDE + e];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      wcount[lane * PLAN_STRIDE + e] = incl - v;
      if (lane == 31) chunk_total[e] = incl;
    }
    __syncthreads();
    if (valid) {
      const int p = base[k] + wcount[warp * PLAN_STRIDE + k] + before;
      pos[i] = p;
      order[p] = i;
    }
    __syncthreads();
    for (int e = tid; e < keys; e += PLAN_THREADS) base[e] += chunk_total[e];
  }
}

}  // namespace d3
