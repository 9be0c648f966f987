// The prompt pass's sort of (token, rank) pairs by expert on the device, for a pass with no host sync: the order of
// drama3/offload.py:141-145 (a stable sort by expert id: within an expert, pairs in (token, rank) order; pairs whose
// id is outside [0, E) sort last, as one more group) and the groups the grouped kernels read, in one launch of one
// block, where the reference reads the per-expert counts back to the host and builds the groups there.
//
// A counting sort in which each of the block's 32 warps owns a contiguous segment of the pairs. Pass 1: a warp
// counts its segment's keys, 32 pairs a round (__match_any_sync groups the equal keys of a round; the group's first
// lane adds the group's size to the warp's own row of counts, so no atomics and no block barrier inside the pass).
// Then, per key, an exclusive scan over the warps' counts and over the keys gives each (warp, key) its first
// position. Pass 2: each warp walks its segment again and places a pair at its (warp, key) position plus its rank
// among the equal keys of its round, then advances that position by the group's size. Segments are in index order
// and a warp's rounds and lanes are too, so equal keys keep their index order, as a stable sort gives.
#pragma once

#include "common.cuh"

namespace d3 {

constexpr int PLAN_THREADS = 1024;
constexpr int PLAN_WARPS = PLAN_THREADS / 32;
constexpr int PLAN_MAX_E = 256;                // experts; one more key holds the out-of-range ids
constexpr int PLAN_STRIDE = PLAN_MAX_E + 1;    // odd row stride of the per-warp count table (conflict-free columns)
constexpr int PLAN_REG_ROUNDS = 16;            // rounds of 32 keys a lane keeps in registers (16384 pairs)

// ids [P] int64 -> order [P] int64 (the pairs in key order), pos [P] int64 (its inverse), groups [E + 1][5] int32
// (expert, slot, 0, first, rows) with key E the out-of-range ids (rows 0 when drop_invalid). One block of
// PLAN_THREADS; E <= PLAN_MAX_E.
__global__ void __launch_bounds__(PLAN_THREADS) prefill_plan_kernel(const int64_t* __restrict__ ids, int P, int E,
                                                                    int drop_invalid, int64_t* __restrict__ order,
                                                                    int64_t* __restrict__ pos,
                                                                    int* __restrict__ groups) {
  __shared__ int start[PLAN_WARPS * PLAN_STRIDE];  // [warp][key]: counts, then first positions, then next positions
  __shared__ int total[PLAN_MAX_E + 1];
  __shared__ int warp_sum[PLAN_WARPS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int keys = E + 1;
  // warp w's segment: [w S, min(P, (w + 1) S)), S a multiple of 32
  const int S = ((P + PLAN_WARPS - 1) / PLAN_WARPS + 31) & ~31;
  const int seg0 = warp * S, seg1 = min(P, seg0 + S);
  auto key_at = [&](int i) {  // past the segment: a key of its own, never counted or placed
    if (i >= seg1) return keys;
    const int64_t v = ids[i];
    return (v >= 0 && v < E) ? (int)v : E;
  };
  int* mine = start + warp * PLAN_STRIDE;
  // the keys of the segment's first PLAN_REG_ROUNDS rounds, loaded together and kept in registers for both passes
  int kreg[PLAN_REG_ROUNDS];
#pragma unroll
  for (int r = 0; r < PLAN_REG_ROUNDS; ++r) kreg[r] = key_at(seg0 + 32 * r + lane);
  // every round of the segment in order: f(key, first pair of the round)
  auto rounds = [&](auto&& f) {
#pragma unroll
    for (int r = 0; r < PLAN_REG_ROUNDS; ++r)
      if (seg0 + 32 * r < seg1) f(kreg[r], seg0 + 32 * r);
    for (int i0 = seg0 + 32 * PLAN_REG_ROUNDS; i0 < seg1; i0 += 32) f(key_at(i0 + lane), i0);
  };
  for (int j = tid; j < PLAN_WARPS * PLAN_STRIDE; j += PLAN_THREADS) start[j] = 0;
  __syncthreads();
  // pass 1: the warp's counts
  rounds([&](int k, int) {
    const unsigned peers = __match_any_sync(0xffffffffu, k);
    if (k < keys && lane == __ffs(peers) - 1) mine[k] += __popc(peers);
    __syncwarp();
  });
  __syncthreads();
  // per key, the exclusive scan of its counts over the warps (warp w scans keys w, w + 32, ...; lane = warp index)
  for (int e = warp; e < keys; e += PLAN_WARPS) {
    const int v = start[lane * PLAN_STRIDE + e];
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    start[lane * PLAN_STRIDE + e] = incl - v;
    if (lane == 31) total[e] = incl;
  }
  __syncthreads();
  // exclusive scan of the key totals (keys <= 257 < PLAN_THREADS: one value a thread): each key's first row
  {
    const int c = tid < keys ? total[tid] : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int w = warp_sum[lane];
      int wi = w;
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
      int* gr = groups + 5 * tid;
      gr[0] = tid;
      gr[1] = tid;
      gr[2] = 0;
      gr[3] = first;
      gr[4] = (tid == E && drop_invalid) ? 0 : c;
      total[tid] = first;  // now the key's first row
    }
  }
  __syncthreads();
  for (int j = tid; j < PLAN_WARPS * keys; j += PLAN_THREADS)
    start[(j / keys) * PLAN_STRIDE + j % keys] += total[j % keys];
  __syncthreads();
  // pass 2: place the warp's pairs
  rounds([&](int k, int i0) {
    const int i = i0 + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, k);
    const int before = __popc(peers & ((1u << lane) - 1u));
    if (k < keys) {
      const int p = mine[k] + before;
      pos[i] = p;
      order[p] = i;
    }
    __syncwarp();
    if (k < keys && before == 0) mine[k] += __popc(peers);
    __syncwarp();
  });
}

}  // namespace d3
