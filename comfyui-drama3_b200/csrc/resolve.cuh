// Slot-cache lookup and least-used eviction for one decode row's k experts of one layer, on the GPU, so that a decode
// step never waits on the host. Same state, same rules and same float arithmetic as drama3/kernels.py:87-191
// (resolve_experts):
//   table[L*E]   a key's slot, -1 (host only) or -2 - slot (its slot is being copied in)
//   owner[count] a slot's key or -1 (free);  pending[count] 1 while a slot is being copied in
//   score[L*E]   use count halving every half_life passes, as of step at[L*E] (-1: never)
//   clock[1]     ticks when layer 0 resolves; now = clock * layers + layer (also written to step[0])
//   reads[3]     hits, fills (read from host memory into a slot), experts left to the CPU
// A missed expert claims the slot with the lowest decayed score (free slots score -1; slots this layer used in this
// pass or pending are excluded; ties to the lower slot), or goes without a slot (plan slot -1) when none is left.
// With `cpu`, the most used misses (their number set by share[0]) stay on the GPU and the rest are marked for the
// CPU (code 2); of those, experts used `admit` times reserve a slot while budget lasts.
// plan[2e] = slot, plan[2e+1] = 0 cached, 1 read from host memory (and fill plan slot when >= 0), 2 left to the CPU.
// Expert ids outside [0, experts) are treated as misses without a slot and recorded in the fault word.
#pragma once

#include "common.cuh"

namespace d3 {

constexpr int RESOLVE_THREADS = 1024;
constexpr int RESOLVE_MAX_K = 32;

__global__ void __launch_bounds__(RESOLVE_THREADS)
    resolve_kernel(const int64_t* __restrict__ ids, int k, int layer, int layers, int experts, int* table, int* owner,
                   float* score, int* at, int* pending, int count, int* clock, int* budget, int* plan, int* reads,
                   int* step, const float* share, double half_life, int cpu, double admit) {
  __shared__ int slot_of[RESOLVE_MAX_K], fill[RESOLVE_MAX_K], valid[RESOLVE_MAX_K];
  __shared__ float uses[RESOLVE_MAX_K];
  __shared__ float red_value[RESOLVE_THREADS / 32];
  __shared__ int red_index[RESOLVE_THREADS / 32];
  __shared__ int now_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
  const int base = layer * experts;
  const float log2_decay = -1.0f / ((float)half_life * layers);
  if (tid == 0) {
    if (layer == 0) clock[0] += 1;
    now_s = clock[0] * layers + layer;
    step[0] = now_s;
  }
  __syncthreads();
  const int now = now_s;
  if (tid < k) {
    long long id = ids[tid];
    int ok = id >= 0 && id < experts;
    valid[tid] = ok;
    if (!ok) {
      record_fault(FAULT_BAD_EXPERT);
      uses[tid] = 0.0f;
      slot_of[tid] = -1;
      fill[tid] = 1;
    } else {
      int key = base + (int)id;
      // score * decay + 1 as one fused multiply-add (what the reference kernel computes)
      float used = at[key] < 0 ? 1.0f : __fmaf_rn(score[key], exp2f(log2_decay * (float)(now - at[key])), 1.0f);
      score[key] = used;
      uses[tid] = used;
      at[key] = now;
      int slot = table[key];
      slot_of[tid] = slot >= 0 ? slot : -1;
      // 3: a CPU expert that may reserve a slot, 4: a miss not yet given to either side
      fill[tid] = slot >= 0 ? 0 : !cpu ? 1 : slot == -1 ? 4 : 2;
    }
  }
  __syncthreads();
  if (tid == 0) {
    int ahead[RESOLVE_MAX_K], misses = 0;
    for (int e = 0; e < k; e++) {
      ahead[e] = 0;
      for (int o = 0; o < k; o++)
        if (fill[e] == 4 && fill[o] == 4 && (uses[o] > uses[e] || (uses[o] == uses[e] && o < e))) ahead[e]++;
      misses += fill[e] == 4;
    }
    // the split that finishes first, rounded towards the CPU by half a GPU expert
    float sh = share[0];
    int gpu = (int)__fmaf_rn((float)misses, sh, 0.5f * (1.0f - sh));
    for (int e = 0; e < k; e++)
      if (fill[e] == 4) fill[e] = ahead[e] < gpu ? 1 : uses[e] >= (float)admit ? 3 : 2;
    int allowed = min(budget[0], budget[1]);
    for (int e = 0; e < k; e++) {
      if (fill[e] != 3) continue;
      int before = 0;
      for (int o = 0; o < k; o++)
        if (fill[o] == 3 && (uses[o] > uses[e] || (uses[o] == uses[e] && o < e))) before++;
      if (before < allowed)
        budget[0] -= 1;
      else
        fill[e] = 5;
    }
    for (int e = 0; e < k; e++) {
      if (fill[e] == 5) fill[e] = 2;
      atomicAdd(reads + (fill[e] == 0 ? 0 : fill[e] == 1 ? 1 : 2), 1);
    }
  }
  __syncthreads();
  for (int e = 0; e < k; e++) {
    if ((fill[e] != 1 && fill[e] != 3) || !valid[e]) continue;
    float value = 3.0e38f;
    int index = 0x7fffffff;
    for (int i = tid; i < count; i += blockDim.x) {
      int key = owner[i];
      float v = key < 0                            ? -1.0f
                : (pending[i] || at[key] == now) ? 3.0e38f
                                                  : __fmul_rn(score[key], exp2f(log2_decay * (float)(now - at[key])));
      if (v < value) {
        value = v;
        index = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, value, o);
      int oi = __shfl_xor_sync(0xffffffffu, index, o);
      if (ov < value || (ov == value && oi < index)) {
        value = ov;
        index = oi;
      }
    }
    if (lane == 0) {
      red_value[warp] = value;
      red_index[warp] = index;
    }
    __syncthreads();
    if (warp == 0) {
      value = lane < warps ? red_value[lane] : 3.0e38f;
      index = lane < warps ? red_index[lane] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, value, o);
        int oi = __shfl_xor_sync(0xffffffffu, index, o);
        if (ov < value || (ov == value && oi < index)) {
          value = ov;
          index = oi;
        }
      }
      // without a slot (every slot this layer's or pending) the GEMVs read the expert from host memory unfilled
      if (lane == 0 && value < 3.0e38f) {
        int key = base + (int)ids[e];
        int old = owner[index];
        if (old >= 0) table[old] = -1;
        owner[index] = key;
        if (fill[e] == 1) {
          table[key] = index;
        } else {
          table[key] = -2 - index;
          pending[index] = 1;
        }
        slot_of[e] = index;
      }
    }
    __syncthreads();
  }
  if (tid < k) {
    plan[2 * tid] = slot_of[tid];
    plan[2 * tid + 1] = fill[tid] == 3 ? 2 : fill[tid];
  }
}

}  // namespace d3
