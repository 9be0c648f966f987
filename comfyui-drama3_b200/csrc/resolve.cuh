// Slot-cache lookup and least-used eviction for one decode row's k experts of one layer, on the GPU, so that a decode
// step never waits on the host. The state arrays and the observable rules are those of the reference's
// resolve_experts (drama3/kernels.py:78-191); the algorithm that applies them is this file's own.
//
// State (one key per (layer, expert): key = layer * experts + expert):
//   table[L*E]   a key's slot, -1 (host memory only) or -2 - slot (its slot is being copied in)
//   owner[count] a slot's key or -1 (free);  pending[count] 1 while a slot is being copied in
//   score[L*E]   use count halving every half_life passes, as of step at[L*E] (-1: never used)
//   clock[1]     ticks when layer 0 resolves; now = clock * layers + layer (also written to step[0])
//   reads[3]     cached hits, misses read from host memory, experts left to the CPU
//   budget[2]    slots a step may still reserve for the CPU's copies, and the cap per layer
// Rules:
//   1. Every routed key counts a use: score = score * 2^(-(now - at) / (half_life * layers)) + 1 (one rounding for
//      the multiply-add), at = now.
//   2. A key with a slot is a hit (code 0). Without a CPU side every miss is read from host memory into a slot
//      (code 1). With one, misses whose key is pending stay on the CPU (code 2); the others are ranked by use
//      (higher first, then lower expert position): the first int(misses * share + (1 - share) / 2) go to the GPU
//      (code 1), the rest to the CPU, and those used at least `admit` times may reserve a slot for the host's copy
//      (code 3, reported as 2) while min(budget[0], budget[1]) lasts, most used first; budget[0] pays for each.
//   3. Misses of code 1 and 3 claim slots in expert-position order. A slot's eviction value is -1 when free, its
//      owner's decayed score otherwise, and it is not a candidate while pending or while its owner was used at
//      `now` (which includes every key of this row). Each claim takes the candidate of lowest (value, slot); the old
//      owner leaves the table. A miss finding no candidate reads host memory without a slot (plan slot -1).
// Design: a claimed slot becomes a non-candidate and no other slot's value changes, so the claims of one call take
// the m lowest (value, slot) candidates in ascending order. Each slot's (value, slot) pair is packed into one
// ordered 64-bit key, and the block extracts the m smallest keys by m rounds of "smallest key above the last one":
// per round a warp minimum, the warps' minima through shared memory, warp 0's minimum of those (two barriers, the
// same m rounds in every thread, no atomics); the claims are then committed in parallel (they touch distinct slots
// and keys). The ranking of step 2 is one warp's: lane e holds expert e and counts the lanes ahead of it.
// plan[2e] = slot, plan[2e+1] = 0 cached, 1 read from host memory (and fill plan slot when >= 0), 2 left to the CPU.
// Expert ids outside [0, experts) are misses without a slot (code 1, never claiming) and set the fault word.
#pragma once

#include "common.cuh"

namespace d3 {

constexpr int RESOLVE_THREADS = 1024;
constexpr int RESOLVE_MAX_K = 32;
constexpr unsigned long long RESOLVE_NO_SLOT = ~0ull;

// Monotone map of a float onto unsigned ints (so that unsigned order is float order; no NaNs here).
__device__ __forceinline__ uint32_t ordered_bits(float v) {
  uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Warp-wide minimum of a 64-bit key.
__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w < v ? w : v;
  }
  return v;
}

// The rank (0 = first) of this lane among the lanes with `in_set`, ordered by `use` descending then lane ascending.
__device__ __forceinline__ int use_rank(float use, bool in_set, int lane) {
  const uint32_t members = __ballot_sync(0xffffffffu, in_set);
  int ahead = 0;
  for (int o = 0; o < 32; o++) {
    float other = __shfl_sync(0xffffffffu, use, o);
    bool counts = ((members >> o) & 1u) && (other > use || (other == use && o < lane));
    ahead += counts;
  }
  return ahead;
}

__global__ void __launch_bounds__(RESOLVE_THREADS)
    resolve_kernel(const int64_t* __restrict__ ids, int k, int layer, int layers, int experts, int* table, int* owner,
                   float* score, int* at, int* pending, int count, int* clock, int* budget, int* plan, int* reads,
                   int* step, const float* share, double half_life, int cpu, double admit) {
  __shared__ unsigned long long picked[RESOLVE_MAX_K];  // the m smallest candidate keys, ascending
  __shared__ unsigned long long warp_best[RESOLVE_THREADS / 32];
  __shared__ int now_s, claims_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float log2_decay = -1.0f / ((float)half_life * layers);
  if (tid < RESOLVE_MAX_K) picked[tid] = RESOLVE_NO_SLOT;
  // ---- warp 0: the row's experts (lane e = expert position e): rules 1 and 2
  int key = -1, code = 1, slot = -1, claim_rank = -1;
  if (warp == 0) {
    int now = 0;
    if (lane == 0) {
      if (layer == 0) clock[0] += 1;
      now = clock[0] * layers + layer;
      step[0] = now;
    }
    now = __shfl_sync(0xffffffffu, now, 0);
    bool mine = lane < k, valid = false;
    float use = 0.0f;
    int entry = -1;
    if (mine) {
      const long long id = ids[lane];
      valid = id >= 0 && id < experts;
      if (!valid) {
        record_fault(FAULT_BAD_EXPERT);
      } else {
        key = layer * experts + (int)id;
        const int last = at[key];
        use = last < 0 ? 1.0f : __fmaf_rn(score[key], exp2f(log2_decay * (float)(now - last)), 1.0f);
        score[key] = use;
        at[key] = now;
        entry = table[key];
        if (entry >= 0) slot = entry;
      }
    }
    if (valid) code = entry >= 0 ? 0 : !cpu ? 1 : entry == -1 ? 4 : 2;  // 4: a miss either side may take
    // CPU split: the most used undecided misses go to the GPU
    const bool undecided = mine && code == 4;
    const int misses = __popc(__ballot_sync(0xffffffffu, undecided));
    const int rank = use_rank(use, undecided, lane);
    if (undecided) {
      const float sh = share[0];
      const int gpu = (int)__fmaf_rn((float)misses, sh, 0.5f * (1.0f - sh));
      code = rank < gpu ? 1 : use >= (float)admit ? 3 : 2;
    }
    // reservations: the most used CPU experts keep theirs while the step's and the layer's budgets last
    const bool asks = mine && code == 3;
    const int order = use_rank(use, asks, lane);
    // every lane takes the shuffle (a full-mask shuffle behind a short-circuit would leave lanes out of it)
    const int allowed = __shfl_sync(0xffffffffu, (lane == 0 && cpu) ? min(budget[0], budget[1]) : 0, 0);
    const bool keeps = asks && order < allowed;
    if (asks && !keeps) code = 2;
    const int kept = __popc(__ballot_sync(0xffffffffu, keeps));
    const int hits = __popc(__ballot_sync(0xffffffffu, mine && code == 0));
    const int fills = __popc(__ballot_sync(0xffffffffu, mine && code == 1));
    const int on_cpu = __popc(__ballot_sync(0xffffffffu, mine && (code == 2 || code == 3)));
    if (lane == 0) {
      if (kept) budget[0] -= kept;
      if (hits) atomicAdd(reads + 0, hits);
      if (fills) atomicAdd(reads + 1, fills);
      if (on_cpu) atomicAdd(reads + 2, on_cpu);
    }
    // claims in expert-position order
    const uint32_t claimers = __ballot_sync(0xffffffffu, valid && (code == 1 || code == 3));
    claim_rank = __popc(claimers & ((1u << lane) - 1u));
    if (!((claimers >> lane) & 1u)) claim_rank = -1;
    if (lane == 0) {
      now_s = now;
      claims_s = __popc(claimers);
    }
  }
  __syncthreads();  // the row's at[] and score[] writes are visible to every thread from here
  // ---- the whole block: the m smallest candidate keys (rule 3)
  const int now = now_s, m = claims_s;
  unsigned long long above = 0;  // every key taken so far is <= above; keys are unique (the slot is in them)
  for (int r = 0; r < m; r++) {  // m is the same in every thread (read after a barrier), and so is every round
    unsigned long long best = RESOLVE_NO_SLOT;
    for (int i = tid; i < count && above != RESOLVE_NO_SLOT; i += RESOLVE_THREADS) {
      const int holder = owner[i];
      float value;
      if (holder < 0) {
        value = -1.0f;
      } else {
        const int last = at[holder];
        if (pending[i] || last == now) continue;
        value = __fmul_rn(score[holder], exp2f(log2_decay * (float)(now - last)));
        value = __fadd_rn(value, 0.0f);  // -0 orders as +0 (equal values tie on the slot)
      }
      const unsigned long long cand = ((unsigned long long)ordered_bits(value) << 32) | (uint32_t)i;
      if ((r == 0 || cand > above) && cand < best) best = cand;
    }
    best = warp_min_u64(best);
    if (lane == 0) warp_best[warp] = best;
    __syncthreads();
    if (warp == 0) {
      const unsigned long long v = warp_min_u64(warp_best[lane]);
      if (lane == 0) picked[r] = v;
    }
    __syncthreads();
    // NO_SLOT: no candidates left, and none in the later rounds (their scans are skipped): those claimers go
    // without a slot
    above = picked[r];
  }
  // ---- commit (warp 0): distinct slots, distinct keys
  if (warp == 0 && lane < k) {
    if (claim_rank >= 0 && claim_rank < m && picked[claim_rank] != RESOLVE_NO_SLOT) {
      const int s = (int)(uint32_t)(picked[claim_rank] & 0xffffffffu);
      const int old = owner[s];
      if (old >= 0) table[old] = -1;
      owner[s] = key;
      if (code == 1) {
        table[key] = s;
      } else {
        table[key] = -2 - s;
        pending[s] = 1;
      }
      slot = s;
    }
    plan[2 * lane] = slot;
    plan[2 * lane + 1] = code == 3 ? 2 : code;
  }
}

}  // namespace d3
