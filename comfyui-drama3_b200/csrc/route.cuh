// Decode routing and the routed combine, batched over rows.
//
// route_rows follows drama3/kernels.py:39-67 (route_experts) row by row: the k largest of n bfloat16 logits in the
// order (value descending, index ascending), and their softmax weights renormalized over those k: expf(l - l_0)
// summed in rank order from rank 0, each weight divided by the sum and rounded to bfloat16. The reference runs one
// 256-thread block per row with an O(n^2) rank count; here one warp owns a row and extracts the k winners by k warp
// arg-max passes, and a block carries 8 rows.
//
// combine_rows follows drama3/kernels.py:69-76 (weighted_sum): out[h] = bf16(sum_e parts[e, h] * w[e]), fp32
// accumulation in e order, fused multiply-add as NVRTC contracts it.
#pragma once

#include "common.cuh"

namespace d3 {

constexpr int ROUTE_WARPS = 8;
constexpr int ROUTE_MAX_N = 1024;

// Better candidate under (value descending, index ascending).
D3_DEV bool route_better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__global__ void __launch_bounds__(ROUTE_WARPS * 32) route_rows(const uint16_t* __restrict__ logits, int rows, int n,
                                                                int k, int64_t* __restrict__ ids,
                                                                float* __restrict__ weights) {
  __shared__ float value[ROUTE_WARPS][ROUTE_MAX_N];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * ROUTE_WARPS + warp;
  if (row >= rows) return;
  float* v = value[warp];
  const uint16_t* src = logits + (size_t)row * n;
  for (int i = lane; i < n; i += 32) v[i] = bf16_to_f32(src[i]);
  __syncwarp();
  // per lane: a bitmask of its own candidates already taken (lane owns indices lane + 32 * m, m < 32)
  uint32_t taken = 0;
  float mine_top = 0.0f;  // lane e keeps the e-th winner's logit
  int mine_id = 0;
  for (int r = 0; r < k; ++r) {
    float bv = -__int_as_float(0x7f800000);
    int bi = 0x7fffffff;
    bool any = false;
    for (int m = 0, i = lane; i < n; ++m, i += 32) {
      if (taken & (1u << m)) continue;
      float x = v[i];
      if (!any || route_better(x, i, bv, bi)) {
        bv = x;
        bi = i;
        any = true;
      }
    }
    if (!any) bi = 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || route_better(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane && bi != 0x7fffffff) taken |= 1u << (bi >> 5);
    if (lane == r) {
      mine_top = bv;
      mine_id = bi;
    }
  }
  const float top0 = __shfl_sync(0xffffffffu, mine_top, 0);
  float total = 0.0f;
  // the reference sums on one thread in rank order
  for (int e = 0; e < k; ++e) {
    float t = __shfl_sync(0xffffffffu, mine_top, e);
    total += expf(t - top0);
  }
  if (lane < k) {
    weights[(size_t)row * k + lane] = bf16_to_f32(f32_to_bf16(expf(mine_top - top0) / total));
    ids[(size_t)row * k + lane] = (int64_t)mine_id;
  }
}

__global__ void combine_rows(const float* __restrict__ parts, const float* __restrict__ weights, int rows, int k, int H,
                             uint16_t* __restrict__ out) {
  int h = blockIdx.x * blockDim.x + threadIdx.x;
  int row = blockIdx.y;
  if (h >= H || row >= rows) return;
  const float* p = parts + (size_t)row * k * H + h;
  const float* w = weights + (size_t)row * k;
  float acc = 0.0f;
  for (int e = 0; e < k; ++e) acc = __fmaf_rn(p[(size_t)e * H], w[e], acc);
  out[(size_t)row * H + h] = f32_to_bf16(acc);
}

}  // namespace d3
