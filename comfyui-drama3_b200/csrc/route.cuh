// Decode routing and the routed combine, batched over rows.
//
// route_rows follows drama3/kernels.py:39-67 (route_experts) row by row: the k largest of n bfloat16 logits in the
// order (value descending, index ascending), and their softmax weights renormalized over those k: expf(l - l_0)
// summed in rank order from rank 0, each weight divided by the sum and rounded to bfloat16. Like the reference, each
// logit's rank is the count of logits ahead of it, so ties, and NaNs, resolve as there; here a group of 128 threads
// owns a row (the reference: a 256-thread block), each rank count reads the row four values at a time, and a block
// carries two rows.
//
// combine_rows follows drama3/kernels.py:69-76 (weighted_sum): out[h] = bf16(sum_e parts[e, h] * w[e]), fp32
// accumulation in e order, fused multiply-add as NVRTC contracts it.
#pragma once

#include "common.cuh"

namespace d3 {

constexpr int ROUTE_GROUP = 128;  // threads per row
constexpr int ROUTE_ROWS = 2;     // rows per block
constexpr int ROUTE_MAX_N = 1024;
constexpr int ROUTE_MAX_K = 32;

// One row's ranking by `threads` threads (this one is t): every logit v[i] (i < n, bf16 values as floats in 16-byte
// aligned shared memory) takes rank = #{j : v[j] > v[i] or (v[j] == v[i] and j < i)}, and the ones ranked below k
// are written to top[rank], top_id[rank] (which the caller zeroed, as the reference does).
D3_DEV void route_rank(const float* v, int n, int k, int t, int threads, float* top, int* top_id) {
  for (int i = t; i < n; i += threads) {
    const float x = v[i];
    int rank = 0, j = 0;
    for (; j + 4 <= n; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(v + j);
      rank += (q.x > x) | ((q.x == x) & (j < i));
      rank += (q.y > x) | ((q.y == x) & (j + 1 < i));
      rank += (q.z > x) | ((q.z == x) & (j + 2 < i));
      rank += (q.w > x) | ((q.w == x) & (j + 3 < i));
    }
    for (; j < n; ++j) rank += (v[j] > x) | ((v[j] == x) & (j < i));
    if (rank < k) {
      top[rank] = x;
      top_id[rank] = i;
    }
  }
}

// The ranked row's ids and weights, threads t < k: expf(top[e] - top[0]) summed from rank 0 in order (every thread
// forms the same sum), each weight the quotient rounded to bf16.
D3_DEV void route_weights(const float* top, const int* top_id, int k, int t, int64_t* __restrict__ ids,
                          float* __restrict__ weights) {
  if (t < k) {
    float total = 0.0f;
    for (int e = 0; e < k; ++e) total += expf(top[e] - top[0]);
    weights[t] = bf16_to_f32(f32_to_bf16(expf(top[t] - top[0]) / total));
    ids[t] = (int64_t)top_id[t];
  }
}

__global__ void __launch_bounds__(ROUTE_ROWS * ROUTE_GROUP) route_rows(const uint16_t* __restrict__ logits, int rows,
                                                                      int n, int k, int64_t* __restrict__ ids,
                                                                      float* __restrict__ weights) {
  __shared__ __align__(16) float value[ROUTE_ROWS][ROUTE_MAX_N];
  __shared__ float top[ROUTE_ROWS][ROUTE_MAX_K];
  __shared__ int top_id[ROUTE_ROWS][ROUTE_MAX_K];
  const int group = threadIdx.x / ROUTE_GROUP, t = threadIdx.x % ROUTE_GROUP;
  const int row = blockIdx.x * ROUTE_ROWS + group;
  if (t < ROUTE_MAX_K) {
    top[group][t] = 0.0f;
    top_id[group][t] = 0;
  }
  if (row < rows) {
    const uint16_t* src = logits + (size_t)row * n;
    for (int i = t; i < n; i += ROUTE_GROUP) value[group][i] = bf16_to_f32(src[i]);
  }
  __syncthreads();
  if (row < rows) route_rank(value[group], n, k, t, ROUTE_GROUP, top[group], top_id[group]);
  __syncthreads();
  if (row < rows) route_weights(top[group], top_id[group], k, t, ids + (size_t)row * k, weights + (size_t)row * k);
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
