// ConvRot rotation of activation rows: x -> x . H256 per group of 256 columns, H256 = h4 (x) h4 (x) h4 (x) h4 / 16
// with h4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]] (drama3/offload.py:170-176, drama3/kernels.py:226-258).
// The butterfly below applies the four radix-4 stages in the reference kernel's order (strides 1, 4, 16, 64) with
// the same expression order, and scales by 1/16 at the end, so its float results are the reference's bit for bit.
// Optionally the row is first SwiGLU(gate | up) = gate / (1 + exp(-gate)) * up of a [rows, 2K] float input (the
// reference's fast-exp form).
#pragma once

#include "common.cuh"

namespace d3 {

// In-place rotation of row[0..K) in shared memory by `nthreads` threads (tid < nthreads); K % 256 == 0. The caller
// synchronizes before (row written) and after (row read); the stages synchronize with `sync` between them.
template <class Sync>
D3_DEV void hadamard256_rows(float* row, int K, int tid, int nthreads, Sync sync) {
  for (int stride = 1; stride < 256; stride *= 4) {
    for (int t = tid; t < K / 4; t += nthreads) {
      int within = t & 63, low = within % stride, high = within / stride;
      int i = (t >> 6) * 256 + high * stride * 4 + low;
      float a = row[i], b = row[i + stride], c = row[i + 2 * stride], d = row[i + 3 * stride];
      row[i] = a + b + c - d;
      row[i + stride] = a + b - c + d;
      row[i + 2 * stride] = a - b + c + d;
      row[i + 3 * stride] = -a + b + c + d;
    }
    sync();
  }
}

D3_DEV float swiglu_fast(float g, float u) { return g / (1.0f + __expf(-g)) * u; }

// One block per row; mode 0: fp32 input [rows, K]; 1: bf16 input [rows, K]; 2: fp32 [rows, 2K] gate | up, SwiGLU
// first. Skipped entirely when only_if[0] == 0 (the output is then left as it was). In place (out == x) is allowed:
// a block reads its whole row before writing it.
__global__ void __launch_bounds__(256) rotate_rows_kernel(const void* x, int mode, int K, float* out,
                                                          const int* __restrict__ only_if) {
  extern __shared__ float row[];
  const int r = blockIdx.x;
  // as a programmatic dependent (inside the fused decode) x is the previous kernel's output
  grid_dependency_wait();
  allow_dependents();
  if (only_if != nullptr && only_if[0] == 0) return;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float v;
    if (mode == 2) {
      const float* f = (const float*)x + (size_t)r * 2 * K;
      v = swiglu_fast(f[i], f[K + i]);
    } else if (mode == 1) {
      v = bf16_to_f32(((const uint16_t*)x)[(size_t)r * K + i]);
    } else {
      v = ((const float*)x)[(size_t)r * K + i];
    }
    row[i] = v;
  }
  __syncthreads();
  hadamard256_rows(row, K, threadIdx.x, blockDim.x, [] { __syncthreads(); });
  for (int i = threadIdx.x; i < K; i += blockDim.x) out[(size_t)r * K + i] = row[i] * 0.0625f;
}

}  // namespace d3
