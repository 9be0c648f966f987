// The shared expert of a decode step in two launches (drama3/model.py:40-47 and the sigmoid-gated add of :123):
//   shared_up:   a = bf16(bf16(silu(g)) * u), g | u = bf16(x W_gu^T)        (gate_up linear, SwiGLU)
//                and, in CTA 0, the gate bf16(sigmoid(bf16(x w_g))) per row
//   shared_down: out = bf16(out + bf16(gate * bf16(a W_d^T)))               (down linear, gated add)
// Every bf16 rounding sits where the reference's bf16 modules round (each linear's output, silu, the product, the
// sigmoid, the gated product and the residual add); the sums are fp32 over exact bf16 products, on the tensor cores
// (mma.sync m16n8k16: the matrices are 4 MB and 2 MB read once, so these launches are bound by memory and latency,
// not by the MMA form). Each CTA bulk-copies its contiguous weight rows into shared memory before it waits on the
// previous grid (the weights do not depend on it), so the copies overlap the previous kernel's tail; the activation
// rows are bulk-copied after the wait and read as A fragments by ldmatrix. x [M, 2048] bf16 with M <= 16 lines; `out`
// is the MoE output the gated shared expert is added to.
#pragma once

#include "router.cuh"

namespace d3 {

constexpr int SH_WARPS = 8;
constexpr int SH_H = 2048;        // hidden size
constexpr int SH_UP_CH = 4;       // intermediate channels per shared_up CTA: 4 gate rows and 4 up rows, one n-tile
constexpr int SH_DOWN_ROWS = 16;  // output rows per shared_down CTA (two n-tiles)
constexpr int SH_UP_PITCH = SH_H + 8;  // padded shared-memory row pitch (elements): conflict-free fragments
constexpr int SH_UP_KSTEPS = SH_H / SH_WARPS / 16;

D3_DEV float bf16r(float v) { return bf16_to_f32(f32_to_bf16(v)); }

D3_DEV float sigmoid_bf16(float v) { return bf16r(1.0f / (1.0f + expf(-bf16r(v)))); }

// a [M, I] bf16 = SwiGLU of the gate_up linear; w_gu [2I, 2048] (gate rows, then up rows); CTA 0 also writes
// gate [M] fp32 = bf16(sigmoid(bf16(x . w_g))). Grid: I / SH_UP_CH CTAs; dynamic shared memory: 9 + 16 rows of
// SH_UP_PITCH elements (the 8 weight rows and w_g in CTA 0, then the rows of x).
__global__ void __launch_bounds__(SH_WARPS * 32)
    shared_up_kernel(const uint16_t* __restrict__ x, int M, const uint16_t* __restrict__ w_gu,
                     const uint16_t* __restrict__ w_g, int I, uint16_t* __restrict__ a, float* __restrict__ gate) {
  extern __shared__ __align__(128) uint8_t sh_smem[];
  uint16_t* ws = reinterpret_cast<uint16_t*>(sh_smem);
  uint16_t* xs = ws + 9 * SH_UP_PITCH;
  __shared__ float part[SH_WARPS][RT_MAX_M][8 + 1];
  __shared__ float part_g[SH_WARPS][RT_MAX_M];
  __shared__ __align__(8) uint64_t bar[2];  // the weight rows, the rows of x
  const int j0 = blockIdx.x * SH_UP_CH;
  const bool with_gate = blockIdx.x == 0;
  D3_GSTAMP(8);
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar[0], (uint32_t)((8 + (with_gate ? 1 : 0)) * SH_H * 2));
    const uint64_t pol = policy_evict_first();
    for (int r = 0; r < 8; ++r) {
      const int src = r < SH_UP_CH ? j0 + r : I + j0 + r - SH_UP_CH;  // gate rows, then the matching up rows
      bulk_g2s(ws + r * SH_UP_PITCH, w_gu + (size_t)src * SH_H, SH_H * 2, &bar[0], pol);
    }
    if (with_gate) bulk_g2s(ws + 8 * SH_UP_PITCH, w_g, SH_H * 2, &bar[0], pol);
  }
  grid_dependency_wait();
  allow_dependents();
  D3_GSTAMP(9);
  if (threadIdx.x == 0) bulk_rows(xs, x, M, SH_H, SH_UP_PITCH, &bar[1], policy_evict_last());
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int k0 = warp * SH_UP_KSTEPS * 16;
  __syncthreads();  // the barriers' initialization is visible to every thread
  const bool ok = mbar_wait(&bar[1], 0) && mbar_wait(&bar[0], 0);
  D3_GSTAMP(10);
  float acc[1][4] = {}, accg[4] = {};
  if (ok) {
    // rows of xs past M are left as they are: an A row only reaches the same C row, which is not read
    const int rows_w[1] = {0};
    mma_rows_smem<1, SH_UP_KSTEPS>(acc, xs, SH_UP_PITCH, ws, SH_UP_PITCH, rows_w, 1, k0);
    if (with_gate) {
      // an n-tile whose 8 B rows are all w_g (row 8): every column of its C holds x . w_g
#pragma unroll 4
      for (int s = 0; s < SH_UP_KSTEPS; ++s) {
        uint32_t af[4];
        frag_a_smem(af, xs, SH_UP_PITCH, k0 + 16 * s);
        const uint16_t* wr = ws + 8 * SH_UP_PITCH + k0 + 16 * s + 2 * c;
        mma_bf16_16816(accg, af[0], af[1], af[2], af[3], *reinterpret_cast<const uint32_t*>(wr),
                       *reinterpret_cast<const uint32_t*>(wr + 8));
      }
    }
  }
  D3_GSTAMP(11);
  part[warp][g][2 * c] = acc[0][0];
  part[warp][g][2 * c + 1] = acc[0][1];
  part[warp][g + 8][2 * c] = acc[0][2];
  part[warp][g + 8][2 * c + 1] = acc[0][3];
  if (c == 0) {
    part_g[warp][g] = accg[0];
    part_g[warp][g + 8] = accg[2];
  }
  __syncthreads();
  if (threadIdx.x < M * SH_UP_CH) {
    const int m = threadIdx.x / SH_UP_CH, j = threadIdx.x - m * SH_UP_CH;
    float gs = 0.0f, us = 0.0f;
#pragma unroll
    for (int q = 0; q < SH_WARPS; ++q) {
      gs += part[q][m][j];
      us += part[q][m][SH_UP_CH + j];
    }
    gs = bf16r(gs);
    us = bf16r(us);
    const float s = bf16r(gs / (1.0f + expf(-gs)));
    a[(size_t)m * I + j0 + j] = f32_to_bf16(s * us);
  } else if (with_gate && threadIdx.x >= 128 && threadIdx.x - 128 < M) {
    const int m = threadIdx.x - 128;
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < SH_WARPS; ++q) s += part_g[q][m];
    gate[m] = sigmoid_bf16(s);
  }
  D3_GSTAMP(12);
}

// out [M, 2048] bf16 += gate * down projection of a [M, I] bf16; w_d [2048, I]; gate [M] fp32 from shared_up.
// KS = I / 128 (the k16 steps of one warp). Grid: 2048 / SH_DOWN_ROWS CTAs; dynamic shared memory: 16 weight rows,
// then 16 rows of a, each I + 8 elements.
template <int KS>
__global__ void __launch_bounds__(SH_WARPS * 32)
    shared_down_kernel(const uint16_t* __restrict__ a, int M, const uint16_t* __restrict__ w_d,
                       const float* __restrict__ gate, uint16_t* __restrict__ out) {
  constexpr int I = KS * 128, PITCH = I + 8;
  extern __shared__ __align__(128) uint8_t sh_smem[];
  uint16_t* ws = reinterpret_cast<uint16_t*>(sh_smem);
  uint16_t* as = ws + SH_DOWN_ROWS * PITCH;
  __shared__ float part[SH_WARPS][RT_MAX_M][2 * 8 + 1];
  __shared__ __align__(8) uint64_t bar[2];  // the weight rows, the rows of a
  const int h0 = blockIdx.x * SH_DOWN_ROWS;
  D3_GSTAMP(16);
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    bulk_rows(ws, w_d + (size_t)h0 * I, SH_DOWN_ROWS, I, PITCH, &bar[0], policy_evict_first());
  }
  grid_dependency_wait();
  allow_dependents();
  D3_GSTAMP(17);
  if (threadIdx.x == 0) bulk_rows(as, a, M, I, PITCH, &bar[1], policy_evict_last());
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int k0 = warp * KS * 16;
  __syncthreads();
  const bool ok = mbar_wait(&bar[1], 0) && mbar_wait(&bar[0], 0);
  D3_GSTAMP(18);
  float acc[2][4] = {};
  const int brow[2] = {0, 8};
  if (ok) mma_rows_smem<2, KS>(acc, as, PITCH, ws, PITCH, brow, 2, k0);
  D3_GSTAMP(19);
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    part[warp][g][nt * 8 + 2 * c] = acc[nt][0];
    part[warp][g][nt * 8 + 2 * c + 1] = acc[nt][1];
    part[warp][g + 8][nt * 8 + 2 * c] = acc[nt][2];
    part[warp][g + 8][nt * 8 + 2 * c + 1] = acc[nt][3];
  }
  __syncthreads();
  if (threadIdx.x < M * SH_DOWN_ROWS) {
    const int m = threadIdx.x / SH_DOWN_ROWS, r = threadIdx.x - m * SH_DOWN_ROWS;
    float d = 0.0f;
#pragma unroll
    for (int q = 0; q < SH_WARPS; ++q) d += part[q][m][r];
    const float shared = bf16r(gate[m] * bf16r(d));
    uint16_t* o = out + (size_t)m * SH_H + h0 + r;
    *o = f32_to_bf16(bf16_to_f32(*o) + shared);
  }
  D3_GSTAMP(20);
}

}  // namespace d3
