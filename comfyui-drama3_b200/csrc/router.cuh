// Router linear and decode routing in one launch: SparseMoeBlock's gate (a bias-free bf16 linear, hidden -> experts)
// followed by kernels.route (drama3/model.py:107-119) for the rows of a decode step (M <= 16 lines).
//
// logits = bf16(x W^T): bf16 products accumulated in fp32 on the tensor cores (mma.sync m16n8k16: the weights are a
// 0.5 MB matrix and the launch is bound by latency, which this form keeps low), summed over the k range of each of
// the 8 warps in a fixed order, rounded to bf16 as the linear's output is. A cluster of 8 CTAs splits the experts.
// Each CTA bulk-copies its experts' weight rows into shared memory before it waits on the previous grid (the
// weights do not depend on it), then bulk-copies the rows of x after it; A fragments come from shared memory by
// ldmatrix. Row r's logits go straight into the shared memory of CTA r % 8 (distributed shared memory), and after
// the cluster barrier each CTA ranks its rows with route_rank / route_weights, the route kernel's arithmetic, so ids
// and weights are those kernels.route gives on the same logits, bit for bit.
#pragma once

#include <cooperative_groups.h>

#include "moe_decode.cuh"
#include "route.cuh"

namespace d3 {

constexpr int RT_CTAS = 8;     // the cluster: experts split over its CTAs
constexpr int RT_WARPS = 8;    // the hidden dimension split over a CTA's warps
constexpr int RT_H = 2048;     // hidden size
constexpr int RT_MAX_E = 256;  // experts (a multiple of 64)
constexpr int RT_MAX_M = 16;   // rows
constexpr int RT_NT = RT_MAX_E / RT_CTAS / 8;  // n-tiles of 8 experts per CTA, at most
constexpr int RT_PITCH = RT_H + 8;             // padded row pitch in shared memory (elements): conflict-free fragments
constexpr int RT_KSTEPS = RT_H / RT_WARPS / 16;  // k16 steps per warp
constexpr int RT_ROWS_PER_CTA = RT_MAX_M / RT_CTAS;  // rows each CTA routes
static_assert(RT_ROWS_PER_CTA * ROUTE_GROUP == RT_WARPS * 32, "a CTA's threads route its rows");

D3_DEV void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A fragments (m16n8k16, row-major A) of the k16 step at column k0 of 16 rows held in shared memory with a row
// pitch of `pitch` elements (a multiple of 8, pitch / 8 odd: the 8 rows an ldmatrix phase reads fall in distinct
// banks).
D3_DEV void frag_a_smem(uint32_t (&a)[4], const uint16_t* rows, int pitch, int k0) {
  const int lane = threadIdx.x & 31, mat = lane >> 3;
  const uint16_t* p = rows + ((lane & 7) + 8 * (mat & 1)) * pitch + k0 + 8 * (mat >> 1);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(smem_u32(p)));
}

// acc[nt] += the A rows `xs` (16 rows in shared memory, pitch `xpitch`) x the weight rows brow[nt] .. + 7 held in
// shared memory (pitch `pitch` elements), over the warp's KSTEPS k16 steps from k0.
template <int NT, int KSTEPS>
D3_DEV void mma_rows_smem(float (&acc)[NT][4], const uint16_t* xs, int xpitch, const uint16_t* w, int pitch,
                          const int (&brow)[NT], int nt_live, int k0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll 4
  for (int s = 0; s < KSTEPS; ++s) {
    uint32_t a[4];
    frag_a_smem(a, xs, xpitch, k0 + 16 * s);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (nt < nt_live) {
        const uint16_t* wr = w + (brow[nt] + g) * pitch + k0 + 16 * s + 2 * c;
        mma_bf16_16816(acc[nt], a[0], a[1], a[2], a[3], *reinterpret_cast<const uint32_t*>(wr),
                       *reinterpret_cast<const uint32_t*>(wr + 8));
      }
    }
  }
}

// Bulk copies of `rows` consecutive rows of K bf16 (from src, row stride K) into shared memory rows of `pitch`
// elements, issued by one thread, completing on `bar` (armed here for their bytes).
D3_DEV void bulk_rows(uint16_t* dst, const uint16_t* src, int rows, int K, int pitch, uint64_t* bar, uint64_t pol) {
  mbar_arrive_expect_tx(bar, (uint32_t)(rows * K * 2));
  for (int r = 0; r < rows; ++r) bulk_g2s(dst + r * pitch, src + (size_t)r * K, (uint32_t)(K * 2), bar, pol);
}

// x [M, 2048] bf16, w [E, 2048] bf16 -> ids [M, k] int64, weights [M, k] fp32 (bf16 values), logits [M, E] bf16 (if
// not null). E % 64 == 0, E <= 256, M <= 16; one cluster of RT_CTAS CTAs; dynamic shared memory: E / RT_CTAS weight
// rows, then 16 rows of x, each RT_PITCH elements.
__global__ void __cluster_dims__(RT_CTAS, 1, 1) __launch_bounds__(RT_WARPS * 32)
    router_kernel(const uint16_t* __restrict__ x, int M, const uint16_t* __restrict__ w, int E, int k,
                  int64_t* __restrict__ ids, float* __restrict__ weights, uint16_t* __restrict__ logits) {
  extern __shared__ __align__(128) uint8_t rt_smem[];
  __shared__ float part[RT_WARPS][RT_MAX_M][RT_MAX_E / RT_CTAS + 1];  // each warp's sums over its k range
  __shared__ __align__(16) float all[RT_ROWS_PER_CTA][RT_MAX_E];      // this CTA's rows: every expert's logits
  __shared__ float top[RT_ROWS_PER_CTA][ROUTE_MAX_K];
  __shared__ int top_id[RT_ROWS_PER_CTA][ROUTE_MAX_K];
  __shared__ __align__(8) uint64_t bar[2];  // the weight rows, the rows of x
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int EC = E / RT_CTAS, e0 = rank * EC, NT = EC / 8;
  uint16_t* ws = reinterpret_cast<uint16_t*>(rt_smem);
  uint16_t* xs = ws + EC * RT_PITCH;
  D3_GSTAMP(0);
  if (threadIdx.x < RT_ROWS_PER_CTA * ROUTE_MAX_K) {
    (&top[0][0])[threadIdx.x] = 0.0f;
    (&top_id[0][0])[threadIdx.x] = 0;
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    bulk_rows(ws, w + (size_t)e0 * RT_H, EC, RT_H, RT_PITCH, &bar[0], policy_evict_first());  // needs no wait
  }
  // as a programmatic dependent, x is the previous kernel's output
  grid_dependency_wait();
  allow_dependents();
  D3_GSTAMP(1);
  if (threadIdx.x == 0) bulk_rows(xs, x, M, RT_H, RT_PITCH, &bar[1], policy_evict_last());
  __syncthreads();  // the barriers' initialization is visible to every thread
  const bool ok = mbar_wait(&bar[1], 0) && mbar_wait(&bar[0], 0);
  D3_GSTAMP(2);
  float acc[RT_NT][4];
  int brow[RT_NT];
#pragma unroll
  for (int nt = 0; nt < RT_NT; ++nt) {
    acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
    brow[nt] = nt * 8;
  }
  // rows of xs past M are left as they are: an A row only reaches the same C row, which is not read
  const int k0 = warp * RT_KSTEPS * 16;
  if (ok) mma_rows_smem<RT_NT, RT_KSTEPS>(acc, xs, RT_PITCH, ws, RT_PITCH, brow, NT, k0);
  D3_GSTAMP(3);
  // C fragments: acc[nt][0..1] = row g, experts nt * 8 + 2c, + 1; acc[nt][2..3] = row g + 8
#pragma unroll
  for (int nt = 0; nt < RT_NT; ++nt) {
    if (nt < NT) {
      part[warp][g][nt * 8 + 2 * c] = acc[nt][0];
      part[warp][g][nt * 8 + 2 * c + 1] = acc[nt][1];
      part[warp][g + 8][nt * 8 + 2 * c] = acc[nt][2];
      part[warp][g + 8][nt * 8 + 2 * c + 1] = acc[nt][3];
    }
  }
  __syncthreads();
  D3_GSTAMP(4);
  for (int i = threadIdx.x; i < M * EC; i += blockDim.x) {
    const int row = i / EC, e = i - row * EC;
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < RT_WARPS; ++q) s += part[q][row][e];
    const uint16_t b = f32_to_bf16(s);
    if (logits) logits[(size_t)row * E + e0 + e] = b;
    float* dst = cluster.map_shared_rank(&all[row / RT_CTAS][0], row % RT_CTAS);
    dst[e0 + e] = bf16_to_f32(b);
  }
  cluster.sync();  // every row's logits are in its CTA's shared memory
  D3_GSTAMP(5);
  const int group = threadIdx.x / ROUTE_GROUP, t = threadIdx.x % ROUTE_GROUP;
  const int row = rank + RT_CTAS * group;
  if (row < M) route_rank(all[group], E, k, t, ROUTE_GROUP, top[group], top_id[group]);
  __syncthreads();
  if (row < M) route_weights(top[group], top_id[group], k, t, ids + (size_t)row * k, weights + (size_t)row * k);
  D3_GSTAMP(6);
}

}  // namespace d3
