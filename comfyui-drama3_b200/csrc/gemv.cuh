// Per-expert decode GEMVs with the reference's slot-cache plan semantics (drama3/kernels.py:274-363, 495-536):
// out[e, n] = expert e's row n . x[e or 0] (x fp32 [1 or k, K]), where expert e is read from its slot (plan code 0)
// or, on a miss, straight from host memory (pinned, mapped: zero-copy over the host link) and copied into its new
// slot on the way (plan slot >= 0). These kernels serve the host-offload slot cache; experts resident in HBM go
// through the fused decode kernels instead.
//
// Differences from the reference kernels, none visible in the results beyond float summation order:
//   - one warp computes two rows and keeps all of its 16-byte loads of both rows in flight before any arithmetic;
//   - the staged x row is swizzled in shared memory (conflict-free 16-byte loads);
//   - expert ids and slots are range-checked (an out-of-range one gives zeros and sets the fault word);
//   - a filled W4/W6 row is written to its slot and used from registers (the reference writes then re-reads it).
#pragma once

#include "common.cuh"
#include "formats.cuh"

namespace d3 {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_RPW = 2;                           // rows per warp
constexpr int GEMV_ROWS = GEMV_WARPS * GEMV_RPW;      // rows per block (the reference's ROWS_PER_BLOCK)
constexpr int GEMV_MAXV = 8;                          // 16-byte vectors per lane per row: K <= 32 * 16 * 8 / 1

struct GemvArgs {
  const float* x;
  int x_rows;
  const int64_t* ids;
  const int* plan;        // [k, 2] (slot, code)
  const int* took_over;   // I8 only
  int late;               // I8 only
  uint8_t* slot_w;        // slot fields
  void* slot_s;           // FP8: float block scales; I8: float row scales; codes: uint8 group scales
  float* slot_c;          // codes: s_channel
  const uint8_t* host_w;  // host fields
  const void* host_s;
  const float* host_c;
  const float* codebook;  // W4
  float* out;             // [k, N]
  int N, K, num_experts, slots;
};

template <int FMT>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_plan_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float xs[];  // K floats, swizzled
  __shared__ float block_scale[32];
  __shared__ float lut[16];
  const int e = blockIdx.y, N = a.N, K = a.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int first = blockIdx.x * GEMV_ROWS;
  const int code = a.plan[2 * e + 1], slot = a.plan[2 * e];
  const long long id = a.ids[e];
  // which experts run: as the reference (I8 leaves CPU experts, code 2, to the host unless `late` and taken over)
  bool run = true, host = code != 0;
  if (FMT == FMT_I8) {
    run = a.late ? (code == 2 && a.took_over[0]) : code != 2;
  }
  const bool id_ok = id >= 0 && id < a.num_experts;
  const bool slot_ok = slot >= 0 && slot < a.slots;
  if (run && ((host && !id_ok) || (!host && !slot_ok) || (host && slot >= a.slots))) {
    if (threadIdx.x == 0) record_fault(host ? (id_ok ? FAULT_BAD_SLOT : FAULT_BAD_EXPERT) : FAULT_BAD_SLOT);
    run = false;
  }
  if (!run) {
    if (threadIdx.x < GEMV_ROWS && first + threadIdx.x < N) a.out[(size_t)e * N + first + threadIdx.x] = 0.0f;
    return;
  }
  const bool fill = (FMT == FMT_I8 ? code == 1 : host) && slot >= 0;
  const int rb = fmt_row_bytes(FMT, K), gb = K / 16;
  const float* xsrc = a.x + (size_t)(a.x_rows == 1 ? 0 : e) * K;
  for (int f = threadIdx.x; f < K / 4; f += blockDim.x) ((float4*)xs)[xswz(f)] = ((const float4*)xsrc)[f];
  if (FMT == FMT_W4 && threadIdx.x < 16) lut[threadIdx.x] = a.codebook[threadIdx.x];
  const size_t base_row = host ? (size_t)id * N : (size_t)slot * N;
  const uint8_t* w = (host ? a.host_w : a.slot_w) + base_row * rb;
  if (FMT == FMT_FP8) {
    const int scols = K / 128, srows = N / 128;
    const float* s = (const float*)(host ? a.host_s : a.slot_s) + (base_row / 128 + first / 128) * scols;
    if (threadIdx.x < scols) {
      float v = s[threadIdx.x];
      block_scale[threadIdx.x] = v;
      if (fill && first % 128 == 0) ((float*)a.slot_s)[((size_t)slot * srows + first / 128) * scols + threadIdx.x] = v;
    }
  }
  __syncthreads();
  const int nv = K / 16;  // 16-column vectors per row
#pragma unroll
  for (int rr = 0; rr < GEMV_RPW; ++rr) {
    const int n = first + warp * GEMV_RPW + rr;
    if (n >= N) break;
    const uint8_t* row = w + (size_t)n * rb;
    uint8_t* dst = a.slot_w + ((size_t)slot * N + n) * rb;
    float acc = 0.0f;
    if (FMT == FMT_FP8 || FMT == FMT_I8) {
      uint4 q[GEMV_MAXV];
#pragma unroll
      for (int j = 0; j < GEMV_MAXV; ++j) {
        const int v = lane + 32 * j;
        if (v < nv) q[j] = __ldcs((const uint4*)row + v);
      }
#pragma unroll
      for (int j = 0; j < GEMV_MAXV; ++j) {
        const int v = lane + 32 * j;
        if (v < nv) {
          if (fill) ((uint4*)dst)[v] = q[j];
          float f[16];
          if (FMT == FMT_FP8)
            dec16_fp8(q[j], f);
          else
            dec16_i8(q[j], f);
          const float4* xr = (const float4*)xs;
          float p = dot16(f, xr + xswz(4 * v), xr + xswz(4 * v + 1), xr + xswz(4 * v + 2), xr + xswz(4 * v + 3));
          acc = FMT == FMT_FP8 ? fmaf(p, block_scale[v / 8], acc) : acc + p;
        }
      }
    } else {
      const uint8_t* grow = (const uint8_t*)(host ? a.host_s : a.slot_s) + (base_row + n) * gb;
      uint8_t* gdst = (uint8_t*)a.slot_s + ((size_t)slot * N + n) * gb;
      for (int v = lane; v < nv; v += 32) {
        const uint2 low = *(const uint2*)(row + 8 * v);
        const uint32_t high = FMT == FMT_W6 ? *(const uint32_t*)(row + K / 2 + 4 * v) : 0u;
        const uint8_t gs = grow[v];
        if (fill) {
          *(uint2*)(dst + 8 * v) = low;
          if (FMT == FMT_W6) *(uint32_t*)(dst + K / 2 + 4 * v) = high;
          gdst[v] = gs;
        }
        float f[16];
        const float s = e4m3_to_f32(gs);
        if (FMT == FMT_W4)
          dec_w4<16>(low, s, lut, f);
        else
          dec_w6<16>(low, high, s, f);
        const float4* xr = (const float4*)xs;
        acc += dot16(f, xr + xswz(4 * v), xr + xswz(4 * v + 1), xr + xswz(4 * v + 2), xr + xswz(4 * v + 3));
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      float rs = 1.0f;
      if (FMT == FMT_I8) {
        rs = ((const float*)(host ? a.host_s : a.slot_s))[base_row + n];
        if (fill) ((float*)a.slot_s)[(size_t)slot * N + n] = rs;
      } else if (fmt_codes(FMT)) {
        rs = (host ? a.host_c : a.slot_c)[base_row + n];
        if (fill) a.slot_c[(size_t)slot * N + n] = rs;
      }
      a.out[(size_t)e * N + n] = acc * rs;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Prompt rows grouped by expert (drama3/kernels.py:365-464, 538-587): group g = (expert, slot, fill, first, rows)
// over sorted rows x; out[r, n] = row n of the group's expert . x[r] (x fp32 [rows, K]). A group reads its expert
// from its slot, or from host memory when it has no slot (-1) or fills it (copying it in). This CUDA-core version
// keeps a tile of 64 dequantized weight rows and 32 activation rows in shared memory per K step.
constexpr int GRP_TN = 64, GRP_TT = 32, GRP_TK = 64;

struct GroupedArgs {
  const float* x;
  const int* groups;  // [g, 5]
  uint8_t* slot_w;
  void* slot_s;
  float* slot_c;
  const uint8_t* host_w;
  const void* host_s;
  const float* host_c;
  const float* codebook;
  float* out;
  int N, K, num_experts, slots, x_rows;
};

// grid (N / 64, groups, ceil(max rows / 32)) would be too large for long groups; instead grid.z strides over
// token tiles of the group.
template <int FMT>
__global__ void __launch_bounds__(256) grouped_plan_kernel(const GroupedArgs a) {
  __shared__ float ws[GRP_TK][GRP_TN + 1];  // dequantized weights, transposed: [k][n]
  __shared__ float xt[GRP_TK][GRP_TT + 1];  // activations, transposed: [k][t]
  __shared__ float lut[16];
  const int* g = a.groups + 5 * blockIdx.y;
  const int expert = g[0], slot = g[1], fill = g[2], gfirst = g[3], grows = g[4];
  const int N = a.N, K = a.K, n0 = blockIdx.x * GRP_TN;
  const bool host = slot < 0 || fill;
  if (grows <= 0) return;
  if ((host && (expert < 0 || expert >= a.num_experts)) || slot >= a.slots || (!host && slot < 0) ||
      gfirst < 0 || gfirst + grows > a.x_rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.z == 0) record_fault(FAULT_BAD_EXPERT);
    return;
  }
  if (FMT == FMT_W4 && threadIdx.x < 16) lut[threadIdx.x] = a.codebook[threadIdx.x];
  const int rb = fmt_row_bytes(FMT, K), gb = K / 16;
  const size_t base_row = host ? (size_t)expert * N : (size_t)slot * N;
  const uint8_t* w = (host ? a.host_w : a.slot_w) + base_row * rb;
  const bool do_fill = fill && slot >= 0 && blockIdx.z == 0;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads: 4 n x 2 t outputs each
  for (int t0 = blockIdx.z * GRP_TT; t0 < grows; t0 += gridDim.z * GRP_TT) {
    float acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += GRP_TK) {
      __syncthreads();
      // weights: 64 rows x 64 columns, 4 groups of 16 columns per row -> 256 work items
      {
        const int r = threadIdx.x >> 2, q = threadIdx.x & 3;  // row, 16-column group within the tile
        const int n = n0 + r, v = (k0 >> 4) + q;
        const uint8_t* row = w + (size_t)n * rb;
        float f[16];
        float scale = 1.0f;
        if (FMT == FMT_FP8 || FMT == FMT_I8) {
          const uint4 qv = ((const uint4*)row)[v];
          if (do_fill) ((uint4*)(a.slot_w + ((size_t)slot * N + n) * rb))[v] = qv;
          if (FMT == FMT_FP8) {
            dec16_fp8(qv, f);
            const float* s = (const float*)(host ? a.host_s : a.slot_s);
            scale = s[(base_row + n) / 128 * (K / 128) + (16 * v) / 128];
            if (do_fill && n % 128 == 0 && (16 * v) % 128 == 0)
              ((float*)a.slot_s)[((size_t)slot * N + n) / 128 * (K / 128) + (16 * v) / 128] = scale;
          } else {
            dec16_i8(qv, f);
          }
        } else {
          const uint2 low = *(const uint2*)(row + 8 * v);
          const uint32_t high = FMT == FMT_W6 ? *(const uint32_t*)(row + K / 2 + 4 * v) : 0u;
          const uint8_t* gs = (const uint8_t*)(host ? a.host_s : a.slot_s) + (base_row + n) * gb;
          if (do_fill) {
            uint8_t* d = a.slot_w + ((size_t)slot * N + n) * rb;
            *(uint2*)(d + 8 * v) = low;
            if (FMT == FMT_W6) *(uint32_t*)(d + K / 2 + 4 * v) = high;
            ((uint8_t*)a.slot_s + ((size_t)slot * N + n) * gb)[v] = gs[v];
          }
          const float s = e4m3_to_f32(gs[v]);
          if (FMT == FMT_W4)
            dec_w4<16>(low, s, lut, f);
          else
            dec_w6<16>(low, high, s, f);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) ws[16 * q + j][r] = f[j] * scale;
      }
      // activations: 32 rows x 64 columns
      for (int i = threadIdx.x; i < GRP_TT * GRP_TK / 4; i += 256) {
        const int t = i / (GRP_TK / 4), c4 = i % (GRP_TK / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + t < grows) v = ((const float4*)(a.x + (size_t)(gfirst + t0 + t) * K + k0))[c4];
        xt[4 * c4 + 0][t] = v.x;
        xt[4 * c4 + 1][t] = v.y;
        xt[4 * c4 + 2][t] = v.z;
        xt[4 * c4 + 3][t] = v.w;
      }
      __syncthreads();
#pragma unroll 8
      for (int kk = 0; kk < GRP_TK; ++kk) {
        float wv[4], xv[2];
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = ws[kk][tx + 16 * i];
        xv[0] = xt[kk][ty];
        xv[1] = xt[kk][ty + 16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[i][0] = fmaf(wv[i], xv[0], acc[i][0]);
          acc[i][1] = fmaf(wv[i], xv[1], acc[i][1]);
        }
      }
    }
    // epilogue: row scales
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = n0 + tx + 16 * i;
      float rs = 1.0f;
      if (FMT == FMT_I8) rs = ((const float*)(host ? a.host_s : a.slot_s))[base_row + n];
      if (fmt_codes(FMT)) rs = (host ? a.host_c : a.slot_c)[base_row + n];
      if (do_fill && t0 == blockIdx.z * GRP_TT && ty == 0) {
        if (FMT == FMT_I8) ((float*)a.slot_s)[(size_t)slot * N + n] = rs;
        if (fmt_codes(FMT)) a.slot_c[(size_t)slot * N + n] = rs;
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int t = t0 + ty + 16 * j;
        if (t < grows) a.out[(size_t)(gfirst + t) * N + n] = acc[i][j] * rs;
      }
    }
  }
}

}  // namespace d3
