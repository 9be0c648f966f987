// Fused decode of a routed-expert MoE layer for M = 1..16 rows (lines decoded together) on sm_100a.
//
// Replaces, for banks resident in HBM, the chain of drama3/offload.py:108-123 (resident_decode): gemv(gate_up) ->
// SwiGLU [-> ConvRot rotate] -> gemv(down) -> weighted_sum, which the reference runs once per row
// (drama3/model.py:111-113). Here all M rows go through one pass that reads each routed expert once:
//
//   up   (K1): the unique experts of the M*k (row, rank) pairs, gate and up rows streamed HBM -> shared memory by
//              1-D bulk copies (cp.async.bulk) on an mbarrier ring filled by one producer warp; eight consumer warps
//              dequantize in registers and write a1[pair, i] = SwiGLU(gate . x, up . x) (fp32).
//   [rot]:     ConvRot formats only, the reference rotate of a1 (rotate_rows_kernel, in place).
//   down (K2): each CTA owns a slice of output columns n0..n1 for every unique expert, so the routed combine
//              out[t, n] = bf16(sum_j w[t, j] * down_{e(t,j)}[n] . a1[t*k+j]) happens inside the CTA, in rank order,
//              deterministic and without atomics. Launched as a programmatic dependent of the kernel before it: it
//              issues its weight copies before waiting for a1, so they overlap the previous kernel's tail.
//
// Formats (the reference's safetensors layouts, drama3/offload.py:72-90,755-766, tools/convert.py:48-82,179-215):
//   FP8  e4m3 rows [E*N, K], fp32 128x128 block scales [E*N/128, K/128]; x used as is.
//   I8   int8 rows [E*N, K], fp32 row scales [E*N]; ConvRot (x rotated per 256 columns).
//   W4   4-bit codes [E*N, K/2] (low nibble = even column), e4m3 group scales [E*N, K/16], fp32 s_channel [E*N],
//        a 16-entry float codebook; weight = clamp(rint(codebook[c] * scale), +-127) (drama3/kernels.py:469-483).
//   W6   6-bit: nibble plane [K/2] then 2-bit high plane [K/4] per row; weight = clamp(rint((c - 32) * scale), +-127).
#pragma once

#include "common.cuh"
#include "rotate.cuh"

namespace d3 {

enum { FMT_FP8 = 0, FMT_I8 = 1, FMT_W4 = 2, FMT_W6 = 3 };

constexpr int DEC_WARPS = 8;                      // consumer warps
constexpr int DEC_THREADS = (DEC_WARPS + 1) * 32;  // + one producer warp
constexpr int DEC_MAX_PAIRS = 128;                 // M * k (16 rows x top-8)
constexpr int DEC_MAX_STAGES = 8;

__host__ __device__ constexpr int fmt_row_bytes(int fmt, int K) {
  return fmt == FMT_W4 ? K / 2 : fmt == FMT_W6 ? 3 * K / 4 : K;
}
__host__ __device__ constexpr bool fmt_rotated(int fmt) { return fmt != FMT_FP8; }
__host__ __device__ constexpr bool fmt_codes(int fmt) { return fmt == FMT_W4 || fmt == FMT_W6; }

// ---------------------------------------------------------------------------------------------------------------
// The pass plan: the M*k (row, rank) pairs sorted by (expert, pair), cut into segments of one expert and at most
// `cap` pairs. Every CTA builds the same plan from ids in its prologue.
struct DecodePlan {
  int nseg;
  int rkey[DEC_MAX_PAIRS];    // expert of the pair at sorted position r (INT_MAX: invalid id)
  int rlocal[DEC_MAX_PAIRS];  // position within its expert's run
  int rlen[DEC_MAX_PAIRS];    // length of that run
  int sorted[DEC_MAX_PAIRS];  // pair at sorted position r
  int seg_expert[DEC_MAX_PAIRS];
  int seg_first[DEC_MAX_PAIRS];
  int seg_count[DEC_MAX_PAIRS];
  int warp_total[DEC_THREADS / 32];
};

// All DEC_THREADS threads call this; P <= DEC_MAX_PAIRS <= DEC_THREADS.
D3_DEV void build_plan(DecodePlan& pl, const int64_t* __restrict__ ids, int P, int E, int cap) {
  __shared__ int key[DEC_MAX_PAIRS];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < P) {
    long long e = ids[tid];
    bool ok = e >= 0 && e < E;
    if (!ok) record_fault(FAULT_BAD_EXPERT);
    key[tid] = ok ? (int)e : 0x7fffffff;
  }
  __syncthreads();
  if (tid < P) {
    const int kp = key[tid];
    int rank = 0, lower = 0, same = 0;
    for (int q = 0; q < P; ++q) {
      int kq = key[q];
      lower += kq < kp;
      same += kq == kp;
      rank += (kq < kp) | ((kq == kp) & (q < tid));
    }
    pl.sorted[rank] = tid;
    pl.rkey[rank] = kp;
    pl.rlocal[rank] = rank - lower;
    pl.rlen[rank] = same;
  }
  __syncthreads();
  const int r = tid;
  const bool start = r < P && pl.rkey[r] != 0x7fffffff && pl.rlocal[r] % cap == 0;
  const unsigned mask = __ballot_sync(0xffffffffu, start);
  if (lane == 0) pl.warp_total[warp] = __popc(mask);
  __syncthreads();
  int offset = 0, total = 0;
  for (int w = 0; w < DEC_THREADS / 32; ++w) {
    int t = pl.warp_total[w];
    offset += w < warp ? t : 0;
    total += t;
  }
  if (start) {
    int s = offset + __popc(mask & ((2u << lane) - 1u)) - 1;
    pl.seg_expert[s] = pl.rkey[r];
    pl.seg_first[s] = r;
    pl.seg_count[s] = min(cap, pl.rlen[r] - pl.rlocal[r]);
  }
  if (tid == 0) pl.nseg = total;
  __syncthreads();
}

// Swizzled float4 slot of float4 index f in a staged activation row: conflict-free 16-byte loads when lane l reads
// float4 4*(l + 32j) + q for fixed (j, q).
D3_DEV int xswz(int f) { return f ^ ((f >> 2) & 7); }
D3_DEV int xswz_elem(int i) { return (xswz(i >> 2) << 2) | (i & 3); }

// ---------------------------------------------------------------------------------------------------------------
// Weight decoding, 16 columns at a time (K1) or 4 / 8 columns (K2).
D3_DEV void dec16_fp8(uint4 w, float (&f)[16]) {
  e4m3x4(w.x, f[0], f[1], f[2], f[3]);
  e4m3x4(w.y, f[4], f[5], f[6], f[7]);
  e4m3x4(w.z, f[8], f[9], f[10], f[11]);
  e4m3x4(w.w, f[12], f[13], f[14], f[15]);
}

D3_DEV void dec4_i8(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  f0 = (float)(int)(signed char)(w & 0xFFu);
  f1 = (float)(int)(signed char)((w >> 8) & 0xFFu);
  f2 = (float)(int)(signed char)((w >> 16) & 0xFFu);
  f3 = (float)((int)w >> 24);
}

D3_DEV void dec16_i8(uint4 w, float (&f)[16]) {
  dec4_i8(w.x, f[0], f[1], f[2], f[3]);
  dec4_i8(w.y, f[4], f[5], f[6], f[7]);
  dec4_i8(w.z, f[8], f[9], f[10], f[11]);
  dec4_i8(w.w, f[12], f[13], f[14], f[15]);
}

D3_DEV float grid_value(float v, float s) { return fmaxf(-127.0f, fminf(127.0f, rintf(v * s))); }

// `n` codes starting at column c0 of a 16-column group (n = 16 or 8): W4 from 8 nibble bytes, W6 adding the 2-bit
// high plane word `high` (2 bits per column of the group).
template <int N>
D3_DEV void dec_w4(uint2 low, float s, const float* __restrict__ lut, float (&f)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    uint32_t code = ((j < 8 ? low.x : low.y) >> (4 * (j & 7))) & 0xFu;
    f[j] = grid_value(lut[code], s);
  }
}
template <int N>
D3_DEV void dec_w6(uint2 low, uint32_t high, float s, float (&f)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    uint32_t code = ((j < 8 ? low.x : low.y) >> (4 * (j & 7))) & 0xFu;
    code |= ((high >> (2 * j)) & 3u) << 4;
    f[j] = grid_value((float)((int)code - 32), s);
  }
}

D3_DEV float dot16(const float (&w)[16], const float4* __restrict__ x0, const float4* __restrict__ x1,
                   const float4* __restrict__ x2, const float4* __restrict__ x3) {
  float4 a = *x0, b = *x1, c = *x2, d = *x3;
  float acc = w[0] * a.x;
  acc = fmaf(w[1], a.y, acc);
  acc = fmaf(w[2], a.z, acc);
  acc = fmaf(w[3], a.w, acc);
  acc = fmaf(w[4], b.x, acc);
  acc = fmaf(w[5], b.y, acc);
  acc = fmaf(w[6], b.z, acc);
  acc = fmaf(w[7], b.w, acc);
  acc = fmaf(w[8], c.x, acc);
  acc = fmaf(w[9], c.y, acc);
  acc = fmaf(w[10], c.z, acc);
  acc = fmaf(w[11], c.w, acc);
  acc = fmaf(w[12], d.x, acc);
  acc = fmaf(w[13], d.y, acc);
  acc = fmaf(w[14], d.z, acc);
  acc = fmaf(w[15], d.w, acc);
  return acc;
}

D3_DEV float dot16r(const float (&w)[16], const float* __restrict__ x) {
  float acc = w[0] * x[0];
#pragma unroll
  for (int j = 1; j < 16; ++j) acc = fmaf(w[j], x[j], acc);
  return acc;
}

// ---------------------------------------------------------------------------------------------------------------
// K1: gate_up + SwiGLU.
struct UpArgs {
  const void* x;  // [M, H]: bf16 when x_bf16, else fp32
  int x_bf16;
  const int64_t* ids;  // [M, k]
  int M, k, E, H, I;
  const uint8_t* w;      // gate_up rows [E * 2I, row_bytes(H)]
  const void* scale;     // FP8: float [E*2I/128, H/128]; I8: float [E*2I]; W4/W6: uint8 e4m3 [E*2I, H/16]
  const float* channel;  // W4/W6: s_channel [E*2I]
  const float* codebook; // W4: [16]
  float* a1;             // [M*k, I]
  int stages;
};

// Rows of one K1 chunk: RPW pair-rows per consumer warp.
template <int FMT, int RPW>
struct UpGeom {
  static constexpr int CH = DEC_WARPS * RPW;  // pair-rows per chunk
};

template <int FMT, int CAP, int NV>
__global__ void __launch_bounds__(DEC_THREADS, 1) moe_up_kernel(const UpArgs a) {
  constexpr int RPW = CAP == 1 ? 1 : 2;
  constexpr int CH = DEC_WARPS * RPW;
  const int H = NV * 512, I = a.I, P = a.M * a.k;
  const int rb = fmt_row_bytes(FMT, H);  // bytes per weight row
  const int gb = H / 16;                  // group-scale bytes per row (codes)
  const int stage_bytes = 2 * CH * rb + (fmt_codes(FMT) ? 2 * CH * gb : 0);
  const int NS = a.stages;

  __shared__ DecodePlan pl;
  __shared__ __align__(8) uint64_t full_bar[DEC_MAX_STAGES], empty_bar[DEC_MAX_STAGES];
  __shared__ float lut[16];
  extern __shared__ __align__(128) uint8_t smem[];
  float* xs = (float*)smem;                                   // CAP rows of H floats (swizzled)
  float* sc = xs + CAP * H;                                   // FP8: the expert's gate_up block scales
  const int sc_floats = FMT == FMT_FP8 ? ((2 * I / 128) * (H / 128) + 3) & ~3 : 0;
  uint8_t* stages = (uint8_t*)(sc + sc_floats);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], DEC_WARPS);
    }
    fence_mbar_init();
  }
  if (FMT == FMT_W4 && tid < 16) lut[tid] = a.codebook[tid];
  // the down kernel may start its prologue (and its weight copies) now
  allow_dependents();
  build_plan(pl, a.ids, P, a.E, CAP);

  const int total = pl.nseg * I;  // pair-rows in this pass
  const int G = gridDim.x;
  const int r0 = (int)((long long)blockIdx.x * total / G), r1 = (int)((long long)(blockIdx.x + 1) * total / G);

  if (warp == DEC_WARPS) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int c = 0;
      for (int q = r0; q < r1; ++c) {
        const int s = q / I, i0 = q - s * I, cn = min(CH, min(I - i0, r1 - q));
        const int st = c % NS;
        if (c >= NS && !mbar_wait(&empty_bar[st], ((c / NS) - 1) & 1)) break;
        const int e = pl.seg_expert[s];
        uint8_t* dst = stages + (size_t)st * stage_bytes;
        const uint8_t* gate = a.w + ((size_t)e * 2 * I + i0) * rb;
        const uint8_t* up = a.w + ((size_t)e * 2 * I + I + i0) * rb;
        uint32_t bytes = 2u * cn * rb;
        if (fmt_codes(FMT)) bytes += 2u * cn * gb;
        mbar_arrive_expect_tx(&full_bar[st], bytes);
        bulk_g2s(dst, gate, cn * rb, &full_bar[st], pol);
        bulk_g2s(dst + CH * rb, up, cn * rb, &full_bar[st], pol);
        if (fmt_codes(FMT)) {
          const uint8_t* gs = (const uint8_t*)a.scale + ((size_t)e * 2 * I + i0) * gb;
          const uint8_t* us = (const uint8_t*)a.scale + ((size_t)e * 2 * I + I + i0) * gb;
          bulk_g2s(dst + 2 * CH * rb, gs, cn * gb, &full_bar[st], pol);
          bulk_g2s(dst + 2 * CH * rb + CH * gb, us, cn * gb, &full_bar[st], pol);
        }
        q += cn;
      }
      // every issued copy lands before this thread leaves (bounded)
      for (int d = max(0, c - NS); d < c; ++d)
        if (!mbar_wait(&full_bar[d % NS], (d / NS) & 1)) break;
    }
    return;
  }

  // ---------------- consumers ----------------
  // A failed (timed-out) wait clears `ok`: the warp then skips its work but still takes part in every named
  // barrier, so no other warp is left waiting on it.
  bool ok = true;
  float xr[CAP == 1 ? NV * 16 : 1];
  int cur = -1, cnt = 0, first = 0, expert = 0;
  int c = 0;
  for (int q = r0; q < r1; ++c) {
    const int s = q / I, i0 = q - s * I, cn = min(CH, min(I - i0, r1 - q));
    if (s != cur) {
      // stage this segment's input rows (and scales)
      named_sync(1, DEC_WARPS * 32);
      cur = s;
      cnt = pl.seg_count[s];
      first = pl.seg_first[s];
      expert = pl.seg_expert[s];
      for (int j = 0; j < cnt; ++j) {
        const int t = pl.sorted[first + j] / a.k;
        float4* dst = (float4*)(xs + j * H);
        for (int f = tid; f < H / 4; f += DEC_WARPS * 32) {
          float4 v;
          if (a.x_bf16) {
            uint2 b = ((const uint2*)((const uint16_t*)a.x + (size_t)t * H))[f];
            v = make_float4(bf16_to_f32(b.x & 0xFFFFu), bf16_to_f32(b.x >> 16), bf16_to_f32(b.y & 0xFFFFu),
                            bf16_to_f32(b.y >> 16));
          } else {
            v = ((const float4*)((const float*)a.x + (size_t)t * H))[f];
          }
          dst[xswz(f)] = v;
        }
      }
      if (FMT == FMT_FP8) {
        const int n = (2 * I / 128) * (H / 128);
        const float* src = (const float*)a.scale + (size_t)expert * n;
        for (int i = tid; i < n; i += DEC_WARPS * 32) sc[i] = src[i];
      }
      named_sync(1, DEC_WARPS * 32);
      if (fmt_rotated(FMT)) {
        for (int j = 0; j < cnt; ++j) {
          float* row = xs + j * H;
          for (int stride = 1; stride < 256; stride *= 4) {
            for (int t = tid; t < H / 4; t += DEC_WARPS * 32) {
              int within = t & 63, low = within % stride, high = within / stride;
              int i = (t >> 6) * 256 + high * stride * 4 + low;
              float* pa = row + xswz_elem(i);
              float* pb = row + xswz_elem(i + stride);
              float* pc = row + xswz_elem(i + 2 * stride);
              float* pd = row + xswz_elem(i + 3 * stride);
              float va = *pa, vb = *pb, vc = *pc, vd = *pd;
              *pa = va + vb + vc - vd;
              *pb = va + vb - vc + vd;
              *pc = va - vb + vc + vd;
              *pd = -va + vb + vc + vd;
            }
            named_sync(1, DEC_WARPS * 32);
          }
        }
      }
      if (CAP == 1) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          const int v = lane + 32 * j;
          const float4* xrow = (const float4*)xs;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            float4 t = xrow[xswz(4 * v + qq)];
            xr[16 * j + 4 * qq + 0] = t.x;
            xr[16 * j + 4 * qq + 1] = t.y;
            xr[16 * j + 4 * qq + 2] = t.z;
            xr[16 * j + 4 * qq + 3] = t.w;
          }
        }
      }
    }
    const int st = c % NS;
    if (ok) ok = mbar_wait(&full_bar[st], (c / NS) & 1);
    const uint8_t* stage = stages + (size_t)st * stage_bytes;
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
      const int ws = warp * RPW + rr;
      if (ok && ws < cn) {
        const int i = i0 + ws;
        const uint8_t* grow = stage + ws * rb;
        const uint8_t* urow = stage + (CH + ws) * rb;
        float ag[CAP], au[CAP];
#pragma unroll
        for (int j = 0; j < CAP; ++j) ag[j] = au[j] = 0.0f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          const int v = lane + 32 * j;  // 16-column group
          float fg[16], fu[16];
          float sg = 1.0f, su = 1.0f;
          if (FMT == FMT_FP8) {
            dec16_fp8(*(const uint4*)(grow + 16 * v), fg);
            dec16_fp8(*(const uint4*)(urow + 16 * v), fu);
            sg = sc[(i / 128) * (H / 128) + v / 8];
            su = sc[((I + i) / 128) * (H / 128) + v / 8];
          } else if (FMT == FMT_I8) {
            dec16_i8(*(const uint4*)(grow + 16 * v), fg);
            dec16_i8(*(const uint4*)(urow + 16 * v), fu);
          } else {
            const uint8_t* gsr = stage + 2 * CH * rb + ws * gb;
            const uint8_t* usr = stage + 2 * CH * rb + (CH + ws) * gb;
            const float gs = e4m3_to_f32(gsr[v]), us = e4m3_to_f32(usr[v]);
            if (FMT == FMT_W4) {
              dec_w4<16>(*(const uint2*)(grow + 8 * v), gs, lut, fg);
              dec_w4<16>(*(const uint2*)(urow + 8 * v), us, lut, fu);
            } else {
              dec_w6<16>(*(const uint2*)(grow + 8 * v), *(const uint32_t*)(grow + H / 2 + 4 * v), gs, fg);
              dec_w6<16>(*(const uint2*)(urow + 8 * v), *(const uint32_t*)(urow + H / 2 + 4 * v), us, fu);
            }
          }
#pragma unroll
          for (int jj = 0; jj < CAP; ++jj) {
            if (jj < cnt) {
              float pg, pu;
              if (CAP == 1) {
                pg = dot16r(fg, xr + 16 * j);
                pu = dot16r(fu, xr + 16 * j);
              } else {
                const float4* xrow = (const float4*)(xs + jj * H);
                const float4 *x0 = xrow + xswz(4 * v), *x1 = xrow + xswz(4 * v + 1), *x2 = xrow + xswz(4 * v + 2),
                             *x3 = xrow + xswz(4 * v + 3);
                pg = dot16(fg, x0, x1, x2, x3);
                pu = dot16(fu, x0, x1, x2, x3);
              }
              ag[jj] = fmaf(pg, sg, ag[jj]);
              au[jj] = fmaf(pu, su, au[jj]);
            }
          }
        }
        float gscale = 1.0f, uscale = 1.0f;
        if (FMT == FMT_I8) {
          // row scales, and the rotation's 1/16 folded in (exact: a power of two)
          gscale = 0.0625f * __ldg((const float*)a.scale + (size_t)expert * 2 * I + i);
          uscale = 0.0625f * __ldg((const float*)a.scale + (size_t)expert * 2 * I + I + i);
        } else if (fmt_codes(FMT)) {
          gscale = 0.0625f * __ldg(a.channel + (size_t)expert * 2 * I + i);
          uscale = 0.0625f * __ldg(a.channel + (size_t)expert * 2 * I + I + i);
        }
#pragma unroll
        for (int jj = 0; jj < CAP; ++jj) {
          if (jj < cnt) {
            float g = warp_sum(ag[jj]) * gscale, u = warp_sum(au[jj]) * uscale;
            if (lane == 0) a.a1[(size_t)pl.sorted[first + jj] * I + i] = swiglu_fast(g, u);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
    q += cn;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// K2: down projection + routed combine, split by output columns.
struct DownArgs {
  const float* a1;  // [M*k, I]: SwiGLU output (rotated for ConvRot formats)
  const int64_t* ids;
  const float* weights;  // [M, k] routing weights
  int M, k, E, H, I;
  const uint8_t* w;  // down rows [E * H, row_bytes(I)]
  const void* scale;  // FP8: float [E*H/128, I/128]; I8: float [E*H]; W4/W6: uint8 [E*H, I/16]
  const float* channel;
  const float* codebook;
  uint16_t* out;  // [M, H] bf16
  int stages;
  int rows_max;  // ceil(H / gridDim.x)
  int cap;
};

template <int FMT, int CAP>
__global__ void __launch_bounds__(DEC_THREADS, 1) moe_down_kernel(const DownArgs a) {
  const int H = a.H, I = a.I, P = a.M * a.k, NS = a.stages, RM = a.rows_max;
  const int rb = fmt_row_bytes(FMT, I);
  const int gb = I / 16;
  const int wbytes = RM * rb + (fmt_codes(FMT) ? RM * gb : 0);  // weight part of a stage, 16-byte multiple
  const int stage_bytes = wbytes + CAP * I * 4;

  __shared__ DecodePlan pl;
  __shared__ __align__(8) uint64_t full_bar[DEC_MAX_STAGES], empty_bar[DEC_MAX_STAGES];
  __shared__ float lut[16];
  extern __shared__ __align__(128) uint8_t smem[];
  float* dots = (float*)smem;  // [P][RM]
  uint8_t* stages = smem + (((size_t)P * RM * 4 + 127) & ~(size_t)127);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = (int)((long long)blockIdx.x * H / gridDim.x), n1 = (int)((long long)(blockIdx.x + 1) * H / gridDim.x);
  const int NR = n1 - n0;
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], DEC_WARPS);
    }
    fence_mbar_init();
  }
  if (FMT == FMT_W4 && tid < 16) lut[tid] = a.codebook[tid];
  for (int i = tid; i < P * RM; i += DEC_THREADS) dots[i] = 0.0f;
  build_plan(pl, a.ids, P, a.E, CAP);
  const int nseg = pl.nseg;

  if (warp == DEC_WARPS) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      // weights of the first stages: they do not depend on the previous kernel
      const int pre = min(NS, nseg);
      for (int c = 0; c < pre; ++c) {
        const int e = pl.seg_expert[c], cnt = pl.seg_count[c];
        uint8_t* dst = stages + (size_t)c * stage_bytes;
        uint32_t bytes = NR * rb + (fmt_codes(FMT) ? NR * gb : 0) + cnt * I * 4;
        mbar_arrive_expect_tx(&full_bar[c], bytes);
        bulk_g2s(dst, a.w + ((size_t)e * H + n0) * rb, NR * rb, &full_bar[c], pol);
        if (fmt_codes(FMT))
          bulk_g2s(dst + RM * rb, (const uint8_t*)a.scale + ((size_t)e * H + n0) * gb, NR * gb, &full_bar[c], pol);
      }
      grid_dependency_wait();  // a1 is complete from here on
      for (int c = 0; c < pre; ++c) {
        const int first = pl.seg_first[c], cnt = pl.seg_count[c];
        uint8_t* dst = stages + (size_t)c * stage_bytes + wbytes;
        for (int j = 0; j < cnt; ++j)
          bulk_g2s(dst + j * I * 4, a.a1 + (size_t)pl.sorted[first + j] * I, I * 4, &full_bar[c], pol);
      }
      for (int c = pre; c < nseg; ++c) {
        const int st = c % NS;
        if (!mbar_wait(&empty_bar[st], ((c / NS) - 1) & 1)) break;
        const int e = pl.seg_expert[c], cnt = pl.seg_count[c], first = pl.seg_first[c];
        uint8_t* dst = stages + (size_t)st * stage_bytes;
        uint32_t bytes = NR * rb + (fmt_codes(FMT) ? NR * gb : 0) + cnt * I * 4;
        mbar_arrive_expect_tx(&full_bar[st], bytes);
        bulk_g2s(dst, a.w + ((size_t)e * H + n0) * rb, NR * rb, &full_bar[st], pol);
        if (fmt_codes(FMT))
          bulk_g2s(dst + RM * rb, (const uint8_t*)a.scale + ((size_t)e * H + n0) * gb, NR * gb, &full_bar[st], pol);
        for (int j = 0; j < cnt; ++j)
          bulk_g2s(dst + wbytes + j * I * 4, a.a1 + (size_t)pl.sorted[first + j] * I, I * 4, &full_bar[st], pol);
      }
      for (int d = max(0, nseg - NS); d < nseg; ++d)
        if (!mbar_wait(&full_bar[d % NS], (d / NS) & 1)) break;
    }
    return;
  }

  // ---------------- consumers ----------------
  bool ok = true;
  for (int c = 0; c < nseg; ++c) {
    const int st = c % NS;
    const int e = pl.seg_expert[c], cnt = pl.seg_count[c], first = pl.seg_first[c];
    if (ok) ok = mbar_wait(&full_bar[st], (c / NS) & 1);
    if (!ok) continue;
    const uint8_t* stage = stages + (size_t)st * stage_bytes;
    const float* xa = (const float*)(stage + wbytes);
    for (int r = warp; r < NR; r += DEC_WARPS) {
      const int n = n0 + r;
      const uint8_t* wrow = stage + r * rb;
      float acc[CAP];
#pragma unroll
      for (int j = 0; j < CAP; ++j) acc[j] = 0.0f;
      if (FMT == FMT_FP8 || FMT == FMT_I8) {
        // lane covers columns 4f..4f+3, f = lane + 32m: block m of 128 columns
        const float* srow = FMT == FMT_FP8 ? (const float*)a.scale + ((size_t)e * H + n) / 128 * (I / 128) : nullptr;
        for (int m = 0; m < I / 128; ++m) {
          const int f = lane + 32 * m;
          const uint32_t wv = *(const uint32_t*)(wrow + 4 * f);
          float w0, w1, w2, w3;
          if (FMT == FMT_FP8)
            e4m3x4(wv, w0, w1, w2, w3);
          else
            dec4_i8(wv, w0, w1, w2, w3);
          const float s = FMT == FMT_FP8 ? __ldg(srow + m) : 1.0f;
#pragma unroll
          for (int j = 0; j < CAP; ++j) {
            if (j < cnt) {
              const float4 x = ((const float4*)(xa + j * I))[f];
              float p = w0 * x.x;
              p = fmaf(w1, x.y, p);
              p = fmaf(w2, x.z, p);
              p = fmaf(w3, x.w, p);
              acc[j] = fmaf(p, s, acc[j]);
            }
          }
        }
      } else {
        // lane covers 8 columns 8u..8u+7, u = lane + 32m (half a 16-column scale group)
        const uint8_t* gsr = stage + RM * rb + r * gb;
        for (int u = lane; u < I / 8; u += 32) {
          const int g = u >> 1;
          const float s = e4m3_to_f32(gsr[g]);
          const uint32_t word = *(const uint32_t*)(wrow + 4 * u);  // nibbles of columns 8u..8u+7
          float wf[8];
          if (FMT == FMT_W4) {
            uint2 l2 = make_uint2(word, 0u);
            dec_w4<8>(l2, s, lut, wf);
          } else {
            const uint32_t hiw = *(const uint16_t*)(wrow + I / 2 + 2 * u);
            dec_w6<8>(make_uint2(word, 0u), hiw, s, wf);
          }
#pragma unroll
          for (int j = 0; j < CAP; ++j) {
            if (j < cnt) {
              const float4 x0 = ((const float4*)(xa + j * I))[2 * u];
              const float4 x1 = ((const float4*)(xa + j * I))[2 * u + 1];
              float p = wf[0] * x0.x;
              p = fmaf(wf[1], x0.y, p);
              p = fmaf(wf[2], x0.z, p);
              p = fmaf(wf[3], x0.w, p);
              p = fmaf(wf[4], x1.x, p);
              p = fmaf(wf[5], x1.y, p);
              p = fmaf(wf[6], x1.z, p);
              p = fmaf(wf[7], x1.w, p);
              acc[j] += p;
            }
          }
        }
      }
      float rscale = 1.0f;
      if (FMT == FMT_I8) rscale = 0.0625f * __ldg((const float*)a.scale + (size_t)e * H + n);
      if (fmt_codes(FMT)) rscale = 0.0625f * __ldg(a.channel + (size_t)e * H + n);
#pragma unroll
      for (int j = 0; j < CAP; ++j) {
        if (j < cnt) {
          float v = warp_sum(acc[j]) * rscale;
          if (lane == 0) dots[pl.sorted[first + j] * RM + r] = v;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
  }
  named_sync(1, DEC_WARPS * 32);
  // routed combine in rank order, as the reference's weighted_sum
  for (int idx = tid; idx < a.M * NR; idx += DEC_WARPS * 32) {
    const int t = idx / NR, r = idx - t * NR;
    float acc = 0.0f;
    for (int j = 0; j < a.k; ++j) acc = __fmaf_rn(dots[(t * a.k + j) * RM + r], a.weights[t * a.k + j], acc);
    a.out[(size_t)t * H + n0 + r] = f32_to_bf16(acc);
  }
}

}  // namespace d3
