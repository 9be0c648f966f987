// One-line decode: drama3/offload.py:108-123 (resident_decode) for one row, as a streaming kernel shaped for that
// case, for e4m3 experts per channel (fp8c) or in the reference's 128 x 128 blocks (fp8), for the reference's int8
// ConvRot rows, and for W4A8 (int4 codes two per byte, bf16 scales per 128 columns, int8 per-row activations). At one line every byte of the pairs' weights
// is used once by one column, so the layer is bound by how early the bytes start to stream and how little waiting
// follows them; the tensor-core decodes (built for 16 lines) spend more on their phase changes than on the bytes.
//
// One CTA per SM: 8 MMA warps and one producer warp. Work:
//   phase 1  the pairs' gate_up rows in units of 4 channels (4 gate + 4 up rows), split evenly over the CTAs in
//            order; two units (16 rows) per MMA tile; SwiGLU to the workspace; each CTA adds the units it finished to
//            its pair's counter (at the pair boundary and at the end).
//   phase 2  split by (pair, row block): CTA b < nv * RB (RB = G / nv) takes pair b / RB and output rows
//            [rb * RR, rb * RR + RR) (RR = ceil(2048 / RB), at most 128: 8 MMA tiles of 16 rows, one a warp); it waits
//            until its pair's counter holds all of the pair's units, reads the pair's SwiGLU row (L2), multiplies its
//            down rows, and writes the fp32 partial; the row block's last CTA to arrive (a counter) sums the pairs'
//            partials in rank order (fp32 fused multiply-adds, as the reference's weighted_sum) and writes bf16.
// One ring of 3 stages of 64 KB carries both phases' weights by per-row bulk copies (one per lane) into padded rows:
// the units (four or eight to a stage: a CTA's whole share fits, so it is all requested at once), then the down rows
// 64 to a stage as the units' stages drain. Measured with no compute, 2 KB copies stream at ~4.2 TB/s aggregate
// through 3 stages of 64 KB per SM, ~3.8 TB/s through 6 of 32 KB and ~3.1 TB/s through 12 of 16 KB; this kernel with
// the down rows prefetched into a region of their own beside a ring of 3 x 32 KB took 18.8 us a layer against 16.1.
//
// e4m3 arithmetic: mma.sync m16n8k32 e4m3 x e4m3 -> f32 with the weights as stored. Activations (the bf16 or fp32
// row, a pair's fp32 SwiGLU row) enter as six e4m3 terms in B's columns: the row is scaled by a power of two that puts
// its largest magnitude in [2^7, 2^8); terms 1-3 are successive roundings to 3 mantissa bits (subnormal steps of 2^-9
// below 2^-6) with exact fp32 residuals; the residual after them is scaled by 2^12 and split the same way into terms
// 4-6, whose columns are scaled back by 2^-12 after the MMA. A bf16 row is exact, an fp32 row keeps ~24 significant
// bits; only magnitudes below 2^-29 of the row's largest are lost. The per-channel scale multiplies the fp32 dot; a
// block scale multiplies the fp32 partial dot of its 128 columns (a warp's phase-1 columns are two blocks, a down
// row's are I / 128), as the reference's block dequantization does before its fp32 sum.
//
// int8 ConvRot arithmetic (the reference's chain: rotate, gemv, rotate(SwiGLU), gemv): the row, and each pair's SwiGLU
// row, rotated per 256 columns in registers (the radix-4 butterfly of the tensor-core int8 decode, tc_rotate16) and
// written as three int8 terms of the rotated row scaled by a power of two that puts its largest magnitude in [32, 64)
// (t1 = rint(y), t2 = rint(128 (y - t1)), t3 = rint(128 (128 (y - t1) - t2)): ~21 significant bits) in B's columns;
// mma.sync m16n8k32 s8 x s8 -> s32 on the int8 rows as stored; D1 + D2 / 128 + D3 / 16384, then the row scale.
//
// W4A8 arithmetic (the format's definition, oracle.moe.gemm_wa8): the row, and each pair's SwiGLU row, quantized to
// int8 by its own max (s = max / 127, q = rint(x / s) clipped, quant_i8_n); mma.sync m16n8k32 s8 x s8 -> s32, exact,
// on the codes expanded in registers: packed byte b (columns 2j, 2j + 1) gives (b << 4) & 0xF0 and b & 0xF0, 16 x
// each signed nibble; in a 32-column chunk the even columns take the MMA's first 16 k slots and the odd ones the
// last 16, and the staged activations follow the same order. Each 128-column group's s32 sum is scaled by its bf16
// group scale into an fp32 sum; the row's s / 16 multiplies the total.
#pragma once

#include "decode_tc.cuh"

namespace d3 {

constexpr int GV_WARPS = 8;                      // MMA warps
constexpr int GV_THREADS = GV_WARPS * 32 + 32;   // + the producer warp
constexpr int GV_MMA_THREADS = GV_WARPS * 32;
constexpr int GV_STAGES = 3;                     // ring stages: four or eight units, or 64 down rows
constexpr int GV_UNIT_CH = 4;                    // channels per unit
constexpr int GV_K = 2048;                       // hidden size (phase-1 K, phase-2 rows)
constexpr int GV_P2_ROWS = 64;                   // down rows per stage
constexpr int GV_MIN_GRID = 128;                 // CTAs needed: 8 pairs x 16 row blocks of at most 128 rows
constexpr int GV_MAX_PAIRS = 8;
constexpr int GV_MAX_TERMS = 6;
constexpr int GV_XPITCH = GV_K + 16;             // bytes per staged activation term (bank-spread)
constexpr float GV_LOW = 1.0f / 4096.0f;         // 2^-12: the second group's weight

// Padded row pitches: a multiple of 16 bytes with an odd number of 16-byte chunks, so the 8 rows an ldmatrix phase
// reads fall in 8 bank groups.
__host__ __device__ constexpr int gv_pitch(int bytes) { return bytes + 16; }

// Per-format layout: bytes per gate_up row and down row, units per ring stage, activation terms (B columns).
template <int FMT>
struct GvFmt {
  static constexpr bool INT4 = false;
  static constexpr bool ROT = false;
  static constexpr bool BLK = FMT == FMT_FP8;  // scales per 128 x 128 block, else per output channel
  static constexpr int ROW1 = GV_K;
  static constexpr int UNITS = 4;
  static constexpr int TERMS = 6;
  __host__ __device__ static constexpr int row2(int I) { return I; }
};
template <>
struct GvFmt<FMT_I8> {
  static constexpr bool INT4 = false;
  static constexpr bool BLK = false;
  static constexpr bool ROT = true;  // ConvRot rows: the activations are rotated and split into int8 terms
  static constexpr int ROW1 = GV_K;
  static constexpr int UNITS = 4;
  static constexpr int TERMS = 3;
  __host__ __device__ static constexpr int row2(int I) { return I; }
};
template <>
struct GvFmt<FMT_W4A8> {
  static constexpr bool ROT = false;
  static constexpr bool INT4 = true;
  static constexpr bool BLK = false;
  static constexpr int ROW1 = GV_K / 2;
  static constexpr int UNITS = 8;
  static constexpr int TERMS = 1;
  __host__ __device__ static constexpr int row2(int I) { return I / 2; }
};

// Shared memory of one format: the ring (stages of UNITS units of padded rows), the activation terms or codes, the
// pair's SwiGLU row, the warps' partial sums (16 rows a tile), the mbarriers. (One layout for all formats, sized for
// the largest, measured 4-5 % slower for the e4m3 formats.)
template <int FMT>
struct GvSmem {
  static constexpr int stage = GvFmt<FMT>::UNITS * 8 * gv_pitch(GvFmt<FMT>::ROW1);
  static constexpr int red_rows = GvFmt<FMT>::UNITS * 8;  // a stage's rows: 16 a tile, UNITS / 2 tiles
  static constexpr int ring = 0;
  static constexpr int xt = ring + GV_STAGES * stage;
  static constexpr int ht = xt + GvFmt<FMT>::TERMS * GV_XPITCH;
  __host__ __device__ static constexpr int red(int I) { return ht + GvFmt<FMT>::TERMS * gv_pitch(I); }
  __host__ __device__ static constexpr int bars(int I) { return red(I) + 2 * GV_WARPS * red_rows * 4; }
  __host__ __device__ static constexpr int total(int I) { return bars(I) + 8 * 2 * GV_STAGES + 128; }
  static_assert(GV_P2_ROWS * gv_pitch(GvFmt<FMT>::row2(768)) <= stage, "64 down rows fit one stage");
};

D3_DEV void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

D3_DEV void mma_e4m3_16832(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

D3_DEV void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// acc += 16 e4m3 rows (rows 0-7 at `lo`, 8-15 at `hi`, pitch `pitch` bytes) x the activation terms at `xt` (term t at
// xt + t * xpitch bytes in B column t; columns 6 and 7 are zero), over 32 columns from kb.
D3_DEV void gv_mma32(float (&acc)[4], const uint8_t* lo, const uint8_t* hi, int pitch, const uint8_t* xt, int xpitch,
                     int kb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  uint32_t w[4];
  ldsm_x4(w, ((lane >> 3) & 1 ? hi : lo) + (lane & 7) * pitch + kb + 16 * (lane >> 4));
  uint32_t b0 = 0u, b1 = 0u;
  if (g < GV_MAX_TERMS) {
    const uint8_t* xr = xt + g * xpitch + kb + 4 * c;
    b0 = *reinterpret_cast<const uint32_t*>(xr);
    b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
  }
  mma_e4m3_16832(acc, w, b0, b1);
}

// acc += 16 packed int4 rows (rows 0-7 at `lo`, 8-15 at `hi`, pitch `pitch` bytes) x the int8 activations at `xq`
// (B column 0, chunk order: even columns, then odd), over 64 columns from kb (two MMAs).
D3_DEV void gv_mma64_i4(int (&acc)[4], const uint8_t* lo, const uint8_t* hi, int pitch, const uint8_t* xq, int kb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  uint32_t w[4];
  ldsm_x4(w, ((lane >> 3) & 1 ? hi : lo) + (lane & 7) * pitch + kb / 2 + 16 * (lane >> 4));
  uint32_t b[4] = {0u, 0u, 0u, 0u};
  if (g == 0) {
#pragma unroll
    for (int h = 0; h < 4; ++h) b[h] = *reinterpret_cast<const uint32_t*>(xq + kb + 16 * h + 4 * c);
  }
  // w[0], w[1]: rows g, g + 8 of columns kb..kb+31; w[2], w[3]: of kb+32..kb+63
  mma_s8_16832(acc, (w[0] << 4) & 0xF0F0F0F0u, (w[1] << 4) & 0xF0F0F0F0u, w[0] & 0xF0F0F0F0u, w[1] & 0xF0F0F0F0u,
               b[0], b[1]);
  mma_s8_16832(acc, (w[2] << 4) & 0xF0F0F0F0u, (w[3] << 4) & 0xF0F0F0F0u, w[2] & 0xF0F0F0F0u, w[3] & 0xF0F0F0F0u,
               b[2], b[3]);
}

// acc += 16 int8 rows (rows 0-7 at `lo`, 8-15 at `hi`, pitch `pitch` bytes) x the three int8 activation terms at
// `xt` (term t at xt + t * xpitch in B column t), over 32 columns from kb.
D3_DEV void gv_mma32_i8(int (&acc)[4], const uint8_t* lo, const uint8_t* hi, int pitch, const uint8_t* xt, int xpitch,
                        int kb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  uint32_t w[4];
  ldsm_x4(w, ((lane >> 3) & 1 ? hi : lo) + (lane & 7) * pitch + kb + 16 * (lane >> 4));
  uint32_t b0 = 0u, b1 = 0u;
  if (g < 3) {
    const uint8_t* xr = xt + g * xpitch + kb + 4 * c;
    b0 = *reinterpret_cast<const uint32_t*>(xr);
    b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
  }
  mma_s8_16832(acc, w[0], w[1], w[2], w[3], b0, b1);
}

// The rows g and g + 8 of the three-term int8 sums (this lane's quad): D1 + D2 / 128 + D3 / 16384, every lane of the
// quad gets the same values.
D3_DEV void gv_i8_term_sums(const int (&acc)[4], float& r_lo, float& r_hi) {
  const int c = threadIdx.x & 3;
  // lane c holds columns 2c, 2c + 1: c = 0 has D1, D2; c = 1 has D3
  float a = c == 0 ? (float)acc[0] + (float)acc[1] * 0.0078125f : c == 1 ? (float)acc[0] * 6.103515625e-05f : 0.0f;
  float b = c == 0 ? (float)acc[2] + (float)acc[3] * 0.0078125f : c == 1 ? (float)acc[2] * 6.103515625e-05f : 0.0f;
  a += __shfl_xor_sync(0xffffffffu, a, 1);
  b += __shfl_xor_sync(0xffffffffu, b, 1);
  a += __shfl_xor_sync(0xffffffffu, a, 2);
  b += __shfl_xor_sync(0xffffffffu, b, 2);
  r_lo = a;
  r_hi = b;
}

// 16 values of a row (rotated, |v * scale| < 64) as three int8 terms, 16 bytes each into dst[t * pitch].
D3_DEV void gv_i8_terms16(const float (&v)[16], float scale, uint8_t* dst, int pitch) {
  uint32_t w[3][4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    w[0][p] = w[1][p] = w[2][p] = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float r = v[4 * p + i] * scale;
#pragma unroll
      for (int t = 0; t < 3; ++t) {
        const float q8 = fminf(127.0f, fmaxf(-127.0f, rintf(r)));
        w[t][p] |= ((uint32_t)(int)q8 & 0xFFu) << (8 * i);
        r = (r - q8) * 128.0f;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 3; ++t) *reinterpret_cast<uint4*>(dst + t * pitch) = make_uint4(w[t][0], w[t][1], w[t][2], w[t][3]);
}

// Byte position of column j (0..31) of a 32-column chunk in the W4A8 activation order: even columns first.
D3_DEV int gv_i4_pos(int j) { return 16 * (j & 1) + 4 * (j >> 3) + ((j >> 1) & 3); }

// The dot products of C rows g and g + 8 (this lane's quad): columns 0-2 at weight 1, 3-5 at 2^-12, summed over the
// quad; every lane of the quad gets the same sums.
D3_DEV void gv_term_sums(const float (&acc)[4], float& r_lo, float& r_hi) {
  const int c = threadIdx.x & 3;
  // lane c holds columns 2c, 2c + 1
  const float w0 = c < 2 ? 1.0f : GV_LOW;
  const float w1 = c == 0 ? 1.0f : GV_LOW;
  const bool live = c < 3;
  float a = live ? acc[0] * w0 + acc[1] * w1 : 0.0f;
  float b = live ? acc[2] * w0 + acc[3] * w1 : 0.0f;
  a += __shfl_xor_sync(0xffffffffu, a, 1);
  b += __shfl_xor_sync(0xffffffffu, b, 1);
  a += __shfl_xor_sync(0xffffffffu, a, 2);
  b += __shfl_xor_sync(0xffffffffu, b, 2);
  r_lo = a;
  r_hi = b;
}

// The power of two s with max * 2^s in [2^7, 2^8) (0 for max 0).
D3_DEV int gv_scale_exp(float m) {
  if (!(m > 0.0f)) return 0;
  const int be = (__float_as_int(m) >> 23) & 255;  // biased exponent (0: subnormal, treated as 2^-126)
  const int e = max(be, 1) - 127;                  // m in [2^e, 2^(e+1))
  return min(127, max(-126, 7 - e));
}
D3_DEV float gv_pow2(int s) { return __int_as_float((127 + s) << 23); }

// The e4m3 byte of t, a value exactly representable in e4m3 (from gv_round3).
D3_DEV uint32_t gv_e4m3_byte(float t) {
  const uint32_t bits = __float_as_uint(t);
  const uint32_t sign = (bits >> 24) & 0x80u;
  const float a = fabsf(t);
  if (a >= 0.015625f) return sign | ((((bits >> 23) & 255u) - 120u) << 3) | ((bits >> 20) & 7u);
  return sign | (uint32_t)(a * 512.0f);
}

// t = y rounded to 3 mantissa bits (to a multiple of 2^-9 below 2^-6): an e4m3 value (|y| < 2^8.5 here).
D3_DEV float gv_round3(float y) {
  if (fabsf(y) >= 0.015625f) return __int_as_float((__float_as_int(y) + 0x80000) & (int)0xFFF00000);
  return rintf(y * 512.0f) * (1.0f / 512.0f);
}

// The six e4m3 terms of v * scale, one byte each into dst[t * pitch].
D3_DEV void gv_terms(float v, float scale, uint8_t* dst, int pitch) {
  float y = v * scale;
#pragma unroll
  for (int grp = 0; grp < 2; ++grp) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const float t = gv_round3(y);
      dst[(3 * grp + i) * pitch] = (uint8_t)gv_e4m3_byte(t);
      y -= t;
    }
    y *= 4096.0f;
  }
}

// Spin (bounded) until *p >= target; acquire. False and the fault word set on timeout.
D3_DEV bool gv_wait_at_least(const unsigned* p, unsigned target) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  if (v >= target) return true;
  const unsigned long long start = globaltimer();
  while (true) {
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    if (globaltimer() - start > WAIT_LIMIT_NS) {
      record_fault(FAULT_WAIT_TIMEOUT);
      return false;
    }
  }
}

// The max |v| over the MMA warps (named barrier 1, `slots` of GV_WARPS floats), every thread's copy.
D3_DEV float gv_block_max(float m, float* slots) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) slots[threadIdx.x >> 5] = m;
  named_sync(1, GV_MMA_THREADS);
  m = slots[0];
#pragma unroll
  for (int w = 1; w < GV_WARPS; ++w) m = fmaxf(m, slots[w]);
  return m;
}

// A weight row's scale for 128-column group `grp`: 1 for per-channel scales (applied after the sum), the block's
// (fp8) or the row's bf16 group scale (W4A8). `row` is the bank row, `groups` the row's groups.
template <int FMT>
D3_DEV float gv_group_scale(const void* scale, size_t row, int groups, int grp) {
  if constexpr (GvFmt<FMT>::INT4) return bf16_to_f32(__ldg((const uint16_t*)scale + row * groups + grp));
  else if constexpr (GvFmt<FMT>::BLK) return __ldg((const float*)scale + row / 128 * groups + grp);
  else return 1.0f;
}

// Synchronization words (zero between calls; every call leaves them zero): a.depart[32 q] counts pair q's finished
// units, a.depart[32 q + 16] its consumers that have passed the wait; a.arrive[rb] counts row block rb's pairs done.
template <int FMT, int I>
__global__ void __launch_bounds__(GV_THREADS, 1) moe_decode_gv_kernel(const DecodeArgs a) {
  using F = GvFmt<FMT>;
  constexpr bool INT4 = F::INT4, ROT = F::ROT, GRP = F::INT4 || F::BLK;  // GRP: scales per 128-column group
  using S = GvSmem<FMT>;
  constexpr int UNITS = F::UNITS, TPS = UNITS / 2;       // units and 16-row tiles per stage
  constexpr int STAGE = S::stage, RED = S::red_rows;
  constexpr int ROW1 = F::ROW1, ROW2 = F::row2(I);
  constexpr int P1 = gv_pitch(ROW1), P2 = gv_pitch(ROW2), HTP = gv_pitch(I);
  constexpr int UPP = I / GV_UNIT_CH;  // units per pair
  constexpr int HPT = (I + GV_MMA_THREADS - 1) / GV_MMA_THREADS;
  constexpr int G1 = GV_K / 128, G2 = I / 128;  // 128-column groups of a gate_up row and of a down row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
  uint8_t* ring = smem + S::ring;
  uint8_t* xt = smem + S::xt;   // the row's terms [TERMS][GV_XPITCH], or its int8 codes (W4A8)
  uint8_t* ht = smem + S::ht;   // the pair's SwiGLU row: [TERMS][HTP] terms, or int8 codes (W4A8)
  float* red = (float*)(smem + S::red(I));  // [2][GV_WARPS][RED]
  uint64_t* bars = (uint64_t*)(smem + S::bars(I));
  uint64_t* full = bars;
  uint64_t* empty = bars + GV_STAGES;
  __shared__ float s_max[GV_WARPS];
  __shared__ int s_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, b = blockIdx.x;
  D3_GSTAMP(0);
  if (tid == 0) {
    for (int s = 0; s < GV_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, GV_WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();
  allow_dependents();
  grid_dependency_wait();
  D3_GSTAMP(1);

  // the plan, computed alike by every thread: valid pairs in rank order and their experts; the unit split; this
  // CTA's phase-2 share
  const int k = a.k;
  long long idv[GV_MAX_PAIRS];
#pragma unroll
  for (int j = 0; j < GV_MAX_PAIRS; ++j) idv[j] = j < k ? a.ids[j] : -1;
  int e_of[GV_MAX_PAIRS], v_of[GV_MAX_PAIRS];
  int nv = 0;
#pragma unroll
  for (int j = 0; j < GV_MAX_PAIRS; ++j) {
    v_of[j] = -1;
    e_of[j] = 0;
    if (j < k) {
      if (idv[j] >= 0 && idv[j] < a.E) {
        v_of[j] = nv;
        e_of[nv] = (int)idv[j];
        ++nv;
      } else if (tid == 0 && b == 0) {
        record_fault(FAULT_BAD_EXPERT);
      }
    }
  }
  if (nv == 0) {  // nothing routed: zeros
    const int z0 = (int)((long long)b * GV_K / G), z1 = (int)((long long)(b + 1) * GV_K / G);
    for (int r = z0 + tid; r < z1; r += blockDim.x) a.out[r] = 0;
    return;
  }
  const int T1 = nv * UPP;
  const int u_lo = (int)((long long)b * T1 / G), u_hi = (int)((long long)(b + 1) * T1 / G);
  const int n1 = u_hi - u_lo;
  const int RB = G / nv, RR = (GV_K + RB - 1) / RB, NRB = (GV_K + RR - 1) / RR;
  const bool p2_live = b < nv * RB && (b % RB) < NRB;
  const int q2 = b / RB, rb = b % RB;
  const int r0 = rb * RR, rows2 = p2_live ? min(GV_K, r0 + RR) - r0 : 0;
  const int nt2 = (rows2 + 15) / 16;                           // down tiles of 16 rows, one a warp
  const int n1s = (n1 + UNITS - 1) / UNITS;                    // unit stages
  const int items = n1s + (rows2 + GV_P2_ROWS - 1) / GV_P2_ROWS;  // + down-row stages
  unsigned* done = a.depart;       // [32 q]: pair q's finished units; [32 q + 16]: its consumers past the wait
  unsigned* block_cnt = a.arrive;  // [rb]: row block rb's pairs done

  if (warp == GV_WARPS) {
    // producer: item i (UNITS units, or 64 down rows) into stage i % GV_STAGES, one row copy a lane
    const uint64_t pol = policy_evict_first();
    for (int i = 0; i < items; ++i) {
      const int s = i % GV_STAGES;
      if (i >= GV_STAGES && !mbar_wait(empty + s, ((i / GV_STAGES) - 1) & 1)) break;
      uint8_t* dst = ring + s * STAGE;
      if (i < n1s) {
        const int units = min(UNITS, n1 - UNITS * i);
        if (lane == 0) mbar_arrive_expect_tx(full + s, (uint32_t)(units * 8 * ROW1));
        __syncwarp();
#pragma unroll
        for (int h = 0; h < UNITS / 4; ++h) {  // 32 rows a pass
          const int r = 32 * h + lane;
          if (r < units * 8) {
            const int u = u_lo + UNITS * i + (r >> 3), v = u / UPP;
            const int ch = (u - v * UPP) * GV_UNIT_CH + (r & 3);
            const int row = e_of[v] * 2 * I + ((r & 7) < 4 ? ch : I + ch);
            bulk_g2s(dst + r * P1, a.w13 + (size_t)row * ROW1, ROW1, full + s, pol);
          }
        }
      } else {
        const int m0 = GV_P2_ROWS * (i - n1s), rows = min(GV_P2_ROWS, rows2 - m0);
        if (lane == 0) mbar_arrive_expect_tx(full + s, (uint32_t)(rows * ROW2));
        __syncwarp();
        for (int r = lane; r < rows; r += 32)
          bulk_g2s(dst + r * P2, a.w2 + ((size_t)e_of[q2] * GV_K + r0 + m0 + r) * ROW2, ROW2, full + s, pol);
      }
    }
    return;
  }

  // ---- MMA warps: the row as terms (e4m3, rotated int8) or int8 codes (W4A8); xmul undoes the row's scaling
  float xmul;
  if constexpr (ROT) {
    // warps 0-3 rotate the row's 8 groups of 256 (a 16-lane half each, 16 contiguous columns a lane)
    float v16[16];
    const int col0 = 256 * (2 * warp + (lane >> 4)) + 16 * (lane & 15);
#pragma unroll
    for (int i = 0; i < 16; ++i) v16[i] = 0.0f;
    if (warp < 4) {
      tc_load16(a.x, a.x_bf16 != 0, col0, v16);
      tc_rotate16(v16);
    }
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v16[i]));
    m = gv_block_max(m, s_max);
    const int e = tc_exponent_i8(m);
    xmul = gv_pow2(-e);
    if (warp < 4) gv_i8_terms16(v16, gv_pow2(e), xt + col0, GV_XPITCH);
    named_sync(1, GV_MMA_THREADS);
  } else {
    float v[8];
    const int c0 = 8 * tid;
    if (a.x_bf16) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>((const uint16_t*)a.x + c0));
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = bf16_to_f32(w4[i] & 0xFFFFu);
        v[2 * i + 1] = bf16_to_f32(w4[i] >> 16);
      }
    } else {
      const float4 p = __ldg(reinterpret_cast<const float4*>((const float*)a.x + c0));
      const float4 q = __ldg(reinterpret_cast<const float4*>((const float*)a.x + c0) + 1);
      v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w; v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    }
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
    m = gv_block_max(m, s_max);
    if constexpr (INT4) {
      // int8 codes, even columns of each 32-column chunk first: this thread's 8 columns are 4 even ones (bytes
      // 4cc..4cc+3 of the chunk) and 4 odd ones (16 + 4cc..)
      const float sq = m / 127.0f;
      float q[8];
      quant_i8_n<8>(v, sq, __frcp_rn(sq), q);
      uint32_t ev = 0, od = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ev |= ((uint32_t)(int)q[2 * i] & 0xFFu) << (8 * i);
        od |= ((uint32_t)(int)q[2 * i + 1] & 0xFFu) << (8 * i);
      }
      uint8_t* chunk = xt + (c0 & ~31);
      *reinterpret_cast<uint32_t*>(chunk + 4 * ((c0 & 31) >> 3)) = ev;
      *reinterpret_cast<uint32_t*>(chunk + 16 + 4 * ((c0 & 31) >> 3)) = od;
      xmul = sq * (1.0f / 16.0f);
    } else {
      const int sx = gv_scale_exp(m);
      xmul = gv_pow2(-sx);
      const float scale = gv_pow2(sx);
#pragma unroll
      for (int i = 0; i < 8; ++i) gv_terms(v[i], scale, xt + c0 + i, GV_XPITCH);
    }
    named_sync(1, GV_MMA_THREADS);
  }

  // ---- phase 1: gate | up dots of this CTA's units, a stage (TPS 16-row tiles) at a time, SwiGLU, to the workspace
  bool ok = true;
  const int kw = warp * (GV_K / GV_WARPS);  // this warp's 256 columns: groups kw / 128 and kw / 128 + 1
  int cur_pair = -1, cur_units = 0;  // warp 0, lane 0: units finished and not yet added to their pair's counter
  for (int i = 0; i < n1s; ++i) {
    const int s = i % GV_STAGES;
    const int units = min(UNITS, n1 - UNITS * i);
    // the SwiGLU threads' per-channel scales (thread t < 4 * UNITS: unit t / 4, channel t % 4), loaded while the
    // stage lands
    const int su = u_lo + UNITS * i + (tid >> 2);
    const bool swi = tid < 4 * units;
    float sg = 1.0f, sup = 1.0f;
    int sv = 0, sch = 0;
    if (swi) {
      sv = su / UPP;
      sch = (su - sv * UPP) * GV_UNIT_CH + (tid & 3);
      if constexpr (!GRP) {
        const float* sc = (const float*)a.s13 + (size_t)e_of[sv] * 2 * I;
        sg = __ldg(sc + sch);
        sup = __ldg(sc + I + sch);
      }
    }
    // group scales: this lane's rows (g of the tile's two units) over the warp's two column groups
    float gs[TPS][2][2];  // [tile][row g / g + 8][group]
#pragma unroll
    for (int tl = 0; tl < TPS; ++tl)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        gs[tl][hr][0] = gs[tl][hr][1] = 0.0f;
        const int uu = UNITS * i + 2 * tl + hr;
        if (GRP && uu < n1) {
          const int g = lane >> 2, u = u_lo + uu, v = u / UPP, ch = (u - v * UPP) * GV_UNIT_CH + (g & 3);
          const size_t row = (size_t)e_of[v] * 2 * I + (g < 4 ? ch : I + ch);
          gs[tl][hr][0] = gv_group_scale<FMT>(a.s13, row, G1, kw / 128);
          gs[tl][hr][1] = gv_group_scale<FMT>(a.s13, row, G1, kw / 128 + 1);
        }
      }
    ok = mbar_wait(full + s, (i / GV_STAGES) & 1) && ok;
    if (i == 0) D3_GSTAMP(2);
    const uint8_t* st = ring + s * STAGE;
    float r_lo[TPS], r_hi[TPS];
    if constexpr (INT4) {
      int acc[TPS][2][4] = {};  // [tile][group]
      if (ok) {
#pragma unroll
        for (int kb = 0; kb < GV_K / GV_WARPS; kb += 64)
#pragma unroll
          for (int tl = 0; tl < TPS; ++tl)
            if (2 * tl < units) {
              const uint8_t* lo = st + 16 * tl * P1;
              gv_mma64_i4(acc[tl][kb >> 7], lo, lo + 8 * P1, P1, xt, kw + kb);
            }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);  // the stage's bytes are in registers: hand it back before the sums
#pragma unroll
      for (int tl = 0; tl < TPS; ++tl) {
        r_lo[tl] = (float)acc[tl][0][0] * gs[tl][0][0] + (float)acc[tl][1][0] * gs[tl][0][1];
        r_hi[tl] = (float)acc[tl][0][2] * gs[tl][1][0] + (float)acc[tl][1][2] * gs[tl][1][1];
      }
    } else if constexpr (ROT) {
      int acc[TPS][2][4] = {};  // [tile][chain]
      if (ok) {
#pragma unroll
        for (int kb = 0; kb < GV_K / GV_WARPS; kb += 64)
#pragma unroll
          for (int tl = 0; tl < TPS; ++tl)
            if (2 * tl < units) {
              const uint8_t* lo = st + 16 * tl * P1;
              gv_mma32_i8(acc[tl][0], lo, lo + 8 * P1, P1, xt, GV_XPITCH, kw + kb);
              gv_mma32_i8(acc[tl][1], lo, lo + 8 * P1, P1, xt, GV_XPITCH, kw + kb + 32);
            }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);  // the stage's bytes are in registers: hand it back before the sums
#pragma unroll
      for (int tl = 0; tl < TPS; ++tl) {
        int t4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) t4[e] = acc[tl][0][e] + acc[tl][1][e];
        gv_i8_term_sums(t4, r_lo[tl], r_hi[tl]);
      }
    } else {
      float acc[TPS][2][2][4] = {};  // [tile][column group][chain]
      if (ok) {
#pragma unroll
        for (int kb = 0; kb < GV_K / GV_WARPS; kb += 64)
#pragma unroll
          for (int tl = 0; tl < TPS; ++tl)
            if (2 * tl < units) {
              const uint8_t* lo = st + 16 * tl * P1;
              gv_mma32(acc[tl][kb >> 7][0], lo, lo + 8 * P1, P1, xt, GV_XPITCH, kw + kb);
              gv_mma32(acc[tl][kb >> 7][1], lo, lo + 8 * P1, P1, xt, GV_XPITCH, kw + kb + 32);
            }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);  // the stage's bytes are in registers: hand it back before the sums
#pragma unroll
      for (int tl = 0; tl < TPS; ++tl) {
        if constexpr (GRP) {
          r_lo[tl] = r_hi[tl] = 0.0f;
#pragma unroll
          for (int blk = 0; blk < 2; ++blk) {
            float t4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) t4[e] = acc[tl][blk][0][e] + acc[tl][blk][1][e];
            float d_lo, d_hi;
            gv_term_sums(t4, d_lo, d_hi);
            r_lo[tl] += d_lo * gs[tl][0][blk];
            r_hi[tl] += d_hi * gs[tl][1][blk];
          }
        } else {
          float t4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            t4[e] = (acc[tl][0][0][e] + acc[tl][0][1][e]) + (acc[tl][1][0][e] + acc[tl][1][1][e]);
          gv_term_sums(t4, r_lo[tl], r_hi[tl]);
        }
      }
    }
    float* rbuf = red + (i & 1) * GV_WARPS * RED;
    if ((lane & 3) == 0)
#pragma unroll
      for (int tl = 0; tl < TPS; ++tl) {
        rbuf[warp * RED + 16 * tl + (lane >> 2)] = r_lo[tl];
        rbuf[warp * RED + 16 * tl + (lane >> 2) + 8] = r_hi[tl];
      }
    named_sync(1, GV_MMA_THREADS);
    if (warp == 0) {
      if (swi) {
        const int row = (tid >> 2) * 8 + (tid & 3);
        float g = 0.0f, u = 0.0f;
#pragma unroll
        for (int w = 0; w < GV_WARPS; ++w) {
          g += rbuf[w * RED + row];
          u += rbuf[w * RED + row + 4];
        }
        g = g * xmul * sg;
        u = u * xmul * sup;
        a.a1[(size_t)sv * I + sch] = g / (1.0f + expf(-g)) * u;
      }
      __syncwarp();
      if (lane == 0) {
        // this stage's units, counted per pair; a pair's count goes out when the next pair starts and at the end
        for (int h = 0; h < units; ++h) {
          const int p = (u_lo + UNITS * i + h) / UPP;
          if (p != cur_pair) {
            if (cur_units) {
              __threadfence();
              atomicAdd(done + 32 * cur_pair, (unsigned)cur_units);
            }
            cur_pair = p;
            cur_units = 0;
          }
          ++cur_units;
        }
        if (i == n1s - 1 && cur_units) {
          __threadfence();
          atomicAdd(done + 32 * cur_pair, (unsigned)cur_units);
        }
      }
    }
  }
  D3_GSTAMP(3);
  if (!p2_live) return;

  // ---- phase 2: wait for the pair's units, then its SwiGLU row as terms or codes
  if (tid == 0) {
    const int pass = gv_wait_at_least(done + 32 * q2, (unsigned)UPP) ? 1 : 0;
    // the last consumer of the pair past the wait clears both of the pair's words for the next call
    if (atomicAdd(done + 32 * q2 + 16, 1u) == (unsigned)(NRB - 1)) {
      done[32 * q2] = 0u;
      done[32 * q2 + 16] = 0u;
    }
    s_flag = pass;
  }
  named_sync(1, GV_MMA_THREADS);
  ok = ok && s_flag != 0;
  D3_GSTAMP(4);
  // the pair's SwiGLU row: HPT strided values a thread, or (rotated int8) 16 contiguous values a lane of the warps
  // holding its groups of 256
  float hv[ROT ? 16 : HPT];
  float m = 0.0f;
  const int hcol0 = 256 * (2 * warp + (lane >> 4)) + 16 * (lane & 15);
  if constexpr (ROT) {
#pragma unroll
    for (int i = 0; i < 16; ++i) hv[i] = 0.0f;
    if (2 * warp < I / 256) {  // warp-uniform: whole warps rotate (a half past the row's groups holds zeros)
      if (hcol0 < I) tc_load16(a.a1 + (size_t)q2 * I, false, hcol0, (float(&)[16])hv);
      tc_rotate16((float(&)[16])hv);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(hv[i]));
  } else {
#pragma unroll
    for (int i = 0; i < HPT; ++i) {
      const int col = tid + i * GV_MMA_THREADS;
      hv[i] = col < I ? __ldcg(a.a1 + (size_t)q2 * I + col) : 0.0f;
      m = fmaxf(m, fabsf(hv[i]));
    }
  }
  // this thread's down scales for its tile rows (per channel, or per 128-column group), loaded while the row lands
  const int row_lo = r0 + 16 * warp + (lane >> 2), row_hi = row_lo + 8;
  const bool live_lo = 16 * warp + (lane >> 2) < rows2, live_hi = 16 * warp + (lane >> 2) + 8 < rows2;
  float sc_lo[GRP ? G2 : 1], sc_hi[GRP ? G2 : 1];
  {
    const size_t blo = (size_t)e_of[q2] * GV_K + row_lo, bhi = (size_t)e_of[q2] * GV_K + row_hi;
    if constexpr (GRP) {
#pragma unroll
      for (int grp = 0; grp < G2; ++grp) {
        sc_lo[grp] = live_lo ? gv_group_scale<FMT>(a.s2, blo, G2, grp) : 0.0f;
        sc_hi[grp] = live_hi ? gv_group_scale<FMT>(a.s2, bhi, G2, grp) : 0.0f;
      }
    } else {
      sc_lo[0] = live_lo ? __ldg((const float*)a.s2 + blo) : 0.0f;
      sc_hi[0] = live_hi ? __ldg((const float*)a.s2 + bhi) : 0.0f;
    }
  }
  m = gv_block_max(m, s_max);  // s_max's phase-1 readers all passed the barriers since
  float hmul;
  if constexpr (ROT) {
    const int e = tc_exponent_i8(m);
    hmul = gv_pow2(-e);
    if (2 * warp < I / 256 && hcol0 < I) gv_i8_terms16((float(&)[16])hv, gv_pow2(e), ht + hcol0, HTP);
  } else if constexpr (INT4) {
    const float sq = m / 127.0f;
    float q[HPT];
    quant_i8_n<HPT>(hv, sq, __frcp_rn(sq), q);
#pragma unroll
    for (int i = 0; i < HPT; ++i) {
      const int col = tid + i * GV_MMA_THREADS;
      if (col < I) ht[(col & ~31) + gv_i4_pos(col & 31)] = (uint8_t)(int)q[i];
    }
    hmul = sq * (1.0f / 16.0f);
  } else {
    const int sh = gv_scale_exp(m);
    const float hscale = gv_pow2(sh);
    hmul = gv_pow2(-sh);
#pragma unroll
    for (int i = 0; i < HPT; ++i) {
      const int col = tid + i * GV_MMA_THREADS;
      if (col < I) gv_terms(hv[i], hscale, ht + col, HTP);
    }
  }
  named_sync(1, GV_MMA_THREADS);
  D3_GSTAMP(5);
  // warp w: down tile w (rows 16 w .. 16 w + 15 of this block), in stage item n1s + w / 4
  if (warp < nt2) {
    const int item = n1s + warp / (GV_P2_ROWS / 16), s = item % GV_STAGES;
    ok = mbar_wait(full + s, (item / GV_STAGES) & 1) && ok;
    const uint8_t* rows = ring + s * STAGE + (warp % (GV_P2_ROWS / 16)) * 16 * P2;
    float r_lo = 0.0f, r_hi = 0.0f;
    if constexpr (INT4) {
      // one 128-column group at a time: two MMA pairs, then its group scales
#pragma unroll
      for (int kb = 0; kb < I; kb += 128) {
        int acc[4] = {0, 0, 0, 0};
        if (ok) {
          gv_mma64_i4(acc, rows, rows + 8 * P2, P2, ht, kb);
          gv_mma64_i4(acc, rows, rows + 8 * P2, P2, ht, kb + 64);
        }
        r_lo += (float)acc[0] * sc_lo[kb / 128];
        r_hi += (float)acc[2] * sc_hi[kb / 128];
      }
    } else if constexpr (ROT) {
      int acc[4][4] = {};
      if (ok) {
#pragma unroll
        for (int kb = 0; kb < I; kb += 128)
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) gv_mma32_i8(acc[c4], rows, rows + 8 * P2, P2, ht, HTP, kb + 32 * c4);
      }
      int t4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) t4[e] = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
      gv_i8_term_sums(t4, r_lo, r_hi);
      r_lo *= sc_lo[0];
      r_hi *= sc_hi[0];
    } else {
      // four chains over the row's columns; with block scales, their term sums fold per column block (128)
      float acc[4][4] = {};
#pragma unroll
      for (int kb = 0; kb < I; kb += 128) {
        if (ok) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) gv_mma32(acc[c4], rows, rows + 8 * P2, P2, ht, HTP, kb + 32 * c4);
        }
        if constexpr (GRP) {
          float t4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) t4[e] = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
          float d_lo, d_hi;
          gv_term_sums(t4, d_lo, d_hi);
          r_lo += d_lo * sc_lo[kb / 128];
          r_hi += d_hi * sc_hi[kb / 128];
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) acc[c4][0] = acc[c4][1] = acc[c4][2] = acc[c4][3] = 0.0f;
        }
      }
      if constexpr (!GRP) {
        float t4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) t4[e] = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
        gv_term_sums(t4, r_lo, r_hi);
        r_lo *= sc_lo[0];
        r_hi *= sc_hi[0];
      }
    }
    if ((lane & 3) == 0) {
      float* part = a.parts + (size_t)q2 * GV_K;
      if (live_lo) part[row_lo] = r_lo * hmul;
      if (live_hi) part[row_hi] = r_hi * hmul;
    }
  }
  named_sync(1, GV_MMA_THREADS);
  D3_GSTAMP(6);
  // the row block's last CTA to finish combines the pairs in rank order
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(block_cnt + rb, 1u);
    const int last = prev == (unsigned)(nv - 1);
    if (last) {
      block_cnt[rb] = 0u;
      __threadfence();
    }
    s_flag = last;
  }
  named_sync(1, GV_MMA_THREADS);
  if (s_flag && tid < rows2) {
    float wj[GV_MAX_PAIRS], pj[GV_MAX_PAIRS];
#pragma unroll
    for (int j = 0; j < GV_MAX_PAIRS; ++j) {
      const int q = v_of[j];
      wj[j] = q >= 0 ? __ldg(a.weights + j) : 0.0f;
      pj[j] = q >= 0 ? __ldcg(a.parts + (size_t)q * GV_K + r0 + tid) : 0.0f;
    }
    float accum = 0.0f;
#pragma unroll
    for (int j = 0; j < GV_MAX_PAIRS; ++j)
      if (v_of[j] >= 0) accum = __fmaf_rn(pj[j], wj[j], accum);
    a.out[r0 + tid] = f32_to_bf16(accum);
  }
  D3_GSTAMP(7);
}

}  // namespace d3
