// Expert weight formats (the reference's layouts) and their in-register decoding.
//
//   FP8  e4m3 rows [E*N, K], fp32 128x128 block scales [E*N/128, K/128] (drama3/offload.py:755-766)
//   I8   int8 ConvRot rows [E*N, K], fp32 row scales [E*N] (tools/convert.py:48-53)
//   W4   4-bit codes [E*N, K/2] (low nibble = even column), e4m3 group-16 scales [E*N, K/16], fp32 s_channel,
//        a 16-entry float codebook: weight = clamp(rint(codebook[c] * scale), +-127) (drama3/kernels.py:469-483)
//   W6   nibble plane [K/2] then 2-bit high plane [K/4] per row: weight = clamp(rint((c - 32) * scale), +-127)
// and the BASELINE layouts (BASELINE.json configs[1..3]; no reference implementation):
//   FP8C e4m3 rows [E*N, K], fp32 per-output-channel scales [E*N]
//   W4A8 int4 (-7..7) two per byte, low nibble = even column; bf16 group-128 scales [E*N, K/128]
//   W6A8 int6 (-31..31) four per three bytes (24-bit little-endian words); bf16 group-128 scales
//   (A8: the activations are quantized to int8 per row, absmax / 127, before every GEMV)
//
// Conversions avoid the slow converter paths measured on B200 (int8 -> float through I2F runs at about 16 per clock
// per SM): e4m3 pairs go to f16 pairs with one cvt (every e4m3 value is an f16), int8 goes to f32 by placing the
// byte in a float's mantissa (byte_perm) and one subtraction, both exact.
#pragma once

#include "common.cuh"

namespace d3 {

enum { FMT_FP8 = 0, FMT_I8 = 1, FMT_W4 = 2, FMT_W6 = 3, FMT_FP8C = 4, FMT_W4A8 = 5, FMT_W6A8 = 6 };
constexpr int FMT_COUNT = 7;
constexpr int A8_GROUP = 128;  // columns per bf16 group scale of W4A8 / W6A8

__host__ __device__ constexpr int fmt_row_bytes(int fmt, int K) {
  return fmt == FMT_W4 || fmt == FMT_W4A8 ? K / 2 : fmt == FMT_W6 || fmt == FMT_W6A8 ? 3 * K / 4 : K;
}
// ConvRot formats: the activations are rotated before the GEMVs
__host__ __device__ constexpr bool fmt_rotated(int fmt) { return fmt == FMT_I8 || fmt == FMT_W4 || fmt == FMT_W6; }
// the reference's codes with e4m3 group-16 scales and an s_channel
__host__ __device__ constexpr bool fmt_codes(int fmt) { return fmt == FMT_W4 || fmt == FMT_W6; }
__host__ __device__ constexpr bool fmt_e4m3(int fmt) { return fmt == FMT_FP8 || fmt == FMT_FP8C; }
// int8 activations and bf16 group-128 scales
__host__ __device__ constexpr bool fmt_a8(int fmt) { return fmt == FMT_W4A8 || fmt == FMT_W6A8; }
// an fp32 scale per weight row (int8 ConvRot, per-channel fp8)
__host__ __device__ constexpr bool fmt_row_scale(int fmt) { return fmt == FMT_I8 || fmt == FMT_FP8C; }
// bytes of per-row group scales staged beside each weight row (e4m3 per 16 columns, or bf16 per 128)
__host__ __device__ constexpr int fmt_gscale_bytes(int fmt, int K) {
  return fmt_codes(fmt) ? K / 16 : fmt_a8(fmt) ? 2 * (K / A8_GROUP) : 0;
}

// Swizzled float4 slot of float4 index f in a staged activation row: conflict-free 16-byte loads when lane l reads
// float4 4*(l + 32j) + q for fixed (j, q). Permutes within aligned groups of eight (rows of K % 32 == 0 floats).
D3_DEV int xswz(int f) { return f ^ ((f >> 2) & 7); }
D3_DEV int xswz_elem(int i) { return (xswz(i >> 2) << 2) | (i & 3); }

// ---------------------------------------------------------------------------------------------------------------
// e4m3 -> f16 pairs (exact)
D3_DEV uint32_t e4m3x2_h2(uint32_t two_bytes) { return e4m3x2_to_h2((uint16_t)two_bytes); }

// d0 += lo(w) * lo(x), d1 += hi(w) * hi(x): f16 inputs, f32 accumulation, full FMA rate on sm_100.
D3_DEV void hfma2_f32(uint32_t w, uint32_t x, float& d0, float& d1) {
  asm("{\n\t.reg .f16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %2;\n\t"
      "mov.b32 {xl, xh}, %3;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.f16 %1, wh, xh, %1;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "r"(w), "r"(x));
}

// int8 x4 -> f32 x4 (exact): the byte (offset to unsigned) becomes the low mantissa byte of 2^23 + u.
D3_DEV void i8x4_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t t = w ^ 0x80808080u;
  const float bias = 8388736.0f;  // 2^23 + 128
  f0 = __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7650)) - bias;
  f1 = __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7651)) - bias;
  f2 = __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7652)) - bias;
  f3 = __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7653)) - bias;
}

// ---------------------------------------------------------------------------------------------------------------
// Float decoders (16 or 8 columns), used where the activations stay fp32.
D3_DEV void dec16_fp8(uint4 w, float (&f)[16]) {
  e4m3x4(w.x, f[0], f[1], f[2], f[3]);
  e4m3x4(w.y, f[4], f[5], f[6], f[7]);
  e4m3x4(w.z, f[8], f[9], f[10], f[11]);
  e4m3x4(w.w, f[12], f[13], f[14], f[15]);
}

D3_DEV void dec16_i8(uint4 w, float (&f)[16]) {
  i8x4_f32(w.x, f[0], f[1], f[2], f[3]);
  i8x4_f32(w.y, f[4], f[5], f[6], f[7]);
  i8x4_f32(w.z, f[8], f[9], f[10], f[11]);
  i8x4_f32(w.w, f[12], f[13], f[14], f[15]);
}

// The int8-grid value of a code: clamp(rint(v * s), +-127), as __float2int_rn and a clamp give it.
D3_DEV float grid_value(float v, float s) { return fmaxf(-127.0f, fminf(127.0f, rintf(v * s))); }

// N codes of a 16-column group starting at column 0 (N = 16) or at the half selected by the caller (N = 8, the
// caller passes the 4 nibble bytes in low.x): W4 through the codebook `lut`, W6 adding two high-plane bits per
// column from `high`.
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
  float p0 = w[0] * a.x, p1 = w[1] * a.y, p2 = w[2] * a.z, p3 = w[3] * a.w;
  p0 = fmaf(w[4], b.x, p0);
  p1 = fmaf(w[5], b.y, p1);
  p2 = fmaf(w[6], b.z, p2);
  p3 = fmaf(w[7], b.w, p3);
  p0 = fmaf(w[8], c.x, p0);
  p1 = fmaf(w[9], c.y, p1);
  p2 = fmaf(w[10], c.z, p2);
  p3 = fmaf(w[11], c.w, p3);
  p0 = fmaf(w[12], d.x, p0);
  p1 = fmaf(w[13], d.y, p1);
  p2 = fmaf(w[14], d.z, p2);
  p3 = fmaf(w[15], d.w, p3);
  return (p0 + p1) + (p2 + p3);
}

}  // namespace d3
