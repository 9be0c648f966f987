// Host-side packers, the on-disk format step before the decode and prompt kernels (the converter's job in the
// reference, tools/convert.py:48-82,179-215): float32 expert rows ->
//   the reference's layouts: e4m3 with 128x128 block scales (fp8), int8 rows in the ConvRot basis with row scales
//   (int8), 4-bit codebook / 6-bit codes with e4m3 group-16 scales and row scales in the ConvRot basis (w4, w6);
//   the BASELINE layouts: per-channel e4m3 (fp8c), W4A8 / W6A8 codes with bf16 scales per 128 columns.
// Plain nearest rounding only (the reference's quantizers live in comfy_kitchen, not part of it), the same arithmetic
// as the repository's reference packers (oracle/moe.py make_bank, quantize_fp8_channel, quantize_wa8); rows are
// split across host threads.
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/drama3_b200.h"

namespace {

// Nearest e4m3 byte of a finite v, ties to the even code, saturating at +-448; the sign bit follows v < 0.
// Below 2^-6 the e4m3 values are the multiples of 2^-9 (codes 0..8 = k), so the code is rint(|v| 2^9), exact since
// scaling by 2^9 is; above, a float's exponent and top 3 mantissa bits are the code plus (127 - 7) << 3 after
// rounding the 20 bits below them to nearest even. Both equal picking the nearer of the two neighbouring e4m3 values
// with ties to the even code.
inline uint8_t to_e4m3(float v) {
  float a = std::fabs(v);
  a = a < 448.0f ? a : 448.0f;
  uint32_t code;
  if (a < 0.015625f) {
    code = (uint32_t)std::nearbyint(a * 512.0f);
  } else {
    uint32_t b;
    std::memcpy(&b, &a, 4);
    code = ((b + 0x7FFFFu + ((b >> 20) & 1u)) >> 20) - (120u << 3);
  }
  return (uint8_t)(code | (v < 0.0f ? 0x80u : 0x00u));
}

// float32 -> bfloat16 bits, nearest-even.
uint16_t to_bf16(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  return (uint16_t)(((uint64_t)b + 0x7FFF + ((b >> 16) & 1)) >> 16);
}

float from_bf16(uint16_t h) {
  const uint32_t b = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

// Run fn(first, last) over [0, rows) in `threads` contiguous parts (threads <= 0: the host's hardware threads).
template <class F>
void parallel_rows(int64_t rows, int threads, F fn) {
  int n = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
  n = (int)std::max<int64_t>(1, std::min<int64_t>(n, rows));
  if (n == 1) {
    fn((int64_t)0, rows);
    return;
  }
  std::vector<std::thread> pool;
  for (int i = 0; i < n; ++i) pool.emplace_back(fn, rows * i / n, rows * (i + 1) / n);
  for (auto& t : pool) t.join();
}

// The regular Hadamard transform of 256 values (the 4-fold Kronecker power of h4 below, symmetric), normalized by
// 1/16, in double: four radix-4 stages. Row times H256 (W x = (W H)(x H) since H is orthogonal and symmetric).
void hadamard256(const float* in, double* out) {
  for (int i = 0; i < 256; ++i) out[i] = in[i];
  for (int stride = 1; stride < 256; stride *= 4) {
    for (int block = 0; block < 256; block += 4 * stride) {
      for (int i = 0; i < stride; ++i) {
        double* v = out + block + i;
        const double a = v[0], b = v[stride], c = v[2 * stride], d = v[3 * stride];
        // h4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]]: out_j = sum_i in_i h4[i][j]
        v[0] = a + b + c - d;
        v[stride] = a + b - c + d;
        v[2 * stride] = a - b + c + d;
        v[3 * stride] = -a + b + c + d;
      }
    }
  }
  for (int i = 0; i < 256; ++i) out[i] *= 1.0 / 16.0;
}

// A row in the ConvRot basis (every 256-column group times H256) and its float32 scale absmax / 127 (1 if zero).
float convrot_row(const float* row, int K, double* r) {
  double m = 0.0;
  for (int g = 0; g < K; g += 256) hadamard256(row + g, r + g);
  for (int j = 0; j < K; ++j) m = std::max(m, std::fabs(r[j]));
  const float s = (float)(m / 127.0);
  return s == 0.0f ? 1.0f : s;
}

inline double clampd(double v, double lo, double hi) { return std::max(lo, std::min(hi, v)); }

}  // namespace

extern "C" int d3_pack_fp8_blocks(const float* w, int64_t rows, int K, uint8_t* codes, float* scales, int threads) {
  if (!w || !codes || !scales || rows < 0 || rows % 128 || K < 128 || K % 128) return D3_ERR_ARG;
  const int KB = K / 128;
  parallel_rows(rows / 128, threads, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      for (int kb = 0; kb < KB; ++kb) {
        float m = 0.0f;
        for (int i = 0; i < 128; ++i)
          for (int j = 0; j < 128; ++j) m = std::max(m, std::fabs(w[(b * 128 + i) * K + kb * 128 + j]));
        float s = m / 448.0f;
        if (s == 0.0f) s = 1.0f;
        scales[b * KB + kb] = s;
        for (int i = 0; i < 128; ++i) {
          const int64_t o = (b * 128 + i) * K + kb * 128;
          for (int j = 0; j < 128; ++j) codes[o + j] = to_e4m3(w[o + j] / s);
        }
      }
    }
  });
  return D3_OK;
}

extern "C" int d3_pack_int8_convrot(const float* w, int64_t rows, int K, int8_t* q, float* scales, int threads) {
  if (!w || !q || !scales || rows < 0 || K < 256 || K % 256) return D3_ERR_ARG;
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    std::vector<double> r(K);
    for (int64_t n = r0; n < r1; ++n) {
      const float s = convrot_row(w + n * K, K, r.data());
      scales[n] = s;
      for (int j = 0; j < K; ++j) q[n * K + j] = (int8_t)clampd(std::nearbyint(r[j] / (double)s), -127.0, 127.0);
    }
  });
  return D3_OK;
}

extern "C" int d3_pack_codes(const float* w, int64_t rows, int K, int bits, const float* codebook, uint8_t* codes,
                             uint8_t* group_scales, float* s_channel, int threads) {
  if (!w || !codes || !group_scales || !s_channel || rows < 0 || K < 256 || K % 256 || (bits != 4 && bits != 6) ||
      (bits == 4 && !codebook))
    return D3_ERR_ARG;
  double top = 31.0;
  if (bits == 4) {
    top = 0.0;
    for (int c = 0; c < 16; ++c) top = std::max(top, (double)std::fabs(codebook[c]));
  }
  const int rb = K * bits / 8, G = K / 16;
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    std::vector<double> r(K);
    std::vector<int> code(K);
    for (int64_t n = r0; n < r1; ++n) {
      const float chan = convrot_row(w + n * K, K, r.data());
      s_channel[n] = chan;
      for (int j = 0; j < K; ++j) r[j] /= (double)chan;  // on the int8 grid
      for (int g = 0; g < G; ++g) {
        const double* t = r.data() + 16 * g;
        double m = 0.0;
        for (int j = 0; j < 16; ++j) m = std::max(m, std::fabs(t[j]));
        const uint8_t gs = to_e4m3((float)std::max(m / top, 1.0 / 64.0));
        group_scales[n * G + g] = gs;
        // the group scale's value: exponent field 1..15 (never subnormal, >= 2^-6), 3 mantissa bits
        const double sv = std::ldexp(1.0 + (gs & 7) / 8.0, (gs >> 3) - 7);
        if (bits == 4) {
          double cand[16];
          for (int c = 0; c < 16; ++c) cand[c] = clampd(std::nearbyint((double)codebook[c] * sv), -127.0, 127.0);
          for (int j = 0; j < 16; ++j) {
            int best = 0;
            double bd = std::fabs(cand[0] - t[j]);
            for (int c = 1; c < 16; ++c) {
              const double d = std::fabs(cand[c] - t[j]);
              if (d < bd) bd = d, best = c;  // the first of equal distances
            }
            code[16 * g + j] = best;
          }
        } else {
          for (int j = 0; j < 16; ++j) code[16 * g + j] = (int)clampd(std::nearbyint(t[j] / sv), -32.0, 31.0) + 32;
        }
      }
      uint8_t* out = codes + n * rb;
      for (int j = 0; j < K / 2; ++j) out[j] = (uint8_t)((code[2 * j] & 0xF) | ((code[2 * j + 1] & 0xF) << 4));
      if (bits == 6) {
        uint8_t* hi = out + K / 2;
        for (int j = 0; j < K / 4; ++j)
          hi[j] = (uint8_t)((code[4 * j] >> 4) | ((code[4 * j + 1] >> 4) << 2) | ((code[4 * j + 2] >> 4) << 4) |
                            ((code[4 * j + 3] >> 4) << 6));
      }
    }
  });
  return D3_OK;
}

extern "C" int d3_pack_fp8c(const float* w, int64_t rows, int K, uint8_t* codes, float* scales, int threads) {
  if (!w || !codes || !scales || rows < 0 || K < 1) return D3_ERR_ARG;
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      const float* row = w + r * K;
      float m = 0.0f;
      for (int j = 0; j < K; ++j) m = std::max(m, std::fabs(row[j]));
      float s = m / 448.0f;
      if (s == 0.0f) s = 1.0f;
      scales[r] = s;
      uint8_t* out = codes + r * K;
      for (int j = 0; j < K; ++j) out[j] = to_e4m3(row[j] / s);
    }
  });
  return D3_OK;
}

extern "C" int d3_pack_wa8(const float* w, int64_t rows, int K, int bits, uint8_t* packed, uint16_t* scales,
                           int threads) {
  if (!w || !packed || !scales || rows < 0 || K < 128 || K % 128 || (bits != 4 && bits != 6)) return D3_ERR_ARG;
  const int qmax = bits == 4 ? 7 : 31, G = K / 128, rb = K * bits / 8;
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    std::vector<int> q(K);
    for (int64_t r = r0; r < r1; ++r) {
      const float* row = w + r * K;
      for (int g = 0; g < G; ++g) {
        float m = 0.0f;
        for (int j = 0; j < 128; ++j) m = std::max(m, std::fabs(row[128 * g + j]));
        float s = m / (float)qmax;
        if (s == 0.0f) s = 1.0f;
        const uint16_t sb = to_bf16(s);
        scales[r * G + g] = sb;
        const double sv = (double)from_bf16(sb);
        for (int j = 0; j < 128; ++j) {
          const double t = std::nearbyint((double)row[128 * g + j] / sv);  // round half to even
          q[128 * g + j] = (int)std::max<double>(-qmax, std::min<double>(qmax, t));
        }
      }
      uint8_t* out = packed + r * rb;
      if (bits == 4) {
        for (int j = 0; j < K / 2; ++j) out[j] = (uint8_t)((q[2 * j] & 0xF) | ((q[2 * j + 1] & 0xF) << 4));
      } else {
        for (int j = 0; j < K / 4; ++j) {
          const uint32_t word = (uint32_t)(q[4 * j] & 0x3F) | ((uint32_t)(q[4 * j + 1] & 0x3F) << 6) |
                                ((uint32_t)(q[4 * j + 2] & 0x3F) << 12) | ((uint32_t)(q[4 * j + 3] & 0x3F) << 18);
          out[3 * j] = (uint8_t)(word & 0xFF);
          out[3 * j + 1] = (uint8_t)((word >> 8) & 0xFF);
          out[3 * j + 2] = (uint8_t)((word >> 16) & 0xFF);
        }
      }
    }
  });
  return D3_OK;
}
