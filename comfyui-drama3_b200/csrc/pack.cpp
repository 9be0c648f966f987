// Host-side packers for the BASELINE expert layouts (the on-disk format step before the decode and prompt kernels):
// float32 expert rows -> per-channel e4m3 (fp8c) or W4A8 / W6A8 codes with bf16 scales per 128 columns. Plain
// rounding only, the same arithmetic as the repository's reference packers (oracle/moe.py quantize_fp8_channel,
// quantize_wa8), byte for byte; rows are split across host threads.
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

}  // namespace

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
