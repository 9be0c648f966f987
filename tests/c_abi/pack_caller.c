/* A plain C caller of the library through include/drama3_b200.h only: packs a seeded float bank with every host
 * packer and prints a checksum line per layout (FNV-1a over the output bytes); with a path argument it also writes
 * the float rows there, so that a caller can pack the same rows another way and compare. Needs no GPU: only host
 * entry points are called. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "drama3_b200.h"

static uint64_t fnv(uint64_t h, const void* p, size_t n) {
  const uint8_t* b = (const uint8_t*)p;
  for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
  return h;
}

/* xorshift64* uniform in [-0.1, 0.1) */
static float next_weight(uint64_t* s) {
  *s ^= *s >> 12;
  *s ^= *s << 25;
  *s ^= *s >> 27;
  const uint64_t r = *s * 2685821657736338717ull;
  return (float)((double)(r >> 11) / 9007199254740992.0 * 0.2 - 0.1);
}

int main(int argc, char** argv) {
  enum { ROWS = 256, K = 512 };
  static const float book[16] = {-1.0f, -0.6962f, -0.5251f, -0.3949f, -0.2844f, -0.1848f, -0.0911f, 0.0f,
                                 0.0796f, 0.1609f, 0.2461f, 0.3379f, 0.4407f, 0.5626f, 0.7230f, 1.0f};
  float* w = malloc(sizeof(float) * ROWS * K);
  uint8_t* codes = malloc((size_t)ROWS * K);
  float* fscale = malloc(sizeof(float) * ROWS * K);
  uint16_t* hscale = malloc(sizeof(uint16_t) * ROWS * K);
  uint8_t* gscale = malloc((size_t)ROWS * K);
  float* chan = malloc(sizeof(float) * ROWS);
  uint64_t seed = 0x9E3779B97F4A7C15ull;
  for (int i = 0; i < ROWS * K; ++i) w[i] = next_weight(&seed);
  if (d3_version() != D3_VERSION) return 2;
  if (argc > 1) { /* the input rows, for the caller to pack the same bank another way */
    FILE* f = fopen(argv[1], "wb");
    if (!f || fwrite(w, sizeof(float), (size_t)ROWS * K, f) != (size_t)ROWS * K) return 5;
    fclose(f);
  }
  uint64_t h;
  if (d3_pack_fp8_blocks(w, ROWS, K, codes, fscale, 2) != D3_OK) return 3;
  h = fnv(fnv(14695981039346656037ull, codes, (size_t)ROWS * K), fscale, sizeof(float) * (ROWS / 128) * (K / 128));
  printf("fp8 %016llx\n", (unsigned long long)h);
  if (d3_pack_int8_convrot(w, ROWS, K, (int8_t*)codes, fscale, 2) != D3_OK) return 3;
  h = fnv(fnv(14695981039346656037ull, codes, (size_t)ROWS * K), fscale, sizeof(float) * ROWS);
  printf("int8 %016llx\n", (unsigned long long)h);
  for (int bits = 4; bits <= 6; bits += 2) {
    if (d3_pack_codes(w, ROWS, K, bits, book, codes, gscale, chan, 2) != D3_OK) return 3;
    h = fnv(14695981039346656037ull, codes, (size_t)ROWS * K * bits / 8);
    h = fnv(fnv(h, gscale, (size_t)ROWS * K / 16), chan, sizeof(float) * ROWS);
    printf("w%d %016llx\n", bits, (unsigned long long)h);
  }
  if (d3_pack_fp8c(w, ROWS, K, codes, fscale, 2) != D3_OK) return 3;
  h = fnv(fnv(14695981039346656037ull, codes, (size_t)ROWS * K), fscale, sizeof(float) * ROWS);
  printf("fp8c %016llx\n", (unsigned long long)h);
  for (int bits = 4; bits <= 6; bits += 2) {
    if (d3_pack_wa8(w, ROWS, K, bits, codes, hscale, 2) != D3_OK) return 3;
    h = fnv(14695981039346656037ull, codes, (size_t)ROWS * K * bits / 8);
    h = fnv(h, hscale, sizeof(uint16_t) * ROWS * K / 128);
    printf("w%da8 %016llx\n", bits, (unsigned long long)h);
  }
  /* argument checks: K not a multiple of 128 / 256 */
  if (d3_pack_wa8(w, ROWS, 200, 4, codes, hscale, 1) != D3_ERR_ARG) return 4;
  if (d3_pack_codes(w, ROWS, 384, 6, book, codes, gscale, chan, 1) != D3_ERR_ARG) return 4;
  free(w);
  free(codes);
  free(fscale);
  free(hscale);
  free(gscale);
  free(chan);
  return 0;
}
