// One-line decode of e4m3 experts, per-channel (fp8c) or in the reference's 128 x 128 blocks (fp8):
// drama3/offload.py:108-123 (resident_decode) for one row, as a streaming kernel shaped for that case. At one line every byte of the pairs' weights is used once by one column, so
// the layer is bound by how early the bytes start to stream and how little waiting follows them; the tensor-core
// decodes (built for 16 lines) spend more on their phase changes than on the bytes at one line.
//
// One CTA per SM: 8 MMA warps and one producer warp. Work:
//   phase 1  the pairs' gate_up rows in units of 4 channels (4 gate + 4 up rows of 2048 e4m3), split evenly over the
//            CTAs in order; two units (16 rows) per MMA tile; SwiGLU to the workspace; each CTA adds the units it
//            finished to its pair's counter (at the pair boundary and at the end).
//   phase 2  split by (pair, row block): CTA b < nv * RB (RB = G / nv) takes pair b / RB and output rows
//            [rb * RR, rb * RR + RR) (RR = ceil(2048 / RB), at most 128: 8 MMA tiles of 16 rows, one a warp); it waits
//            until its pair's counter holds all of the pair's units, reads the pair's SwiGLU row (768 values, L2),
//            multiplies its down rows, and writes the fp32 partial; the row block's last CTA to arrive (a counter)
//            sums the pairs' partials in rank order (fp32 fused multiply-adds, as the reference's weighted_sum) and
//            writes bf16.
// One ring of 3 stages of 32 rows carries both phases' weights by per-row bulk copies (one per lane) into padded
// rows: the units four to a stage (a CTA's whole share fits, so it is all requested at once), then the down rows 64
// to a stage as the units' stages drain. Measured with no compute, 2 KB copies stream at ~4.2 TB/s aggregate through
// 3 stages of 64 KB per SM, ~3.8 TB/s through 6 of 32 KB and ~3.1 TB/s through 12 of 16 KB; this kernel with the down
// rows prefetched into a region of their own beside a ring of 3 x 32 KB took 18.8 us a layer against 16.1 us.
//
// Arithmetic: mma.sync m16n8k32 e4m3 x e4m3 -> f32 with the weights as stored. Activations (the bf16 or fp32 row, a
// pair's fp32 SwiGLU row) enter as six e4m3 terms in B's columns: the row is scaled by a power of two that puts its
// largest magnitude in [2^7, 2^8); terms 1-3 are successive roundings to 3 mantissa bits (subnormal steps of 2^-9
// below 2^-6) with exact fp32 residuals; the residual after them is scaled by 2^12 and split the same way into terms
// 4-6, whose columns are scaled back by 2^-12 after the MMA. A bf16 row is exact, an fp32 row keeps ~24 significant
// bits; only magnitudes below 2^-29 of the row's largest are lost. The per-channel scale multiplies the fp32 dot; a
// block scale multiplies the fp32 partial dot of its 128 columns (a warp's phase-1 columns are two blocks, a down row's
// are I / 128), as the reference's block dequantization does before its fp32 sum.
#pragma once

#include "moe_decode.cuh"

namespace d3 {

constexpr int GV_WARPS = 8;                      // MMA warps
constexpr int GV_THREADS = GV_WARPS * 32 + 32;   // + the producer warp
constexpr int GV_MMA_THREADS = GV_WARPS * 32;
constexpr int GV_STAGES = 3;                     // ring stages: four units (32 rows) or 64 down rows
constexpr int GV_UNIT_CH = 4;                    // channels per unit
constexpr int GV_K = 2048;                       // hidden size (phase-1 K, phase-2 rows)
constexpr int GV_P1_PITCH = GV_K + 16;           // bytes per staged row: 129 x 16, so 8 rows hit 8 bank groups
constexpr int GV_STAGE_UNITS = 4;
constexpr int GV_STAGE_BYTES = 8 * GV_STAGE_UNITS * GV_P1_PITCH;
constexpr int GV_P2_ROWS = 64;                   // down rows per stage
constexpr int GV_MIN_GRID = 128;                 // CTAs needed: 8 pairs x 16 row blocks of at most 128 rows
constexpr int GV_MAX_PAIRS = 8;
constexpr int GV_TERMS = 6;                      // B columns in use: terms 1-3, then terms 4-6 scaled by 2^12
constexpr int GV_XPITCH = GV_K + 16;             // bytes per staged activation term (bank-spread)
constexpr float GV_LOW = 1.0f / 4096.0f;         // 2^-12: the second group's weight

__host__ __device__ constexpr int gv_p2_pitch(int I) { return I + 16; }

struct GvSmem {
  static constexpr int ring = 0;
  static constexpr int xt = ring + GV_STAGES * GV_STAGE_BYTES;
  static constexpr int ht = xt + GV_TERMS * GV_XPITCH;
  __host__ __device__ static constexpr int red(int I) { return ht + GV_TERMS * gv_p2_pitch(I); }
  __host__ __device__ static constexpr int bars(int I) { return red(I) + 2 * GV_WARPS * 32 * 4; }
  __host__ __device__ static constexpr int total(int I) { return bars(I) + 8 * 2 * GV_STAGES + 128; }
};
static_assert(GV_P2_ROWS * gv_p2_pitch(768) <= GV_STAGE_BYTES, "64 down rows fit one stage");

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

// acc += 16 e4m3 rows (rows 0-7 at `lo`, 8-15 at `hi`, pitch `pitch` bytes) x the activation terms at `xt` (term t at
// xt + t * xpitch bytes in B column t; columns 6 and 7 are zero), over 32 columns from kb.
D3_DEV void gv_mma32(float (&acc)[4], const uint8_t* lo, const uint8_t* hi, int pitch, const uint8_t* xt, int xpitch,
                     int kb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  uint32_t w[4];
  ldsm_x4(w, ((lane >> 3) & 1 ? hi : lo) + (lane & 7) * pitch + kb + 16 * (lane >> 4));
  uint32_t b0 = 0u, b1 = 0u;
  if (g < GV_TERMS) {
    const uint8_t* xr = xt + g * xpitch + kb + 4 * c;
    b0 = *reinterpret_cast<const uint32_t*>(xr);
    b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
  }
  mma_e4m3_16832(acc, w, b0, b1);
}

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

// Synchronization words (zero between calls; every call leaves them zero): a.depart[32 q] counts pair q's finished
// units, a.depart[32 q + 16] its consumers that have passed the wait; a.arrive[rb] counts row block rb's pairs done.
template <int FMT, int I>
__global__ void __launch_bounds__(GV_THREADS, 1) moe_decode_gv_kernel(const DecodeArgs a) {
  constexpr bool BLK = FMT == FMT_FP8;  // scales per 128 x 128 block, else per output channel
  constexpr int UPP = I / GV_UNIT_CH;  // units per pair
  constexpr int P2P = gv_p2_pitch(I);
  constexpr int HPT = (I + GV_MMA_THREADS - 1) / GV_MMA_THREADS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
  uint8_t* ring = smem + GvSmem::ring;
  uint8_t* xt = smem + GvSmem::xt;   // [GV_TERMS][GV_XPITCH]: the row's terms
  uint8_t* ht = smem + GvSmem::ht;   // [GV_TERMS][P2P]: the pair's SwiGLU row's terms
  float* red = (float*)(smem + GvSmem::red(I));  // [2][GV_WARPS][32]
  uint64_t* bars = (uint64_t*)(smem + GvSmem::bars(I));
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
  const int nt2 = (rows2 + 15) / 16;                                   // down tiles of 16 rows, one a warp
  const int n1s = (n1 + GV_STAGE_UNITS - 1) / GV_STAGE_UNITS;            // unit stages
  const int items = n1s + (rows2 + GV_P2_ROWS - 1) / GV_P2_ROWS;         // + down-row stages
  unsigned* done = a.depart;       // [32 q]: pair q's finished units; [32 q + 16]: its consumers past the wait
  unsigned* block_cnt = a.arrive;  // [rb]: row block rb's pairs done

  if (warp == GV_WARPS) {
    // producer: item i (four units, or 64 down rows) into stage i % GV_STAGES, one row copy a lane
    const uint64_t pol = policy_evict_first();
    for (int i = 0; i < items; ++i) {
      const int s = i % GV_STAGES;
      if (i >= GV_STAGES && !mbar_wait(empty + s, ((i / GV_STAGES) - 1) & 1)) break;
      uint8_t* dst = ring + s * GV_STAGE_BYTES;
      if (i < n1s) {
        const int units = min(GV_STAGE_UNITS, n1 - GV_STAGE_UNITS * i);
        if (lane == 0) mbar_arrive_expect_tx(full + s, (uint32_t)(units * 8 * GV_K));
        __syncwarp();
        if (lane < units * 8) {
          const int u = u_lo + GV_STAGE_UNITS * i + (lane >> 3), v = u / UPP;
          const int ch = (u - v * UPP) * GV_UNIT_CH + (lane & 3);
          const int row = e_of[v] * 2 * I + ((lane & 7) < 4 ? ch : I + ch);
          bulk_g2s(dst + lane * GV_P1_PITCH, a.w13 + (size_t)row * GV_K, GV_K, full + s, pol);
        }
      } else {
        const int m0 = GV_P2_ROWS * (i - n1s), rows = min(GV_P2_ROWS, rows2 - m0);
        if (lane == 0) mbar_arrive_expect_tx(full + s, (uint32_t)(rows * I));
        __syncwarp();
        for (int r = lane; r < rows; r += 32)
          bulk_g2s(dst + r * P2P, a.w2 + ((size_t)e_of[q2] * GV_K + r0 + m0 + r) * I, I, full + s, pol);
      }
    }
    return;
  }

  // ---- MMA warps: the row's terms
  float x_inv;
  {
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
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_max[warp] = m;
    named_sync(1, GV_MMA_THREADS);
    m = s_max[0];
#pragma unroll
    for (int w = 1; w < GV_WARPS; ++w) m = fmaxf(m, s_max[w]);
    const int sx = gv_scale_exp(m);
    x_inv = gv_pow2(-sx);
    const float scale = gv_pow2(sx);
#pragma unroll
    for (int i = 0; i < 8; ++i) gv_terms(v[i], scale, xt + c0 + i, GV_XPITCH);
    named_sync(1, GV_MMA_THREADS);
  }

  // ---- phase 1: gate | up dots of this CTA's units, a stage (two 16-row tiles) at a time, SwiGLU, to the workspace
  bool ok = true;
  const int kw = warp * (GV_K / GV_WARPS);
  int cur_pair = -1, cur_units = 0;  // warp 0, lane 0: units finished and not yet added to their pair's counter
  for (int i = 0; i < n1s; ++i) {
    const int s = i % GV_STAGES;
    const int units = min(GV_STAGE_UNITS, n1 - GV_STAGE_UNITS * i);
    // the SwiGLU threads' scales (thread t < 16: unit t / 4, channel t % 4), loaded while the stage lands
    const int su = u_lo + GV_STAGE_UNITS * i + (tid >> 2);
    const bool swi = tid < 4 * units;
    float sg = 1.0f, sup = 1.0f;
    int sv = 0, sch = 0;
    if (swi) {
      sv = su / UPP;
      sch = (su - sv * UPP) * GV_UNIT_CH + (tid & 3);
      if (!BLK) {
        const float* sc = (const float*)a.s13 + (size_t)e_of[sv] * 2 * I;
        sg = __ldg(sc + sch);
        sup = __ldg(sc + I + sch);
      }
    }
    // block scales: this lane's rows (g of units 2 tl, 2 tl + 1) over the warp's two column blocks
    float bs[2][2][2] = {};  // [tile][row g / g + 8][block]
    if (BLK) {
      const int g = lane >> 2;
#pragma unroll
      for (int tl = 0; tl < 2; ++tl)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int uu = GV_STAGE_UNITS * i + 2 * tl + hr;
          if (uu < n1) {
            const int u = u_lo + uu, v = u / UPP, ch = (u - v * UPP) * GV_UNIT_CH + (g & 3);
            const int row = e_of[v] * 2 * I + (g < 4 ? ch : I + ch);
            const float* sc = (const float*)a.s13 + (size_t)(row / 128) * (GV_K / 128) + kw / 128;
            bs[tl][hr][0] = __ldg(sc);
            bs[tl][hr][1] = __ldg(sc + 1);
          }
        }
    }
    ok = mbar_wait(full + s, (i / GV_STAGES) & 1) && ok;
    if (i == 0) D3_GSTAMP(2);
    const uint8_t* st = ring + s * GV_STAGE_BYTES;
    float acc[2][2][2][4] = {};  // [tile][column block][chain]
    if (ok) {
#pragma unroll
      for (int kb = 0; kb < GV_K / GV_WARPS; kb += 64) {
#pragma unroll
        for (int tl = 0; tl < 2; ++tl) {
          if (tl == 0 || units > 2) {
            const uint8_t* lo = st + 16 * tl * GV_P1_PITCH;
            gv_mma32(acc[tl][kb >> 7][0], lo, lo + 8 * GV_P1_PITCH, GV_P1_PITCH, xt, GV_XPITCH, kw + kb);
            gv_mma32(acc[tl][kb >> 7][1], lo, lo + 8 * GV_P1_PITCH, GV_P1_PITCH, xt, GV_XPITCH, kw + kb + 32);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    float* rbuf = red + (i & 1) * GV_WARPS * 32;
#pragma unroll
    for (int tl = 0; tl < 2; ++tl) {
      float r_lo = 0.0f, r_hi = 0.0f;
      if constexpr (BLK) {
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          float t4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) t4[e] = acc[tl][blk][0][e] + acc[tl][blk][1][e];
          float d_lo, d_hi;
          gv_term_sums(t4, d_lo, d_hi);
          r_lo += d_lo * bs[tl][0][blk];
          r_hi += d_hi * bs[tl][1][blk];
        }
      } else {
        float t4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) t4[e] = (acc[tl][0][0][e] + acc[tl][0][1][e]) + (acc[tl][1][0][e] + acc[tl][1][1][e]);
        gv_term_sums(t4, r_lo, r_hi);
      }
      if ((lane & 3) == 0) {
        rbuf[warp * 32 + 16 * tl + (lane >> 2)] = r_lo;
        rbuf[warp * 32 + 16 * tl + (lane >> 2) + 8] = r_hi;
      }
    }
    named_sync(1, GV_MMA_THREADS);
    if (warp == 0) {
      if (swi) {
        const int row = (tid >> 2) * 8 + (tid & 3);
        float g = 0.0f, u = 0.0f;
#pragma unroll
        for (int w = 0; w < GV_WARPS; ++w) {
          g += rbuf[w * 32 + row];
          u += rbuf[w * 32 + row + 4];
        }
        g = g * x_inv * sg;
        u = u * x_inv * sup;
        a.a1[(size_t)sv * I + sch] = g / (1.0f + expf(-g)) * u;
      }
      __syncwarp();
      if (lane == 0) {
        // this stage's units, counted per pair; a pair's count goes out when the next pair starts and at the end
        for (int h = 0; h < units; ++h) {
          const int p = (u_lo + GV_STAGE_UNITS * i + h) / UPP;
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

  // ---- phase 2: wait for the pair's units, then its SwiGLU row as terms
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
  float hv[HPT];
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < HPT; ++i) {
    const int col = tid + i * GV_MMA_THREADS;
    hv[i] = col < I ? __ldcg(a.a1 + (size_t)q2 * I + col) : 0.0f;
    m = fmaxf(m, fabsf(hv[i]));
  }
  // this thread's down scales for its tile rows (per channel, or per 128-column block), loaded while the row lands
  constexpr int NKB2 = I / 128;
  const int row_lo = r0 + 16 * warp + (lane >> 2), row_hi = row_lo + 8;
  const bool live_lo = 16 * warp + (lane >> 2) < rows2, live_hi = 16 * warp + (lane >> 2) + 8 < rows2;
  float sc_lo[BLK ? NKB2 : 1], sc_hi[BLK ? NKB2 : 1];
  if (BLK) {
    const float* s2b = (const float*)a.s2;
    const size_t blo = ((size_t)e_of[q2] * GV_K + row_lo) / 128 * NKB2, bhi = ((size_t)e_of[q2] * GV_K + row_hi) / 128 * NKB2;
#pragma unroll
    for (int kb = 0; kb < (BLK ? NKB2 : 1); ++kb) {
      sc_lo[kb] = live_lo ? __ldg(s2b + blo + kb) : 0.0f;
      sc_hi[kb] = live_hi ? __ldg(s2b + bhi + kb) : 0.0f;
    }
  } else {
    const float* s2 = (const float*)a.s2 + (size_t)e_of[q2] * GV_K;
    sc_lo[0] = live_lo ? __ldg(s2 + row_lo) : 0.0f;
    sc_hi[0] = live_hi ? __ldg(s2 + row_hi) : 0.0f;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) s_max[warp] = m;  // s_max's phase-1 readers all passed the barriers since
  named_sync(1, GV_MMA_THREADS);
  m = s_max[0];
#pragma unroll
  for (int w = 1; w < GV_WARPS; ++w) m = fmaxf(m, s_max[w]);
  const int sh = gv_scale_exp(m);
  const float hscale = gv_pow2(sh), h_inv = gv_pow2(-sh);
#pragma unroll
  for (int i = 0; i < HPT; ++i) {
    const int col = tid + i * GV_MMA_THREADS;
    if (col < I) gv_terms(hv[i], hscale, ht + col, P2P);
  }
  named_sync(1, GV_MMA_THREADS);
  D3_GSTAMP(5);
  // warp w: down tile w (rows 16 w .. 16 w + 15 of this block), in stage item n1s + w / 4
  if (warp < nt2) {
    const int item = n1s + warp / (GV_P2_ROWS / 16), s = item % GV_STAGES;
    ok = mbar_wait(full + s, (item / GV_STAGES) & 1) && ok;
    // four chains over the row's columns; with block scales, their term sums fold per column block (128)
    float r_lo = 0.0f, r_hi = 0.0f;
    const uint8_t* rows = ring + s * GV_STAGE_BYTES + (warp % (GV_P2_ROWS / 16)) * 16 * P2P;
    float acc[4][4] = {};
#pragma unroll
    for (int kb = 0; kb < I; kb += 128) {
      if (ok) {
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) gv_mma32(acc[c4], rows, rows + 8 * P2P, P2P, ht, P2P, kb + 32 * c4);
      }
      if constexpr (BLK) {
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
    if constexpr (!BLK) {
      float t4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) t4[e] = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
      gv_term_sums(t4, r_lo, r_hi);
    }
    if ((lane & 3) == 0) {
      float* part = a.parts + (size_t)q2 * GV_K;
      if (live_lo) part[row_lo] = r_lo * h_inv * (BLK ? 1.0f : sc_lo[0]);
      if (live_hi) part[row_hi] = r_hi * h_inv * (BLK ? 1.0f : sc_hi[0]);
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
