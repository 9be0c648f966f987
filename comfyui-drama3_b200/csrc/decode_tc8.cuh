// The routed-expert decode of M <= 16 lines on the tensor cores for W4A8 banks (int4 weights
// two per byte along K, bf16 scales per 128 columns, activations quantized to int8 per row): tcgen05.mma kind::i8
// with int32 accumulation, which is exact. Same plan, phases, scratch, dataflow start of phase 2 and combine as
// moe_decode_tc_kernel; what differs is the A operand and the scales:
//
//   * TMA brings the packed int4 rows (64 bytes per 128 columns) into a raw ring; two converter warps turn each
//     stage into an int8 A stage: a packed byte b (columns 2j, 2j+1 in its low / high nibble) becomes the bytes
//     (b << 4) & 0xF0 and b & 0xF0, i.e. 16 x the signed nibble, exact in int8. Within every 32 columns the even
//     columns go first and the odd ones after; the B rows are staged with the same order, and a dot product does
//     not depend on it. No shift back is needed: the epilogue folds the 1/16 into the scales.
//   * B: the lines' rows (phase 1) or the segment's pairs' a1 rows (phase 2), each quantized to int8 per row
//     (s = max|x| / 127, q = rint(x * (1 / s)) clipped to +-127: quant_i8_n) - one exact term.
//   * Every 128-column group has its own bf16 scale per row, so each group's MMAs (4 of K = 32) go to a TMEM region
//     of their own (16 columns: the lines or pairs); a tile's groups fill 16 regions (256 columns), two tiles in
//     flight, and the epilogue warps fold a finished tile's regions into fp32 registers, acc += group scale x int32
//     sum (a fold per group, handing each region back at once, measured slower: the round trip paced the MMAs).
#pragma once
#include "decode_tc.cuh"

namespace d3 {

constexpr int T8_RAW_ST = 6;         // raw ring: 128 rows x 64 packed bytes = 128 int4 columns a stage
constexpr int T8_RAW_BYTES = 8192;
constexpr int T8_A_ST = 8;           // int8 A ring: 128 rows x 128 bytes (deep: a stage comes back only once its
                                     // MMAs have completed)
constexpr int T8_BUF_COLS = 256;     // TMEM columns of one tile: 16 groups x 16 columns
constexpr int T8_CONV0 = 192;        // converter threads: warps 6-7
constexpr int T8_BREGION = 32768;    // phase-1 B (16 lines x 2048) or two phase-2 B buffers (16 pairs x <= 768)
constexpr int T8_TMEM_COLS = 512;   // two tiles

struct T8Smem {
  static constexpr int raw = 0;
  static constexpr int astage = raw + T8_RAW_ST * T8_RAW_BYTES;
  static constexpr int breg = astage + T8_A_ST * TC_ABYTES;
  static constexpr int xchg = breg + T8_BREGION;  // float [128][17]
  static constexpr int bars = xchg + 128 * TC_XPITCH * 4;
  static constexpr int tmem = bars + 40 * 8;
  static constexpr int linv = tmem + 16;     // float [16]: line scales
  static constexpr int spair = linv + 64;    // int [2][16]: phase-2 B rows' pairs
  static constexpr int sinv = spair + 128;   // float [2][16]: their scales
  static constexpr int end = sinv + 128;
  static constexpr int launch = end + 1024;  // + alignment slack
};

// 32 consecutive values of a bf16 or fp32 row from global memory (L2).
D3_DEV void t8_load32(const void* src, bool bf16, size_t i, float (&v)[32]) {
  tc_load16(src, bf16, i, (float(&)[16])v[0]);
  tc_load16(src, bf16, i + 16, (float(&)[16])v[16]);
}

// The bytes of one 32-column chunk of int8 codes in the A stages' column order: the 16 even columns, then the 16
// odd ones (byte i of word p: column 8p + 2i, then 8p + 2i + 1).
D3_DEV void t8_store_chunk(uint8_t* b, int rows, int n, int c, const float (&q)[32]) {
  uint32_t w[8];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      uint32_t r = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) r |= ((uint32_t)(int)q[8 * p + 2 * i + h] & 0xFFu) << (8 * i);
      w[4 * h + p] = r;
    }
  *reinterpret_cast<uint4*>(b + tc_b_offset(rows, n, 2 * c)) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(b + tc_b_offset(rows, n, 2 * c + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
}

// One 32-column chunk c of a B row n quantized to int8 by s (quant_i8_n), into a K-major 128-byte-swizzled operand
// of `rows` rows in the A stages' column order.
D3_DEV void t8_write_chunk(uint8_t* b, int rows, int n, int c, const float (&v)[32], float s) {
  float q[32];
  quant_i8_n<32>(v, s, __frcp_rn(s), q);
  t8_store_chunk(b, rows, n, c, q);
}

// 16 consecutive TMEM columns of this warp's lanes, without waiting (tcgen05.wait::ld before the registers are read).
D3_DEV void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// The epilogue's fold of tile tn (TMEM buffer tn & 1, NK groups of 16 int32 columns at `taddr` = this warp's lanes):
// acc[j] = sum over groups g of scale[g] x column 16g + j, the bf16 group scales packed two per word in gw. Waits
// (bounded) for the tile, then hands the buffer back. Four groups are loaded per wait.
template <int NK>
D3_DEV void t8_fold(float (&acc)[16], const uint32_t* gw, uint32_t taddr, int tn, uint64_t* acc_full,
                    uint64_t* acc_empty, bool& ok, int lane) {
  const int buf = tn & 1;
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
  if (ok) ok = mbar_wait(acc_full + buf, (tn >> 1) & 1);
  ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: the warp agrees
  tc_fence_after();
  if (ok) {
#pragma unroll
    for (int k0 = 0; k0 < NK; k0 += 4) {
      uint32_t v[4][16];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (k0 + u < NK) tmem_ld16_async(taddr + buf * T8_BUF_COLS + (k0 + u) * 16, v[u]);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (k0 + u < NK) {
          const int kb = k0 + u;
          const float gs = bf16_to_f32((kb & 1) ? gw[kb >> 1] >> 16 : gw[kb >> 1] & 0xFFFFu);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = fmaf((float)(int)v[u][j], gs, acc[j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(acc_empty + buf);
}

// ---------------------------------------------------------------------------------------------------------------
template <bool XBF, int NKB2>
__global__ void __launch_bounds__(TC_THREADS, 1)
    moe_decode_tc8_kernel(const __grid_constant__ CUtensorMap map13, const __grid_constant__ CUtensorMap map2,
                          const DecodeArgs a) {
  constexpr int H = DEC_H, NKB1 = H / 128;
  constexpr int I = NKB2 * 128;
  constexpr int TPS1 = I / TC_U1, TPS2 = H / TC_R2;
  constexpr int B2BYTES = TC_CAP * I;  // one phase-2 B buffer

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* raw = smem + T8Smem::raw;
  uint8_t* astage = smem + T8Smem::astage;
  uint8_t* breg = smem + T8Smem::breg;
  float* xchg = (float*)(smem + T8Smem::xchg);
  uint64_t* bars = (uint64_t*)(smem + T8Smem::bars);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + T8_RAW_ST;
  uint64_t* a_full = raw_empty + T8_RAW_ST;
  uint64_t* a_empty = a_full + T8_A_ST;
  uint64_t* acc_full = a_empty + T8_A_ST;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* b1_full = acc_empty + 2;
  uint64_t* b2_full = b1_full + 1;
  uint32_t* tmem_slot = (uint32_t*)(smem + T8Smem::tmem);
  float* linv = (float*)(smem + T8Smem::linv);
  int* spair = (int*)(smem + T8Smem::spair);
  float* sinv = (float*)(smem + T8Smem::sinv);
  __shared__ DecodePlan pl;
  // the plan's counting-sort scratch lives in the raw ring, which no copy touches before the plan is built
  int* ecnt = (int*)raw;
  int* ebase = ecnt + TC_MAX_E;
  int* esegb = ebase + TC_MAX_E;
  __shared__ float c_w[DEC_MAX_PAIRS];
  __shared__ unsigned char c_ok[DEC_MAX_PAIRS];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = a.M * a.k, G = gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < T8_RAW_ST; ++s) {
      mbar_init(raw_full + s, 1);
      mbar_init(raw_empty + s, 2);
    }
    for (int s = 0; s < T8_A_ST; ++s) {
      mbar_init(a_full + s, 2);
      mbar_init(a_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(acc_full + s, 1);
      mbar_init(acc_empty + s, 4);
    }
    mbar_init(b1_full, 1);
    mbar_init(b2_full, 1);
    mbar_init(b2_full + 1, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, T8_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // programmatic dependent launch: inputs and the workspace are touched only after the previous grid has completed
  allow_dependents();
  grid_dependency_wait();
  const long long my_id = tid < P ? a.ids[tid] : 0;
  const float my_w = tid < P ? a.weights[tid] : 0.0f;
  tc_plan(pl, ecnt, ebase, esegb, my_id, P, a.E, TC_CAP, a.e_first, a.e_count);
  if (tid < P) {
    c_ok[tid] = my_id >= a.e_first && my_id < (long long)a.e_first + a.e_count && my_id < a.E;
    c_w[tid] = my_w;
  }
  const int nseg = pl.nseg;
  const int t1_lo = (int)((long long)blockIdx.x * nseg * TPS1 / G);
  const int t1_hi = (int)((long long)(blockIdx.x + 1) * nseg * TPS1 / G);
  const int t2_lo = (int)((long long)blockIdx.x * nseg * TPS2 / G);
  const int t2_hi = (int)((long long)(blockIdx.x + 1) * nseg * TPS2 / G);
  const int s2a = t2_lo / TPS2, s2n = t2_hi > t2_lo ? (t2_hi - 1) / TPS2 - s2a + 1 : 0;
  const int nkb = (t1_hi - t1_lo) * NKB1 + (t2_hi - t2_lo) * NKB2;  // this CTA's 128-column groups, both phases
  bool ok = true;
  // few segments: each 128-row block is combined by its last-arriving phase-2 tile (no grid barrier)
  const bool last_arrive = nseg <= a.lastarrive_nseg;

  if (warp == 0) {
    // ---------------- TMA producer: packed rows ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int c = 0;
      for (int t = t1_lo; t < t1_hi && ok; ++t) {
        const int s = t / TPS1, ub = t - s * TPS1, e = pl.seg_expert[s];
        const int grow = e * 2 * I + ub * TC_U1;
        for (int kb = 0; kb < NKB1; ++kb, ++c) {
          const int rs = c % T8_RAW_ST;
          ok = mbar_wait(raw_empty + rs, ((c / T8_RAW_ST) & 1) ^ 1);
          if (!ok) break;
          mbar_arrive_expect_tx(raw_full + rs, T8_RAW_BYTES);
          tma_load_2d_hint(raw + rs * T8_RAW_BYTES, &map13, kb * 64, grow, raw_full + rs, pol);
          tma_load_2d_hint(raw + rs * T8_RAW_BYTES + T8_RAW_BYTES / 2, &map13, kb * 64, grow + I, raw_full + rs, pol);
        }
      }
      for (int t = t2_lo; t < t2_hi && ok; ++t) {
        const int s = t / TPS2, rb = t - s * TPS2, e = pl.seg_expert[s];
        const int row = e * H + rb * TC_R2;
        for (int kb = 0; kb < NKB2; ++kb, ++c) {
          const int rs = c % T8_RAW_ST;
          ok = mbar_wait(raw_empty + rs, ((c / T8_RAW_ST) & 1) ^ 1);
          if (!ok) break;
          mbar_arrive_expect_tx(raw_full + rs, T8_RAW_BYTES);
          tma_load_2d_hint(raw + rs * T8_RAW_BYTES, &map2, kb * 64, row, raw_full + rs, pol);
        }
      }
      // every issued copy lands before this thread leaves (bounded)
      for (int d = max(0, c - T8_RAW_ST); d < c; ++d)
        if (!mbar_wait(raw_full + d % T8_RAW_ST, (d / T8_RAW_ST) & 1)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: a tile's groups (4 MMAs of K = 32 each) into its 16-column TMEM regions ----------
    if (lane == 0) {
      const uint32_t a_s = smem_u32(astage), b_s = smem_u32(breg);
      const uint32_t idesc = t8_idesc(TC_CAP);
      int c = 0, tn = 0;
      if (t1_hi > t1_lo) ok = mbar_wait(b1_full, 0);
      tc_fence_after();
      auto tile = [&](uint32_t bbase, int nk) {
        const int buf = tn & 1;
        ok = mbar_wait(acc_empty + buf, ((tn >> 1) & 1) ^ 1);
        tc_fence_after();
        for (int kb = 0; kb < nk && ok; ++kb, ++c) {
          const int st = c % T8_A_ST;
          ok = mbar_wait(a_full + st, (c / T8_A_ST) & 1);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_i8(tmem + buf * T8_BUF_COLS + kb * 16, umma_desc_sw128(a_s + st * TC_ABYTES + 32 * ks),
                    umma_desc_sw128(bbase + kb * TC_CAP * 128 + 32 * ks), idesc, ks != 0 ? 1u : 0u);
          umma_commit(a_empty + st);
        }
        umma_commit(acc_full + buf);
        ++tn;
      };
      for (int t = t1_lo; t < t1_hi && ok; ++t) tile(b_s, NKB1);
      int cur = -1;
      for (int t = t2_lo; t < t2_hi && ok; ++t) {
        const int s = t / TPS2, bb = s - s2a;
        if (bb > 1) {
          record_fault(FAULT_WAIT_TIMEOUT);
          break;
        }
        if (s != cur) {
          ok = mbar_wait(b2_full + bb, 0);
          if (!ok) break;
          tc_fence_after();
          cur = s;
        }
        tile(b_s + bb * B2BYTES, NKB2);
      }
    }
  } else if (warp >= 6) {
    // ---------------- converters: packed int4 stage -> int8 A stage ----------------
    const int ct = tid - T8_CONV0;
    for (int c = 0; c < nkb; ++c) {
      const int rs = c % T8_RAW_ST, st = c % T8_A_ST;
      if (ok) ok = mbar_wait(raw_full + rs, (c / T8_RAW_ST) & 1);
      if (ok) ok = mbar_wait(a_empty + st, ((c / T8_A_ST) & 1) ^ 1);
      const uint8_t* src = raw + rs * T8_RAW_BYTES;
      uint8_t* dst = astage + st * TC_ABYTES;
      if (ok) {
        // all 8 loads first: stores to the A stage could alias them for all the compiler knows
        uint4 w[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) w[m] = *reinterpret_cast<const uint4*>(src + 16 * (ct + 64 * m));
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int u = ct + 64 * m, row = u >> 2, ch = u & 3;  // 16 packed bytes: 32 columns of one row
          const uint4 lo = make_uint4((w[m].x << 4) & 0xF0F0F0F0u, (w[m].y << 4) & 0xF0F0F0F0u,
                                      (w[m].z << 4) & 0xF0F0F0F0u, (w[m].w << 4) & 0xF0F0F0F0u);
          const uint4 hi = make_uint4(w[m].x & 0xF0F0F0F0u, w[m].y & 0xF0F0F0F0u, w[m].z & 0xF0F0F0F0u,
                                      w[m].w & 0xF0F0F0F0u);
          *reinterpret_cast<uint4*>(dst + tc_b_offset(128, row, 2 * ch)) = lo;
          *reinterpret_cast<uint4*>(dst + tc_b_offset(128, row, 2 * ch + 1)) = hi;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(a_full + st);
        mbar_arrive(raw_empty + rs);
      }
    }
  }
  if (warp >= 2) {
    // ---------------- helpers (warps 2-5: staging and epilogue; 2-7: barriers and combine) ----------------
    const int hid = tid - TC_HELP0;
    int tn = 0;  // tile sequence (TMEM buffer tn & 1)
    if (warp < 6) {
      const int hw = warp - 2, quarter = warp & 3, row = 32 * quarter + lane;
      const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
      // phase-1 B: every line quantized to int8, one warp per line (lines past M stay unwritten: never read)
      if (t1_hi > t1_lo) {
        // the warp's lines hw, hw + 4, ...; a lane holds columns 32 lane .. + 31 and 1024 + 32 lane .. + 31 of a
        // line. The loads of NB lines are issued together, then the lines are quantized one by one.
        constexpr int EB = XBF ? 2 : 4, XW = 64 * EB / 16, NB = XBF ? 4 : 1;
        for (int n0 = hw; n0 < a.M; n0 += 4 * NB) {
          uint4 xr[NB][XW];
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const int n = n0 + 4 * b;
#pragma unroll
            for (int w = 0; w < XW; ++w) {
              const int u = w / (XW / 2), k = w % (XW / 2);
              xr[b][w] = n < a.M ? __ldcg(reinterpret_cast<const uint4*>(
                                       (const uint8_t*)a.x + ((size_t)n * H + 32 * (lane + 32 * u)) * EB + 16 * k))
                                 : make_uint4(0u, 0u, 0u, 0u);
            }
          }
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const int n = n0 + 4 * b;
            if (n >= a.M) break;
            float v[2][32];
            float m = 0.0f;
#pragma unroll
            for (int w = 0; w < XW; ++w) {
              const int u = w / (XW / 2), k = w % (XW / 2);
              const uint32_t ww[4] = {xr[b][w].x, xr[b][w].y, xr[b][w].z, xr[b][w].w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                if (XBF) {
                  v[u][8 * k + 2 * h] = bf16_to_f32(ww[h] & 0xFFFFu);
                  v[u][8 * k + 2 * h + 1] = bf16_to_f32(ww[h] >> 16);
                } else {
                  v[u][4 * k + h] = __uint_as_float(ww[h]);
                }
              }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
              for (int i = 0; i < 32; ++i) m = fmaxf(m, fabsf(v[u][i]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float s = __fdiv_rn(m, 127.0f);
#pragma unroll
            for (int u = 0; u < 2; ++u) t8_write_chunk(breg, TC_LINES, n, lane + 32 * u, v[u], s);
            if (lane == 0) linv[n] = s;
          }
        }
        fence_async_smem();
        named_sync(3, TC_EPI);
        if (tid == TC_HELP0) mbar_arrive(b1_full);
      }
      // phase-1 epilogue: per tile, the 16 groups folded with each row's bf16 group scales, then SwiGLU
      unsigned* seg_done = a.arrive;
      for (int t = t1_lo; t < t1_hi; ++t) {
        const int s = t / TPS1, ub = t - s * TPS1, e = pl.seg_expert[s];
        const int i = ub * TC_U1 + (row & (TC_U1 - 1));
        const size_t wrow = (size_t)e * 2 * I + (row < TC_U1 ? i : I + i);
        const uint4* gp = reinterpret_cast<const uint4*>((const uint16_t*)a.s13 + wrow * NKB1);
        const uint4 g0 = __ldg(gp), g1 = __ldg(gp + 1);
        const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        float acc[TC_LINES];
        t8_fold<NKB1>(acc, gw, tmem + lane_base, tn, acc_full, acc_empty, ok, lane);
        ++tn;
#pragma unroll
        for (int l = 0; l < TC_LINES; ++l) xchg[row * TC_XPITCH + l] = ok ? acc[l] : 0.0f;
        named_sync(3, TC_EPI);
        if (row < TC_U1) {
          const int first = pl.seg_first[s], cnt = pl.seg_count[s];
          for (int j = 0; j < cnt; ++j) {
            const int pair = pl.sorted[first + j], line = pair / a.k;
            const float sl = linv[line] * 0.0625f;  // the A bytes hold 16 x the codes
            a.a1[(size_t)pair * I + i] = swiglu_fast(xchg[row * TC_XPITCH + line] * sl,
                                                     xchg[(row + TC_U1) * TC_XPITCH + line] * sl);
          }
        }
        named_sync(3, TC_EPI);
        if (tid == TC_HELP0) {
          __threadfence();
          atomicAdd(seg_done + s, 1u);
        }
      }
      // phase-2 B, segment by segment (at most two): once every phase-1 tile of the segment is done (bounded
      // wait), its pairs' a1 rows quantized to int8, one warp per row
      __shared__ int s_ready;
      for (int bb = 0; bb < s2n; ++bb) {
        const int s = s2a + bb, cnt = pl.seg_count[s], first = pl.seg_first[s];
        if (tid == TC_HELP0) {
          int okw = 1;
          unsigned seen;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(seg_done + s) : "memory");
          if (seen < (unsigned)TPS1) {
            const unsigned long long start = globaltimer();
            while (true) {
              asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(seg_done + s) : "memory");
              if (seen >= (unsigned)TPS1) break;
              if (globaltimer() - start > WAIT_LIMIT_NS) {
                record_fault(FAULT_WAIT_TIMEOUT);
                okw = 0;
                break;
              }
            }
          }
          s_ready = okw;
        }
        named_sync(3, TC_EPI);
        ok = ok && s_ready;
        for (int j = hw; j < cnt; j += 4) {
          const int pair = pl.sorted[first + j];
          constexpr int CH = I / 32;  // 32-column chunks a row (<= 24: one per lane)
          float v[32];
          float m = 0.0f;
          if (lane < CH) {
            t8_load32(a.a1, false, (size_t)pair * I + 32 * lane, v);
#pragma unroll
            for (int q = 0; q < 32; ++q) m = fmaxf(m, fabsf(v[q]));
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          const float sc = __fdiv_rn(m, 127.0f);
          if (lane < CH) t8_write_chunk(breg + bb * B2BYTES, TC_CAP, j, lane, v, sc);
          if (lane == 0) {
            spair[bb * TC_CAP + j] = pair;
            sinv[bb * TC_CAP + j] = sc * 0.0625f;
          }
        }
        fence_async_smem();
        named_sync(3, TC_EPI);
        if (tid == TC_HELP0) mbar_arrive(b2_full + bb);
      }
      // phase-2 epilogue: parts[pair, row] = sum over groups of group scale x int32 sum, x the pair's scale / 16
      for (int t = t2_lo; t < t2_hi; ++t) {
        const int s = t / TPS2, rb = t - s * TPS2, bb = s - s2a, e = pl.seg_expert[s];
        const int r = rb * TC_R2 + row;
        const uint32_t* gp = reinterpret_cast<const uint32_t*>((const uint16_t*)a.s2 + ((size_t)e * H + r) * NKB2);
        uint32_t gw[NKB2 / 2];
#pragma unroll
        for (int q = 0; q < NKB2 / 2; ++q) gw[q] = __ldg(gp + q);
        float acc[TC_CAP];
        t8_fold<NKB2>(acc, gw, tmem + lane_base, tn, acc_full, acc_empty, ok, lane);
        ++tn;
        if (ok && bb <= 1) {
          const int cnt = pl.seg_count[s];
#pragma unroll
          for (int j = 0; j < TC_CAP; ++j)
            if (j < cnt) __stcg(a.parts + (size_t)spair[bb * TC_CAP + j] * H + r, acc[j] * sinv[bb * TC_CAP + j]);
        }
        if (last_arrive) tc_block_done(a, c_ok, c_w, rb, nseg, ok);
      }
    }
    if (last_arrive) {
      // the row blocks were combined by their last tiles; the last CTA out clears the counters for the next call
      tc_exit_count(a, nseg, G);
    } else {
    // every CTA's parts are written; each CTA combines an even share of the columns
    ok = grid_barrier<TC_HELPERS, TC_HELP0>(a.barrier, G) && ok;
    if (blockIdx.x == 0)
      for (int s = hid; s < nseg; s += TC_HELPERS) a.arrive[s] = 0u;  // the segment counters, for the next call
    int q0, q1;
    split_range(H / 4, blockIdx.x, G, q0, q1);
    combine_columns(a, c_ok, c_w, 4 * q0, 4 * q1, ok, TC_HELP0, TC_HELPERS);
    if (a.ex) {
      // exchange: once every CTA has pushed its columns, raise this rank's flag on every rank
      named_sync(2, TC_HELPERS);
      if (tid == TC_HELP0 && ep_geometry_ok(*a.ex, a.M, H)) {
        __threadfence_system();
        if (atomicAdd(a.ep_done, 1u) + 1u == (unsigned)G) {
          tc_raise_flags(*a.ex);
          *a.ep_done = 0u;
        }
      }
    }
    }  // grid-barrier combine
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, T8_TMEM_COLS);
  }
}

}  // namespace d3
