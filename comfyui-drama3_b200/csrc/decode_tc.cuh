// The routed-expert decode of M <= 16 lines on the 5th-generation tensor cores, for e4m3 rows with per-output-channel
// fp32 scales (the fp8c layout). Same plan, phases, scratch and combine as moe_decode_kernel; what changes is how a
// weight byte meets the activations:
//
//   * the e4m3 weight tiles go from HBM to shared memory by TMA and straight into tcgen05.mma kind::f8f6f4 as the A
//     operand - no conversion, no register fragments;
//   * the activations become the B operand as a sum of e4m3 terms: y = x * 2^e (e per row, so that max|y| lies in
//     [128, 256)), t1 = e4m3(y), t2 = e4m3(y - t1), ... Each term is exact in fp32 and every product of two e4m3
//     numbers is exact, so D = W t1 + W t2 + ... is the fp32 dot product with y rounded to the terms' precision:
//     2 terms hold a bf16 value exactly (8 significant bits, 4 per term) and 3 / 4 terms keep 12 / 16 bits of an
//     fp32 one. The terms sit side by side along N, so one MMA computes all of them;
//   * the accumulators live in TMEM (two buffers, so a tile's epilogue overlaps the next tile's MMAs).
//
// Phase 1 (gate_up + SwiGLU): a tile is 64 gate rows and the matching 64 up rows of one expert (M = 128) over all H
// columns; B holds every line's terms (N = 16 lines x terms), staged once per call, so a segment needs no staging of
// its own - the epilogue picks the columns of the segment's lines. Phase 2 (down): a tile is 128 down rows over all I
// columns; B holds the segment's pairs' a1 rows (N = 16 pairs x 4 terms), two segments' worth. The work of each phase
// is split across the grid by whole tiles, in proportion, so a CTA's phase-2 segments are mostly its own phase-1 ones.
// Between the phases no grid-wide wait: a segment's phase-2 staging waits (bounded) for the count of its finished
// phase-1 tiles. With many segments the combine follows a grid barrier, each CTA taking an even share of the columns;
// with few (one or two lines: DecodeArgs::lastarrive_nseg) each 128-row block is combined by the CTA whose phase-2
// tile completes it, and no CTA waits for the others.
//
// Roles (8 warps): warp 0 lane 0 issues the TMA loads, warp 1 owns TMEM and lane 0 issues the MMAs, warps 2-5 are
// the TMEM epilogue (one warp per lane quarter), warps 2-7 stage the B operands and run the combine.
#pragma once
#include "grouped_mma.cuh"
#include "moe_decode.cuh"

namespace d3 {

#ifdef D3_TRACE
// Trace builds: globaltimer at milestones and clock64 wait totals, kept in shared memory, one row per CTA.
#define TC_STAMP(slot) s_trace[slot] = globaltimer()
#define TC_ADD(slot, v) s_trace[slot] += (v)
#else
#define TC_STAMP(slot)
#define TC_ADD(slot, v)
#endif

constexpr int TC_WARPS = 8;
constexpr int TC_THREADS = TC_WARPS * 32;
constexpr int TC_HELP0 = 64;          // first helper thread (warp 2)
constexpr int TC_HELPERS = 192;       // warps 2-7
constexpr int TC_EPI = 128;           // warps 2-5
constexpr int TC_STAGES = 6;          // A ring depth
constexpr int TC_ABYTES = 16384;      // one A stage: 128 rows x 128 bytes
constexpr int TC_U1 = 64;             // phase-1 units (a gate row and its up row) per tile
constexpr int TC_R2 = 128;            // phase-2 rows per tile
constexpr int TC_LINES = 16;          // phase-1 B rows per term: the (at most 16) lines
constexpr int TC_CAP = 16;            // pairs per segment
constexpr int TC_TERMS2 = 4;          // phase-2 terms (a1 is fp32)
constexpr int TC_N2 = TC_CAP * TC_TERMS2;
constexpr int TC_BREGION = 98304;     // phase-1 B (<= 48 rows x 2048) or two phase-2 B buffers (64 rows x <= 768)
constexpr int TC_XPITCH = 17;         // exchange row pitch (floats)
constexpr int TC_TMEM_COLS = 128;     // two accumulators of <= 64 columns
constexpr int TC_MAX_E = 512;         // experts per rank the plan's counting sort holds
constexpr int TC_I8_TERMS = 3;        // int8 activation terms: about 22 bits of the row maximum (two, 15 bits, measured
                                      // 1.25e-3 rel-L2 on bf16 outputs at one line)

struct TcSmem {
  static constexpr int ring = 0;
  static constexpr int breg = ring + TC_STAGES * TC_ABYTES;
  static constexpr int xchg = breg + TC_BREGION;                       // float [128][17]
  static constexpr int bars = xchg + 128 * TC_XPITCH * 4;              // 19 mbarriers
  static constexpr int tmem = bars + 24 * 8;
  static constexpr int linv = tmem + 16;                               // float [16]: phase-1 line scales
  static constexpr int lmax = linv + 64;                               // int [16]
  static constexpr int spair = lmax + 64;                              // int [2][16]: phase-2 B rows' pairs
  static constexpr int sinv = spair + 128;                             // float [2][16]
  static constexpr int smax = sinv + 128;                              // int [2][16]
  static constexpr int end = smax + 128;
  static constexpr int launch = end + 1024;                            // + alignment slack
};

// Instruction descriptor, kind::f8f6f4: f32 accumulator, e4m3 A and B, both K-major, M = 128, N = n.
D3_DEV uint32_t tc_idesc(int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24); }

D3_DEV void umma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One MMA of the tensor-core decode: kind::i8 (s32 accumulators) for int8 rows, kind::f8f6f4 (f32) for e4m3 rows.
template <bool I8>
D3_DEV void tc_umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  if constexpr (I8)
    umma_i8(tmem_d, adesc, bdesc, idesc, accumulate);
  else
    umma_f8(tmem_d, adesc, bdesc, idesc, accumulate);
}

// 2-D tiled TMA load with an L2 cache hint.
D3_DEV void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Two fp32 -> packed e4m3 x2 (round to nearest even, saturating): `lo` in the low byte.
D3_DEV uint32_t f32x2_e4m3(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Packed e4m3 x2 -> the two values as fp32 (exact).
D3_DEV float2 e4m3x2_f32(uint32_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Byte offset of (row n, 16-byte chunk q of the K bytes) in a K-major, 128-byte-swizzled operand of `rows` rows:
// 128-column blocks of rows x 128 bytes, 8-row atoms of 1024 bytes, chunk index XOR (row % 8).
D3_DEV uint32_t tc_b_offset(int rows, int n, int q) {
  return (uint32_t)((q >> 3) * rows * 128 + (n >> 3) * 1024 + (n & 7) * 128 + (((q & 7) ^ (n & 7)) << 4));
}

// Power-of-two scale for a row of maximum magnitude m: m * 2^e in [128, 256) (1 for an all-zero row).
D3_DEV int tc_exponent(float m) {
  if (!(m > 0.0f) || !(m < 3.0e38f)) return 0;
  const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
  return min(100, max(-100, 7 - ex));
}

// 16 consecutive values of a row as `terms` e4m3 terms of y = v * scale, written as 16-byte chunks: term t of the
// row goes to B row t * tstride + n.
template <int TERMS>
D3_DEV void tc_write_terms(uint8_t* b, int rows, int n, int tstride, int q, const float (&v)[16], float scale) {
  float y[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) y[i] = v[i] * scale;
#pragma unroll
  for (int t = 0; t < TERMS; ++t) {
    uint32_t w[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t lo = f32x2_e4m3(y[4 * p], y[4 * p + 1]), hi = f32x2_e4m3(y[4 * p + 2], y[4 * p + 3]);
      w[p] = lo | (hi << 16);
      if (t + 1 < TERMS) {
        const float2 a = e4m3x2_f32(lo), c = e4m3x2_f32(hi);
        y[4 * p] -= a.x;
        y[4 * p + 1] -= a.y;
        y[4 * p + 2] -= c.x;
        y[4 * p + 3] -= c.y;
      }
    }
    *reinterpret_cast<uint4*>(b + tc_b_offset(rows, t * tstride + n, q)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ConvRot rotation of 256-column groups held 16 contiguous values a lane: lane L (of a 16-lane group, L = lane % 16)
// holds the group's columns 16 L .. 16 L + 15. H256 = h4 (x) h4 (x) h4 (x) h4 / 16 acts on the four base-4 digits of
// the column index: the two low ones inside the lane, the two high ones across lanes. One radix-4 stage of h4
// (rows [1,1,1,-1], [1,1,-1,1], [1,-1,1,1], [-1,1,1,1]) gives output p = (sum of the four inputs) - 2 x input 3 - p.
// The stages run in the reference's order (digit 0 first); float results agree with it to rounding.
D3_DEV void tc_h4_regs(float (&v)[16], int base, int stride) {
  const float a = v[base], b = v[base + stride], c = v[base + 2 * stride], d = v[base + 3 * stride];
  const float s = (a + b) + (c + d);
  v[base] = s - 2.0f * d;
  v[base + stride] = s - 2.0f * c;
  v[base + 2 * stride] = s - 2.0f * b;
  v[base + 3 * stride] = s - 2.0f * a;
}

D3_DEV float tc_h4_lanes(float v, int x1, int x2, int mirror) {
  float s = v + __shfl_xor_sync(0xffffffffu, v, x1);
  s += __shfl_xor_sync(0xffffffffu, s, x2);
  return s - 2.0f * __shfl_xor_sync(0xffffffffu, v, mirror);
}

// The whole warp calls it (shuffles); each 16-lane half rotates its own group.
D3_DEV void tc_rotate16(float (&v)[16]) {
#pragma unroll
  for (int b = 0; b < 16; b += 4) tc_h4_regs(v, b, 1);
#pragma unroll
  for (int i = 0; i < 4; ++i) tc_h4_regs(v, i, 4);
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = tc_h4_lanes(v[i], 1, 2, 3);
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = 0.0625f * tc_h4_lanes(v[i], 4, 8, 12);
}

// Power-of-two scale for int8 terms: m * 2^e in [32, 64) (1 for an all-zero row).
D3_DEV int tc_exponent_i8(float m) {
  if (!(m > 0.0f) || !(m < 3.0e38f)) return 0;
  const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
  return min(100, max(-100, 5 - ex));
}

// 16 consecutive values of a row as TERMS int8 terms of y = v * scale (|y| < 64): t1 = rint(y), t2 = rint(128 (y -
// t1)), t3 = rint(128 (128 (y - t1) - t2)), so y = t1 + t2 / 128 (+ t3 / 16384) to within 2^-8 (2^-15); term t of
// the row goes to B row t * tstride + n as 16-byte chunks of a K-major, 128-byte-swizzled operand.
template <int TERMS>
D3_DEV void tc_write_i8_terms(uint8_t* b, int rows, int n, int tstride, int q, const float (&v)[16], float scale) {
  uint32_t w[TERMS][4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
#pragma unroll
    for (int t = 0; t < TERMS; ++t) w[t][p] = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float r = v[4 * p + i] * scale;
#pragma unroll
      for (int t = 0; t < TERMS; ++t) {
        const float q8 = fminf(127.0f, fmaxf(-127.0f, rintf(r)));
        w[t][p] |= ((uint32_t)(int)q8 & 0xFFu) << (8 * i);
        r = (r - q8) * 128.0f;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < TERMS; ++t)
    *reinterpret_cast<uint4*>(b + tc_b_offset(rows, t * tstride + n, q)) = make_uint4(w[t][0], w[t][1], w[t][2], w[t][3]);
}

// The s32 accumulators of TERMS int8 terms as one float: D1 + D2 / 128 (+ D3 / 16384); each |D| < 2^24, exact.
template <int TERMS>
D3_DEV float tc_i8_sum(const float* v, int stride) {
  float sum = (float)__float_as_int(v[0]) + (float)__float_as_int(v[stride]) * 0.0078125f;
  if constexpr (TERMS > 2) sum += (float)__float_as_int(v[2 * stride]) * 6.103515625e-05f;
  return sum;
}

D3_DEV void tc_load16(const void* src, bool bf16, size_t i, float (&v)[16]) {
  if (bf16) {
    const uint4* p = reinterpret_cast<const uint4*>((const uint16_t*)src + i);
    const uint4 a = __ldcg(p), b = __ldcg(p + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      v[2 * u] = bf16_to_f32(w[u] & 0xFFFFu);
      v[2 * u + 1] = bf16_to_f32(w[u] >> 16);
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>((const float*)src + i);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4 f = __ldcg(p + u);
      v[4 * u] = f.x;
      v[4 * u + 1] = f.y;
      v[4 * u + 2] = f.z;
      v[4 * u + 3] = f.w;
    }
  }
}

// The plan by counting sort (all TC_THREADS threads; `id` is pair tid's expert id, loaded by the caller): pairs
// grouped by expert in expert order, segments of one expert and at most `cap` pairs. Within an expert the pairs
// keep the order their atomic slots came in - every MMA column is computed on its own, so the order changes no
// result. ecnt / ebase / esegb: shared scratch of TC_MAX_E ints each (e_count <= TC_MAX_E, checked by the host).
D3_DEV void tc_plan(DecodePlan& pl, int* ecnt, int* ebase, int* esegb, long long id, int P, int E, int cap,
                    int e_first, int e_count) {
  const int tid = threadIdx.x, lane = tid & 31;
  for (int e = tid; e < e_count; e += TC_THREADS) ecnt[e] = 0;
  int key = -1;
  if (tid < P) {
    if (id < 0 || id >= E) record_fault(FAULT_BAD_EXPERT);
    if (id >= e_first && id < (long long)e_first + e_count && id < E) key = (int)(id - e_first);
  }
  __syncthreads();
  const int slot = key >= 0 ? atomicAdd(ecnt + key, 1) : 0;
  __syncthreads();
  if (tid < 32) {
    // exclusive scans of the pair counts and the segment counts: lane L takes experts 16L .. 16L + 15
    int pc[TC_MAX_E / 32], sc[TC_MAX_E / 32];
    int ps = 0, ss = 0;
#pragma unroll
    for (int i = 0; i < TC_MAX_E / 32; ++i) {
      const int e = (TC_MAX_E / 32) * lane + i;
      const int n = e < e_count ? ecnt[e] : 0;
      pc[i] = n;
      sc[i] = (n + cap - 1) / cap;
      ps += pc[i];
      ss += sc[i];
    }
    int pi = ps, si = ss;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, pi, o), b = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) {
        pi += a;
        si += b;
      }
    }
    int pb = pi - ps, sb = si - ss;
#pragma unroll
    for (int i = 0; i < TC_MAX_E / 32; ++i) {
      const int e = (TC_MAX_E / 32) * lane + i;
      if (e < e_count) {
        ebase[e] = pb;
        esegb[e] = sb;
      }
      pb += pc[i];
      sb += sc[i];
    }
    if (lane == 31) pl.nseg = si;
  }
  __syncthreads();
  if (key >= 0) pl.sorted[ebase[key] + slot] = tid;
  for (int e = tid; e < e_count; e += TC_THREADS) {
    const int n = ecnt[e];
    for (int j = 0; j * cap < n; ++j) {
      const int s = esegb[e] + j;
      pl.seg_expert[s] = e;
      pl.seg_first[s] = ebase[e] + j * cap;
      pl.seg_count[s] = min(cap, n - j * cap);
    }
  }
  __syncthreads();
}

// Raise this rank's flag for the current call on every rank of the exchange (after its partial is pushed).
D3_DEV void tc_raise_flags(const EpExchange& ex) {
  const unsigned ep = *(volatile const unsigned*)ex.epoch + 1u;
  __threadfence_system();
  for (int r = 0; r < ex.world; ++r) {
    unsigned* f = ex.flags[r] + (ep & 1u) * EP_MAX_RANKS + ex.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(ep) : "memory");
  }
}

// Combine by last arrival (few segments): once a phase-2 tile's parts rows are written, the epilogue threads (TC_EPI,
// from TC_HELP0) count the tile for its 128-row block; the tile that completes the block (one per segment) combines
// those rows, with the same arithmetic as the grid-wide combine, so the output is the same bit for bit. With the
// peer exchange, the block's rows go to every rank, and the block that completes all H / 128 raises the flags.
// Counters: a.blocks[rb] (reset by the block's combiner) and a.ep_done (reset by the flag raiser).
D3_DEV void tc_block_done(const DecodeArgs& a, const unsigned char* c_ok, const float* c_w, int rb, int nseg,
                          bool ok) {
  __shared__ int s_last;
  named_sync(3, TC_EPI);
  if (threadIdx.x == TC_HELP0) {
    __threadfence();
    s_last = atomicAdd(a.blocks + rb, 1u) + 1u == (unsigned)nseg;
  }
  named_sync(3, TC_EPI);
  if (!s_last) return;  // the same value in every participant
  __threadfence();
  combine_columns(a, c_ok, c_w, rb * TC_R2, rb * TC_R2 + TC_R2, ok, TC_HELP0, TC_EPI);
  named_sync(3, TC_EPI);
  if (threadIdx.x == TC_HELP0) {
    a.blocks[rb] = 0u;  // every tile of the block has counted: nothing adds to it again in this call
    if (a.ex && ep_geometry_ok(*a.ex, a.M, DEC_H)) {
      __threadfence_system();
      if (atomicAdd(a.ep_done, 1u) + 1u == (unsigned)(DEC_H / TC_R2)) {
        tc_raise_flags(*a.ex);
        *a.ep_done = 0u;
      }
    }
  }
}

// Combine by last arrival: every helper of this CTA is past its staging waits and combines; the last CTA to get
// here clears the segment counters (a.arrive) and this count (a.depart[0]) for the next call.
D3_DEV void tc_exit_count(const DecodeArgs& a, int nseg, int G) {
  named_sync(1, TC_HELPERS);
  if (threadIdx.x == TC_HELP0) {
    __threadfence();
    if (atomicAdd(a.depart, 1u) + 1u == (unsigned)G) {
      for (int s = 0; s < nseg; ++s) a.arrive[s] = 0u;
      a.depart[0] = 0u;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// FMT: FMT_FP8C (e4m3 rows, kind::f8f6f4, e4m3 activation terms) or FMT_I8 (int8 ConvRot rows, kind::i8: the
// activation rows rotated while staged and written as three int8 terms, s32 accumulators).
template <int FMT, bool XBF, int NKB2>
__global__ void __launch_bounds__(TC_THREADS, 1)
    moe_decode_tc_kernel(const __grid_constant__ CUtensorMap map13, const __grid_constant__ CUtensorMap map2,
                         const DecodeArgs a) {
  constexpr bool I8 = FMT == FMT_I8;
  constexpr int T1 = I8 ? TC_I8_TERMS : XBF ? 2 : 3;  // phase-1 terms
  constexpr int N1 = TC_LINES * T1;         // 32 / 48
  constexpr int T2 = I8 ? TC_I8_TERMS : TC_TERMS2;  // phase-2 terms
  constexpr int N2 = TC_CAP * T2;           // 48 / 64
  constexpr int H = DEC_H, NKB1 = H / 128;  // 16 column blocks in phase 1
  constexpr int I = NKB2 * 128;
  constexpr int TPS1 = I / TC_U1, TPS2 = H / TC_R2;
  constexpr int B2BYTES = N2 * I;           // one phase-2 B buffer

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ring = smem + TcSmem::ring;
  uint8_t* breg = smem + TcSmem::breg;
  float* xchg = (float*)(smem + TcSmem::xchg);
  uint64_t* bars = (uint64_t*)(smem + TcSmem::bars);
  uint64_t* full = bars;
  uint64_t* empty = bars + TC_STAGES;
  uint64_t* acc_full = bars + 2 * TC_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* b1_full = acc_empty + 2;
  uint64_t* b2_full = b1_full + 1;
  uint32_t* tmem_slot = (uint32_t*)(smem + TcSmem::tmem);
  float* linv = (float*)(smem + TcSmem::linv);
  int* lmax = (int*)(smem + TcSmem::lmax);
  int* spair = (int*)(smem + TcSmem::spair);
  float* sinv = (float*)(smem + TcSmem::sinv);
  int* smax = (int*)(smem + TcSmem::smax);
  __shared__ DecodePlan pl;
  __shared__ int ecnt[TC_MAX_E], ebase[TC_MAX_E], esegb[TC_MAX_E];
  __shared__ float c_w[DEC_MAX_PAIRS];
  __shared__ unsigned char c_ok[DEC_MAX_PAIRS];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = a.M * a.k, G = gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(acc_full + s, 1);
      mbar_init(acc_empty + s, 4);
      mbar_init(b2_full + s, 1);
    }
    mbar_init(b1_full, 1);
    fence_mbar_init();
  }
  if (tid < 16) lmax[tid] = 0;
  if (tid < 32) smax[tid] = 0;
#ifdef D3_TRACE
  if (tid < 32) s_trace[tid] = 0;
#endif
  if (warp == 1) tmem_alloc(tmem_slot, TC_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) TC_STAMP(0);
  // programmatic dependent launch: inputs and the workspace are touched only after the previous grid has completed
  allow_dependents();
  grid_dependency_wait();
  if (tid == 0) TC_STAMP(12);
  // phase-1 B rows (lines) of this helper warp: hw, hw + 6, hw + 12; their loads are issued before the plan is built
  // (bf16: all three rows; fp32: the first), so they land while it is
  constexpr int XW = XBF ? 2 : 4;  // 16-byte words per 16-column chunk
  constexpr int PRE = XBF ? 3 : 1;
  const int hw = warp - 2;
  uint4 xr[PRE][4][XW];
  if (warp >= 2) {
#pragma unroll
    for (int r = 0; r < PRE; ++r) {
      const int n = hw + 6 * r;
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < XW; ++w)
          xr[r][u][w] = (n < TC_LINES && n < a.M)
                            ? __ldcg(reinterpret_cast<const uint4*>((const uint8_t*)a.x +
                                                                     ((size_t)n * H + 16 * (lane + 32 * u)) * (XBF ? 2 : 4)) + w)
                            : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  // phase-1 B (warps 2-7, after the plan): every line's terms, one warp per line; the warp holds the whole row, so
  // the row maximum is a warp reduction
  auto stage_b1 = [&]() {
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        const int n = hw + 6 * r;
        if (n >= TC_LINES || n >= a.M) break;  // rows past M stay unwritten: the epilogue never reads their columns
        uint4 cur[4][XW];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int w = 0; w < XW; ++w)
            cur[u][w] = r < PRE ? xr[r < PRE ? r : 0][u][w]
                        : (n < a.M ? __ldcg(reinterpret_cast<const uint4*>((const uint8_t*)a.x +
                                                                           ((size_t)n * H + 16 * (lane + 32 * u)) * 4) + w)
                                   : make_uint4(0u, 0u, 0u, 0u));
        float v[4][16];
        float m = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (XBF) {
#pragma unroll
            for (int w = 0; w < 2; ++w) {
              const uint32_t ww[4] = {cur[u][w].x, cur[u][w].y, cur[u][w].z, cur[u][w].w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                v[u][8 * w + 2 * h] = bf16_to_f32(ww[h] & 0xFFFFu);
                v[u][8 * w + 2 * h + 1] = bf16_to_f32(ww[h] >> 16);
              }
            }
          } else {
#pragma unroll
            for (int w = 0; w < XW; ++w) {
              v[u][4 * w] = __uint_as_float(cur[u][w].x);
              v[u][4 * w + 1] = __uint_as_float(cur[u][w].y);
              v[u][4 * w + 2] = __uint_as_float(cur[u][w].z);
              v[u][4 * w + 3] = __uint_as_float(cur[u][w].w);
            }
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[u][i]));
        }
        if constexpr (I8) {
          // ConvRot: the row in the weights' rotated basis (lanes 16h .. 16h + 15 hold group 2u + h), then its max
          m = 0.0f;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            tc_rotate16(v[u]);
#pragma unroll
            for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[u][i]));
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const int e = I8 ? tc_exponent_i8(m) : tc_exponent(m);
        const float scale = __uint_as_float((uint32_t)(e + 127) << 23);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if constexpr (I8)
            tc_write_i8_terms<T1>(breg, N1, n, TC_LINES, lane + 32 * u, v[u], scale);
          else
            tc_write_terms<T1>(breg, N1, n, TC_LINES, lane + 32 * u, v[u], scale);
        }
        if (lane == 0) linv[n] = __uint_as_float((uint32_t)(127 - e) << 23);
      }
      fence_async_smem();
      named_sync(1, TC_HELPERS);
      if (tid == TC_HELP0) {
        mbar_arrive(b1_full);
        TC_STAMP(2);
      }
  };
  const long long my_id = tid < P ? a.ids[tid] : 0;
  const float my_w = tid < P ? a.weights[tid] : 0.0f;
  if (tid == 0) TC_STAMP(13);
  tc_plan(pl, ecnt, ebase, esegb, my_id, P, a.E, TC_CAP, a.e_first, a.e_count);
  if (tid == 0) TC_STAMP(14);
  if (tid < P) {
    c_ok[tid] = my_id >= a.e_first && my_id < (long long)a.e_first + a.e_count && my_id < a.E;
    c_w[tid] = my_w;
  }
  if (warp >= 2) stage_b1();
  const int nseg = pl.nseg;
  const int t1_lo = (int)((long long)blockIdx.x * nseg * TPS1 / G);
  const int t1_hi = (int)((long long)(blockIdx.x + 1) * nseg * TPS1 / G);
  const int t2_lo = (int)((long long)blockIdx.x * nseg * TPS2 / G);
  const int t2_hi = (int)((long long)(blockIdx.x + 1) * nseg * TPS2 / G);
  // phase-2 segments of this CTA: at most two (its range is at most TPS2 tiles when nseg <= G, which the host checks)
  const int s2a = t2_lo / TPS2, s2n = t2_hi > t2_lo ? (t2_hi - 1) / TPS2 - s2a + 1 : 0;
  bool ok = true;
  // few segments: each 128-row block is combined by its last-arriving phase-2 tile (no grid barrier)
  const bool last_arrive = nseg <= a.lastarrive_nseg;
  if (tid == 0) TC_STAMP(1);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int c = 0;
      for (int t = t1_lo; t < t1_hi && ok; ++t) {
        const int s = t / TPS1, ub = t - s * TPS1, e = pl.seg_expert[s];
        const int grow = e * 2 * I + ub * TC_U1;
        for (int kb = 0; kb < NKB1; ++kb, ++c) {
          const int st = c % TC_STAGES;
#ifdef D3_TRACE
          const long long w0 = clock64();
#endif
          ok = mbar_wait(empty + st, ((c / TC_STAGES) & 1) ^ 1);
          TC_ADD(20, clock64() - w0);
          if (!ok) break;
          mbar_arrive_expect_tx(full + st, TC_ABYTES);
          tma_load_2d_hint(ring + st * TC_ABYTES, &map13, kb * 128, grow, full + st, pol);
          tma_load_2d_hint(ring + st * TC_ABYTES + TC_ABYTES / 2, &map13, kb * 128, grow + I, full + st, pol);
        }
      }
      for (int t = t2_lo; t < t2_hi && ok; ++t) {
        const int s = t / TPS2, rb = t - s * TPS2, e = pl.seg_expert[s];
        const int row = e * H + rb * TC_R2;
        for (int kb = 0; kb < NKB2; ++kb, ++c) {
          const int st = c % TC_STAGES;
#ifdef D3_TRACE
          const long long w0 = clock64();
#endif
          ok = mbar_wait(empty + st, ((c / TC_STAGES) & 1) ^ 1);
          TC_ADD(21, clock64() - w0);
          if (!ok) break;
          mbar_arrive_expect_tx(full + st, TC_ABYTES);
          tma_load_2d_hint(ring + st * TC_ABYTES, &map2, kb * 128, row, full + st, pol);
        }
      }
      // every issued copy lands before this thread leaves (bounded)
      for (int d = max(0, c - TC_STAGES); d < c; ++d)
        if (!mbar_wait(full + d % TC_STAGES, (d / TC_STAGES) & 1)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t ring_s = smem_u32(ring), b_s = smem_u32(breg);
      const uint32_t id1 = I8 ? t8_idesc(N1) : tc_idesc(N1), id2 = I8 ? t8_idesc(N2) : tc_idesc(N2);
      int c = 0, tn = 0;
      if (t1_hi > t1_lo) ok = mbar_wait(b1_full, 0);
      TC_STAMP(3);
      tc_fence_after();
      for (int t = t1_lo; t < t1_hi && ok; ++t, ++tn) {
        const int buf = tn & 1;
        ok = mbar_wait(acc_empty + buf, ((tn >> 1) & 1) ^ 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * 64;
        for (int kb = 0; kb < NKB1; ++kb, ++c) {
          const int st = c % TC_STAGES;
#ifdef D3_TRACE
          const long long w0 = clock64();
#endif
          ok = mbar_wait(full + st, (c / TC_STAGES) & 1);
          TC_ADD(22, clock64() - w0);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc_umma<I8>(d, umma_desc_sw128(ring_s + st * TC_ABYTES + 32 * ks),
                        umma_desc_sw128(b_s + kb * N1 * 128 + 32 * ks), id1, (kb | ks) != 0 ? 1u : 0u);
          umma_commit(empty + st);
        }
        umma_commit(acc_full + buf);
      }
      TC_STAMP(4);
      int cur = -1;
      for (int t = t2_lo; t < t2_hi && ok; ++t, ++tn) {
        const int s = t / TPS2, bb = s - s2a;
        if (s != cur) {
          if (bb > 1) {
            record_fault(FAULT_WAIT_TIMEOUT);
            ok = false;
            break;
          }
          ok = mbar_wait(b2_full + bb, 0);
          if (bb == 0) TC_STAMP(7);
          if (!ok) break;
          tc_fence_after();
          cur = s;
        }
        const int buf = tn & 1;
        ok = mbar_wait(acc_empty + buf, ((tn >> 1) & 1) ^ 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * 64;
        for (int kb = 0; kb < NKB2; ++kb, ++c) {
          const int st = c % TC_STAGES;
#ifdef D3_TRACE
          const long long w0 = clock64();
#endif
          ok = mbar_wait(full + st, (c / TC_STAGES) & 1);
          TC_ADD(23, clock64() - w0);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc_umma<I8>(d, umma_desc_sw128(ring_s + st * TC_ABYTES + 32 * ks),
                    umma_desc_sw128(b_s + bb * B2BYTES + kb * N2 * 128 + 32 * ks), id2,
                    (kb | ks) != 0 ? 1u : 0u);
          umma_commit(empty + st);
        }
        umma_commit(acc_full + buf);
      }
      TC_STAMP(8);
    }
  } else {
    // ---------------- helpers: staging, epilogue, combine ----------------
    const int hid = tid - TC_HELP0;  // helper thread 0..191
    unsigned* seg_done = a.arrive;  // per segment: phase-1 tiles finished (all CTAs), zero between calls
    int tn = 0;
    if (warp < 6) {
      // phase-1 epilogue: per tile, every line's gate / up sums, then SwiGLU for the segment's pairs
      const int quarter = warp & 3, row = 32 * quarter + lane;
      const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
      for (int t = t1_lo; t < t1_hi; ++t, ++tn) {
        const int buf = tn & 1;
        if (ok) ok = mbar_wait(acc_full + buf, (tn >> 1) & 1);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: the warp agrees
        tc_fence_after();
        float v[N1];
        if (ok) {
#pragma unroll
          for (int cb = 0; cb < N1 / 16; ++cb) tmem_ld16(tmem + lane_base + buf * 64 + 16 * cb, (float(&)[16])v[16 * cb]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + buf);
#pragma unroll
        for (int l = 0; l < TC_LINES; ++l) {
          float sum = v[l];
          if constexpr (I8) {
            sum = tc_i8_sum<T1>(v + l, TC_LINES);
          } else {
#pragma unroll
            for (int tt = 1; tt < T1; ++tt) sum += v[tt * TC_LINES + l];
          }
          xchg[row * TC_XPITCH + l] = ok ? sum : 0.0f;
        }
        named_sync(3, TC_EPI);
        const int s = t / TPS1;
        if (row < TC_U1) {
          const int ub = t - s * TPS1, e = pl.seg_expert[s];
          const int i = ub * TC_U1 + row;
          const float gsc = __ldg((const float*)a.s13 + (size_t)e * 2 * I + i);
          const float usc = __ldg((const float*)a.s13 + (size_t)e * 2 * I + I + i);
          const int first = pl.seg_first[s], cnt = pl.seg_count[s];
          for (int j = 0; j < cnt; ++j) {
            const int pair = pl.sorted[first + j], line = pair / a.k;
            const float sl = linv[line];
            a.a1[(size_t)pair * I + i] = swiglu_fast(xchg[row * TC_XPITCH + line] * (gsc * sl),
                                                     xchg[(row + TC_U1) * TC_XPITCH + line] * (usc * sl));
          }
        }
        named_sync(3, TC_EPI);
        if (tid == TC_HELP0) {
          // the tile's a1 columns are written (the barrier orders the epilogue's stores before this fence)
          __threadfence();
          atomicAdd(seg_done + s, 1u);
        }
      }
    }
    if (tid == TC_HELP0) TC_STAMP(5);
    // phase-2 B, segment by segment (at most two): once every phase-1 tile of the segment is done (bounded wait),
    // its pairs' a1 rows as 4 terms, two rows per warp (16 lanes a row)
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
        if (bb == 0) TC_STAMP(6);
      }
      named_sync(1, TC_HELPERS);
      ok = ok && s_ready;
      constexpr int CPL = I / 16 / 16;  // chunks per lane (16 lanes a row)
      for (int jp = hw; 2 * jp < cnt; jp += TC_HELPERS / 32) {  // rows past cnt stay unwritten (never read)
        const int j = 2 * jp + (lane >> 4), sub = lane & 15;
        const bool live = j < cnt;
        const int pair = live ? pl.sorted[first + j] : 0;
        float v[CPL][16];
        float m = 0.0f;
#pragma unroll
        for (int u = 0; u < CPL; ++u) {
          if (live) {
            tc_load16(a.a1, false, (size_t)pair * I + 16 * (sub + 16 * u), v[u]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[u][i] = 0.0f;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[u][i]));
        }
        if constexpr (I8) {
          // ConvRot on the SwiGLU rows (as the reference's rotate(swiglu=True)): group u is lane sub's chunk u
          m = 0.0f;
#pragma unroll
          for (int u = 0; u < CPL; ++u) {
            tc_rotate16(v[u]);
#pragma unroll
            for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[u][i]));
          }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const int e = I8 ? tc_exponent_i8(m) : tc_exponent(m);
        const float scale = __uint_as_float((uint32_t)(e + 127) << 23);
        if (live)
#pragma unroll
          for (int u = 0; u < CPL; ++u) {
            if constexpr (I8)
              tc_write_i8_terms<T2>(breg + bb * B2BYTES, N2, j, TC_CAP, sub + 16 * u, v[u], scale);
            else
              tc_write_terms<T2>(breg + bb * B2BYTES, N2, j, TC_CAP, sub + 16 * u, v[u], scale);
          }
        if (live && sub == 0) {
          spair[bb * TC_CAP + j] = pair;
          sinv[bb * TC_CAP + j] = __uint_as_float((uint32_t)(127 - e) << 23);
        }
      }
      fence_async_smem();
      named_sync(1, TC_HELPERS);
      if (hid == 0) mbar_arrive(b2_full + bb);
    }
    // phase-2 epilogue: parts[pair, row] = the pair's terms summed x row scale x 2^-e
    if (warp < 6) {
      const int quarter = warp & 3;
      const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
      for (int t = t2_lo; t < t2_hi; ++t, ++tn) {
        const int buf = tn & 1;
        if (ok) ok = mbar_wait(acc_full + buf, (tn >> 1) & 1);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        float v[N2];
        if (ok) {
#pragma unroll
          for (int cb = 0; cb < N2 / 16; ++cb)
            tmem_ld16(tmem + lane_base + buf * 64 + 16 * cb, (float(&)[16])v[16 * cb]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + buf);
        const int s = t / TPS2, rb = t - s * TPS2, bb = s - s2a, e = pl.seg_expert[s];
        if (ok && bb <= 1) {
          const int r = rb * TC_R2 + 32 * quarter + lane;
          const float sc = __ldg((const float*)a.s2 + (size_t)e * H + r);
          const int cnt = pl.seg_count[s];
#pragma unroll
          for (int j = 0; j < TC_CAP; ++j) {
            if (j < cnt) {
              float sum = v[j];
              if constexpr (I8) {
                sum = tc_i8_sum<T2>(v + j, TC_CAP);
              } else {
#pragma unroll
                for (int tt = 1; tt < T2; ++tt) sum += v[tt * TC_CAP + j];
              }
              __stcg(a.parts + (size_t)spair[bb * TC_CAP + j] * H + r, sum * (sc * sinv[bb * TC_CAP + j]));
            }
          }
        }
        if (last_arrive) tc_block_done(a, c_ok, c_w, rb, nseg, ok);
      }
    }
    if (last_arrive) {
      // the row blocks were combined by their last tiles; the last CTA out clears the counters for the next call
      if (tid == TC_HELP0) TC_STAMP(9);
      tc_exit_count(a, nseg, G);
    } else {
    // every CTA's parts are written; each CTA combines an even share of the columns
    if (tid == TC_HELP0) TC_STAMP(9);
    ok = grid_barrier<TC_HELPERS, TC_HELP0>(a.barrier, G) && ok;
    if (tid == TC_HELP0) TC_STAMP(10);
    // every CTA is past its phase-2 staging: CTA 0 clears the segment counters for the next call
    if (blockIdx.x == 0)
      for (int s = hid; s < nseg; s += TC_HELPERS) seg_done[s] = 0u;
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
#ifdef D3_TRACE
  if (tid == 0) {
    TC_STAMP(11);
    if (blockIdx.x < 1024)
      for (int t = 0; t < 32; ++t) g_trace[blockIdx.x][t] = s_trace[t];
  }
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TC_TMEM_COLS);
  }
}

}  // namespace d3
