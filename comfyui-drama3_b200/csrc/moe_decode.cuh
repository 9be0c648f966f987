// Fused decode of a routed-expert MoE layer for M = 1..16 rows (lines decoded together) on sm_100a.
//
// Replaces, for banks resident in HBM, the chain of drama3/offload.py:108-123 (resident_decode): gemv(gate_up) ->
// SwiGLU [-> ConvRot rotate] -> gemv(down) -> weighted_sum, which the reference runs once per row
// (drama3/model.py:111-113). Here all M rows go through one persistent kernel (one CTA per SM) that reads each
// routed expert once:
//
//   plan      every CTA sorts the M*k (row, rank) pairs by expert: segments of one expert and at most 8 pairs.
//   phase 1   gate_up + SwiGLU: the segments' gate and up rows, split evenly over the CTAs as contiguous ranges of
//             (segment, i) pair-rows; a1[pair, i] = SwiGLU(gate_i . x, up_i . x) to global scratch (fp32).
//   barrier   grid-wide; or, with few segments (nseg * 8 <= CTAs, e.g. one or two rows), each segment owns a
//             contiguous group of CTAs for both phases and only the group waits for its own a1
//   phase 2   down: the segments' down rows, split the same way; parts[pair, n] = down_n . a1[pair] (fp32 scratch).
//   combine   out[t, n] = bf16(sum_j w[t, j] * parts[t*k + j, n]) in rank order (the reference's weighted_sum
//             order), one CTA per output: after a second grid-wide barrier each CTA sums an even share of the
//             columns; in group mode each CTA instead adds the down rows it finished to a per-64-column-block
//             counter, and the CTA that completes a block sums it and resets the counter (no second wait).
//             Deterministic either way.
//
// Data movement: weights reach shared memory through 1-D bulk copies (cp.async.bulk, the untiled TMA path) issued
// by one producer warp on an mbarrier ring that runs through both phases, so the down rows stream in while phase 1
// finishes and while the CTAs wait at the barrier.
//
// Arithmetic: tensor cores (mma.sync m16n8k16, f16 inputs, f32 accumulation). A = 16 weight rows converted in
// registers to f16 exactly (e4m3 by cvt; int8 by byte placement; W4/W6 by the reference's int8-grid decode), B = the
// segment's pairs (up to 8 columns) staged as f16: x * 2^e for bf16 rows (exact), or an f16 hi + lo pair for fp32
// rows (~22 significant bits, two MMAs). A tile costs the same for 1 or 8 pairs, so the work per CTA is the bytes it
// streams whatever the routing. The k index is permuted identically for A and B inside each 64-column chunk so that
// a lane loads 16 contiguous weight columns and 16 contiguous activation halves; a dot product is order-free.
// Each chunk's k range is split over the eight consumer warps and reduced through shared memory.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "formats.cuh"
#include "rotate.cuh"

namespace d3 {

#ifdef D3_TRACE
// Compile-time phase timestamps (build with -DD3_TRACE): per CTA, globaltimer at the kernel's milestones, and in SM
// clock cycles (clock64, cheap to read) the time the first consumer warp and the epilogue warp spent waiting for
// data, staging inputs, computing and handing off. Off in normal builds.
// The counters live in shared memory while the kernel runs (a global read-modify-write per chunk would stall the
// consumer warps and distort what is measured); the CTA's row is written out once at the end.
__device__ unsigned long long g_trace[1024][32];
__shared__ unsigned long long s_trace[32];
#define D3_STAMP(slot) \
  if (threadIdx.x == 0) s_trace[slot] = globaltimer()
#define D3_ADD(slot, v) \
  if (threadIdx.x == 0) s_trace[slot] += (v)
#define D3_ADD_EPI(slot, v) \
  if (threadIdx.x == DEC_WARPS * 32) s_trace[slot] += (v)
// globaltimer at a milestone of a short kernel, straight into this CTA's row of the table
#define D3_GSTAMP(slot) \
  if (threadIdx.x == 0) g_trace[blockIdx.x][slot] = globaltimer()
#else
#define D3_STAMP(slot)
#define D3_ADD(slot, v)
#define D3_ADD_EPI(slot, v)
#define D3_GSTAMP(slot)
#endif

constexpr int DEC_WARPS = 8;                       // consumer warps
constexpr int DEC_THREADS = (DEC_WARPS + 2) * 32;  // + the epilogue warp and the producer warp
constexpr int DEC_CONSUMERS = DEC_WARPS * 32;
constexpr int DEC_MAX_PAIRS = 128;  // M * k
constexpr int DEC_MAX_STAGES = 8;
constexpr int DEC_MAX_CAP = 8;  // pairs per segment = the MMA's N
constexpr int DEC_H = 2048;     // hidden size the kernels are built for
constexpr int DEC_CH1 = 8;      // phase-1 pair-rows per chunk: one 16-row tile (8 gate rows, 8 up rows)
constexpr int DEC_CH2 = 32;     // phase-2 rows per chunk: two 16-row tiles
constexpr int DEC_PAD = 8;      // halves of padding per staged row (conflict-free fragment loads)

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

// All DEC_THREADS threads call this; P <= DEC_MAX_PAIRS <= DEC_THREADS. Expert parallelism: only ids in
// [e_first, e_first + e_count) are this rank's (local expert id - e_first); the others are skipped, and only ids
// outside [0, E) are faults.
template <int NT = DEC_THREADS>
D3_DEV void build_plan(DecodePlan& pl, const int64_t* __restrict__ ids, int P, int E, int cap, int e_first,
                       int e_count) {
  __shared__ __align__(16) int key[DEC_MAX_PAIRS];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < DEC_MAX_PAIRS) {
    int kv = 0x7fffffff;  // positions past P: no expert, ranked after every pair
    if (tid < P) {
      const long long e = ids[tid];
      if (e < 0 || e >= E) record_fault(FAULT_BAD_EXPERT);
      const bool mine = e >= e_first && e < (long long)e_first + e_count && e < E;
      if (mine) kv = (int)(e - e_first);
    }
    key[tid] = kv;
  }
  __syncthreads();
  if (tid < P) {
    const int kp = key[tid];
    int rank = 0, lower = 0, same = 0;
    // the keys four per load, through the padding after P (which never ranks below a pair or ties with a valid one)
#pragma unroll 8
    for (int q0 = 0; q0 < P; q0 += 4) {
      const int4 k4 = *reinterpret_cast<const int4*>(key + q0);
      const int kq[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        lower += kq[u] < kp;
        same += kq[u] == kp;
        rank += (kq[u] < kp) | ((kq[u] == kp) & (q0 + u < tid));
      }
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
  for (int w = 0; w < NT / 32; ++w) {
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

// ---------------------------------------------------------------------------------------------------------------
// Staged activation columns of the MMA (one per pair of the current segment): f16 [8][K + DEC_PAD], the hi term,
// then for fp32 sources the lo term in a second such block. inv[j] = 2^-e (times 1/16 for ConvRot rows) undoes the
// staging scale on the dot products.
__host__ __device__ constexpr int stage_row_halves(int K) { return K + DEC_PAD; }

// 2^e such that max * 2^e lies in [2^14, 2^15): f16 then holds every value of the row below 65504.
D3_DEV int stage_exponent(float m) {
  if (!(m > 0.0f) || !(m < 3.0e38f)) return 0;
  const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
  return min(100, max(-100, 14 - ex));
}

// The 8 values lane `lane` owns of item (row j, 256-column group q): columns 256q + 8 lane .. + 7 of source row
// rows[j] (bf16, or fp32 read at L2).
D3_DEV void stage_load(const void* src, bool bf16, size_t base, float (&v)[8]) {
  if (bf16) {
    const uint4 b = *(const uint4*)((const uint16_t*)src + base);
    const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[2 * u] = bf16_to_f32(w[u] & 0xFFFFu);
      v[2 * u + 1] = bf16_to_f32(w[u] >> 16);
    }
  } else {
    const float4 f0 = __ldcg((const float4*)((const float*)src + base));
    const float4 f1 = __ldcg((const float4*)((const float*)src + base) + 1);
    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
    v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
  }
}

// Stage `cnt` rows of K columns (source row rows[j]) as the MMA's columns, by the eight MMA warps, in work items of
// (row, 256-column group) spread over the warps. Pass A bounds each row's staged values: the exact max |x| of a
// plain row; for a rotated row 16 * max over groups of the group's 2-norm (each output of the unscaled butterfly,
// 16 times a normalized-Hadamard row dotted with the group, is within that). Pass B reloads the values (L2), rotates
// each group with the reference's butterfly when `rotate` (in the warp's own 256-float scratch; the groups are
// independent), scales by 2^e so the bound sits in [2^14, 2^15) and converts to f16 (hi, and lo when `two`); with
// `int8q` (W4A8 / W6A8) it instead quantizes the row to int8 by its exact max (inv = the int8 scale).
// Uses named barrier 1 (MMA warps); rowmax[] must be zero on entry.
D3_DEV void stage_rows(__half* xin, float* inv, int* rowmax, float* wscratch, const void* src, bool bf16,
                       const int* rows, int cnt, int K, bool rotate, bool two, bool int8q = false) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = K / 256, items = cnt * groups;
  for (int it = warp; it < items; it += DEC_WARPS) {
    const int j = it / groups, q = it - j * groups;
    float v[8];
    stage_load(src, bf16, (size_t)rows[j] * K + 256 * q + 8 * lane, v);
    float m = 0.0f;
    if (rotate) {
#pragma unroll
      for (int u = 0; u < 8; ++u) m = fmaf(v[u], v[u], m);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
      m = 16.0f * sqrtf(m) * 1.001f;
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) m = fmaxf(m, fabsf(v[u]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    if (lane == 0) atomicMax(rowmax + j, __float_as_int(m));  // non-negative floats order as ints
  }
  named_sync(1, DEC_CONSUMERS);
  const int RH = stage_row_halves(K);
  for (int it = warp; it < items; it += DEC_WARPS) {
    const int j = it / groups, q = it - j * groups;
    float v[8];
    stage_load(src, bf16, (size_t)rows[j] * K + 256 * q + 8 * lane, v);
    if (rotate) {
      float* row = wscratch + warp * 256;
#pragma unroll
      for (int u = 0; u < 8; ++u) row[8 * lane + u] = v[u];
      __syncwarp();
#pragma unroll
      for (int stride = 1; stride < 256; stride *= 4) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int tt = lane + 32 * h, low = tt % stride, high = tt / stride;
          const int i = high * stride * 4 + low;
          const float va = row[i], vb = row[i + stride], vc = row[i + 2 * stride], vd = row[i + 3 * stride];
          row[i] = va + vb + vc - vd;
          row[i + stride] = va + vb - vc + vd;
          row[i + 2 * stride] = va - vb + vc + vd;
          row[i + 3 * stride] = -va + vb + vc + vd;
        }
        __syncwarp();
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = row[8 * lane + u];
      __syncwarp();
    }
    __half* hi = xin + (size_t)j * RH + 256 * q + 8 * lane;
    __half* lo = xin + (size_t)(DEC_MAX_CAP + j) * RH + 256 * q + 8 * lane;
    if (int8q) {
      // per-row int8 quantization (W4A8 / W6A8): s = max|x| / 127, q = clamp(rint(x / s), +-127), IEEE division
      const float s = __fdiv_rn(__int_as_float(rowmax[j]), 127.0f);
      float qv[8];
      quant_i8_n<8>(v, s, __frcp_rn(s), qv);
      uint32_t hw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float q0 = qv[2 * u];
        const float q1 = qv[2 * u + 1];
        hw[u] = (uint32_t)__half_as_ushort(__float2half_rn(q0)) |
                ((uint32_t)__half_as_ushort(__float2half_rn(q1)) << 16);
      }
      *(uint4*)hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      if (q == 0 && lane == 0) inv[j] = s;
      continue;
    }
    const int e = stage_exponent(__int_as_float(rowmax[j]));
    const float scale = __uint_as_float((uint32_t)(e + 127) << 23);
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float s0 = v[2 * u] * scale, s1 = v[2 * u + 1] * scale;
      const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
      hw[u] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      const __half l0 = __float2half_rn(s0 - __half2float(h0)), l1 = __float2half_rn(s1 - __half2float(h1));
      lw[u] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    *(uint4*)hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    if (two) *(uint4*)lo = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    if (q == 0 && lane == 0) inv[j] = (rotate ? 0.0625f : 1.0f) * __uint_as_float((uint32_t)(127 - e) << 23);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// MMA and the A-fragment builders. For a lane (g = lane / 4, c = lane % 4) and a 64-column chunk, the lane owns
// columns 16c .. 16c + 15 of the chunk; k16-step j of the chunk uses columns 16c + 4j + {0, 1} (A register 0 / 1 of
// the step: fragment slots 2c, 2c+1) and 16c + 4j + {2, 3} (registers 2 / 3: slots 2c+8, 2c+9). a[2j] holds the
// first pair of f16 values, a[2j + 1] the second.
D3_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

D3_DEV uint32_t pack_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// int8 x2 (low bytes of w) -> exact f16 x2: the unsigned byte as the mantissa of 1024 + u, minus 1152.
D3_DEV uint32_t i8x2_h2(uint32_t w_xor80, uint32_t sel) {
  const uint32_t m = __byte_perm(w_xor80, 0x64646464u, sel);
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(0x64806480u));  // 1152.0 in both halves
  return r;
}

// The 16 columns a lane owns in one weight row, as 8 f16x2 registers. `row` points at the row's bytes,
// `col` is the first column (64 * kc + 16c); W4/W6 also read the row's group scales `srow` (one e4m3 byte per 16
// columns) and the codebook `lut`.
// Signed 4-bit / 6-bit codes -> exact f16 pairs: the code, sign bit flipped, as the low mantissa bits of 1024, minus
// 1024 + 8 (or + 32).
D3_DEV uint32_t s4x2_h2(uint32_t byte) {
  const uint32_t h = (((byte & 0xFu) | ((byte & 0xF0u) << 12)) ^ 0x00080008u) | 0x64006400u;
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64086408u));  // 1032.0 in both halves
  return r;
}
D3_DEV uint32_t s6x2_h2(uint32_t c0, uint32_t c1) {
  const uint32_t h = ((c0 | (c1 << 16)) ^ 0x00200020u) | 0x64006400u;
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64206420u));  // 1056.0 in both halves
  return r;
}

template <int FMT>
D3_DEV void build_a(const uint8_t* row, const uint8_t* srow, int col, int K, const float* lut, uint32_t (&a)[8]) {
  if (FMT == FMT_W4A8) {
    // 16 nibbles: byte i holds columns 2i (low) and 2i + 1. Sign bits flipped once per word; byte i copied into both
    // halves (prmt), low nibble and high nibble (times 16) into the mantissas of 1024 (lop3), then one f16x2 FMA:
    // lo * 1 - 1032, hi * 1/16 - 72 (both exact).
    const uint2 p = *(const uint2*)(row + col / 2);
    const uint32_t w[2] = {p.x ^ 0x88888888u, p.y ^ 0x88888888u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t t = __byte_perm(w[i >> 2], 0u, (uint32_t)((i & 3) | 0x40 | ((i & 3) << 8) | 0x4000));
      const uint32_t h = (t & 0x00F0000Fu) | 0x64006400u;
      asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(a[i]) : "r"(h), "r"(0x2C003C00u), "r"(0xD480E408u));
    }
  } else if (FMT == FMT_W6A8) {
    // 16 six-bit codes in 12 bytes: code i at bit 6i of the little-endian 96-bit word
    const uint32_t* p = (const uint32_t*)(row + (col / 16) * 12);
    const uint32_t w[3] = {p[0], p[1], p[2]};
    uint32_t c[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int bit = 6 * i, k = bit >> 5, off = bit & 31;
      c[i] = __funnelshift_r(w[k], k < 2 ? w[k + 1] : 0u, off) & 63u;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = s6x2_h2(c[2 * i], c[2 * i + 1]);
  } else if (fmt_e4m3(FMT) || FMT == FMT_I8) {
    const uint4 q = *(const uint4*)(row + col);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (fmt_e4m3(FMT)) {
        a[2 * j] = e4m3x2_h2(w[j] & 0xFFFFu);
        a[2 * j + 1] = e4m3x2_h2(w[j] >> 16);
      } else {
        const uint32_t t = w[j] ^ 0x80808080u;
        a[2 * j] = i8x2_h2(t, 0x4140);
        a[2 * j + 1] = i8x2_h2(t, 0x4342);
      }
    }
  } else {
    const uint2 low = *(const uint2*)(row + col / 2);
    const uint32_t high = FMT == FMT_W6 ? *(const uint32_t*)(row + K / 2 + col / 4) : 0u;
    const float s = e4m3_to_f32(srow[col / 16]);
    float f[16];
    if (FMT == FMT_W4)
      dec_w4<16>(low, s, lut, f);
    else
      dec_w6<16>(low, high, s, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = pack_h2(f[2 * j], f[2 * j + 1]);
  }
}

// Activation fragment of column (pair) g for the lane's 16 columns: 8 b32 registers (pairs of halves).
D3_DEV void load_b(const __half* xrow, int col, uint32_t (&b)[8]) {
  const uint4 u0 = *(const uint4*)(xrow + col), u1 = *(const uint4*)(xrow + col + 8);
  b[0] = u0.x;
  b[1] = u0.y;
  b[2] = u0.z;
  b[3] = u0.w;
  b[4] = u1.x;
  b[5] = u1.y;
  b[6] = u1.z;
  b[7] = u1.w;
}

// ---------------------------------------------------------------------------------------------------------------
// Expert-parallel exchange over peer memory (one node, up to 8 ranks). Every rank holds an exchange area: fp32
// slots [2][world][M_max * H] (two sets, alternating by call parity), flags [2][8] and its call counter `epoch`. A
// decode pushes this rank's fp32 partial into its slot of every rank's area (P2P stores over NVLink for peers) and
// then, once all its CTAs have, raises flag[parity][rank] = epoch + 1 on every rank (system-scope release); the
// reduce kernel waits for all ranks' flags, sums the slots in rank order and advances the counter (the word after the
// counter counts the reduce's finished CTAs). A rank can run at
// most one call ahead of a peer's reduce (its next reduce needs the peer's next push), so two slot sets suffice.
constexpr int EP_MAX_RANKS = 8;
struct EpExchange {
  float* slots[EP_MAX_RANKS];     // rank r's area (this rank's own pointer, or the IPC mapping of a peer's)
  unsigned* flags[EP_MAX_RANKS];  // rank r's flags [2][EP_MAX_RANKS]
  unsigned* epoch;                // this rank's call counter
  int world, rank, m_max, h;      // the area's geometry: slots [2][world][m_max * h]
};

__device__ __forceinline__ bool ep_geometry_ok(const EpExchange& ex, int M, int H) {
  return ex.world >= 1 && ex.world <= EP_MAX_RANKS && ex.rank >= 0 && ex.rank < ex.world && M <= ex.m_max &&
         H == ex.h;
}

struct DecodeArgs {
  const void* x;  // [M, H]: bf16 when x_bf16, else fp32
  int x_bf16;
  const int64_t* ids;    // [M, k]
  const float* weights;  // [M, k]
  int M, k, E, H, I;
  const uint8_t* w13;  // gate_up rows [E * 2I, row_bytes(H)]
  const void* s13;     // FP8: float [E*2I/128, H/128]; I8: float [E*2I]; W4/W6: uint8 e4m3 [E*2I, H/16]
  const float* c13;    // W4/W6: s_channel [E*2I]
  const float* cb13;   // W4: codebook [16]
  const uint8_t* w2;   // down rows [E * H, row_bytes(I)]
  const void* s2;
  const float* c2;
  const float* cb2;
  uint16_t* out;                // [M, H] bf16 (or null, with out_f32)
  float* out_f32;               // [M, H] fp32 partial sums of this rank's experts (expert parallelism), or null
  int e_first, e_count;         // this rank's experts: ids in [e_first, e_first + e_count); the banks hold them
  const EpExchange* ex;         // expert parallelism over peer memory: push the partial to every rank, or null
  unsigned* ep_done;            // scratch: combine-completion counter for the exchange, zero between calls
  float* a1;                    // scratch [M*k, I]
  float* parts;                 // scratch [M*k, H]
  unsigned long long* barrier;  // scratch: zero before the first call; grows by gridDim.x per grid-wide barrier
  unsigned* blocks;             // scratch [DEC_H / DEC_CB]: combine counters, zero between calls
  unsigned* arrive;             // scratch [DEC_MAX_GRID]: group-barrier counters, zero between calls
  unsigned* depart;             // scratch [DEC_MAX_GRID]
  int stages, stage_bytes, cap;
  int lastarrive_nseg;          // tensor-core decodes: at most this many segments combine per 128-row block by the
                                // block's last-arriving tile instead of after a grid barrier
};

constexpr int DEC_CB = 64;          // columns per combine block
constexpr int DEC_MAX_GRID = 256;   // CTAs the group counters cover
// The workspace tail holding the synchronization words (at the end of the caller's workspace): the ticket
// (8 bytes), the block counters at +64, arrive at +512, depart at +1536 (unsigned each). Zero before the first
// call; every call leaves them zero (the ticket a multiple of the grid size), unless it recorded a fault.
constexpr int DEC_SYNC_BYTES = 4096;

// Warp roles: DEC_WARPS MMA warps, then the epilogue warp (reductions and stores), then the producer warp.
constexpr int DEC_EPI = DEC_WARPS, DEC_PROD = DEC_WARPS + 1;
constexpr int DEC_ALL = DEC_THREADS;
constexpr int DEC_RED = 4;  // partial-sum slots between the MMA warps and the epilogue warp

// One chunk's partial sums (per MMA warp and lane) and what the epilogue needs to finish it.
struct RedSlot {
  float4 part[DEC_WARPS * 32];
  int pair[DEC_MAX_CAP];
  float inv[DEC_MAX_CAP];
  float rsc[DEC_CH2];  // fp8c / int8: the chunk's row scales (phase 1: gate rows, then up rows at +8)
  int r, cn, cnt, e;
};

// Row scales (fp8c / int8) ride with their chunk: each span is copied from the 16-byte boundary at or below its first
// scale, into a 64-byte (phase 1: gate, then up) or 160-byte (phase 2) area after the chunk's rows.
constexpr int DEC_RS1 = 64, DEC_RS2 = 160;

// Shared-memory layout of the decode kernel (dynamic part), shared with the host launcher.
struct DecodeSmem {
  int scratch, in, inv, rowmax, table, red, ring, total;
};

template <int FMT, bool XBF>
__host__ __device__ inline DecodeSmem decode_smem(int H, int I, int stages, int stage_bytes) {
  DecodeSmem s{};
  s.scratch = 0;
  const int scratch_bytes = fmt_rotated(FMT) ? DEC_WARPS * 256 * 4 : 0;
  s.in = scratch_bytes;
  // phase 1: hi (and lo unless bf16 rows of an fp8 bank) blocks of 8 rows of H; phase 2: hi and lo of I
  const int terms1 = ((fmt_e4m3(FMT) && XBF) || fmt_a8(FMT)) ? 1 : 2;
  const int in1 = terms1 * DEC_MAX_CAP * stage_row_halves(H) * 2, in2 = 2 * DEC_MAX_CAP * stage_row_halves(I) * 2;
  s.inv = s.in + (in1 > in2 ? in1 : in2);
  s.rowmax = s.inv + 4 * DEC_MAX_CAP;
  s.table = s.rowmax + 4 * DEC_MAX_CAP;
  const int t = FMT == FMT_FP8 ? (2 * I / 128) * (H / 128) : 0;  // >= (H/128)(I/128)
  s.red = s.table + ((4 * t + 15) / 16) * 16;
  s.ring = s.red + DEC_RED * (int)sizeof(RedSlot);
  s.ring = (s.ring + 127) / 128 * 128;
  s.total = s.ring + stages * stage_bytes;
  return s;
}

// Bytes of one ring stage: a phase-1 chunk (8 gate rows, 8 up rows, and their group scales) or a phase-2 chunk.
// A phase-2 chunk's group scales are copied from the 16-byte boundary below their first byte (W4A8 / W6A8 rows of
// I = 768 hold 12 scale bytes), hence the 32 spare bytes.
template <int FMT>
__host__ __device__ constexpr int decode_stage_bytes(int H, int I) {
  return (2 * DEC_CH1 * (fmt_row_bytes(FMT, H) + fmt_gscale_bytes(FMT, H)) + (fmt_row_scale(FMT) ? 2 * DEC_RS1 : 0)) >
                 (DEC_CH2 * (fmt_row_bytes(FMT, I) + fmt_gscale_bytes(FMT, I)) + 32 +
                  (fmt_row_scale(FMT) ? DEC_RS2 : 0))
             ? 2 * DEC_CH1 * (fmt_row_bytes(FMT, H) + fmt_gscale_bytes(FMT, H)) + (fmt_row_scale(FMT) ? 2 * DEC_RS1 : 0)
             : DEC_CH2 * (fmt_row_bytes(FMT, I) + fmt_gscale_bytes(FMT, I)) + 32 + (fmt_row_scale(FMT) ? DEC_RS2 : 0);
}

// The contiguous range [lo, hi) of `total` work items owned by CTA `b` of `g`.
D3_DEV void split_range(int total, int b, int g, int& lo, int& hi) {
  lo = (int)((long long)b * total / g);
  hi = (int)((long long)(b + 1) * total / g);
}

// Grid-wide barrier of one CTA per SM, taken by the MMA warps and the epilogue warp (named barrier 2), by tickets on
// a 64-bit counter that starts at zero and only grows: a round completes when the counter reaches the round's end.
// Bounded: after WAIT_LIMIT_NS the fault word is set and false returned.
// Participants: the NT threads from LEADER on, on named barrier 2.
template <int NT = DEC_CONSUMERS + 32, int LEADER = 0>
D3_DEV bool grid_barrier(unsigned long long* counter, unsigned nblocks) {
  __shared__ int passed;
  named_sync(2, NT);
  if (threadIdx.x == LEADER) {
    __threadfence();
    const unsigned long long ticket = atomicAdd(counter, 1ull);
    const unsigned long long target = (ticket / nblocks + 1) * nblocks;
    int ok = 1;
    unsigned long long seen;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(seen) : "l"(counter) : "memory");
    if (seen < target) {
      const unsigned long long start = globaltimer();
      while (true) {
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(seen) : "l"(counter) : "memory");
        if (seen >= target) break;
        if (globaltimer() - start > WAIT_LIMIT_NS) {
          record_fault(FAULT_WAIT_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    passed = ok;
  }
  named_sync(2, NT);
  return passed != 0;
}

// Barrier of the `n` CTAs of one segment group (same participants as grid_barrier): arrive, wait for all n
// arrivals, depart; the last to depart zeroes both counters for the next call (every member has passed the wait by
// then). Bounded like grid_barrier.
D3_DEV bool group_barrier(unsigned* arrive, unsigned* depart, unsigned n) {
  __shared__ int passed;
  named_sync(2, DEC_CONSUMERS + 32);
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(arrive, 1u);
    int ok = 1;
    unsigned seen;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(arrive) : "memory");
    if (seen < n) {
      const unsigned long long start = globaltimer();
      while (true) {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(arrive) : "memory");
        if (seen >= n) break;
        if (globaltimer() - start > WAIT_LIMIT_NS) {
          record_fault(FAULT_WAIT_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    passed = ok;
    if (ok && atomicAdd(depart, 1u) == n - 1) {
      atomicExch(arrive, 0u);
      atomicExch(depart, 0u);
    }
  }
  named_sync(2, DEC_CONSUMERS + 32);
  return passed != 0;
}

// The phase-1 and phase-2 ranges of CTA b of G for nseg segments: contiguous even splits of the whole
// (segment, row) space, or, in group mode, CTA b belongs to segment b * nseg / G and splits that segment's rows with
// the other CTAs of its group. Returns the group (segment) or -1, and its size.
D3_DEV int decode_ranges(int nseg, int I, int H, int b, int G, bool grouped, int& lo1, int& hi1, int& lo2, int& hi2,
                         int& gsz) {
  if (!grouped) {
    split_range(nseg * I, b, G, lo1, hi1);
    split_range(nseg * H, b, G, lo2, hi2);
    gsz = G;
    return -1;
  }
  const int s = (int)((long long)b * nseg / G);
  const int b0 = (int)(((long long)s * G + nseg - 1) / nseg), b1 = (int)(((long long)(s + 1) * G + nseg - 1) / nseg);
  gsz = b1 - b0;
  int l, h;
  split_range(I, b - b0, gsz, l, h);
  lo1 = s * I + l;
  hi1 = s * I + h;
  split_range(H, b - b0, gsz, l, h);
  lo2 = s * H + l;
  hi2 = s * H + h;
  return s;
}

// ---------------------------------------------------------------------------------------------------------------
// The activation fragments a warp uses for every chunk of a segment (its k range is the same in each): phase 1 the
// four 64-column chunks kc = warp + 8m, phase 2 the NKC chunks kc = warp % 4 + 4m. Loaded once per segment.
constexpr int P1_KC = DEC_H / 64 / DEC_WARPS;

template <bool TWO>
D3_DEV void load_b1(const __half* xin, uint32_t (&bh)[P1_KC][8], uint32_t (&bl)[TWO ? P1_KC : 1][8]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const __half* xh = xin + (size_t)g * stage_row_halves(DEC_H);
  const __half* xl = xin + (size_t)(DEC_MAX_CAP + g) * stage_row_halves(DEC_H);
#pragma unroll
  for (int m = 0; m < P1_KC; ++m) {
    const int col = 64 * (warp + DEC_WARPS * m) + 16 * c;
    load_b(xh, col, bh[m]);
    if (TWO) load_b(xl, col, bl[m]);
  }
}

template <int NKC>
D3_DEV void load_b2(const __half* xin, int I, uint32_t (&bh)[NKC][8], uint32_t (&bl)[NKC][8]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const __half* xh = xin + (size_t)g * stage_row_halves(I);
  const __half* xl = xin + (size_t)(DEC_MAX_CAP + g) * stage_row_halves(I);
#pragma unroll
  for (int m = 0; m < NKC; ++m) {
    const int col = 64 * ((warp & 3) + 4 * m) + 16 * c;
    load_b(xh, col, bh[m]);
    load_b(xl, col, bl[m]);
  }
}

// Phase 1, one chunk, one MMA warp: the warp's four 64-column chunks of the 16-row tile (rows 0-7: gate rows i0..,
// rows 8-15: up rows i0..) against the segment's activation fragments.
template <int FMT, bool TWO>
D3_DEV float4 p1_chunk(const DecodeArgs& a, const uint8_t* stage, int i0, const uint32_t (&bh)[P1_KC][8],
                       const uint32_t (&bl)[TWO ? P1_KC : 1][8], const float* table, const float* lut) {
  constexpr int H = DEC_H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int I = a.I, rb = fmt_row_bytes(FMT, H), gb = fmt_gscale_bytes(FMT, H);
  const uint8_t* grow = stage + g * rb;
  const uint8_t* urow = stage + (DEC_CH1 + g) * rb;
  const uint8_t* gsrow = stage + 2 * DEC_CH1 * rb + g * gb;
  const uint8_t* usrow = stage + 2 * DEC_CH1 * rb + (DEC_CH1 + g) * gb;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int m = 0; m < P1_KC; ++m) {
    const int kc = warp + DEC_WARPS * m, col = 64 * kc + 16 * c;
    uint32_t ga[8], ua[8];
    build_a<FMT>(grow, gsrow, col, H, lut, ga);
    build_a<FMT>(urow, usrow, col, H, lut, ua);
    float t0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, t1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float(&t)[4] = (j & 1) ? t1 : t0;  // two independent accumulation chains
      mma16816(t, ga[2 * j], ua[2 * j], ga[2 * j + 1], ua[2 * j + 1], bh[m][2 * j], bh[m][2 * j + 1]);
      if (TWO) mma16816(t, ga[2 * j], ua[2 * j], ga[2 * j + 1], ua[2 * j + 1], bl[m][2 * j], bl[m][2 * j + 1]);
    }
    if (FMT == FMT_FP8) {
      // 128 x 128 block scales of rows (gate i0 + g, up I + i0 + g) and this chunk's columns (rows past a partial
      // tile are stale and discarded; their block index is clamped into the table)
      const float sg = table[min((i0 + g) / 128, 2 * I / 128 - 1) * (H / 128) + kc / 2];
      const float su = table[min((I + i0 + g) / 128, 2 * I / 128 - 1) * (H / 128) + kc / 2];
      acc[0] = fmaf(t0[0] + t1[0], sg, acc[0]);
      acc[1] = fmaf(t0[1] + t1[1], sg, acc[1]);
      acc[2] = fmaf(t0[2] + t1[2], su, acc[2]);
      acc[3] = fmaf(t0[3] + t1[3], su, acc[3]);
    } else if (fmt_a8(FMT)) {
      // bf16 group-128 scales of the gate / up row (the chunk's 64 columns lie in group kc / 2)
      const float sg = bf16_to_f32(*(const uint16_t*)(gsrow + 2 * (kc / 2)));
      const float su = bf16_to_f32(*(const uint16_t*)(usrow + 2 * (kc / 2)));
      acc[0] = fmaf(t0[0] + t1[0], sg, acc[0]);
      acc[1] = fmaf(t0[1] + t1[1], sg, acc[1]);
      acc[2] = fmaf(t0[2] + t1[2], su, acc[2]);
      acc[3] = fmaf(t0[3] + t1[3], su, acc[3]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] += t0[q] + t1[q];
    }
  }
  return make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// Phase 2, one chunk, one MMA warp: tile warp / 4 (rows 16 * tile .. of the chunk), 64-column chunks kc = warp % 4 + 4m.
// soff: where the chunk's first group-scale byte sits past the stage's scale area (W4A8 / W6A8, see
// decode_stage_bytes).
template <int FMT, int NKC>
D3_DEV float4 p2_chunk(const DecodeArgs& a, const uint8_t* stage, int n0, int soff, const uint32_t (&bh)[NKC][8],
                       const uint32_t (&bl)[NKC][8], const float* table, const float* lut) {
  constexpr bool TWO2 = !fmt_a8(FMT);  // int8-quantized a1 is one exact f16 term
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int H = DEC_H, I = a.I, rb = fmt_row_bytes(FMT, I), gb = fmt_gscale_bytes(FMT, I);
  const int tile = warp >> 2, r_lo = 16 * tile + g, r_hi = r_lo + 8;
  const uint8_t* lrow = stage + r_lo * rb;
  const uint8_t* hrow = stage + r_hi * rb;
  const uint8_t* lsrow = stage + DEC_CH2 * rb + soff + r_lo * gb;
  const uint8_t* hsrow = stage + DEC_CH2 * rb + soff + r_hi * gb;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int m = 0; m < NKC; ++m) {
    const int kc = (warp & 3) + 4 * m, col = 64 * kc + 16 * c;
    uint32_t la[8], ha[8];
    build_a<FMT>(lrow, lsrow, col, I, lut, la);
    build_a<FMT>(hrow, hsrow, col, I, lut, ha);
    float t0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, t1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mma16816(t0, la[2 * j], ha[2 * j], la[2 * j + 1], ha[2 * j + 1], bh[m][2 * j], bh[m][2 * j + 1]);
      if (TWO2) mma16816(t1, la[2 * j], ha[2 * j], la[2 * j + 1], ha[2 * j + 1], bl[m][2 * j], bl[m][2 * j + 1]);
    }
    if (FMT == FMT_FP8) {
      const float sl = table[min((n0 + r_lo) / 128, H / 128 - 1) * (I / 128) + kc / 2];
      const float sh = table[min((n0 + r_hi) / 128, H / 128 - 1) * (I / 128) + kc / 2];
      acc[0] = fmaf(t0[0] + t1[0], sl, acc[0]);
      acc[1] = fmaf(t0[1] + t1[1], sl, acc[1]);
      acc[2] = fmaf(t0[2] + t1[2], sh, acc[2]);
      acc[3] = fmaf(t0[3] + t1[3], sh, acc[3]);
    } else if (fmt_a8(FMT)) {
      const float sl = bf16_to_f32(*(const uint16_t*)(lsrow + 2 * (kc / 2)));
      const float sh = bf16_to_f32(*(const uint16_t*)(hsrow + 2 * (kc / 2)));
      acc[0] = fmaf(t0[0] + t1[0], sl, acc[0]);
      acc[1] = fmaf(t0[1] + t1[1], sl, acc[1]);
      acc[2] = fmaf(t0[2] + t1[2], sh, acc[2]);
      acc[3] = fmaf(t0[3] + t1[3], sh, acc[3]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] += t0[q] + t1[q];
    }
  }
  return make_float4(acc[0], acc[1], acc[2], acc[3]);
}

D3_DEV float f4get(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// ---------------------------------------------------------------------------------------------------------------
// The MMA warps' work for one phase: every chunk of the CTA's range [lo, hi) in order; the segment's activation
// fragments are staged and loaded at each segment change; each chunk's partial sums go to the epilogue warp through
// the RedSlot ring. `c` counts chunks across both phases (ring positions). Returns false after a failed wait.
template <int FMT, bool XBF, int NKC, int PHASE>
D3_DEV bool mma_phase(const DecodeArgs& a, const DecodePlan& pl, int lo, int hi, int& c, bool ok, uint8_t* ring,
                      uint64_t* full_bar, uint64_t* empty_bar, uint64_t* rfull, uint64_t* rempty, RedSlot* red,
                      __half* xin, float* inv, int* rowmax, float* wscratch, float* table, const float* lut,
                      int* pair_in, int* rows_in) {
  constexpr bool ROT = fmt_rotated(FMT);
  constexpr bool A8 = fmt_a8(FMT);
  constexpr bool TWO1 = !((fmt_e4m3(FMT) && XBF) || A8);
  constexpr int KC = PHASE == 1 ? P1_KC : NKC;
  constexpr bool TWO = PHASE == 1 ? TWO1 : true;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = DEC_H, I = a.I, NS = a.stages, SB = a.stage_bytes;
  const int per = PHASE == 1 ? I : H, ch = PHASE == 1 ? DEC_CH1 : DEC_CH2;
  uint32_t bh[KC][8], bl[TWO ? KC : 1][8];
  int cur = -1, cnt = 0, e = 0;
  // Each chunk's sums go to the epilogue as soon as they are computed (handing them off one chunk later, after the
  // next chunk's MMAs were issued, measured slower).
  int pv_c = -1, pv_r = 0, pv_cn = 0;
  float4 pv_part = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float pv_rsv = 0.0f;
  auto handoff = [&]() {
    const int slot = pv_c % DEC_RED;
#ifdef D3_TRACE
    const unsigned long long th0 = (unsigned long long)clock64();
#endif
    if (pv_c >= DEC_RED && ok) ok = mbar_wait(&rempty[slot], ((pv_c / DEC_RED) - 1) & 1);
#ifdef D3_TRACE
    D3_ADD(PHASE == 1 ? 15 : 21, (unsigned long long)clock64() - th0);
#endif
#ifdef D3_TRACE
    const unsigned long long th1 = (unsigned long long)clock64();
#endif
    RedSlot& rs = red[slot];
    rs.part[warp * 32 + lane] = pv_part;
    if (fmt_row_scale(FMT) && warp == 0) rs.rsc[lane] = pv_rsv;
    if (warp == 0) {
      if (lane < DEC_MAX_CAP) {
        rs.pair[lane] = pair_in[lane];
        rs.inv[lane] = inv[lane];
      }
      if (lane == 0) {
        rs.r = pv_r;
        rs.cn = pv_cn;
        rs.cnt = cnt;
        rs.e = e;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&rfull[slot]);
    pv_c = -1;
#ifdef D3_TRACE
    D3_ADD(24, (unsigned long long)clock64() - th1);
#endif
  };
#ifdef D3_TRACE
  unsigned long long t_it = (unsigned long long)clock64();
#endif
  for (int q = lo; q < hi; ++c) {
    const int s = q / per, r = q - s * per, cn = min(ch, min(per - r, hi - q));
    if (s != cur) {
      // a new segment: stage its pairs' rows (x in phase 1, a1 in phase 2) once all warps left the last one
#ifdef D3_TRACE
      const unsigned long long tn0 = (unsigned long long)clock64();
#endif
      named_sync(1, DEC_CONSUMERS);
#ifdef D3_TRACE
      D3_ADD(7, (unsigned long long)clock64() - tn0);
#endif
      cur = s;
      cnt = pl.seg_count[s];
      e = pl.seg_expert[s];
      const int first = pl.seg_first[s];
      if (tid < cnt) {
        pair_in[tid] = pl.sorted[first + tid];
        rows_in[tid] = PHASE == 1 ? pl.sorted[first + tid] / a.k : pl.sorted[first + tid];
        rowmax[tid] = 0;
      }
      if (FMT == FMT_FP8) {
        const int n = PHASE == 1 ? (2 * I / 128) * (H / 128) : (H / 128) * (I / 128);
        const float* src = (const float*)(PHASE == 1 ? a.s13 : a.s2) + (size_t)e * n;
        for (int t = tid; t < n; t += DEC_CONSUMERS) table[t] = src[t];
      }
      named_sync(1, DEC_CONSUMERS);
#ifdef D3_TRACE
      const unsigned long long ts0 = (unsigned long long)clock64();
#endif
      // a1 holds SwiGLU outputs; ConvRot formats rotate them, as the reference's rotate(swiglu=True) does
      if (PHASE == 1)
        stage_rows(xin, inv, rowmax, wscratch, a.x, a.x_bf16 != 0, rows_in, cnt, H, ROT, TWO1, A8);
      else
        stage_rows(xin, inv, rowmax, wscratch, a.a1, false, rows_in, cnt, I, ROT, !A8, A8);
      named_sync(1, DEC_CONSUMERS);
      if (PHASE == 1)
        load_b1<TWO1>(xin, (uint32_t(&)[P1_KC][8])bh, (uint32_t(&)[TWO1 ? P1_KC : 1][8])bl);
      else
        load_b2<NKC>(xin, I, (uint32_t(&)[NKC][8])bh, (uint32_t(&)[NKC][8])bl);
#ifdef D3_TRACE
      D3_ADD(PHASE == 1 ? 8 : 10, (unsigned long long)clock64() - ts0);
      D3_ADD(12, 1);
#endif
    }
    const int st = c % NS;
#ifdef D3_TRACE
    const unsigned long long tw0 = (unsigned long long)clock64();
    D3_ADD(25, tw0 - t_it);
#endif
    if (ok) ok = mbar_wait(&full_bar[st], (c / NS) & 1);
#ifdef D3_TRACE
    D3_ADD(PHASE == 1 ? 9 : 11, (unsigned long long)clock64() - tw0);
    if (c == 0) D3_STAMP(13);
    const unsigned long long tc0 = (unsigned long long)clock64();
#endif
    float4 part = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (ok) {
      if (PHASE == 1)
        part = p1_chunk<FMT, TWO1>(a, ring + (size_t)st * SB, r, (const uint32_t(&)[P1_KC][8])bh,
                                   (const uint32_t(&)[TWO1 ? P1_KC : 1][8])bl, table, lut);
      else
        part = p2_chunk<FMT, NKC>(a, ring + (size_t)st * SB, r,
                                  A8 ? (int)((((size_t)e * H + r) * fmt_gscale_bytes(FMT, I)) & 15) : 0,
                                  (const uint32_t(&)[NKC][8])bh, (const uint32_t(&)[NKC][8])bl, table, lut);
    }
    // fp8c / int8: warp 0 takes the chunk's row scales out of the stage before it is released
    float rsv = 0.0f;
    if (fmt_row_scale(FMT) && warp == 0 && ok) {
      const uint8_t* stg = ring + (size_t)st * SB;
      if (PHASE == 1) {
        const size_t base = (size_t)e * 2 * I + r + (lane < 8 ? 0 : I);
        if (lane < 16 && (lane & 7) < cn)
          rsv = *(const float*)(stg + 2 * DEC_CH1 * fmt_row_bytes(FMT, H) + (lane < 8 ? 0 : DEC_RS1) +
                                ((base * 4) & 15) + (lane & 7) * 4);
      } else {
        const size_t base = (size_t)e * H + r;
        if (lane < cn) rsv = *(const float*)(stg + DEC_CH2 * fmt_row_bytes(FMT, I) + ((base * 4) & 15) + lane * 4);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
#ifdef D3_TRACE
    D3_ADD(PHASE == 1 ? 16 : 20, (unsigned long long)clock64() - tc0);
    D3_ADD(PHASE == 1 ? 18 : 22, 1);
#endif
    pv_c = c;
    pv_r = r;
    pv_cn = cn;
    pv_part = part;
    pv_rsv = rsv;
    handoff();
    q += cn;
#ifdef D3_TRACE
    const unsigned long long t_now = (unsigned long long)clock64();
    D3_ADD(PHASE == 1 ? 23 : 14, t_now - t_it);
    t_it = t_now;
#endif
  }
  return ok;
}

// The routed combine of columns [n0, n1) for every row, in rank order (the reference's weighted_sum order), by the
// CTA's MMA and epilogue warps. valid[p] / w[p]: pair p's id is in range / its routing weight (shared memory). The
// k parts of an output are loaded together (independent L2 loads), then summed in order.
// Run by the nt threads from t0 on.
D3_DEV void combine_columns(const DecodeArgs& a, const unsigned char* valid, const float* w, int n0, int n1, bool ok,
                            int t0 = 0, int nt = DEC_CONSUMERS + 32) {
  // four adjacent columns a thread (n0, n1 multiples of 4): 16-byte loads of the parts and 16-byte stores (peer
  // stores included)
  const int NQ = (n1 - n0) >> 2, H = DEC_H;
  float* dst32 = a.out_f32;
  size_t slot = 0;
  int world = 0;
  if (a.ex) {
    // this rank's slot in every rank's area (call parity set)
    const EpExchange& ex = *a.ex;
    if (ep_geometry_ok(ex, a.M, H)) {
      const unsigned ep = *(volatile const unsigned*)ex.epoch + 1u;
      slot = (size_t)((ep & 1u) * ex.world + ex.rank) * ex.m_max * H;
      world = ex.world;
    } else if (threadIdx.x == t0) {
      record_fault(FAULT_EXCHANGE);
    }
    dst32 = nullptr;
  }
  const bool out8 = ((uintptr_t)a.out & 7u) == 0;
  for (int idx = threadIdx.x - t0; idx < a.M * NQ; idx += nt) {
    const int t = idx / NQ, n = n0 + 4 * (idx - t * NQ);
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int j0 = 0; j0 < a.k; j0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int p = t * a.k + j0 + u;
        v[u] = (ok && j0 + u < a.k && valid[p]) ? __ldcg(reinterpret_cast<const float4*>(a.parts + (size_t)p * H + n))
                                                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (j0 + u < a.k) {
          const float wt = w[t * a.k + j0 + u];
          acc.x = __fmaf_rn(v[u].x, wt, acc.x);
          acc.y = __fmaf_rn(v[u].y, wt, acc.y);
          acc.z = __fmaf_rn(v[u].z, wt, acc.z);
          acc.w = __fmaf_rn(v[u].w, wt, acc.w);
        }
    }
    if (a.ex) {
      for (int r = 0; r < world; ++r)
        *reinterpret_cast<float4*>(a.ex->slots[r] + slot + (size_t)t * H + n) = acc;
    } else if (dst32) {
      *reinterpret_cast<float4*>(dst32 + (size_t)t * H + n) = acc;
    } else {
      uint16_t* o = a.out + (size_t)t * H + n;
      const uint16_t b0 = f32_to_bf16(acc.x), b1 = f32_to_bf16(acc.y), b2 = f32_to_bf16(acc.z),
                     b3 = f32_to_bf16(acc.w);
      if (out8) {
        *reinterpret_cast<uint2*>(o) = make_uint2((uint32_t)b0 | ((uint32_t)b1 << 16), (uint32_t)b2 | ((uint32_t)b3 << 16));
      } else {
        o[0] = b0;
        o[1] = b1;
        o[2] = b2;
        o[3] = b3;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
template <int FMT, bool XBF, int NKC>
__global__ void __launch_bounds__(DEC_ALL, 1) moe_decode_kernel(const DecodeArgs a) {
  constexpr bool ROT = fmt_rotated(FMT);
  constexpr bool TWO1 = !((fmt_e4m3(FMT) && XBF) || fmt_a8(FMT));  // phase-1 activations need the lo term
  const int H = DEC_H, I = a.I, P = a.M * a.k, NS = a.stages, SB = a.stage_bytes;
  const int rb1 = fmt_row_bytes(FMT, H), gb1 = fmt_gscale_bytes(FMT, H), rb2 = fmt_row_bytes(FMT, I),
            gb2 = fmt_gscale_bytes(FMT, I);

  __shared__ DecodePlan pl;
  __shared__ __align__(8) uint64_t full_bar[DEC_MAX_STAGES], empty_bar[DEC_MAX_STAGES];
  __shared__ __align__(8) uint64_t rfull[DEC_RED], rempty[DEC_RED];
  __shared__ float lut1[16], lut2[16];
  __shared__ int rows_in[DEC_MAX_CAP], pair_in[DEC_MAX_CAP];
  extern __shared__ __align__(128) uint8_t smem[];
  const DecodeSmem L = decode_smem<FMT, XBF>(H, I, NS, SB);
  float* wscratch = (float*)(smem + L.scratch);
  __half* xin = (__half*)(smem + L.in);
  float* inv = (float*)(smem + L.inv);
  int* rowmax = (int*)(smem + L.rowmax);
  float* table = (float*)(smem + L.table);
  RedSlot* red = (RedSlot*)(smem + L.red);
  uint8_t* ring = smem + L.ring;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#ifdef D3_TRACE
  if (tid == 0)
    for (int t = 0; t < 32; ++t) s_trace[t] = 0;
#endif
  D3_STAMP(0);
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], DEC_WARPS);
    }
    for (int s = 0; s < DEC_RED; ++s) {
      mbar_init(&rfull[s], DEC_WARPS);
      mbar_init(&rempty[s], 1);
    }
    fence_mbar_init();
  }
  // programmatic dependent launch: the next kernel in the stream may be scheduled onto SMs this grid frees; this one
  // reads its inputs and touches the workspace only after the previous grid has completed
  allow_dependents();
  grid_dependency_wait();
  if (FMT == FMT_W4 && tid < 16) {
    lut1[tid] = a.cb13[tid];
    lut2[tid] = a.cb2[tid];
  }
  build_plan(pl, a.ids, P, a.E, a.cap, a.e_first, a.e_count);
  D3_STAMP(1);
  const int nseg = pl.nseg, G = gridDim.x;
  // group mode needs at least 8 CTAs per segment, so that a CTA's down rows (H / 8 = 256 at most) span <= 5 blocks
  const bool grouped = nseg > 0 && nseg * 8 <= G && G <= DEC_MAX_GRID;
  int lo1, hi1, lo2, hi2, gsz;
  const int grp = decode_ranges(nseg, I, H, blockIdx.x, G, grouped, lo1, hi1, lo2, hi2, gsz);

  if (warp == DEC_PROD) {
    // ---------------- producer: phase-1 chunks, then phase-2 chunks, through one ring ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int c = 0;
      bool ok = true;
      for (int phase = 1; phase <= 2 && ok; ++phase) {
        const int lo = phase == 1 ? lo1 : lo2, hi = phase == 1 ? hi1 : hi2, per = phase == 1 ? I : H;
        const int ch = phase == 1 ? DEC_CH1 : DEC_CH2;
        for (int q = lo; q < hi; ++c) {
          const int s = q / per, r = q - s * per, cn = min(ch, min(per - r, hi - q));
          const int st = c % NS;
          if (c >= NS && !mbar_wait(&empty_bar[st], ((c / NS) - 1) & 1)) {
            ok = false;
            break;
          }
          const int e = pl.seg_expert[s];
          uint8_t* dst = ring + (size_t)st * SB;
          if (phase == 1) {
            const size_t g0 = (size_t)e * 2 * I + r, u0 = g0 + I;
            // row scales (fp8c / int8): 16-byte-aligned spans around each set of cn scales
            const size_t a0 = (g0 * 4) & ~(size_t)15, a1 = ((g0 + cn) * 4 + 15) & ~(size_t)15;
            const size_t b0 = (u0 * 4) & ~(size_t)15, b1 = ((u0 + cn) * 4 + 15) & ~(size_t)15;
            const uint32_t rsb = fmt_row_scale(FMT) ? (uint32_t)(a1 - a0 + b1 - b0) : 0u;
            const uint32_t bytes = 2u * cn * rb1 + 2u * cn * gb1 + rsb;
            mbar_arrive_expect_tx(&full_bar[st], bytes);
            bulk_g2s(dst, a.w13 + g0 * rb1, cn * rb1, &full_bar[st], pol);
            bulk_g2s(dst + DEC_CH1 * rb1, a.w13 + u0 * rb1, cn * rb1, &full_bar[st], pol);
            if (fmt_row_scale(FMT)) {
              const uint8_t* sc = (const uint8_t*)a.s13;
              uint8_t* rs = dst + 2 * DEC_CH1 * rb1;
              bulk_g2s(rs, sc + a0, (uint32_t)(a1 - a0), &full_bar[st], pol);
              bulk_g2s(rs + DEC_RS1, sc + b0, (uint32_t)(b1 - b0), &full_bar[st], pol);
            }
            if (gb1 > 0) {
              const uint8_t* sc = (const uint8_t*)a.s13;
              bulk_g2s(dst + 2 * DEC_CH1 * rb1, sc + g0 * gb1, cn * gb1, &full_bar[st], pol);
              bulk_g2s(dst + 2 * DEC_CH1 * rb1 + DEC_CH1 * gb1, sc + u0 * gb1, cn * gb1, &full_bar[st], pol);
            }
          } else {
            const size_t n0 = (size_t)e * H + r;
            // group scales (W4/W6/A8) or row scales (fp8c / int8), from the 16-byte boundary at or below their
            // first byte to one at or above their end
            const int sb = gb2 > 0 ? gb2 : (fmt_row_scale(FMT) ? 4 : 0);
            const size_t s0 = (n0 * sb) & ~(size_t)15, s1 = ((n0 + cn) * sb + 15) & ~(size_t)15;
            const uint32_t sbytes = sb > 0 ? (uint32_t)(s1 - s0) : 0u;
            const uint8_t* ssrc = (const uint8_t*)a.s2;
            mbar_arrive_expect_tx(&full_bar[st], cn * rb2 + sbytes);
            bulk_g2s(dst, a.w2 + n0 * rb2, cn * rb2, &full_bar[st], pol);
            if (sb > 0) bulk_g2s(dst + DEC_CH2 * rb2, ssrc + s0, sbytes, &full_bar[st], pol);
          }
          q += cn;
        }
      }
      // every issued copy lands before this thread leaves (bounded)
      for (int d = max(0, c - NS); d < c; ++d)
        if (!mbar_wait(&full_bar[d % NS], (d / NS) & 1)) break;
    }
    return;
  }

  bool ok = true;
  if (warp == DEC_EPI) {
    // ---------------- epilogue: reduce each chunk's partial sums, scale, store ----------------
    int c = 0;
    for (int phase = 1; phase <= 2; ++phase) {
      if (phase == 2)
        ok = (grouped ? group_barrier(a.arrive + grp, a.depart + grp, gsz) : grid_barrier(a.barrier, G)) && ok;
      const int lo = phase == 1 ? lo1 : lo2, hi = phase == 1 ? hi1 : hi2, per = phase == 1 ? I : H;
      const int ch = phase == 1 ? DEC_CH1 : DEC_CH2;
      for (int q = lo; q < hi; ++c) {
        const int s = q / per, r = q - s * per, cn = min(ch, min(per - r, hi - q));
        const int slot = c % DEC_RED;
#ifdef D3_TRACE
        const unsigned long long te0 = (unsigned long long)clock64();
#endif
        if (ok) ok = mbar_wait(&rfull[slot], (c / DEC_RED) & 1);
#ifdef D3_TRACE
        const unsigned long long te1 = (unsigned long long)clock64();
        D3_ADD_EPI(17, te1 - te0);
#endif
        const RedSlot& rs = red[slot];
        const int cnt = rs.cnt, e = rs.e;
        // lane L finishes what lane L of the MMA warps holds: rows g, g + 8 of the tile x pairs 2c, 2c + 1
        const int g = lane >> 2, n0 = 2 * (lane & 3), n1 = n0 + 1;
        if (ok && phase == 1) {
          float4 sum = rs.part[lane];
#pragma unroll
          for (int w = 1; w < DEC_WARPS; ++w) {
            const float4 v = rs.part[w * 32 + lane];
            sum.x += v.x;
            sum.y += v.y;
            sum.z += v.z;
            sum.w += v.w;
          }
          // x, y: gate row g for pairs n0, n1; z, w: up row g
          if (g < cn) {
            const int i = r + g;
            float gsc = 1.0f, usc = 1.0f;
            if (fmt_row_scale(FMT)) {
              gsc = rs.rsc[g];
              usc = rs.rsc[DEC_CH1 + g];
            } else if (fmt_codes(FMT)) {
              gsc = __ldg(a.c13 + (size_t)e * 2 * I + i);
              usc = __ldg(a.c13 + (size_t)e * 2 * I + I + i);
            }
            if (n0 < cnt) {
              const float s0 = rs.inv[n0];
              a.a1[(size_t)rs.pair[n0] * I + i] = swiglu_fast(sum.x * (gsc * s0), sum.z * (usc * s0));
            }
            if (n1 < cnt) {
              const float s1 = rs.inv[n1];
              a.a1[(size_t)rs.pair[n1] * I + i] = swiglu_fast(sum.y * (gsc * s1), sum.w * (usc * s1));
            }
          }
        } else if (ok) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            float4 sum = rs.part[(4 * t) * 32 + lane];
#pragma unroll
            for (int w = 1; w < 4; ++w) {
              const float4 v = rs.part[(4 * t + w) * 32 + lane];
              sum.x += v.x;
              sum.y += v.y;
              sum.z += v.z;
              sum.w += v.w;
            }
            // x, y: row 16t + g for pairs n0, n1; z, w: row 16t + g + 8
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const int row = 16 * t + g + 8 * half;
              if (row < cn) {
                const int nrow = r + row;
                float sc = 1.0f;
                if (fmt_row_scale(FMT)) sc = rs.rsc[row];
                if (fmt_codes(FMT)) sc = __ldg(a.c2 + (size_t)e * H + nrow);
                const float v0 = half ? sum.z : sum.x, v1 = half ? sum.w : sum.y;
                if (n0 < cnt) __stcg(a.parts + (size_t)rs.pair[n0] * H + nrow, v0 * (sc * rs.inv[n0]));
                if (n1 < cnt) __stcg(a.parts + (size_t)rs.pair[n1] * H + nrow, v1 * (sc * rs.inv[n1]));
              }
            }
          }
        }
#ifdef D3_TRACE
        D3_ADD_EPI(19, (unsigned long long)clock64() - te1);
#endif
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[slot]);
        q += cn;
      }
    }
  } else {
    // ---------------- MMA warps ----------------
    int c = 0;
    ok = mma_phase<FMT, XBF, NKC, 1>(a, pl, lo1, hi1, c, ok, ring, full_bar, empty_bar, rfull, rempty, red, xin, inv,
                                     rowmax, wscratch, table, lut1, pair_in, rows_in);
    D3_STAMP(2);
    ok = (grouped ? group_barrier(a.arrive + grp, a.depart + grp, gsz) : grid_barrier(a.barrier, G)) && ok;
    D3_STAMP(3);
    ok = mma_phase<FMT, XBF, NKC, 2>(a, pl, lo2, hi2, c, ok, ring, full_bar, empty_bar, rfull, rempty, red, xin, inv,
                                     rowmax, wscratch, table, lut2, pair_in, rows_in);
    D3_STAMP(4);
  }
  D3_STAMP(5);
  // ---------------- combine ----------------
  __shared__ int s_nblk, s_blk[DEC_H / DEC_CB];
  __shared__ float c_w[DEC_MAX_PAIRS];
  __shared__ unsigned char c_ok[DEC_MAX_PAIRS];
  if (tid < P) {
    const long long id = a.ids[tid];
    c_ok[tid] = nseg > 0 && id >= a.e_first && id < (long long)a.e_first + a.e_count && id < a.E;
    c_w[tid] = a.weights[tid];
  }
  if (!grouped) {
    // grid-wide: every CTA's parts are written; each CTA combines an even share of the columns
    ok = grid_barrier(a.barrier, G) && ok;
    int q0, q1;
    split_range(H / 4, blockIdx.x, G, q0, q1);
    combine_columns(a, c_ok, c_w, 4 * q0, 4 * q1, ok);
  } else {
    // group mode: the CTA that completes a 64-column block (its counter reaching nseg * 64 finished down rows) sums
    // that block; no second wait
    named_sync(2, DEC_CONSUMERS + 32);  // the epilogue's parts stores are done
    if (tid == 0) {
      int nb = 0;
      if (ok && hi2 > lo2) {
        __threadfence();
        // one segment's rows [r, end): at most 256 rows (G >= 8 nseg CTAs share H rows), so at most 5 blocks; the
        // counter updates are issued together, then checked
        const int r = lo2 % H, end = r + (hi2 - lo2), b0 = r / DEC_CB, nblk = min(8, (end - 1) / DEC_CB - b0 + 1);
        unsigned old[8], cnt[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int lo = max(r, (b0 + i) * DEC_CB), hi = min(end, (b0 + i + 1) * DEC_CB);
          cnt[i] = i < nblk ? (unsigned)(hi - lo) : 0u;
          old[i] = i < nblk ? atomicAdd(a.blocks + b0 + i, cnt[i]) : 0u;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < nblk && old[i] + cnt[i] == (unsigned)(nseg * DEC_CB)) s_blk[nb++] = b0 + i;
        __threadfence();
      }
      s_nblk = nb;
    }
    named_sync(2, DEC_CONSUMERS + 32);
    for (int i = 0; i < s_nblk; ++i) {
      const int b = s_blk[i];
      combine_columns(a, c_ok, c_w, b * DEC_CB, (b + 1) * DEC_CB, ok);
      if (tid == 0) a.blocks[b] = 0u;
    }
  }
  if (a.ex) {
    // exchange: once every column block of this rank's partial has been pushed, raise this rank's flag on every rank
    // (grid mode: every CTA pushed its share of the columns; group mode: the CTAs that completed blocks pushed them)
    named_sync(2, DEC_CONSUMERS + 32);  // this CTA's pushes are issued
    if (tid == 0 && ep_geometry_ok(*a.ex, a.M, H)) {
      const unsigned share = grouped ? (unsigned)s_nblk : 1u, total = grouped ? (unsigned)(H / DEC_CB) : (unsigned)G;
      if (share > 0) {
        // one system-scope fence for the CTA: the barrier orders its threads' pushes before it, and it orders them
        // before the count that releases them (the pattern of a grid barrier, at system scope)
        __threadfence_system();
        if (atomicAdd(a.ep_done, share) + share == total) {
          const EpExchange& ex = *a.ex;
          const unsigned ep = *(volatile const unsigned*)ex.epoch + 1u;
          __threadfence_system();
          for (int r = 0; r < ex.world; ++r) {
            unsigned* f = ex.flags[r] + (ep & 1u) * EP_MAX_RANKS + ex.rank;
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(ep) : "memory");
          }
          *a.ep_done = 0u;
        }
      }
    }
  }
  D3_STAMP(6);
#ifdef D3_TRACE
  if (tid == 0 && blockIdx.x < 1024)
    for (int t = 0; t < 32; ++t) g_trace[blockIdx.x][t] = s_trace[t];
#endif
}

// The exchange's reduce on one rank: every CTA waits (bounded) until each rank has raised its flag for this call,
// then sums 4 columns a thread, out[t, n..n+3] = bf16(sum over ranks r in order of slot r); the last CTA to finish
// advances this rank's call counter (the counter word after it counts finished CTAs). Launched with programmatic
// dependent launch: it may be scheduled while the decode still runs, and reads nothing before that grid completes.
constexpr int EP_REDUCE_THREADS = 256;
__global__ void __launch_bounds__(EP_REDUCE_THREADS) ep_reduce_kernel(const EpExchange* __restrict__ exp, int M, int H,
                                                                      uint16_t* __restrict__ out) {
  __shared__ int s_ok;
  __shared__ unsigned s_ep;
  allow_dependents();
  grid_dependency_wait();
  const EpExchange& ex = *exp;
  if (threadIdx.x == 0) {
    const unsigned ep = *(volatile const unsigned*)ex.epoch + 1u;
    int ok = ep_geometry_ok(ex, M, H) && H % 4 == 0;
    if (!ok) record_fault(FAULT_EXCHANGE);
    const unsigned* flags = ok ? ex.flags[ex.rank] + (ep & 1u) * EP_MAX_RANKS : nullptr;
    const unsigned long long start = globaltimer();
    for (int r = 0; r < ex.world && ok; ++r) {
      while (true) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
        if ((int)(v - ep) >= 0) break;
        if (globaltimer() - start > WAIT_LIMIT_NS) {
          record_fault(FAULT_WAIT_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
    s_ep = ep;
  }
  __syncthreads();
  const int ok = s_ok;
  const unsigned ep = s_ep;
  const int q = blockIdx.x * EP_REDUCE_THREADS + threadIdx.x;  // a group of 4 columns
  if (q * 4 < M * H) {
    const int t = (q * 4) / H, n = q * 4 - t * H;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (ok) {
      const float* base = ex.slots[ex.rank] + (size_t)(ep & 1u) * ex.world * ex.m_max * H;
      for (int r = 0; r < ex.world; ++r) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(base + ((size_t)r * ex.m_max + t) * H + n));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    }
    uint2 packed;
    packed.x = (uint32_t)f32_to_bf16(acc.x) | ((uint32_t)f32_to_bf16(acc.y) << 16);
    packed.y = (uint32_t)f32_to_bf16(acc.z) | ((uint32_t)f32_to_bf16(acc.w) << 16);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + n) = packed;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* done = ex.epoch + 1;
    __threadfence();
    if (atomicAdd(done, 1u) + 1u == gridDim.x) {
      *done = 0u;
      *(volatile unsigned*)ex.epoch = ep;
    }
  }
}

}  // namespace d3
