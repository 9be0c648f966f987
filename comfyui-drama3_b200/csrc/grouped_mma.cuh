// Grouped expert GEMM for a prompt's rows on the 5th-generation tensor cores: out[row, n] = the rows of each group
// (sorted by expert, fp32) against their expert's weight rows, as the reference's grouped kernels compute it
// (drama3/kernels.py:365-464, 538-587: fp8 block-scaled, int8 ConvRot, W4A8 / W6A8 codes), for banks held whole on
// the GPU.
//
// Work unit = (token tile of up to 128 rows of one group, block of 128 weight rows). Per unit, D[128 x N] (weight
// rows x the tile's rows rounded up to 16) accumulates in tensor memory, in one of two MMA forms:
//   kind::f16 (fp8 blocks, int8 ConvRot, W4 / W6 codes; f32 accumulators, K = 16, 64 columns a chunk):
//     A = 128 weight rows, converted exactly to f16 in shared memory (every e4m3 value, every int8 and every
//         int8-grid code is an f16), K-major with the 128-byte swizzle;
//     B = the tile's rows as two f16 terms, hi = f16(x * 2^e) and lo = f16(x * 2^e - hi) (e per row puts its max in
//         [2^14, 2^15)); the products are exact; two MMAs per K step.
//   kind::i8 (W4A8 / W6A8; s32 accumulators, K = 32, 128 columns a chunk):
//     A = the int4 / int6 codes expanded to int8 (16 x code, 4 x code), B = the rows' int8 codes; the sums are exact.
// B is laid out by the staging kernel in global memory exactly as the MMA reads it from shared memory, so one 1-D
// bulk copy per term moves a chunk's operand block.
// Scales that vary every 128 columns (fp8 blocks, W4A8 / W6A8 groups) are folded every 128 columns: the MMA thread
// cycles through four regions of 128 tensor-memory columns and the fold warps add scale x partial into registers;
// the other formats fold once per unit and apply the row scale (int8 scale, W4/W6 s_channel).
//
// Warps (352 threads, one CTA per SM, persistent over units):
//   0     raw-weight producer: 2-D TMA tile loads (128 columns x 128 rows, hardware-swizzled so the converters'
//         row reads hit distinct banks) into a 4-stage ring of 16 KB
//   1     activation producer: one bulk copy per term and chunk into a 3-stage ring; a tile of R rows copies and
//         multiplies only its first round_up(R, 16) rows (MMA N = that), which matters for the many small groups of
//         a skewed routing
//   2     MMA issuer (one elected thread) and owner of the 512 tensor-memory columns (4 accumulator regions)
//   3-6   converters: thread = weight row, raw bytes -> f16 or int8, written swizzled into the A stage
//   7-10  fold + epilogue: tcgen05.ld of their 32-lane quarter, scale, accumulate, write fp32 rows
// Every wait is bounded (2 s) and records FAULT_WAIT_TIMEOUT instead of hanging.
#pragma once

#include <cuda.h>

#include "formats.cuh"
#include "moe_decode.cuh"
#include "rotate.cuh"

namespace d3 {

#ifdef D3_TRACE
// Trace builds only: per CTA, cycles each role spent waiting at each barrier (clock64), and counters.
//   0 raw producer / raw_empty   1 B producer / mma_empty   2 MMA / acc_empty   3 MMA / a_full   4 MMA / b_full
//   5 converters / raw_full      6 converters / mma_empty   7 fold / acc_full   8 units   9 total cycles
//   10 converter busy cycles     11 MMA issue cycles     12 fold tmem-load + fma cycles     13 fold epilogue cycles
//   14 converter fence + arrive cycles
__device__ unsigned long long g_gm_trace[1024][16];
#define GM_T0() const long long _t0 = clock64()
#define GM_TADD(slot) \
  if (blockIdx.x < 1024) atomicAdd(&g_gm_trace[blockIdx.x][slot], (unsigned long long)(clock64() - _t0))
#else
#define GM_T0()
#define GM_TADD(slot)
#endif

constexpr int GM_M = 128;              // weight rows per unit (one fp8 scale block)
constexpr int GM_NT = 128;             // token rows per tile
constexpr int GM_KC = 64;              // columns per MMA chunk: one 128-byte swizzle atom of f16
constexpr int GM_RKC = 128;            // columns per raw-weight stage (two MMA chunks)
constexpr int GM_RAW_ST = 4;           // raw weight ring depth
constexpr int GM_MMA_ST = 3;           // operand ring depth (A f16 + B hi/lo)
constexpr int GM_RAW_BYTES = 16384;    // one raw stage: up to 128 bytes x 128 rows
constexpr int GM_A_BYTES = GM_M * GM_KC * 2;      // 16 KB
constexpr int GM_B_BYTES = GM_NT * GM_KC * 2;     // 16 KB per term
constexpr int GM_WARPS = 11;
constexpr int GM_THREADS = GM_WARPS * 32;
constexpr int GM_CONV0 = 3, GM_FOLD0 = 7;         // first converter / fold warp
constexpr int GM_REGIONS = 4;                      // accumulator regions of GM_NT columns: the MMAs run up to three
constexpr int GM_TMEM_COLS = GM_REGIONS * GM_NT;   // folds ahead of the fold warps (one CTA per SM: all 512 columns)

struct GroupedTile {
  int group;  // index into groups[]
  int row0;   // first sorted row of the tile
  int rows;   // rows in the tile (1..128)
  int slot;   // the group's slot (its expert's index in the bank): groups[5 group + 1]
};

// Byte offset of 16-byte chunk c (columns 8c..8c+7 of a 64-column chunk) of row r in a K-major, 128-byte-swizzled
// operand block: 8-row atoms of 1024 bytes, chunk c of row r stored at position c ^ (r % 8). TMA's 128-byte swizzle
// writes the same pattern.
__host__ __device__ constexpr uint32_t sw128_offset(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Bytes of the staged activations of `tiles` tiles with K columns, and of the whole workspace.
__host__ __device__ constexpr size_t gm_staged_bytes(int tiles, int K) {
  return (size_t)tiles * (size_t)(K / GM_KC) * 2u * GM_B_BYTES;
}
__host__ __device__ constexpr size_t gm_workspace_bytes(int tiles, int K) {
  return gm_staged_bytes(tiles, K) + (size_t)tiles * GM_NT * 4u + (size_t)tiles * sizeof(GroupedTile) + 256u;
}

// ---------------------------------------------------------------------------------------------------------------
// Staging: one block (8 warps) per (tile slot, 16-row slice of the tile), so a full tile's rows are spread over 8
// blocks. Block (t, s) finds its (group, tile of the group) from the groups' row counts, slice 0 writes the tile table
// entry, and the block converts its slice of the tile's rows (zeros past the group's end, up to the MMA width) to
// the hi / lo f16 operand blocks (or int8 codes) plus inv[row] = 2^-e (times 1/16 after a rotation; 0 for padding
// rows). Block (0, 0) also writes the number of tiles. A warp owns a row (lane l: columns 256 q + 8 l .. + 7), so
// the row's bound is exact: with a rotation the rotated row stays in registers; without one the warp reads the row
// twice (its bound, then the conversion), which keeps few values in registers and many warps resident.
//   source row of sorted row s: x[row_index ? row_index[s] : s], fp32 or bf16 (src_bf16)
//   mode bit GM_SWIGLU: the source row holds 2K columns, gate then up; the staged value is SiLU(gate) * up in the
//        fast-exp form of the reference's rotate kernel (drama3/kernels.py:233-236)
//   mode bit GM_ROTATE: each 256-column group is rotated by the reference's radix-4 butterfly (ConvRot,
//        drama3/kernels.py:240-256), the 1/16 folded into inv
// Needs K % 256 == 0, K <= 2048.
//   mode bit GM_INT8 (W4A8 / W6A8): the row is quantized to int8 by its exact max (s = max / 127, q = rint(x / s)
//        clamped, IEEE division) and staged as int8 operand blocks of 128 columns for kind::i8; inv = s
enum { GM_ROTATE = 1, GM_SWIGLU = 2, GM_INT8 = 4 };
constexpr int GM_STAGE_ROWS = 16;  // rows of a tile per staging block (grid: tile slots x GM_NT / GM_STAGE_ROWS)
constexpr int GM_STAGE_PREFETCH = 9;  // chunks of 32 group counts a staging block loads up front (257 groups)

D3_DEV float gm_load(const void* x, bool bf16, size_t i) {
  return bf16 ? bf16_to_f32(((const uint16_t*)x)[i]) : ((const float*)x)[i];
}

D3_DEV void gm_load8(const void* x, bool bf16, size_t base, float* v) {
  if (bf16) {
    const uint4 b = __ldg((const uint4*)((const uint16_t*)x + base));
    const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[2 * u] = bf16_to_f32(w[u] & 0xFFFFu);
      v[2 * u + 1] = bf16_to_f32(w[u] >> 16);
    }
  } else {
    const float4 a = __ldg((const float4*)((const float*)x + base));
    const float4 b = __ldg((const float4*)((const float*)x + base) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

template <bool ROT>
__global__ void __launch_bounds__(256, ROT ? 2 : 3) gm_stage_kernel(const void* __restrict__ x, int src_bf16,
                                                       const int64_t* __restrict__ row_index, int mode,
                                                       const int* __restrict__ groups, int G, int K, int max_tiles,
                                                       uint8_t* __restrict__ staged, float* __restrict__ inv,
                                                       GroupedTile* __restrict__ table, int* __restrict__ ntiles) {
  __shared__ int s_group, s_local, s_total;
  __shared__ float scratch[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x, slice = blockIdx.y;
  if (warp == 0) {
    // the row counts of the first GM_STAGE_PREFETCH x 32 groups, loaded together (one memory latency, not one per
    // 32 groups); groups past them are read in the loop
    int pre[GM_STAGE_PREFETCH];
#pragma unroll
    for (int m = 0; m < GM_STAGE_PREFETCH; ++m) {
      const int g = 32 * m + lane;
      pre[m] = g < G ? groups[5 * g + 4] : 0;
    }
    int base = 0, found_g = -1, found_l = 0;
    // one chunk of 32 groups (g = c0 + lane holds n rows): find tile slot t among the chunk's tiles
    auto chunk = [&](int c0, int n) {
      const int tiles = (max(0, n) + GM_NT - 1) / GM_NT;
      int incl = tiles;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int excl = incl - tiles;
      const unsigned hit = __ballot_sync(0xffffffffu, t >= base + excl && t < base + incl);
      const int src = hit ? __ffs(hit) - 1 : 0;
      const int src_excl = __shfl_sync(0xffffffffu, excl, src);
      if (hit && found_g < 0) {
        found_g = c0 + src;
        found_l = t - base - src_excl;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    };
#pragma unroll
    for (int m = 0; m < GM_STAGE_PREFETCH; ++m)
      if (32 * m < G) chunk(32 * m, pre[m]);
    for (int c0 = 32 * GM_STAGE_PREFETCH; c0 < G; c0 += 32)
      chunk(c0, c0 + lane < G ? groups[5 * (c0 + lane) + 4] : 0);
    if (lane == 0) {
      s_group = found_g;
      s_local = found_l;
      s_total = base;
      if (t == 0 && slice == 0) {
        *ntiles = min(base, max_tiles);
        if (base > max_tiles) record_fault(FAULT_TILES);
      }
    }
  }
  __syncthreads();
  if (s_group < 0 || t >= s_total) return;
  const int g = s_group;
  const int first = groups[5 * g + 3], count = groups[5 * g + 4];
  const int row0 = first + s_local * GM_NT, rows = min(GM_NT, count - s_local * GM_NT);
  if (threadIdx.x == 0 && slice == 0) table[t] = GroupedTile{g, row0, rows, groups[5 * g + 1]};
  const bool bf16 = src_bf16 != 0, swiglu = (mode & GM_SWIGLU) != 0;  // GM_ROTATE: the ROT instance
  const bool int8q = (mode & GM_INT8) != 0;
  const int nkc = K / GM_KC, nq = K / 256;
  const size_t pitch = swiglu ? 2 * (size_t)K : (size_t)K;
  uint8_t* tile_base = staged + (size_t)t * nkc * 2 * GM_B_BYTES;
  const int width = (rows + 15) & ~15;  // rows the GEMM reads (its MMA N)
  const int j_end = min(width, GM_STAGE_ROWS * (slice + 1));
  float* row = scratch[warp];
  // columns 256 q + 8 lane .. + 7 of a source row (through SwiGLU when asked; zeros for padding rows)
  auto load_q = [&](int q, size_t src_row, bool live, float* v) {
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = 0.0f;
    if (live) {
      const size_t base = src_row * pitch + 256 * q + 8 * lane;
      gm_load8(x, bf16, base, v);
      if (swiglu) {
        float up[8];
        gm_load8(x, bf16, base + K, up);
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = swiglu_fast(v[u], up[u]);
      }
    }
  };
  // the same columns of staged row j: int8 codes (GM_INT8), or the hi / lo f16 terms of v * scale
  auto store_q = [&](int q, int j, const float* v, float scale, float qs) {
    if (int8q) {
      // int8 operand blocks of 128 columns (one per kind::i8 MMA chunk, GM_B_BYTES apart): columns 256q + 8 lane
      // .. + 7 are chunk 2q + lane / 16, the (lane & 1) half of 16-byte piece (lane % 16) / 2
      float qv[8];
      quant_i8_n<8>(v, qs, __frcp_rn(qs), qv);
      uint32_t b[2] = {0u, 0u};
#pragma unroll
      for (int u = 0; u < 8; ++u) b[u >> 2] |= ((uint32_t)(int)qv[u] & 0xFFu) << (8 * (u & 3));
      uint8_t* blk = tile_base + (size_t)(2 * q + (lane >> 4)) * GM_B_BYTES;
      *(uint2*)(blk + sw128_offset(j, (lane & 15) >> 1) + 8 * (lane & 1)) = make_uint2(b[0], b[1]);
      return;
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float s0 = v[2 * u] * scale, s1 = v[2 * u + 1] * scale;
      const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
      hw[u] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      const __half l0 = __float2half_rn(s0 - __half2float(h0)), l1 = __float2half_rn(s1 - __half2float(h1));
      lw[u] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    // columns 256q + 8 lane .. + 7: chunk kc = 4q + lane / 8, 16-byte piece c = lane % 8
    const int kc = 4 * q + (lane >> 3), c = lane & 7;
    uint8_t* blk = tile_base + (size_t)kc * 2 * GM_B_BYTES;
    *(uint4*)(blk + sw128_offset(j, c)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *(uint4*)(blk + GM_B_BYTES + sw128_offset(j, c)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  };
  for (int j = GM_STAGE_ROWS * slice + warp; j < j_end; j += 8) {
    const bool live = j < rows;
    const size_t src_row = live ? (size_t)(row_index ? row_index[row0 + j] : row0 + j) : 0;
    float m = 0.0f;
    float v[ROT ? 8 : 1][8];  // ROT: the whole rotated row; otherwise one 256-column group at a time
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q >= nq) break;
      float* vq = v[ROT ? q : 0];
      load_q(q, src_row, live, vq);
      if (ROT) {
#pragma unroll
        for (int u = 0; u < 8; ++u) row[8 * lane + u] = vq[u];
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
        for (int u = 0; u < 8; ++u) vq[u] = row[8 * lane + u];
        __syncwarp();
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) m = fmaxf(m, fabsf(vq[u]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int e = stage_exponent(m);
    const float scale = __uint_as_float((uint32_t)(e + 127) << 23);
    const float qs = __fdiv_rn(m, 127.0f);  // int8 scale (GM_INT8)
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q >= nq) break;
      if (!ROT) load_q(q, src_row, live, v[0]);  // the second pass reads the row again (from L1 / L2)
      store_q(q, j, v[ROT ? q : 0], scale, qs);
    }
    if (lane == 0)
      inv[(size_t)t * GM_NT + j] =
          !live ? 0.0f : int8q ? qs : (ROT ? 0.0625f : 1.0f) * __uint_as_float((uint32_t)(127 - e) << 23);
  }
}

// Combine of a prompt pass (drama3/offload.py:146-149): out[t, :] = sum over k of weight[t, k] * sorted[pos[t*k + k'], :]
// in rank order (fmaf), rounded to bf16 (or kept fp32 with out_f32). pos = the sorted position of pair (t, k'). One
// block per token.
__global__ void __launch_bounds__(256) gm_combine_kernel(const float* __restrict__ sorted, const int64_t* __restrict__ pos,
                                                         const void* __restrict__ weights, int w_bf16, int k, int H,
                                                         void* __restrict__ out, int out_f32) {
  const int t = blockIdx.x;
  for (int n = 4 * threadIdx.x; n < H; n += 4 * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < k; ++r) {
      const float w = w_bf16 ? bf16_to_f32(((const uint16_t*)weights)[(size_t)t * k + r])
                             : ((const float*)weights)[(size_t)t * k + r];
      const float4 p = __ldg((const float4*)(sorted + (size_t)pos[(size_t)t * k + r] * H + n));
      acc.x = __fmaf_rn(w, p.x, acc.x);
      acc.y = __fmaf_rn(w, p.y, acc.y);
      acc.z = __fmaf_rn(w, p.z, acc.z);
      acc.w = __fmaf_rn(w, p.w, acc.w);
    }
    if (out_f32) {
      *(float4*)((float*)out + (size_t)t * H + n) = acc;
    } else {
      uint2 o;
      o.x = (uint32_t)f32_to_bf16(acc.x) | ((uint32_t)f32_to_bf16(acc.y) << 16);
      o.y = (uint32_t)f32_to_bf16(acc.z) | ((uint32_t)f32_to_bf16(acc.w) << 16);
      *(uint2*)((uint16_t*)out + (size_t)t * H + n) = o;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05 / TMA primitives (inline PTX, sm_100a)

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart (SBO), version 1.
D3_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both K-major, M = 128, N = n (16..128, % 16).
D3_DEV uint32_t gm_idesc(int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(GM_M >> 4) << 24); }

// MMA width of a tile of `rows` rows.
D3_DEV int gm_width(int rows) { return (rows + 15) & ~15; }

D3_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::i8: s32 accumulator, signed 8-bit A and B, both K-major, M = 128, N = n.
D3_DEV uint32_t t8_idesc(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

D3_DEV void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued so far has completed.
D3_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

D3_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
D3_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Generic-proxy shared-memory writes made visible to the async proxy (the tensor cores' operand reads).
D3_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

D3_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
D3_DEV void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 lanes (lane = row): v[i] = column col + i of row (lane base + lane).
D3_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 2-D tiled TMA load of box (x, y) of `map` into shared memory, completing on `bar`.
D3_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}


// ---------------------------------------------------------------------------------------------------------------
struct GmArgs {
  const uint8_t* staged;
  const float* inv;
  const GroupedTile* table;
  const int* ntiles;
  const int* groups;
  const void* scale;       // fp8: fp32 blocks [E*N/128, K/128]; int8: fp32 [E*N]; W4/W6: e4m3 [E*N, K/16]
  const float* s_channel;  // W4/W6
  const float* codebook;   // W4
  float* out;
  int N, K, max_units;
  int bank_rows;           // rows in the bank (E*N): slot indices beyond it are skipped
};

constexpr int GM_UNIT_CAP = 64;  // units per CTA whose description is cached in shared memory

// One unit as every role needs it: the weight rows' first bank row (wrow < 0: skipped; -1 also records a bad slot),
// the tile, its rows and its first sorted row.
struct GmUnit {
  int wrow, tile, rows, row0;
};

struct GmSmem {
  static constexpr int a = 0;
  static constexpr int b = a + GM_MMA_ST * GM_A_BYTES;
  static constexpr int raw = b + GM_MMA_ST * 2 * GM_B_BYTES;
  static constexpr int bars = raw + GM_RAW_ST * GM_RAW_BYTES;
  // raw_full, raw_empty [GM_RAW_ST]; a_full, b_full, mma_empty [GM_MMA_ST]; acc_full, acc_empty [GM_REGIONS]
  static constexpr int nbars = 2 * GM_RAW_ST + 3 * GM_MMA_ST + 2 * GM_REGIONS;
  static constexpr int tmem = bars + nbars * 8;
  static constexpr int lut = tmem + 16;
  static constexpr int units = lut + 64;  // GmUnit [GM_UNIT_CAP]: this CTA's first units
  static constexpr int inv = units + GM_UNIT_CAP * 16;  // float [4][GM_NT]: the tile rows' 2^-e, a copy per fold warp
  static constexpr int total = inv + 4 * GM_NT * 4;
  static constexpr int launch = total + 1024;  // slack to align the base to 1024 bytes
};

// Raw bytes per weight row in one raw stage (128 columns): fp8 / fp8c / int8 128, W4 nibbles 64, W6 nibbles 64 +
// plane 32, W4A8 64, W6A8 96.
template <int FMT>
__host__ __device__ constexpr int gm_raw_row_bytes() {
  return fmt_e4m3(FMT) || FMT == FMT_I8 ? 128 : FMT == FMT_W4 || FMT == FMT_W4A8 ? 64 : 96;
}
// Formats folded every 128 columns (a scale per 128-column block of each row): fp8 blocks, W4A8 / W6A8 groups.
template <int FMT>
__host__ __device__ constexpr bool gm_folds() {
  return FMT == FMT_FP8 || fmt_a8(FMT);
}

// The unit (tile, row block) a CTA takes k-th, or false past the end.
D3_DEV bool gm_unit(const GmArgs& a, int ntiles, int u, int& tile, int& rb) {
  const int RB = a.N / GM_M;
  if (u >= ntiles * RB || u >= a.max_units) return false;
  tile = u / RB;
  rb = u - tile * RB;
  return true;
}

// Unit u's description, read from the tile table.
D3_DEV GmUnit gm_unit_read(const GmArgs& a, int tile, int rb) {
  const GroupedTile tl = a.table[tile];
  const int wrow = tl.slot * a.N + rb * GM_M;
  GmUnit g;
  g.wrow = tl.slot < 0 || wrow >= a.bank_rows ? -1 : wrow + GM_M > a.bank_rows ? -2 : wrow;
  g.tile = tile;
  g.rows = tl.rows;
  g.row0 = tl.row0;
  return g;
}

// The CTA's i-th unit (u = blockIdx.x + i * gridDim.x): from the shared-memory cache for the first GM_UNIT_CAP,
// read from the table past them; false past the end.
D3_DEV bool gm_unit_at(const GmArgs& a, const GmUnit* cache, int ntiles, int i, GmUnit& out) {
  int tile, rb;
  if (!gm_unit(a, ntiles, blockIdx.x + i * gridDim.x, tile, rb)) return false;
  out = i < GM_UNIT_CAP ? cache[i] : gm_unit_read(a, tile, rb);
  return true;
}

// Convert half h (64 columns) of a raw stage's weight row r to f16 and store it swizzled into the A stage. The raw
// stage holds TMA tiles with the hardware swizzle of their row width: 128-byte rows (fp8, int8) put 16-byte chunk c of
// row r at c ^ (r % 8); 64-byte rows (W4/W6 nibbles) at c ^ ((r / 2) % 4); 32-byte rows (the W6 high plane) at
// c ^ ((r / 4) % 2).
template <int FMT>
D3_DEV void gm_convert(const uint8_t* raw, int h, uint8_t* astage, int r, uint32_t sbytes, const float* lut) {
  if (FMT == FMT_W4A8) {
    // 64-byte rows (swizzled like the W4 nibbles): 16-column group g = 4h + p is 8 bytes
    const uint8_t* low = raw + r * 64;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int g = 4 * h + p;
      const uint2 lw = *(const uint2*)(low + (((g >> 1) ^ ((r >> 1) & 3)) << 4) + 8 * (g & 1));
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = s4x2_h2(((i < 4 ? lw.x : lw.y) >> (8 * (i & 3))) & 0xFFu);
      *(uint4*)(astage + sw128_offset(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
      *(uint4*)(astage + sw128_offset(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  } else if (FMT == FMT_W6A8) {
    // 96-byte rows, no swizzle: 16-column group g = 4h + p is 12 bytes at 12 g
    const uint8_t* row = raw + r * 96;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t* q = (const uint32_t*)(row + 12 * (4 * h + p));
      const uint32_t w[3] = {q[0], q[1], q[2]};
      uint32_t c[16], o[8];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int bit = 6 * i, k = bit >> 5, off = bit & 31;
        c[i] = __funnelshift_r(w[k], k < 2 ? w[k + 1] : 0u, off) & 63u;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = s6x2_h2(c[2 * i], c[2 * i + 1]);
      *(uint4*)(astage + sw128_offset(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
      *(uint4*)(astage + sw128_offset(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  } else if (fmt_e4m3(FMT) || FMT == FMT_I8) {
    const uint8_t* row = raw + r * 128;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int cc = 4 * h + p;
      const uint4 q = *(const uint4*)(row + ((cc ^ (r & 7)) << 4));
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (fmt_e4m3(FMT)) {
          o[2 * j] = e4m3x2_h2(w[j] & 0xFFFFu);
          o[2 * j + 1] = e4m3x2_h2(w[j] >> 16);
        } else {
          const uint32_t t = w[j] ^ 0x80808080u;
          o[2 * j] = i8x2_h2(t, 0x4140);
          o[2 * j + 1] = i8x2_h2(t, 0x4342);
        }
      }
      *(uint4*)(astage + sw128_offset(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
      *(uint4*)(astage + sw128_offset(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  } else {
    // four 16-column groups g = 4h + p: nibbles 8 bytes each, W6 high plane 4 bytes each
    const uint8_t* low = raw + r * 64;
    const uint8_t* high = raw + GM_M * 64 + r * 32;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int g = 4 * h + p;
      const uint2 lw = *(const uint2*)(low + (((g >> 1) ^ ((r >> 1) & 3)) << 4) + 8 * (g & 1));
      const uint32_t hb =
          FMT == FMT_W6 ? *(const uint32_t*)(high + (((g >> 2) ^ ((r >> 2) & 1)) << 4) + 4 * (g & 3)) : 0u;
      const float s = e4m3_to_f32((sbytes >> (8 * p)) & 0xFFu);
      float f[16];
      if (FMT == FMT_W4)
        dec_w4<16>(lw, s, lut, f);
      else
        dec_w6<16>(lw, hb, s, f);
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = pack_h2(f[2 * j], f[2 * j + 1]);
      *(uint4*)(astage + sw128_offset(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
      *(uint4*)(astage + sw128_offset(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
}

// W4A8 / W6A8 on kind::i8: a raw stage's weight row r (128 columns) as int8 into the A stage, K-major with the
// 128-byte swizzle, 16 columns per 16-byte piece. Each code becomes an exact int8 multiple of itself placed in the
// byte's high bits (int4: 16 x code, int6: 4 x code); gm_i8_unscale undoes the factor in the fold.
template <int FMT>
D3_DEV void gm_convert_i8(const uint8_t* raw, uint8_t* astage, int r) {
  if (FMT == FMT_W6A8) {
    // 96-byte rows, no swizzle: 16-column group g is 12 bytes (three words) at 12 g; four 6-bit codes per 24 bits
    const uint4* row = (const uint4*)(raw + r * 96);
    uint32_t w[24];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const uint4 q = row[i];
      w[4 * i] = q.x; w[4 * i + 1] = q.y; w[4 * i + 2] = q.z; w[4 * i + 3] = q.w;
    }
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const uint32_t w0 = w[3 * g], w1 = w[3 * g + 1], w2 = w[3 * g + 2];
      const uint32_t t[4] = {w0, __funnelshift_r(w0, w1, 24), __funnelshift_r(w1, w2, 16), w2 >> 8};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = ((t[i] << 2) & 0xFCu) | ((t[i] << 4) & 0xFC00u) | ((t[i] << 6) & 0xFC0000u) |
               ((t[i] << 8) & 0xFC000000u);
      *(uint4*)(astage + sw128_offset(r, g)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    // 64-byte rows with the hardware swizzle of their width (16-byte chunk c of row r at c ^ ((r / 2) % 4)):
    // group g is 8 bytes, byte i holding columns 2i (low nibble) and 2i + 1
    const uint8_t* low = raw + r * 64;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const uint2 lw = *(const uint2*)(low + (((g >> 1) ^ ((r >> 1) & 3)) << 4) + 8 * (g & 1));
      const uint32_t wv[2] = {lw.x, lw.y};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t lo = (wv[i] << 4) & 0xF0F0F0F0u, hi = wv[i] & 0xF0F0F0F0u;
        o[2 * i] = __byte_perm(lo, hi, 0x5140);
        o[2 * i + 1] = __byte_perm(lo, hi, 0x7362);
      }
      *(uint4*)(astage + sw128_offset(r, g)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// The factor gm_convert_i8 put on every code, undone: 1/4 (int6), 1/16 (int4). Powers of two, so exact.
template <int FMT>
__host__ __device__ constexpr float gm_i8_unscale() {
  return FMT == FMT_W6A8 ? 0.25f : 0.0625f;
}

template <int FMT>
__global__ void __launch_bounds__(GM_THREADS, 1)
    grouped_mma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap pmap, GmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = (uint64_t*)(smem + GmSmem::bars);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + GM_RAW_ST;
  uint64_t* a_full = bars + 2 * GM_RAW_ST;
  uint64_t* b_full = a_full + GM_MMA_ST;
  uint64_t* mma_empty = b_full + GM_MMA_ST;
  uint64_t* acc_full = mma_empty + GM_MMA_ST;
  uint64_t* acc_empty = acc_full + GM_REGIONS;
  uint32_t* tmem_slot = (uint32_t*)(smem + GmSmem::tmem);
  float* lut = (float*)(smem + GmSmem::lut);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef D3_TRACE
  const long long t_kernel = clock64();
  if (threadIdx.x == 0 && blockIdx.x < 1024)
    for (int i = 0; i < 16; ++i) g_gm_trace[blockIdx.x][i] = 0;
#endif
  if (threadIdx.x == 0) {
    for (int i = 0; i < GM_RAW_ST; ++i) {
      mbar_init(raw_full + i, 1);
      mbar_init(raw_empty + i, 4);
    }
    for (int i = 0; i < GM_MMA_ST; ++i) {
      mbar_init(a_full + i, 4);
      mbar_init(b_full + i, 1);
      mbar_init(mma_empty + i, 1);
    }
    for (int i = 0; i < GM_REGIONS; ++i) {
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 4);
    }
    fence_mbar_init();
  }
  if (FMT == FMT_W4 && threadIdx.x < 16) lut[threadIdx.x] = a.codebook[threadIdx.x];
  if (warp == 2) tmem_alloc(tmem_slot, GM_TMEM_COLS);
  const int ntiles = *a.ntiles;
  // the CTA's first units, described once for every role (one table read each, all in flight together)
  GmUnit* units = (GmUnit*)(smem + GmSmem::units);
  if (threadIdx.x < GM_UNIT_CAP) {
    int tile, rb;
    if (gm_unit(a, ntiles, blockIdx.x + threadIdx.x * gridDim.x, tile, rb))
      units[threadIdx.x] = gm_unit_read(a, tile, rb);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // W4A8 / W6A8 (int8 activations) run kind::i8: int8 A and B, 128 columns (128 bytes of a row) per MMA chunk, one
  // raw stage each; the other formats run kind::f16 with 64 columns per chunk, two chunks per raw stage
  constexpr bool I8 = fmt_a8(FMT);
  constexpr int KC = I8 ? 128 : GM_KC;
  const int nkc = a.K / KC;
  const size_t tile_bytes = (size_t)(a.K / GM_KC) * 2 * GM_B_BYTES;  // staged bytes per tile (the f16 layout's)
  constexpr int chunk_bytes = I8 ? GM_B_BYTES : 2 * GM_B_BYTES;      // staged bytes per chunk
  const int G = gridDim.x;
  bool ok = true;

  if (warp == 0) {
    // raw weights: TMA tiles of the unit's 128 rows, chunk by chunk
    if (lane == 0) {
      int rs = 0;
      uint32_t rph = 0;
      GmUnit un;
      for (int i = 0; ok && gm_unit_at(a, units, ntiles, i, un); ++i) {
        const int wrow = un.wrow;
        if (wrow < 0) continue;
        for (int kr = 0; kr < a.K / GM_RKC && ok; ++kr) {
          {
            GM_T0();
            ok = mbar_wait(raw_empty + rs, rph ^ 1);
            GM_TADD(0);
          }
          if (!ok) break;
          uint8_t* dst = smem + GmSmem::raw + rs * GM_RAW_BYTES;
          mbar_arrive_expect_tx(raw_full + rs, GM_M * gm_raw_row_bytes<FMT>());
          if (fmt_e4m3(FMT) || FMT == FMT_I8) {
            tma_load_2d(dst, &wmap, kr * 128, wrow, raw_full + rs);
          } else if (FMT == FMT_W4A8) {
            tma_load_2d(dst, &wmap, kr * 64, wrow, raw_full + rs);
          } else if (FMT == FMT_W6A8) {
            tma_load_2d(dst, &wmap, kr * 96, wrow, raw_full + rs);
          } else {
            tma_load_2d(dst, &wmap, kr * 64, wrow, raw_full + rs);
            if (FMT == FMT_W6) tma_load_2d(dst + GM_M * 64, &pmap, a.K / 2 + kr * 32, wrow, raw_full + rs);
          }
          if (++rs == GM_RAW_ST) {
            rs = 0;
            rph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // staged activations: the operand blocks of each chunk (hi and lo for kind::f16, the int8 block for kind::i8)
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      int ms = 0;
      uint32_t mph = 0;
      GmUnit un;
      for (int i = 0; ok && gm_unit_at(a, units, ntiles, i, un); ++i) {
        if (un.wrow < 0) continue;
        const uint8_t* src = a.staged + (size_t)un.tile * tile_bytes;
        const uint32_t bytes = (uint32_t)gm_width(un.rows) * 128u;  // rows x 128 bytes per term
        for (int kc = 0; kc < nkc && ok; ++kc) {
          {
            GM_T0();
            ok = mbar_wait(mma_empty + ms, mph ^ 1);
            GM_TADD(1);
          }
          if (!ok) break;
          uint8_t* dst = smem + GmSmem::b + ms * 2 * GM_B_BYTES;
          const uint8_t* blk = src + (size_t)kc * chunk_bytes;
          mbar_arrive_expect_tx(b_full + ms, fmt_a8(FMT) ? bytes : 2 * bytes);
          bulk_g2s(dst, blk, bytes, b_full + ms, keep);
          if (!fmt_a8(FMT)) bulk_g2s(dst + GM_B_BYTES, blk + GM_B_BYTES, bytes, b_full + ms, keep);
          if (++ms == GM_MMA_ST) {
            ms = 0;
            mph ^= 1;
          }
        }
      }
    }
  } else if (warp == 2) {
    // MMA issuer
    if (lane == 0) {
      int ms = 0, folds = 0;
      uint32_t mph = 0;
      const int kbc = gm_folds<FMT>() ? 128 / KC : nkc;  // chunks per fold
      GmUnit un;
      for (int i = 0; ok && gm_unit_at(a, units, ntiles, i, un); ++i) {
        if (un.wrow < 0) continue;
        uint32_t acc = 0;
        const uint32_t idesc = I8 ? t8_idesc(gm_width(un.rows)) : gm_idesc(gm_width(un.rows));
        for (int kc = 0; kc < nkc && ok; ++kc) {
          if (kc % kbc == 0) {
            const int region = folds % GM_REGIONS;
            {
              GM_T0();
              ok = mbar_wait(acc_empty + region, ((folds / GM_REGIONS) & 1) ^ 1);
              GM_TADD(2);
            }
            if (!ok) break;
            tc_fence_after();
            acc = tmem + region * GM_NT;
          }
          {
            GM_T0();
            ok = mbar_wait(a_full + ms, mph);
            GM_TADD(3);
          }
          {
            GM_T0();
            ok = ok && mbar_wait(b_full + ms, mph);
            GM_TADD(4);
          }
          if (!ok) break;
          GM_T0();
          tc_fence_after();
          const uint32_t as = smem_u32(smem + GmSmem::a + ms * GM_A_BYTES);
          const uint32_t bs = smem_u32(smem + GmSmem::b + ms * 2 * GM_B_BYTES);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {  // K steps of 32 bytes: 16 f16 or 32 int8 columns
            const uint64_t ad = umma_desc_sw128(as + 32 * ks);
            const uint32_t accumulate = (kc % kbc != 0 || ks != 0) ? 1u : 0u;
            if (I8) {
              umma_i8(acc, ad, umma_desc_sw128(bs + 32 * ks), idesc, accumulate);
            } else {
              umma_f16(acc, ad, umma_desc_sw128(bs + 32 * ks), idesc, accumulate);
              if (!fmt_a8(FMT)) umma_f16(acc, ad, umma_desc_sw128(bs + GM_B_BYTES + 32 * ks), idesc, 1u);
            }
          }
          umma_commit(mma_empty + ms);
          if (kc % kbc == kbc - 1) {
            umma_commit(acc_full + folds % GM_REGIONS);
            ++folds;
          }
          GM_TADD(11);
          if (++ms == GM_MMA_ST) {
            ms = 0;
            mph ^= 1;
          }
        }
      }
    }
  } else if (warp < GM_FOLD0) {
    // converters: thread = weight row of the unit
    const int r = threadIdx.x - GM_CONV0 * 32;
    int rs = 0, ms = 0;
    uint32_t rph = 0, mph = 0;
    GmUnit un;
    for (int i = 0; ok && gm_unit_at(a, units, ntiles, i, un); ++i) {
      const int wrow = un.wrow;
      if (wrow < 0) continue;
      const uint8_t* srow = FMT == FMT_W4 || FMT == FMT_W6
                                ? (const uint8_t*)a.scale + (size_t)(wrow + r) * (a.K / 16)
                                : nullptr;
      // W4 / W6 group scales: four bytes a chunk, loaded one chunk ahead of their use
      uint32_t snext = srow ? __ldg((const uint32_t*)srow) : 0u;
      for (int kc = 0; kc < nkc && ok; ++kc) {
        const int h = kc & 1;
        const bool first = I8 || h == 0, last = I8 || h == 1;  // this chunk's raw stage: first / last use
        const uint32_t sbytes = snext;
        if (srow && kc + 1 < nkc) snext = __ldg((const uint32_t*)(srow + 4 * (kc + 1)));
        {
          GM_T0();
          ok = (!first || mbar_wait(raw_full + rs, rph));
          if (r == 0) GM_TADD(5);
        }
        {
          GM_T0();
          ok = ok && mbar_wait(mma_empty + ms, mph ^ 1);
          if (r == 0) GM_TADD(6);
        }
        if (!ok) break;
        {
          GM_T0();
          if constexpr (I8)
            gm_convert_i8<FMT>(smem + GmSmem::raw + rs * GM_RAW_BYTES, smem + GmSmem::a + ms * GM_A_BYTES, r);
          else
            gm_convert<FMT>(smem + GmSmem::raw + rs * GM_RAW_BYTES, h, smem + GmSmem::a + ms * GM_A_BYTES, r,
                            sbytes, lut);
          if (r == 0) GM_TADD(10);
        }
        {
          GM_T0();
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (last) mbar_arrive(raw_empty + rs);
            mbar_arrive(a_full + ms);
          }
          if (r == 0) GM_TADD(14);
        }
        if (last && ++rs == GM_RAW_ST) {
          rs = 0;
          rph ^= 1;
        }
        if (++ms == GM_MMA_ST) {
          ms = 0;
          mph ^= 1;
        }
      }
    }
  } else {
    // fold + epilogue: this warp's quarter of the 128 accumulator lanes (weight rows)
    const int quarter = warp & 3;
    const int r = 32 * quarter + lane;
    const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
    const int kbc = gm_folds<FMT>() ? 128 / KC : nkc;
    const int nfold = nkc / kbc;  // at most 16 (K <= 2048)
    // fold f's scale of the unit whose weight rows start at wrow: the 128 x 128 block's (fp8), or this row's bf16
    // group scale times the int8 expansion's 1/4 or 1/16 (W4A8 / W6A8); loaded one fold ahead of its use
    auto fold_scale = [&](int wrow, int f) -> float {
      if (FMT == FMT_FP8) return __ldg((const float*)a.scale + (size_t)(wrow / 128) * (a.K / 128) + f);
      return bf16_to_f32(__ldg((const uint16_t*)a.scale + (size_t)(wrow + r) * (a.K / 128) + f)) *
             gm_i8_unscale<FMT>();
    };
    int folds = 0;
    GmUnit un;
    for (int i = 0; ok && gm_unit_at(a, units, ntiles, i, un); ++i) {
      if (un.wrow < 0) {
        if (un.wrow == -1) record_fault(FAULT_BAD_SLOT);
      } else {
        // the tile rows' factors, copied into this warp's own shared-memory row while the unit's MMAs run, so the
        // epilogue's stores do not wait on global loads (the warp's previous epilogue has read the row already)
        float* inv = (float*)(smem + GmSmem::inv) + quarter * GM_NT;
#pragma unroll
        for (int m = 0; m < GM_NT / 32; ++m)
          inv[lane + 32 * m] = __ldg(a.inv + (size_t)un.tile * GM_NT + lane + 32 * m);
        float* dst = a.out + (size_t)un.row0 * a.N + (un.wrow % a.N) + r;
        if (gm_folds<FMT>()) {
          // one fold per 128 columns: acc += scale x partial (fp8: the 128 x 128 block's; W4A8 / W6A8: the row's
          // bf16 group scale)
          float acc[GM_NT];
#pragma unroll
          for (int j = 0; j < GM_NT; ++j) acc[j] = 0.0f;
          float s_cur = fold_scale(un.wrow, 0), s_nxt = 0.0f;
          for (int f = 0; f < nfold && ok; ++f) {
            const int region = folds % GM_REGIONS;
            if (f + 1 < nfold) s_nxt = fold_scale(un.wrow, f + 1);  // in flight while this fold's MMAs finish
            {
              GM_T0();
              ok = mbar_wait(acc_full + region, (folds / GM_REGIONS) & 1);
              if (r == 0) GM_TADD(7);
            }
            if (!ok) break;
            tc_fence_after();
            GM_T0();
            const float s = s_cur;
            s_cur = s_nxt;
#pragma unroll
            for (int c = 0; c < GM_NT / 16; ++c) {
              if (16 * c >= un.rows) break;
              float v[16];
              tmem_ld16(tmem + lane_base + region * GM_NT + 16 * c, v);
              if (I8) {  // s32 partials of one 128-column group: |sum| < 2^24, exact as floats
#pragma unroll
                for (int q = 0; q < 16; ++q) v[q] = (float)(int)__float_as_uint(v[q]);
              }
#pragma unroll
              for (int q = 0; q < 16; ++q) acc[16 * c + q] = fmaf(s, v[q], acc[16 * c + q]);
            }
            if (r == 0) GM_TADD(12);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + region);
            ++folds;
          }
          if (!ok) break;
          GM_T0();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < GM_NT; ++j)
            if (j < un.rows) dst[(size_t)j * a.N] = acc[j] * inv[j];
          if (r == 0) GM_TADD(13);
        } else {
          // one fold per unit: the row scale (int8 scale, W4/W6 s_channel) and each row's 2^-e, straight to out
          const int region = folds % GM_REGIONS;
          const float rs = fmt_row_scale(FMT) ? __ldg((const float*)a.scale + un.wrow + r)
                                              : __ldg(a.s_channel + un.wrow + r);
          {
            GM_T0();
            ok = mbar_wait(acc_full + region, (folds / GM_REGIONS) & 1);
            if (r == 0) GM_TADD(7);
          }
          if (!ok) break;
          tc_fence_after();
          __syncwarp();
#pragma unroll 1
          for (int c = 0; 16 * c < un.rows; ++c) {
            float v[16];
            tmem_ld16(tmem + lane_base + region * GM_NT + 16 * c, v);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const int j = 16 * c + q;
              if (j < un.rows) dst[(size_t)j * a.N] = v[q] * inv[j] * rs;
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty + region);
          ++folds;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
#ifdef D3_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) {
    g_gm_trace[blockIdx.x][9] = clock64() - t_kernel;
    int n = 0, tile, rb;
    for (int u = blockIdx.x; gm_unit(a, ntiles, u, tile, rb); u += G) ++n;
    g_gm_trace[blockIdx.x][8] = n;
  }
#endif
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, GM_TMEM_COLS);
  }
}

}  // namespace d3
