// Device helpers shared by every kernel of the routed-expert path: number formats (bfloat16, float8 e4m3), warp
// reductions, and the sm_100a asynchronous-copy machinery (mbarriers, bulk copies global -> shared, programmatic
// dependent launch). Every wait here is bounded by %globaltimer and reports a fault word instead of spinning forever.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define D3_DEV __device__ __forceinline__

namespace d3 {

// ---------------------------------------------------------------------------------------------------------------
// Fault word: set by a kernel that gave up a wait or skipped an out-of-range index; read and cleared by the host
// (d3_take_fault). One word per device, in this library's module.
enum : unsigned {
  FAULT_WAIT_TIMEOUT = 1u,  // an mbarrier or flag wait ran past its time limit
  FAULT_BAD_EXPERT = 2u,    // an expert id outside [0, E): the pair was skipped
  FAULT_BAD_SLOT = 4u,      // a slot index outside [0, count): the expert was skipped
  FAULT_TILES = 8u,         // the groups need more row tiles than the caller sized: the excess rows were skipped
  FAULT_EXCHANGE = 16u,     // an expert-parallel exchange area that does not fit the call: nothing was exchanged
};
__device__ unsigned int g_fault;

D3_DEV void record_fault(unsigned bits) { atomicOr(&g_fault, bits); }

constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;  // 2 s: far beyond any legal wait in these kernels

D3_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------------------------
// Number formats.
D3_DEV float bf16_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// float -> bfloat16 bits, round to nearest, ties to even (what a cast does for finite values).
D3_DEV uint16_t f32_to_bf16(float v) {
  uint32_t b = __float_as_uint(v);
  return (uint16_t)((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);
}

// Two float8 e4m3 values (low byte first) -> two halves, exactly (every e4m3 value is a half), by the hardware
// converter.
D3_DEV uint32_t e4m3x2_to_h2(uint16_t two) {
  uint32_t out;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(two));
  return out;
}

D3_DEV float h_lo(uint32_t h2) {
  float f;
  asm("{ .reg .f16 a, b; mov.b32 {a, b}, %1; cvt.f32.f16 %0, a; }" : "=f"(f) : "r"(h2));
  return f;
}
D3_DEV float h_hi(uint32_t h2) {
  float f;
  asm("{ .reg .f16 a, b; mov.b32 {a, b}, %1; cvt.f32.f16 %0, b; }" : "=f"(f) : "r"(h2));
  return f;
}

// Four e4m3 bytes of a word (byte 0 first) -> four floats.
D3_DEV void e4m3x4(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  uint32_t lo = e4m3x2_to_h2((uint16_t)(w & 0xFFFFu)), hi = e4m3x2_to_h2((uint16_t)(w >> 16));
  f0 = h_lo(lo);
  f1 = h_hi(lo);
  f2 = h_lo(hi);
  f3 = h_hi(hi);
}

// A single e4m3 byte -> float.
D3_DEV float e4m3_to_f32(uint32_t b) { return h_lo(e4m3x2_to_h2((uint16_t)(b & 0xFFu))); }

D3_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------------------------------------------
// Shared-memory mbarriers and bulk copies (cp.async.bulk, the untiled TMA path).
D3_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

D3_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

D3_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

D3_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

D3_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

D3_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `bar` with parity `parity` to complete; false (and the fault word set) after WAIT_LIMIT_NS.
D3_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long start = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - start > WAIT_LIMIT_NS) {
      record_fault(FAULT_WAIT_TIMEOUT);
      return false;
    }
  }
}

// The int8 activation quantization of N values: rint(x / s) clipped to +-127 (s = max|x| / 127; 0 when s == 0), with
// the quotient rounded correctly but without a division: r = __frcp_rn(s), y = x * r, then one correction step
// y' = y + r (x - y s) with fused multiply-adds (Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990), which gives the correctly rounded quotient from a correctly
// rounded reciprocal. Rounding x * r alone flips ties: with bf16 rows, x = max / 2 (x / s = 63.5) is common. A
// division, or an exact fix-up branch, in these loops made them several times slower.
template <int N>
D3_DEV void quant_i8_n(const float* v, float s, float r, float* q) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float y = v[i] * r;
    const float yq = fmaf(fmaf(-y, s, v[i]), r, y);
    q[i] = s > 0.0f ? fminf(127.0f, fmaxf(-127.0f, rintf(yq))) : 0.0f;
  }
}

D3_DEV uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

D3_DEV uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// `bytes` (a multiple of 16, both addresses 16-byte aligned) from global memory into this CTA's shared memory,
// completing on `bar`'s transaction count.
D3_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch: a dependent grid may start its prologue (which touches nothing the primary grid
// writes) early; it calls grid_dependency_wait() before reading the primary's output.
D3_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
D3_DEV void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier over the first `threads` threads of the block (ids 1..15; 0 is __syncthreads).
D3_DEV void named_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

}  // namespace d3
