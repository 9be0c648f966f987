// C ABI of the B200 routed-expert library (declared in include/drama3_b200.h). Every entry point checks its
// arguments, launches on the caller's stream, allocates nothing and never synchronizes (except d3_take_fault),
// so calls can be captured in CUDA graphs. Return value 0 or a D3_ERR_* code.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>

#include <cudaTypedefs.h>

#include "../../include/drama3_b200.h"
#include "common.cuh"
#include "gemv.cuh"
#include "grouped_mma.cuh"
#include "moe_decode.cuh"
#include "decode_tc.cuh"
#include "decode_tc8.cuh"
#include "decode_gv.cuh"
#include "resolve.cuh"
#include "router.cuh"
#include "shared.cuh"
#include "plan.cuh"
#include "rotate.cuh"
#include "route.cuh"

namespace {

thread_local int g_last_cuda = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return D3_OK;
  g_last_cuda = (int)e;
  return D3_ERR_CUDA;
}

int launch_status() { return cuda_status(cudaGetLastError()); }

bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int sms = 0;
  int smem_optin = 0;
  int cc = 0;
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];

int device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return D3_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sms == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    d.cc = major * 10 + minor;
  }
  *out = d;
  if (d.cc != 100) return D3_ERR_DEVICE;
  return D3_OK;
}

// Raise a kernel's dynamic shared-memory ceiling (once per device and kernel).
template <class K>
int allow_smem(K kernel, int bytes) {
  if (bytes <= 48 * 1024) return D3_OK;
  return cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

template <class K, class... Args>
int launch(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, args...));
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// A 2-D byte tensor [rows, row_bytes] read in boxes of box_bytes x 128 rows, with the shared-memory swizzle of that
// row width (128, 64 or 32 bytes).
bool byte_tile_map(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                   uint32_t box_rows = 128, bool swizzled = true) {
  const CUtensorMapSwizzle swizzle = !swizzled           ? CU_TENSOR_MAP_SWIZZLE_NONE
                                     : box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                     : box_bytes == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                     : box_bytes == 32  ? CU_TENSOR_MAP_SWIZZLE_32B
                                                        : CU_TENSOR_MAP_SWIZZLE_NONE;
  PFN_cuTensorMapEncodeTiled_v12000 fn = tensor_map_encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_bytes, box_rows};
  cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int static_smem(const void* kernel) {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) return 0;
  return (int)fa.sharedSizeBytes;
}

}  // namespace

extern "C" {

int d3_version(void) { return D3_VERSION; }

const char* d3_error_string(int code) {
  switch (code) {
    case D3_OK: return "ok";
    case D3_ERR_ARG: return "invalid argument (shape, count or format)";
    case D3_ERR_ALIGN: return "pointer not aligned as required (16 bytes for weight rows and activations)";
    case D3_ERR_CUDA: return "CUDA error at launch (see d3_last_cuda_error)";
    case D3_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case D3_ERR_WORKSPACE: return "workspace too small";
    case D3_ERR_TOO_LARGE: return "shape beyond the library-held scratch (at most 128 routed pairs, intermediate <= 768)";
    default: return "unknown error";
  }
}

int d3_last_cuda_error(void) { return g_last_cuda; }

int d3_device_check(void) {
  DeviceInfo d;
  return device_info(&d);
}

#ifdef D3_TRACE
// Trace builds only: copy the per-CTA phase timestamps (uint64 [1024][24]) to host memory.
int d3_trace_read(void* dst) { return cuda_status(cudaMemcpyFromSymbol(dst, d3::g_trace, sizeof(d3::g_trace))); }
// Trace builds only: the grouped GEMM's per-CTA wait counters (uint64 [1024][16]).
int d3_gm_trace_read(void* dst) {
  return cuda_status(cudaMemcpyFromSymbol(dst, d3::g_gm_trace, sizeof(d3::g_gm_trace)));
}
#endif

int d3_take_fault(unsigned int* fault) {
  if (fault == nullptr) return D3_ERR_ARG;
  unsigned int v = 0, zero = 0;
  int st = cuda_status(cudaMemcpyFromSymbol(&v, d3::g_fault, sizeof(v)));
  if (st) return st;
  st = cuda_status(cudaMemcpyToSymbol(d3::g_fault, &zero, sizeof(zero)));
  *fault = v;
  return st;
}

// ------------------------------------------------------------------------------------------------------------
int d3_route(const uint16_t* logits, int rows, int n, int k, int64_t* ids, float* weights, void* stream) {
  if (rows < 0 || n < 1 || n > d3::ROUTE_MAX_N || k < 1 || k > 32 || k > n) return D3_ERR_ARG;
  if (!logits || !ids || !weights) return D3_ERR_ARG;
  if (rows == 0) return D3_OK;
  dim3 grid((rows + d3::ROUTE_ROWS - 1) / d3::ROUTE_ROWS);
  d3::route_rows<<<grid, d3::ROUTE_ROWS * d3::ROUTE_GROUP, 0, (cudaStream_t)stream>>>(logits, rows, n, k, ids, weights);
  return launch_status();
}

int d3_weighted_sum(const float* parts, const float* weights, int rows, int k, int H, uint16_t* out, void* stream) {
  if (rows < 0 || k < 1 || H < 1 || rows > 65535 || !parts || !weights || !out) return D3_ERR_ARG;
  if (rows == 0) return D3_OK;
  dim3 grid((H + 255) / 256, rows);
  d3::combine_rows<<<grid, 256, 0, (cudaStream_t)stream>>>(parts, weights, rows, k, H, out);
  return launch_status();
}

int d3_rotate(const void* x, int mode, int rows, int K, float* out, const int* only_if, void* stream) {
  if (rows < 0 || K < 256 || K % 256 != 0 || K > 12288 || mode < 0 || mode > 2 || !x || !out) return D3_ERR_ARG;
  if (rows == 0) return D3_OK;
  int smem = K * 4;
  int st = allow_smem(d3::rotate_rows_kernel, smem);
  if (st) return st;
  d3::rotate_rows_kernel<<<rows, 256, smem, (cudaStream_t)stream>>>(x, mode, K, out, only_if);
  return launch_status();
}

int d3_router(const void* x, int M, int H, const void* w, int E, int k, int64_t* ids, float* weights, void* logits,
              void* stream) {
  if (!x || !w || !ids || !weights) return D3_ERR_ARG;
  if (M < 1 || M > d3::RT_MAX_M || H != d3::RT_H || E < 64 || E > d3::RT_MAX_E || E % 64 || k < 1 || k > 32 ||
      k > E)
    return D3_ERR_ARG;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(logits, 2)) return D3_ERR_ALIGN;
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  const int smem = (E / d3::RT_CTAS + d3::RT_MAX_M) * d3::RT_PITCH * 2;
  if (int st = allow_smem(d3::router_kernel, smem)) return st;
  return launch(d3::router_kernel, dim3(d3::RT_CTAS), dim3(d3::RT_WARPS * 32), smem, (cudaStream_t)stream, true,
                (const uint16_t*)x, M, (const uint16_t*)w, E, k, ids, weights, (uint16_t*)logits);
}

extern "C++" {
template <int KS>
static int shared_down(const void* scratch, int M, const void* w_d, const float* gate, void* out, cudaStream_t s) {
  const int smem = (d3::SH_DOWN_ROWS + d3::RT_MAX_M) * (KS * 128 + 8) * 2;
  if (int st = allow_smem(d3::shared_down_kernel<KS>, smem)) return st;
  return launch(d3::shared_down_kernel<KS>, dim3(d3::SH_H / d3::SH_DOWN_ROWS), dim3(d3::SH_WARPS * 32), smem, s, true,
                (const uint16_t*)scratch, M, (const uint16_t*)w_d, gate, (uint16_t*)out);
}
}

int d3_shared_expert(const void* x, int M, int H, const void* w_gu, const void* w_d, const void* w_g, int I,
                     void* scratch, void* out, void* stream) {
  if (!x || !w_gu || !w_d || !w_g || !scratch || !out) return D3_ERR_ARG;
  if (M < 1 || M > d3::RT_MAX_M || H != d3::SH_H || I < 256 || I > 1024 || I % 256) return D3_ERR_ARG;
  if (!aligned(x, 16) || !aligned(w_gu, 16) || !aligned(w_d, 16) || !aligned(w_g, 16) || !aligned(scratch, 16) ||
      !aligned(out, 2))
    return D3_ERR_ALIGN;
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  cudaStream_t s = (cudaStream_t)stream;
  // scratch: a [M, I] bf16, then the gate [M] fp32
  float* gate = reinterpret_cast<float*>((uint16_t*)scratch + (size_t)M * I);
  const int smem_up = (9 + d3::RT_MAX_M) * d3::SH_UP_PITCH * 2;
  if (int st = allow_smem(d3::shared_up_kernel, smem_up)) return st;
  if (int st = launch(d3::shared_up_kernel, dim3(I / d3::SH_UP_CH), dim3(d3::SH_WARPS * 32), smem_up, s, true,
                      (const uint16_t*)x, M, (const uint16_t*)w_gu, (const uint16_t*)w_g, I, (uint16_t*)scratch,
                      gate))
    return st;
  switch (I / 128) {
    case 2: return shared_down<2>(scratch, M, w_d, gate, out, s);
    case 4: return shared_down<4>(scratch, M, w_d, gate, out, s);
    case 6: return shared_down<6>(scratch, M, w_d, gate, out, s);
    default: return shared_down<8>(scratch, M, w_d, gate, out, s);
  }
}

int d3_prefill_plan(const int64_t* ids, int P, int E, int drop_invalid, int64_t* order, int64_t* pos, int* groups,
                    void* stream) {
  if (P < 0 || E < 1 || E > d3::PLAN_MAX_E || !groups || (P > 0 && (!ids || !order || !pos))) return D3_ERR_ARG;
  d3::prefill_plan_kernel<<<1, d3::PLAN_THREADS, 0, (cudaStream_t)stream>>>(ids, P, E, drop_invalid, order, pos,
                                                                           groups);
  return launch_status();
}

int d3_resolve(const int64_t* ids, int k, int layer, int layers, int experts, int* table, int* owner, float* score,
               int* at, int* pending, int count, int* clock, int* budget, int* plan, int* reads, int* step,
               const float* share, double half_life, int cpu, double admit, void* stream) {
  if (k < 1 || k > d3::RESOLVE_MAX_K || layers < 1 || layer < 0 || layer >= layers || experts < 1 || count < 1)
    return D3_ERR_ARG;
  if ((long long)layers * experts > 0x7fffffffLL) return D3_ERR_ARG;
  if (!ids || !table || !owner || !score || !at || !pending || !clock || !budget || !plan || !reads || !step || !share)
    return D3_ERR_ARG;
  d3::resolve_kernel<<<1, d3::RESOLVE_THREADS, 0, (cudaStream_t)stream>>>(ids, k, layer, layers, experts, table, owner,
                                                                         score, at, pending, count, clock, budget,
                                                                         plan, reads, step, share, half_life, cpu,
                                                                         admit);
  return launch_status();
}

// ------------------------------------------------------------------------------------------------------------
static int gemv_common(int fmt, const d3::GemvArgs& a, int k, void* stream) {
  // K % 32: the swizzled staging of x permutes float4 slots within aligned groups of eight
  if (k < 1 || k > 65535 || a.N < 16 || a.N % 16 || a.K < 32 || a.K % 32 || a.K > 32 * 16 * d3::GEMV_MAXV)
    return D3_ERR_ARG;
  if (a.x_rows != 1 && a.x_rows != k) return D3_ERR_ARG;
  if (a.num_experts < 1 || a.slots < 0) return D3_ERR_ARG;
  if (fmt == d3::FMT_FP8 && (a.N % 128 || a.K % 128)) return D3_ERR_ARG;
  if ((fmt == d3::FMT_W4 || fmt == d3::FMT_W6) && (a.K % 256)) return D3_ERR_ARG;
  if (fmt == d3::FMT_W4 && !a.codebook) return D3_ERR_ARG;
  if (!a.x || !a.ids || !a.plan || !a.host_w || !a.host_s || !a.out) return D3_ERR_ARG;
  if (!aligned(a.x, 16) || !aligned(a.host_w, 16) || (a.slot_w && !aligned(a.slot_w, 16))) return D3_ERR_ALIGN;
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  dim3 grid(a.N / d3::GEMV_ROWS, k);
  int smem = a.K * 4;
  cudaStream_t s = (cudaStream_t)stream;
  switch (fmt) {
    case d3::FMT_FP8:
      if (int st = allow_smem(d3::gemv_plan_kernel<d3::FMT_FP8>, smem)) return st;
      d3::gemv_plan_kernel<d3::FMT_FP8><<<grid, d3::GEMV_WARPS * 32, smem, s>>>(a);
      break;
    case d3::FMT_I8:
      if (int st = allow_smem(d3::gemv_plan_kernel<d3::FMT_I8>, smem)) return st;
      d3::gemv_plan_kernel<d3::FMT_I8><<<grid, d3::GEMV_WARPS * 32, smem, s>>>(a);
      break;
    case d3::FMT_W4:
      if (int st = allow_smem(d3::gemv_plan_kernel<d3::FMT_W4>, smem)) return st;
      d3::gemv_plan_kernel<d3::FMT_W4><<<grid, d3::GEMV_WARPS * 32, smem, s>>>(a);
      break;
    case d3::FMT_W6:
      if (int st = allow_smem(d3::gemv_plan_kernel<d3::FMT_W6>, smem)) return st;
      d3::gemv_plan_kernel<d3::FMT_W6><<<grid, d3::GEMV_WARPS * 32, smem, s>>>(a);
      break;
    default: return D3_ERR_ARG;
  }
  return launch_status();
}

int d3_gemv_fp8(const float* x, int x_rows, const int64_t* ids, const int* plan, int k, uint8_t* slot_w,
                float* slot_s, const uint8_t* host_w, const float* host_s, float* out, int N, int K,
                int num_experts, int slots, void* stream) {
  d3::GemvArgs a = {x, x_rows, ids, plan, nullptr, 0, slot_w, slot_s, nullptr, host_w, host_s, nullptr,
                    nullptr, out, N, K, num_experts, slots};
  return gemv_common(d3::FMT_FP8, a, k, stream);
}

int d3_gemv_int8(const float* x, int x_rows, const int64_t* ids, const int* plan, const int* took_over, int late,
                 int k, int8_t* slot_w, float* slot_s, const int8_t* host_w, const float* host_s, float* out, int N,
                 int K, int num_experts, int slots, void* stream) {
  if (!took_over) return D3_ERR_ARG;
  d3::GemvArgs a = {x, x_rows, ids, plan, took_over, late, (uint8_t*)slot_w, slot_s, nullptr, (const uint8_t*)host_w,
                    host_s, nullptr, nullptr, out, N, K, num_experts, slots};
  return gemv_common(d3::FMT_I8, a, k, stream);
}

int d3_gemv_codes(const float* x, int x_rows, const int64_t* ids, const int* plan, int k, uint8_t* slot_w,
                  uint8_t* slot_r, float* slot_c, const uint8_t* host_w, const uint8_t* host_r,
                  const float* host_c, const float* codebook, int bits, float* out, int N, int K, int num_experts,
                  int slots, void* stream) {
  if (bits != 4 && bits != 6) return D3_ERR_ARG;
  if (!host_c) return D3_ERR_ARG;
  d3::GemvArgs a = {x, x_rows, ids, plan, nullptr, 0, slot_w, slot_r, slot_c, host_w, host_r, host_c,
                    codebook, out, N, K, num_experts, slots};
  return gemv_common(bits == 4 ? d3::FMT_W4 : d3::FMT_W6, a, k, stream);
}

// ------------------------------------------------------------------------------------------------------------
static int grouped_common(int fmt, const d3::GroupedArgs& a, int n_groups, void* stream) {
  if (n_groups < 0 || n_groups > 65535 || a.N < 64 || a.N % 64 || a.K < 64 || a.K % 64 || a.x_rows < 0)
    return D3_ERR_ARG;
  if (fmt == d3::FMT_FP8 && (a.N % 128 || a.K % 128)) return D3_ERR_ARG;
  if ((fmt == d3::FMT_W4 || fmt == d3::FMT_W6) && (a.K % 256)) return D3_ERR_ARG;
  if (fmt == d3::FMT_W4 && !a.codebook) return D3_ERR_ARG;
  if (!a.x || !a.groups || !a.host_w || !a.host_s || !a.out) return D3_ERR_ARG;
  if (!aligned(a.x, 16) || !aligned(a.host_w, 16) || (a.slot_w && !aligned(a.slot_w, 16))) return D3_ERR_ALIGN;
  if (n_groups == 0 || a.x_rows == 0) return D3_OK;
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  int z = (a.x_rows + d3::GRP_TT - 1) / d3::GRP_TT;
  if (z > 64) z = 64;
  dim3 grid(a.N / d3::GRP_TN, n_groups, z);
  cudaStream_t s = (cudaStream_t)stream;
  switch (fmt) {
    case d3::FMT_FP8: d3::grouped_plan_kernel<d3::FMT_FP8><<<grid, 256, 0, s>>>(a); break;
    case d3::FMT_I8: d3::grouped_plan_kernel<d3::FMT_I8><<<grid, 256, 0, s>>>(a); break;
    case d3::FMT_W4: d3::grouped_plan_kernel<d3::FMT_W4><<<grid, 256, 0, s>>>(a); break;
    case d3::FMT_W6: d3::grouped_plan_kernel<d3::FMT_W6><<<grid, 256, 0, s>>>(a); break;
    default: return D3_ERR_ARG;
  }
  return launch_status();
}

int d3_grouped_fp8(const float* x, int x_rows, const int* groups, int n_groups, uint8_t* slot_w, float* slot_s,
                   const uint8_t* host_w, const float* host_s, float* out, int N, int K, int num_experts, int slots,
                   void* stream) {
  d3::GroupedArgs a = {x, groups, slot_w, slot_s, nullptr, host_w, host_s, nullptr, nullptr, out, N, K, num_experts,
                       slots, x_rows};
  return grouped_common(d3::FMT_FP8, a, n_groups, stream);
}

int d3_grouped_int8(const float* x, int x_rows, const int* groups, int n_groups, int8_t* slot_w, float* slot_s,
                    const int8_t* host_w, const float* host_s, float* out, int N, int K, int num_experts, int slots,
                    void* stream) {
  d3::GroupedArgs a = {x, groups, (uint8_t*)slot_w, slot_s, nullptr, (const uint8_t*)host_w, host_s, nullptr,
                       nullptr, out, N, K, num_experts, slots, x_rows};
  return grouped_common(d3::FMT_I8, a, n_groups, stream);
}

int d3_grouped_codes(const float* x, int x_rows, const int* groups, int n_groups, uint8_t* slot_w, uint8_t* slot_r,
                     float* slot_c, const uint8_t* host_w, const uint8_t* host_r, const float* host_c,
                     const float* codebook, int bits, float* out, int N, int K, int num_experts, int slots,
                     void* stream) {
  if (bits != 4 && bits != 6) return D3_ERR_ARG;
  if (!host_c) return D3_ERR_ARG;
  d3::GroupedArgs a = {x, groups, slot_w, slot_r, slot_c, host_w, host_r, host_c, codebook, out, N, K, num_experts,
                       slots, x_rows};
  return grouped_common(bits == 4 ? d3::FMT_W4 : d3::FMT_W6, a, n_groups, stream);
}

// ------------------------------------------------------------------------------------------------------------
// Grouped expert GEMM on the tensor cores (banks held whole on the GPU).

int d3_grouped_mma_tile_rows(void) { return d3::GM_NT; }

size_t d3_grouped_mma_workspace(int tiles, int K) {
  if (tiles < 0 || K < 256) return 0;
  return d3::gm_workspace_bytes(tiles, K);
}

int d3_grouped_mma(int fmt, const void* x, int x_bf16, const int64_t* row_index, int mode, const int* groups,
                   int n_groups, int tiles, const void* weight, const void* scale, const float* s_channel,
                   const float* codebook, int bank_rows, float* out, int N, int K, void* workspace,
                   size_t workspace_bytes, void* stream) {
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  if (fmt < 0 || fmt >= d3::FMT_COUNT || n_groups < 0 || tiles < 0) return D3_ERR_ARG;
  if (mode < 0 || mode > (d3::GM_ROTATE | d3::GM_SWIGLU)) return D3_ERR_ARG;
  if (d3::fmt_a8(fmt)) mode |= d3::GM_INT8;  // A8 formats always quantize their inputs to int8
  if (N < d3::GM_M || N % d3::GM_M || K < 256 || K % 256 || K > 2048 || bank_rows < N || bank_rows % d3::GM_M)
    return D3_ERR_ARG;
  if (!x || !groups || !weight || !scale || !out || !workspace) return D3_ERR_ARG;
  if ((fmt == d3::FMT_W4 || fmt == d3::FMT_W6) && !s_channel) return D3_ERR_ARG;
  if (fmt == d3::FMT_W4 && !codebook) return D3_ERR_ARG;
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(weight, 16) || !aligned(scale, 4) || !aligned(workspace, 256))
    return D3_ERR_ALIGN;
  if (workspace_bytes < d3::gm_workspace_bytes(tiles, K)) return D3_ERR_WORKSPACE;
  if (tiles == 0 || n_groups == 0) return D3_OK;
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  uint8_t* staged = ws;
  float* inv = (float*)(ws + d3::gm_staged_bytes(tiles, K));
  d3::GroupedTile* table = (d3::GroupedTile*)(inv + (size_t)tiles * d3::GM_NT);
  int* ntiles = (int*)(table + tiles);
  CUtensorMap wmap, pmap;
  const uint64_t row_bytes = (uint64_t)d3::fmt_row_bytes(fmt, K);
  // one raw stage = 128 columns: fp8 / fp8c / int8 128 bytes per row; W4 / W6 nibbles and W4A8 64; W6A8 96; the W6
  // high plane 32
  const uint32_t box = d3::fmt_e4m3(fmt) || fmt == d3::FMT_I8 ? 128 : fmt == d3::FMT_W6A8 ? 96 : 64;
  if (!byte_tile_map(&wmap, weight, row_bytes, (uint64_t)bank_rows, box)) return D3_ERR_ARG;
  pmap = wmap;
  if (fmt == d3::FMT_W6 && !byte_tile_map(&pmap, weight, row_bytes, (uint64_t)bank_rows, 32)) return D3_ERR_ARG;
  if (int st = launch((mode & d3::GM_ROTATE) ? d3::gm_stage_kernel<true> : d3::gm_stage_kernel<false>,
                      dim3(tiles, d3::GM_NT / d3::GM_STAGE_ROWS), dim3(256), 0, s, false, x, x_bf16, row_index, mode,
                      groups, n_groups, K, tiles, staged, inv, table, ntiles))
    return st;
  const int units = tiles * (N / d3::GM_M);
  d3::GmArgs a = {staged, inv, table, ntiles, groups, scale, s_channel, codebook, out, N, K, units, bank_rows};
  const int smem = d3::GmSmem::launch;
  const dim3 grid(units < d.sms ? units : d.sms);
  switch (fmt) {
#define D3_GM_CASE(F)                                                                    \
  case F: {                                                                              \
    if (int st = allow_smem(d3::grouped_mma_kernel<F>, smem)) return st;                 \
    return launch(d3::grouped_mma_kernel<F>, grid, dim3(d3::GM_THREADS), smem, s, false, wmap, pmap, a); \
  }
    D3_GM_CASE(d3::FMT_FP8)
    D3_GM_CASE(d3::FMT_I8)
    D3_GM_CASE(d3::FMT_W4)
    D3_GM_CASE(d3::FMT_W6)
    D3_GM_CASE(d3::FMT_FP8C)
    D3_GM_CASE(d3::FMT_W4A8)
    D3_GM_CASE(d3::FMT_W6A8)
#undef D3_GM_CASE
  }
  return D3_ERR_ARG;
}

int d3_prefill_combine(const float* sorted, const int64_t* pos, const void* weights, int w_bf16, int T, int k, int H,
                       void* out, int out_f32, void* stream) {
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  if (T < 0 || k < 1 || k > 64 || H < 4 || H % 4 || !sorted || !pos || !weights || !out) return D3_ERR_ARG;
  if (!aligned(sorted, 16) || !aligned(out, out_f32 ? 16 : 8)) return D3_ERR_ALIGN;
  if (T == 0) return D3_OK;
  return launch(d3::gm_combine_kernel, dim3(T), dim3(256), 0, (cudaStream_t)stream, false, sorted, pos, weights, w_bf16,
                k, H, out, out_f32);
}

// ------------------------------------------------------------------------------------------------------------
// Fused decode.
// Pairs a segment of one expert carries (the MMA's 8 columns): at most 8. An expert routed to more of the rows is
// cut into several segments, each reading it again.
static int cap_for(int M) { return M < d3::DEC_MAX_CAP ? M : d3::DEC_MAX_CAP; }

static size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t d3_moe_decode_workspace(int M, int k, int I) {
  if (M < 1 || k < 1 || I < 1) return 0;
  const size_t P = (size_t)M * k;
  return align256(P * I * 4) + align256(P * d3::DEC_H * 4) + d3::DEC_SYNC_BYTES;
}

}  // extern "C"

template <int FMT, bool XBF, int NKC>
static int decode_launch(const d3::DecodeArgs& a0, const DeviceInfo& d, cudaStream_t s) {
  auto kern = d3::moe_decode_kernel<FMT, XBF, NKC>;
  d3::DecodeArgs a = a0;
  const int SB = d3::decode_stage_bytes<FMT>(d3::DEC_H, a.I);
  const int limit = d.smem_optin - static_smem((const void*)kern);
  int ns = d3::DEC_MAX_STAGES;
  while (ns > 2 && d3::decode_smem<FMT, XBF>(d3::DEC_H, a.I, ns, SB).total > limit) --ns;
  const int smem = d3::decode_smem<FMT, XBF>(d3::DEC_H, a.I, ns, SB).total;
  if (smem > limit) return D3_ERR_ARG;
  a.stages = ns;
  a.stage_bytes = SB;
  if (int st = allow_smem(kern, smem)) return st;
  return launch(kern, dim3(d.sms), dim3(d3::DEC_ALL), smem, s, true, a);
}

template <int FMT, bool XBF>
static int decode_nkc(const d3::DecodeArgs& a, const DeviceInfo& d, cudaStream_t s) {
  switch (a.I) {
    case 512: return decode_launch<FMT, XBF, 2>(a, d, s);
    case 768: return decode_launch<FMT, XBF, 3>(a, d, s);
    default: return D3_ERR_ARG;
  }
}

// The tensor-core decode (per-channel e4m3 rows; faster than the mma.sync decode at every line count measured, 1-16):
// on unless D3_DECODE_TC=0 in the environment at the call, from D3_DECODE_TC_MIN lines (default 1) on (both kept for
// comparing the two kernels on the same inputs).
static bool decode_tc_enabled() {
  const char* v = getenv("D3_DECODE_TC");
  return !(v && v[0] == '0');
}

// The one-line streaming decode of per-channel e4m3 experts (moe_decode_gv_kernel); D3_DECODE_GV=0 turns it off.
static bool decode_gv_enabled() {
  const char* v = getenv("D3_DECODE_GV");
  return !(v && v[0] == '0');
}

template <int FMT, int I>
static int decode_gv_launch(const d3::DecodeArgs& a, const DeviceInfo& d, cudaStream_t s) {
  auto kern = d3::moe_decode_gv_kernel<FMT, I>;
  const int smem = d3::GvSmem<FMT>::total(I);
  if (int st = allow_smem(kern, smem)) return st;
  return launch(kern, dim3(d.sms), dim3(d3::GV_THREADS), smem, s, true, a);
}

// Segment counts up to which the tensor-core decodes combine each 128-row block as soon as its last tile is done;
// above it they combine after a grid barrier. D3_LASTARRIVE_NSEG sets it (default 0: always the grid barrier).
static int lastarrive_nseg() {
  const char* v = getenv("D3_LASTARRIVE_NSEG");
  return v ? atoi(v) : 0;
}

static int decode_tc_min_lines() {
  const char* v = getenv("D3_DECODE_TC_MIN");
  return v ? atoi(v) : 1;
}

template <int FMT, bool XBF, int NKB2>
static int decode_tc_launch(const d3::DecodeArgs& a, const CUtensorMap& m13, const CUtensorMap& m2,
                            const DeviceInfo& d, cudaStream_t s) {
  auto kern = d3::moe_decode_tc_kernel<FMT, XBF, NKB2>;
  const int smem = d3::TcSmem::launch;
  if (int st = allow_smem(kern, smem)) return st;
  return launch(kern, dim3(d.sms), dim3(d3::TC_THREADS), smem, s, true, m13, m2, a);
}

// e4m3 (fp8c) or int8 ConvRot rows: one byte a weight either way
template <int FMT>
static int decode_tc(const d3::DecodeArgs& a, const DeviceInfo& d, cudaStream_t s) {
  CUtensorMap m13, m2;
  // gate_up rows [e_count * 2I, H] in boxes of 64 rows x 128 bytes; down rows [e_count * H, I] in 128 x 128
  if (!byte_tile_map(&m13, a.w13, (uint64_t)a.H, (uint64_t)a.e_count * 2 * a.I, 128, 64)) return D3_ERR_ARG;
  if (!byte_tile_map(&m2, a.w2, (uint64_t)a.I, (uint64_t)a.e_count * a.H, 128, 128)) return D3_ERR_ARG;
  switch (a.I) {
    case 512:
      return a.x_bf16 ? decode_tc_launch<FMT, true, 4>(a, m13, m2, d, s) : decode_tc_launch<FMT, false, 4>(a, m13, m2, d, s);
    case 768:
      return a.x_bf16 ? decode_tc_launch<FMT, true, 6>(a, m13, m2, d, s) : decode_tc_launch<FMT, false, 6>(a, m13, m2, d, s);
    default: return D3_ERR_ARG;
  }
}

template <bool XBF, int NKB2>
static int decode_tc8_launch(const d3::DecodeArgs& a, const CUtensorMap& m13, const CUtensorMap& m2,
                             const DeviceInfo& d, cudaStream_t s) {
  auto kern = d3::moe_decode_tc8_kernel<XBF, NKB2>;
  const int smem = d3::T8Smem::launch;
  if (int st = allow_smem(kern, smem)) return st;
  return launch(kern, dim3(d.sms), dim3(d3::TC_THREADS), smem, s, true, m13, m2, a);
}

// W4A8 on the tensor cores: packed rows in boxes of 64 bytes (128 int4 columns), unswizzled (the converter warps
// read them row by row)
static int decode_tc8(const d3::DecodeArgs& a, const DeviceInfo& d, cudaStream_t s) {
  CUtensorMap m13, m2;
  if (!byte_tile_map(&m13, a.w13, (uint64_t)a.H / 2, (uint64_t)a.e_count * 2 * a.I, 64, 64, false)) return D3_ERR_ARG;
  if (!byte_tile_map(&m2, a.w2, (uint64_t)a.I / 2, (uint64_t)a.e_count * a.H, 64, 128, false)) return D3_ERR_ARG;
  switch (a.I) {
    case 512: return a.x_bf16 ? decode_tc8_launch<true, 4>(a, m13, m2, d, s) : decode_tc8_launch<false, 4>(a, m13, m2, d, s);
    case 768: return a.x_bf16 ? decode_tc8_launch<true, 6>(a, m13, m2, d, s) : decode_tc8_launch<false, 6>(a, m13, m2, d, s);
    default: return D3_ERR_ARG;
  }
}

// The host-side checks of a decode call's arguments other than its workspace: 0 or an error code. Every decode entry
// point runs them before it asks the runtime anything or puts anything on the stream.
static int check_decode(int fmt, const void* x, int M, int k, int E, int e_first, int e_count, int H, int I,
                        const int64_t* ids, const float* weights, const uint8_t* w13, const void* s13,
                        const float* c13, const uint8_t* w2, const void* s2, const float* c2,
                        const float* codebook13, const float* codebook2, bool has_out, const void* exchange) {
  if (fmt < 0 || fmt >= d3::FMT_COUNT) return D3_ERR_ARG;
  if (M < 1 || M > 16 || k < 1 || k > 32 || M * k > d3::DEC_MAX_PAIRS || E < 1) return D3_ERR_ARG;
  if (e_first < 0 || e_count < 1 || e_first + e_count > E) return D3_ERR_ARG;
  if (H != d3::DEC_H || (I != 512 && I != 768)) return D3_ERR_ARG;
  if (!x || !ids || !weights || !w13 || !s13 || !w2 || !s2 || !has_out) return D3_ERR_ARG;
  if (d3::fmt_codes(fmt) && (!c13 || !c2)) return D3_ERR_ARG;
  if (fmt == d3::FMT_W4 && (!codebook13 || !codebook2)) return D3_ERR_ARG;
  if (!aligned(x, 16) || !aligned(w13, 16) || !aligned(w2, 16) || !aligned(s13, 16) || !aligned(s2, 16) ||
      !aligned(exchange, 8))
    return D3_ERR_ALIGN;
  return D3_OK;
}

static int decode_common(int fmt, const void* x, int x_bf16, int M, int k, int E, int e_first, int e_count, int H,
                         int I, const int64_t* ids, const float* weights, const uint8_t* w13, const void* s13,
                         const float* c13, const uint8_t* w2, const void* s2, const float* c2,
                         const float* codebook13, const float* codebook2, uint16_t* out, float* out_f32,
                         const void* exchange, void* workspace, size_t workspace_bytes, void* stream) {
  if (int st = check_decode(fmt, x, M, k, E, e_first, e_count, H, I, ids, weights, w13, s13, c13, w2, s2, c2,
                            codebook13, codebook2, out || out_f32 || exchange, exchange))
    return st;
  if (!workspace) return D3_ERR_ARG;
  if (workspace_bytes < d3_moe_decode_workspace(M, k, I)) return D3_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return D3_ERR_ALIGN;
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  const size_t P = (size_t)M * k;
  uint8_t* ws = (uint8_t*)workspace;
  float* a1 = (float*)ws;
  float* parts = (float*)(ws + align256(P * I * 4));
  // the synchronization words sit at the end of the caller's workspace, so a workspace reused for several shapes
  // keeps them in one place
  uint8_t* tail = ws + ((workspace_bytes - d3::DEC_SYNC_BYTES) & ~(size_t)255);
  auto* barrier = (unsigned long long*)tail;
  auto* words = (unsigned*)tail;
  const int cap = cap_for(M);
  d3::DecodeArgs a = {x, x_bf16, ids, weights, M, k, E, H, I, w13, s13, c13, codebook13, w2, s2, c2, codebook2,
                      out, out_f32, e_first, e_count, (const d3::EpExchange*)exchange, words + 4, a1, parts, barrier,
                      words + 16, words + 128, words + 384, 0, 0, cap, lastarrive_nseg()};
  cudaStream_t s = (cudaStream_t)stream;
  // e4m3 rows (per channel or in 128 x 128 blocks), int8 ConvRot rows and W4A8 at one line: the streaming kernel (its row blocks of
  // 2048 / (G / pairs) rows fit 8 tiles of 16 from 128 CTAs; its counters cover 256)
  if ((fmt == d3::FMT_FP8C || fmt == d3::FMT_FP8 || fmt == d3::FMT_W4A8 || fmt == d3::FMT_I8) && M == 1 &&
      k <= d3::GV_MAX_PAIRS && out && !out_f32 && !exchange && e_first == 0 && d.sms >= d3::GV_MIN_GRID &&
      d.sms <= d3::DEC_MAX_GRID && decode_gv_enabled()) {
    if (fmt == d3::FMT_I8)
      return a.I == 768 ? decode_gv_launch<d3::FMT_I8, 768>(a, d, s) : decode_gv_launch<d3::FMT_I8, 512>(a, d, s);
    if (fmt == d3::FMT_FP8)
      return a.I == 768 ? decode_gv_launch<d3::FMT_FP8, 768>(a, d, s) : decode_gv_launch<d3::FMT_FP8, 512>(a, d, s);
    if (fmt == d3::FMT_W4A8)
      return a.I == 768 ? decode_gv_launch<d3::FMT_W4A8, 768>(a, d, s) : decode_gv_launch<d3::FMT_W4A8, 512>(a, d, s);
    return a.I == 768 ? decode_gv_launch<d3::FMT_FP8C, 768>(a, d, s) : decode_gv_launch<d3::FMT_FP8C, 512>(a, d, s);
  }
  // per-channel e4m3: the tensor-core kernel (its phase-2 split needs one CTA per segment at least: at most
  // M * k <= 128 segments)
  if (fmt == d3::FMT_FP8C && M >= decode_tc_min_lines() && d.sms >= d3::DEC_MAX_PAIRS && e_count <= d3::TC_MAX_E &&
      decode_tc_enabled())
    return decode_tc<d3::FMT_FP8C>(a, d, s);
  // int8 ConvRot: from 3 lines (each CTA rotates the lines' rows while staging them, which costs more than the
  // mma.sync decode saves at one or two lines: 27.3 against 24.2 us a layer at one line, 43.9 against 50.1 at four)
  if (fmt == d3::FMT_I8 && M >= std::max(3, decode_tc_min_lines()) && d.sms >= d3::DEC_MAX_PAIRS &&
      e_count <= d3::TC_MAX_E && decode_tc_enabled())
    return decode_tc<d3::FMT_I8>(a, d, s);
  if (fmt == d3::FMT_W4A8 && M >= decode_tc_min_lines() && d.sms >= d3::DEC_MAX_PAIRS && e_count <= d3::TC_MAX_E &&
      decode_tc_enabled())
    return decode_tc8(a, d, s);
  switch (fmt) {
    case d3::FMT_FP8:
      return x_bf16 ? decode_nkc<d3::FMT_FP8, true>(a, d, s) : decode_nkc<d3::FMT_FP8, false>(a, d, s);
    case d3::FMT_I8: return decode_nkc<d3::FMT_I8, true>(a, d, s);
    case d3::FMT_W4: return decode_nkc<d3::FMT_W4, true>(a, d, s);
    case d3::FMT_W6: return decode_nkc<d3::FMT_W6, true>(a, d, s);
    case d3::FMT_FP8C:
      return x_bf16 ? decode_nkc<d3::FMT_FP8C, true>(a, d, s) : decode_nkc<d3::FMT_FP8C, false>(a, d, s);
    case d3::FMT_W4A8: return decode_nkc<d3::FMT_W4A8, true>(a, d, s);
    case d3::FMT_W6A8: return decode_nkc<d3::FMT_W6A8, true>(a, d, s);
  }
  return D3_ERR_ARG;
}

extern "C" int d3_moe_decode(int fmt, const void* x, int x_bf16, int M, int k, int E, int H, int I, const int64_t* ids,
                             const float* weights, const uint8_t* w13, const void* s13, const float* c13,
                             const uint8_t* w2, const void* s2, const float* c2, const float* codebook13,
                             const float* codebook2, uint16_t* out, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (!out) return D3_ERR_ARG;
  return decode_common(fmt, x, x_bf16, M, k, E, 0, E, H, I, ids, weights, w13, s13, c13, w2, s2, c2, codebook13,
                       codebook2, out, nullptr, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int d3_moe_decode_ep(int fmt, const void* x, int x_bf16, int M, int k, int E, int e_first, int e_count,
                                int H, int I, const int64_t* ids, const float* weights, const uint8_t* w13,
                                const void* s13, const float* c13, const uint8_t* w2, const void* s2, const float* c2,
                                const float* codebook13, const float* codebook2, float* partial,
                                const void* exchange, void* workspace, size_t workspace_bytes, void* stream) {
  if (!partial && !exchange) return D3_ERR_ARG;
  if (partial && !aligned(partial, 16)) return D3_ERR_ALIGN;
  return decode_common(fmt, x, x_bf16, M, k, E, e_first, e_count, H, I, ids, weights, w13, s13, c13, w2, s2, c2,
                       codebook13, codebook2, nullptr, exchange ? nullptr : partial, exchange, workspace,
                       workspace_bytes, stream);
}

// ------------------------------------------------------------------------------------------------------------
// Expert-parallel exchange over peer memory.

extern "C" size_t d3_ep_exchange_bytes(int world, int m_max, int H) {
  if (world < 1 || world > d3::EP_MAX_RANKS || m_max < 1 || H < 1) return 0;
  return align256((size_t)2 * world * m_max * H * 4) + 256;
}

extern "C" int d3_ep_reduce(const void* exchange, int M, int H, void* out, void* stream) {
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  if (!exchange || !out || M < 1 || H < 1) return D3_ERR_ARG;
  if (H % 4) return D3_ERR_ARG;
  if (!aligned(exchange, 8) || !aligned(out, 8)) return D3_ERR_ALIGN;
  const int blocks = (int)(((size_t)M * H / 4 + d3::EP_REDUCE_THREADS - 1) / d3::EP_REDUCE_THREADS);
  return launch(d3::ep_reduce_kernel, dim3(blocks), dim3(d3::EP_REDUCE_THREADS), 0, (cudaStream_t)stream, true,
                (const d3::EpExchange*)exchange, M, H, (uint16_t*)out);
}

namespace {
PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuMemGetAddressRange_v3020)p;
  });
  return fn;
}
}  // namespace

extern "C" int d3_ipc_handle(const void* ptr, void* handle, size_t* offset) {
  if (!ptr || !handle || !offset) return D3_ERR_ARG;
  PFN_cuMemGetAddressRange_v3020 fn = address_range_fn();
  if (!fn) return D3_ERR_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return D3_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (int st = cuda_status(cudaIpcGetMemHandle(&h, (void*)base))) return st;
  memcpy(handle, &h, sizeof(h));
  *offset = (size_t)((uintptr_t)ptr - (uintptr_t)base);
  return D3_OK;
}

extern "C" int d3_ipc_open(const void* handle, size_t offset, void** ptr, void** base) {
  if (!handle || !ptr || !base) return D3_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  if (int st = cuda_status(cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess))) return st;
  *base = b;
  *ptr = (void*)((uintptr_t)b + offset);
  return D3_OK;
}

extern "C" int d3_ipc_close(void* base) {
  if (!base) return D3_ERR_ARG;
  return cuda_status(cudaIpcCloseMemHandle(base));
}

// ------------------------------------------------------------------------------------------------------------
// Fused decode without a caller-provided workspace, for callers that cannot allocate device memory themselves.
// The scratch is this file-scope array, sized for the largest decode the kernel takes (16 rows x top-8 = 128 routed
// pairs, intermediate 768, hidden 2048): 1,445,888 bytes that every GPU loading the library holds until exit.
// Host code cannot use the array's name as a device address: set-up, once per device with that device current,
// asks the runtime for the address (cudaGetSymbolAddress) and keeps it.
namespace {

constexpr size_t kStaticScratchBytes = 128u * 768u * 4u + 128u * 2048u * 4u + d3::DEC_SYNC_BYTES;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

void* g_static_ptr[kMaxDevices];

// The device address of g_static_scratch on the current device (set up on first use: not inside a stream capture).
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return D3_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_static_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (int st = cuda_status(cudaGetSymbolAddress(&p, g_static_scratch))) return st;
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return D3_OK;
}

}  // namespace

extern "C" int d3_moe_decode_static(int fmt, const void* x, int x_bf16, int M, int k, int E, int H, int I,
                                    const int64_t* ids, const float* weights, const uint8_t* w13, const void* s13,
                                    const float* c13, const uint8_t* w2, const void* s2, const float* c2,
                                    const float* codebook13, const float* codebook2, uint16_t* out, void* stream) {
  if (M < 1 || k < 1 || I < 1) return D3_ERR_ARG;
  if ((long long)M * k > 128 || I > 768 || d3_moe_decode_workspace(M, k, I) > kStaticScratchBytes)
    return D3_ERR_TOO_LARGE;
  // every other argument is checked before the array is looked up or anything is put on the stream
  if (int st = check_decode(fmt, x, M, k, E, 0, E, H, I, ids, weights, w13, s13, c13, w2, s2, c2, codebook13,
                            codebook2, out != nullptr, nullptr))
    return st;
  DeviceInfo d;
  if (int st = device_info(&d)) return st;
  void* ws = nullptr;
  if (int st = static_scratch(&ws)) return st;
  // The array keeps the last call's contents; of them only the synchronization words at its end must start at zero
  // (every call leaves them so, but a call that recorded a fault may not). Cleared on the stream, ahead of the
  // kernel.
  unsigned char* tail = (unsigned char*)ws + kStaticScratchBytes - d3::DEC_SYNC_BYTES;
  if (int st = cuda_status(cudaMemsetAsync(tail, 0, d3::DEC_SYNC_BYTES, (cudaStream_t)stream))) return st;
  return d3_moe_decode(fmt, x, x_bf16, M, k, E, H, I, ids, weights, w13, s13, c13, w2, s2, c2, codebook13, codebook2,
                       out, ws, kStaticScratchBytes, stream);
}
