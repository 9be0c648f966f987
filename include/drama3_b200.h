/* drama3_b200: the routed-expert MoE path of ComfyUI-Drama3, as a C ABI over hand-written sm_100a (B200) kernels.
 *
 * Conventions for every entry point:
 *   - all tensor arguments are device pointers (or pinned, mapped host pointers where a "host_*" field says so);
 *   - `stream` is a cudaStream_t (NULL: the legacy default stream); the call launches on it and returns without
 *     synchronizing, so calls can be captured in CUDA graphs;
 *   - nothing is allocated: outputs and workspaces are the caller's;
 *   - the return value is D3_OK (0) or a D3_ERR_* code, checked before any launch;
 *   - kernels never trap on bad data: an out-of-range expert id or slot is skipped (zeros) and recorded in a
 *     per-device fault word that d3_take_fault() reads and clears; a wait that runs past its limit does the same.
 *
 * Each entry cites the reference interface it replaces, as path:line inside PedroMarinhoDev/ComfyUI-Drama3. The
 * reference launches these computations from Python (drama3/kernels.py) through NVRTC; there is no C FFI there.
 */
#ifndef DRAMA3_B200_H
#define DRAMA3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define D3_VERSION 100

#define D3_OK 0
#define D3_ERR_ARG 1       /* a shape, count, format or null pointer the kernels do not take */
#define D3_ERR_ALIGN 2     /* a weight, activation or workspace pointer not 16-byte aligned */
#define D3_ERR_CUDA 3      /* the launch failed; d3_last_cuda_error() has the cudaError_t */
#define D3_ERR_DEVICE 4    /* the current device is not compute capability 10.0 */
#define D3_ERR_WORKSPACE 5 /* the workspace is smaller than d3_moe_decode_workspace() */
#define D3_ERR_TOO_LARGE 6 /* beyond the library-held scratch of d3_moe_decode_static() */

/* Weight formats of the fused decode (the reference's safetensors layouts; drama3/offload.py:72-90,755-766). */
#define D3_FMT_FP8 0  /* e4m3 rows + fp32 128x128 block scales */
#define D3_FMT_INT8 1 /* int8 ConvRot rows + fp32 row scales */
#define D3_FMT_W4 2   /* 4-bit codes + e4m3 group-16 scales + s_channel + 16-entry codebook, ConvRot */
#define D3_FMT_W6 3   /* 6-bit codes (nibble plane + 2-bit plane) + e4m3 group-16 scales + s_channel, ConvRot */
/* The BASELINE layouts (no counterpart in the reference; d3_moe_decode and d3_grouped_mma): */
#define D3_FMT_FP8C 4 /* e4m3 rows + fp32 per-output-channel scales [E*N] */
#define D3_FMT_W4A8 5 /* int4 (-7..7) two per byte, low nibble = even column; bf16 group-128 scales [E*N, K/128];
                       * activations quantized to int8 per row (absmax / 127) before each GEMV */
#define D3_FMT_W6A8 6 /* int6 (-31..31), four per three bytes (24-bit little-endian words); bf16 group-128 scales;
                       * int8 activations as W4A8 */

int d3_version(void);
const char* d3_error_string(int code);
int d3_last_cuda_error(void);

/* D3_OK when the current device is an sm_100 GPU; stands in for the reference's availability probe
 * drama3/kernels.py:604-615 (available), which there falls back to PyTorch; here there is no fallback. */
int d3_device_check(void);

/* Reads and clears the current device's fault word (synchronous). Bits: D3_FAULT_WAIT (1) a wait timed out,
 * D3_FAULT_EXPERT (2) an expert id out of range, D3_FAULT_SLOT (4) a slot out of range, D3_FAULT_TILES (8) a
 * grouped GEMM given fewer row tiles than its groups need, D3_FAULT_EXCHANGE (16) an expert-parallel exchange area
 * whose geometry does not fit the call. No counterpart in the reference, whose kernels do not check indices. */
#define D3_FAULT_WAIT 1u
#define D3_FAULT_EXPERT 2u
#define D3_FAULT_SLOT 4u
#define D3_FAULT_TILES 8u
#define D3_FAULT_EXCHANGE 16u
int d3_take_fault(unsigned int* fault);

/* Decode routing, `rows` independent rows: ids [rows, k] (int64) and weights [rows, k] (fp32 holding bfloat16
 * values) of logits [rows, n] (bfloat16): the k largest by (value desc, index asc) and their softmax weights
 * renormalized over them. n <= 1024, k <= 32.
 * Replaces drama3/kernels.py:39-67 (route_experts) and its launcher :647-653 (route), which take one row. */
int d3_route(const uint16_t* logits, int rows, int n, int k, int64_t* ids, float* weights, void* stream);

/* out [rows, H] (bfloat16) = sum_e parts[row*k + e, :] * weights[row*k + e], fp32 in e order.
 * Replaces drama3/kernels.py:69-76 (weighted_sum) and :656-661. */
int d3_weighted_sum(const float* parts, const float* weights, int rows, int k, int H, uint16_t* out, void* stream);

/* ConvRot rotation of rows: mode 0 fp32 x [rows, K], 1 bfloat16 x [rows, K], 2 fp32 x [rows, 2K] gate|up with
 * SwiGLU first; out fp32 [rows, K] (out may equal x); skipped when only_if (device int, may be NULL) is 0.
 * K % 256 == 0. Replaces drama3/kernels.py:222-258 (rotate_rows) and :636-644 (rotate). */
int d3_rotate(const void* x, int mode, int rows, int K, float* out, const int* only_if, void* stream);

/* The prompt pass's sort of its (token, rank) pairs by expert, on the device, in one launch (replaces the host-side
 * sort and group list of drama3/offload.py:141-145, which reads the counts back to the host): ids [P] int64 ->
 * order [P] int64 (pairs by expert id, within an expert in index order; ids outside [0, E) last), pos [P] int64 (the
 * inverse of order), groups [E + 1][5] int32 (expert, slot = expert, 0, first row, rows; group E holds the
 * out-of-range ids, with 0 rows when drop_invalid). 1 <= E <= 256. */
int d3_prefill_plan(const int64_t* ids, int P, int E, int drop_invalid, int64_t* order, int64_t* pos, int* groups,
                    void* stream);

/* The router of a decode step in one launch: SparseMoeBlock's gate linear (drama3/model.py:115, a bias-free bf16
 * linear hidden -> experts) and kernels.route (drama3/kernels.py:647-653) on its output. x [M, H] bf16, w [E, H]
 * bf16 -> ids [M, k] int64, weights [M, k] fp32 (bf16 values, renormalized softmax of the k largest logits), and the
 * logits [M, E] bf16 when `logits` is not null. The logits are the bf16 rounding of fp32 sums of the exact products;
 * ids and weights are kernels.route's on them. M <= 16, H == 2048, E % 64 == 0, E <= 256, k <= min(32, E); x and w
 * 16-byte aligned. */
int d3_router(const void* x, int M, int H, const void* w, int E, int k, int64_t* ids, float* weights, void* logits,
              void* stream);

/* The shared expert of a decode step, sigmoid-gated and added to the MoE output, in two launches (drama3/model.py:40-47
 * and :123: out + sigmoid(shared_expert_gate(x)) * shared_expert(x)). x [M, H] bf16; w_gu [2I, H] bf16 (gate rows,
 * then up rows), w_d [H, I] bf16, w_g [H] bf16 (the gate linear's one row); scratch: M * I bf16 then M fp32 of the
 * caller's (the SwiGLU rows and the gate values between the launches); out [M, H] bf16, updated in place. bf16
 * rounding where the reference's bf16 modules round. M <= 16, H == 2048, I in {256, 512, 768, 1024}; x, the weights
 * and scratch 16-byte aligned. */
int d3_shared_expert(const void* x, int M, int H, const void* w_gu, const void* w_d, const void* w_g, int I,
                     void* scratch, void* out, void* stream);

/* Slot-cache lookup and eviction for one decode row's k experts of `layer`; writes plan [k, 2] (slot, code) and
 * updates the cache state in place. Same state arrays and semantics as drama3/kernels.py:78-191 (resolve_experts),
 * launcher :618-625 (resolve); k <= 32. */
int d3_resolve(const int64_t* ids, int k, int layer, int layers, int experts, int* table, int* owner, float* score,
               int* at, int* pending, int count, int* clock, int* budget, int* plan, int* reads, int* step,
               const float* share, double half_life, int cpu, double admit, void* stream);

/* Per-expert GEMVs under a slot plan: out [k, N] fp32 = expert e's rows . x[e or 0] (x fp32 [x_rows, K],
 * x_rows 1 or k). Expert e comes from slot plan[2e] (code 0) or from host memory expert ids[e] (code != 0,
 * mapped pinned memory), filling its slot when plan[2e] >= 0. num_experts bounds ids, slots bounds plan slots.
 * Replace drama3/kernels.py:316-363 (gemv_fp8) / :674-681, :274-314 (gemv_int8) / :664-671, :495-536
 * (gemv_codes) / :703-713. N % 16 == 0, K % 32 == 0, K <= 4096 (fp8 N, K % 128; codes K % 256). */
int d3_gemv_fp8(const float* x, int x_rows, const int64_t* ids, const int* plan, int k, uint8_t* slot_w,
                float* slot_s, const uint8_t* host_w, const float* host_s, float* out, int N, int K,
                int num_experts, int slots, void* stream);
int d3_gemv_int8(const float* x, int x_rows, const int64_t* ids, const int* plan, const int* took_over, int late,
                 int k, int8_t* slot_w, float* slot_s, const int8_t* host_w, const float* host_s, float* out, int N,
                 int K, int num_experts, int slots, void* stream);
int d3_gemv_codes(const float* x, int x_rows, const int64_t* ids, const int* plan, int k, uint8_t* slot_w,
                  uint8_t* slot_r, float* slot_c, const uint8_t* host_w, const uint8_t* host_r,
                  const float* host_c, const float* codebook, int bits, float* out, int N, int K, int num_experts,
                  int slots, void* stream);

/* Prompt rows grouped by expert: groups [n_groups, 5] int32 (expert, slot, fill, first, rows) over x fp32
 * [x_rows, K] sorted by expert; out [x_rows, N] fp32 (rows outside every group untouched).
 * Replace drama3/kernels.py:408-464 (grouped_fp8) / :694-700, :365-406 (grouped_int8) / :684-691, :538-587
 * (grouped_codes) / :716-724. N % 64 == 0, K % 64 == 0. */
int d3_grouped_fp8(const float* x, int x_rows, const int* groups, int n_groups, uint8_t* slot_w, float* slot_s,
                   const uint8_t* host_w, const float* host_s, float* out, int N, int K, int num_experts, int slots,
                   void* stream);
int d3_grouped_int8(const float* x, int x_rows, const int* groups, int n_groups, int8_t* slot_w, float* slot_s,
                    const int8_t* host_w, const float* host_s, float* out, int N, int K, int num_experts, int slots,
                    void* stream);
int d3_grouped_codes(const float* x, int x_rows, const int* groups, int n_groups, uint8_t* slot_w, uint8_t* slot_r,
                     float* slot_c, const uint8_t* host_w, const uint8_t* host_r, const float* host_c,
                     const float* codebook, int bits, float* out, int N, int K, int num_experts, int slots,
                     void* stream);

/* The grouped kernels above on the tensor cores, for banks held whole on the GPU (every group's `slot` column is the
 * expert's index in the bank; `fill` is ignored): the same outputs as d3_grouped_fp8 / _int8 / _codes for
 * drama3/offload.py:126-149 (resident_prefill), up to summation order. fmt = D3_FMT_*; weight / scale / s_channel /
 * codebook are the bank's fields (fp8: e4m3 rows + fp32 128x128 blocks; int8: rows + fp32 row scales; W4/W6: codes
 * + e4m3 group-16 scales + fp32 s_channel, codebook float[16] for W4), bank_rows = rows in the bank (E * N).
 * Sorted row s of the GEMM input is x[row_index ? row_index[s] : s] (fp32, or bf16 when x_bf16), transformed by
 * `mode`: D3_GM_SWIGLU (x rows hold 2K columns, gate then up: SiLU(gate) * up, the reference rotate kernel's form),
 * then D3_GM_ROTATE (ConvRot over each 256 columns, as kernels.rotate) - so a prompt pass needs no separate gather,
 * SwiGLU or rotation launches. tiles = sum over groups of ceil(rows / d3_grouped_mma_tile_rows()) (an upper bound
 * is allowed: the kernels count the tiles on the device; fewer records D3_FAULT_TILES and skips the rows past them).
 * Groups of 0 rows get no tile, so a caller may list every expert and build the groups on the device.
 * N % 128 == 0, K % 256 == 0, K <= 2048; x, out and weight 16-byte aligned, workspace 256-byte aligned,
 * d3_grouped_mma_workspace(tiles, K) bytes (no initial state). No counterpart in the reference's kernel set beyond
 * the grouped kernels it replaces for resident banks. */
#define D3_GM_ROTATE 1
#define D3_GM_SWIGLU 2
int d3_grouped_mma_tile_rows(void);
size_t d3_grouped_mma_workspace(int tiles, int K);
int d3_grouped_mma(int fmt, const void* x, int x_bf16, const int64_t* row_index, int mode, const int* groups,
                   int n_groups, int tiles, const void* weight, const void* scale, const float* s_channel,
                   const float* codebook, int bank_rows, float* out, int N, int K, void* workspace,
                   size_t workspace_bytes, void* stream);

/* The combine of a prompt pass (drama3/offload.py:146-149): out[t] = sum over k' of weights[t, k'] *
 * sorted[pos[t * k + k']] (fp32 [rows, H]; pos = each pair's row in the sorted order), in rank order, into out
 * [T, H]: bf16 (rounded to nearest even), or fp32 when out_f32. weights fp32 or bf16 (w_bf16). H % 4 == 0. */
int d3_prefill_combine(const float* sorted, const int64_t* pos, const void* weights, int w_bf16, int T, int k, int H,
                       void* out, int out_f32, void* stream);

/* Bytes of workspace d3_moe_decode needs for M rows, top-k and expert width I. */
size_t d3_moe_decode_workspace(int M, int k, int I);

/* Fused decode of M rows (1..16) through their routed experts held whole in device memory:
 *   out [M, H] bf16 = sum_j weights[t, j] * down_{ids[t,j]}(SwiGLU(gate_up_{ids[t,j]} . x[t]))
 * with x [M, H] (bfloat16 when x_bf16, else fp32), ids [M, k] int64, weights [M, k] fp32. Banks in the reference
 * layouts, flattened over experts: w13 [E*2I, row] (gate rows then up rows per expert), w2 [E*H, row];
 * s13/s2: fp8 block scales (fp32 [E*N/128, K/128]), int8 row scales (fp32 [E*N]) or code group scales
 * (uint8 e4m3 [E*N, K/16]); c13/c2: s_channel (codes only); codebook13/2: W4 codebooks (fp32 [16]).
 * ConvRot formats rotate x and the SwiGLU output as the reference does. Each unique expert of the M*k pairs is
 * read once (an expert routed to more than 8 of the rows is read once per 8 of them). H == 2048, I % 128 == 0 (% 256 for ConvRot formats), M*k <= 128.
 * Replaces the chain drama3/offload.py:108-123 (resident_decode) = gemv -> SwiGLU/rotate -> gemv -> weighted_sum,
 * which drama3/model.py:111-113 runs once per row of a lines-at-once batch. */
int d3_moe_decode(int fmt, const void* x, int x_bf16, int M, int k, int E, int H, int I, const int64_t* ids,
                  const float* weights, const uint8_t* w13, const void* s13, const float* c13, const uint8_t* w2,
                  const void* s2, const float* c2, const float* codebook13, const float* codebook2, uint16_t* out,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Expert parallelism: d3_moe_decode of this rank's experts only. The banks hold experts [e_first, e_first +
 * e_count) of the E routed ones (bank expert 0 = expert e_first); pairs routed elsewhere are skipped (not faults);
 * partial [M, H] fp32 receives the routing-weighted sum over this rank's pairs, in rank order. Summing the ranks'
 * partials (in rank order) and rounding to bf16 gives the whole decode. No counterpart in the reference (one GPU). */
int d3_moe_decode_ep(int fmt, const void* x, int x_bf16, int M, int k, int E, int e_first, int e_count, int H, int I,
                     const int64_t* ids, const float* weights, const uint8_t* w13, const void* s13, const float* c13,
                     const uint8_t* w2, const void* s2, const float* c2, const float* codebook13,
                     const float* codebook2, float* partial, const void* exchange, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Expert parallelism over peer memory (NVLink P2P stores, one node, up to 8 ranks): `exchange` (device memory) is
 * the struct { float* slots[8]; unsigned* flags[8]; unsigned* epoch; int world, rank, m_max, h; } where slots[r] /
 * flags[r] address rank r's exchange area (d3_ep_exchange_bytes(world, m_max, H) bytes, zeroed: fp32 slots
 * [2][world][m_max][H], then at the next 256-byte boundary flags [2][8], this rank's call counter and one scratch
 * word) - the caller's own area for r == rank, the IPC mapping (d3_ipc_open) of the peers' - and epoch the counter
 * in the caller's area. With it, d3_moe_decode_ep pushes the partial into every rank's area instead of `partial` and
 * raises this rank's flag there; d3_ep_reduce then waits (bounded; fault bit 1 on timeout) for every rank's flag,
 * writes out [M, H] bf16 (8-byte aligned, H a multiple of 4) = the partials summed in rank order, and advances the
 * counter. Every rank makes the same calls in the same order; M <= m_max and H == h, else nothing is exchanged and
 * D3_FAULT_EXCHANGE is set. No counterpart in the reference (one GPU). */
/* Host-side packers (CPU, no device work), float32 rows w [rows, K] -> the expert layouts the kernels read, by plain
 * nearest rounding (round half to even throughout). Rows are split across `threads` host threads (<= 0: all
 * hardware threads). Inputs are finite. They replace the converter step tools/convert.py:48-82,179-215, whose own
 * quantizers (comfy_kitchen, absent) are not reproduced: the codes here are the nearest ones, not GPTQ's.
 *   d3_pack_fp8_blocks:   (fp8, tools/convert.py:179-189) e4m3 [rows, K] and fp32 128x128 block scales
 *                         [rows / 128, K / 128] = block absmax / 448 (1 for an all-zero block); rows, K % 128 == 0.
 *   d3_pack_int8_convrot: (int8, tools/convert.py:48-53) each 256-column group times the normalized 256-point
 *                         Hadamard matrix (drama3/offload.py:170-176), then int8 [rows, K] = rint(r / s) clipped to
 *                         +-127 with fp32 row scales s = absmax(r) / 127; K % 256 == 0.
 *   d3_pack_codes:        (w4 / w6, tools/convert.py:61-82; the layout drama3/kernels.py:466-483 decodes) rotated
 *                         as int8, t = r / s_channel (s_channel = absmax(r) / 127), e4m3 group scales per 16 columns
 *                         g = max(absmax(t) / top, 2^-6) (top = max |codebook| for bits 4, 31 for bits 6); bits 4:
 *                         the code c (first of equal distances) whose clip(rint(codebook[c] g), +-127) is nearest to
 *                         t, nibbles two per byte (low nibble first) [rows, K / 2]; bits 6: c = clip(rint(t / g),
 *                         -32, 31) + 32 as the same nibble plane followed by a 2-bit plane of c >> 4, four per byte
 *                         [rows, K / 4]. codebook: 16 floats (bits 4 only). K % 256 == 0.
 *   d3_pack_fp8c:         (BASELINE configs[1]) e4m3 [rows, K] (saturating at +-448) and fp32 row scales [rows] =
 *                         absmax / 448 (1 for an all-zero row).
 *   d3_pack_wa8:          ([3]) bits 4: two codes per byte along K (low nibble first); bits 6:
 *                         four codes per three bytes (little-endian 24-bit words); bf16 scales [rows, K / 128] =
 *                         absmax / qmax per 128 columns (qmax 7 / 31; 1 for an all-zero group), codes rint(x / scale)
 *                         clipped to +-qmax. K % 128 == 0. */
int d3_pack_fp8_blocks(const float* w, int64_t rows, int K, uint8_t* codes, float* scales, int threads);
int d3_pack_int8_convrot(const float* w, int64_t rows, int K, int8_t* q, float* scales, int threads);
int d3_pack_codes(const float* w, int64_t rows, int K, int bits, const float* codebook, uint8_t* codes,
                  uint8_t* group_scales, float* s_channel, int threads);
int d3_pack_fp8c(const float* w, int64_t rows, int K, uint8_t* codes, float* scales, int threads);
int d3_pack_wa8(const float* w, int64_t rows, int K, int bits, uint8_t* packed, uint16_t* scales, int threads);

size_t d3_ep_exchange_bytes(int world, int m_max, int H);
int d3_ep_reduce(const void* exchange, int M, int H, void* out, void* stream);
int d3_ipc_handle(const void* ptr, void* handle /* 64 bytes */, size_t* offset);
int d3_ipc_open(const void* handle, size_t offset, void** ptr, void** base);
int d3_ipc_close(void* base);

/* d3_moe_decode without a workspace argument. No counterpart in the reference: it is for callers that cannot
 * allocate device memory themselves, such as a plugin whose host application's memory manager owns every device
 * allocation, or a C host that links this library without any device allocator. The scratch is an array inside the
 * library (1,445,888 bytes, held on every GPU that loads it until the process exits), so the call allocates nothing
 * and calls no allocating routine. Limits: at most 128 routed pairs (M * k), intermediate size <= 768; larger shapes
 * return D3_ERR_TOO_LARGE; other bad arguments return the codes d3_moe_decode gives, before anything is put on
 * the stream. The first call on a device sets up the array's device address (synchronous); make it
 * before any stream capture. All calls share the one array: calls that overlap on the GPU race, so issue them on
 * one stream (or order them). Each call clears the array's barrier word on `stream` before its kernel. */
int d3_moe_decode_static(int fmt, const void* x, int x_bf16, int M, int k, int E, int H, int I, const int64_t* ids,
                         const float* weights, const uint8_t* w13, const void* s13, const float* c13,
                         const uint8_t* w2, const void* s2, const float* c2, const float* codebook13,
                         const float* codebook2, uint16_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DRAMA3_B200_H */
