"""Benchmark: MoE decode tokens/s of the routed-expert path on B200 (FP8 experts with
per-output-channel scales, 16 lines, 48 layers as configs[4]).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference] [--lines 16] [--layers 48]
                    [--kind fp8c] [--no-extras] [--prefill-only]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

A step is one decode pass of `lines` rows (16: lines decoded together) through 48 MoE layers of the BASELINE shape
(hidden 2048, 128 experts, top-8, intermediate 768, SwiGLU), each layer with its own expert banks (default fp8c:
e4m3 rows + fp32 per-output-channel scales) and its own seeded routing: 29 GB of experts, far
larger than L2, so every step streams its experts from HBM (no flush needed). Inputs are resident in HBM; the timed
region replays one CUDA graph per step and is bracketed by cudaProfilerStart/Stop, so `ncu --profile-from-start off`
sees exactly its launches; `--layers 4` is the small case for multi-pass captures (the same banks and routing as the
first 4 layers of the full run).

One GPU: `value` is that decode. N > 1 GPUs: `value` is expert parallelism, one 16-line job over all N GPUs (strong
scaling): rank r holds experts expert_range(128, r, N) of every layer, every rank decodes all 16 lines over its own
experts, and each layer's fp32 partials are exchanged over NVLink by the decode kernel itself (peer stores into every
rank's exchange area) and summed in rank order. Timing: CUDA events, max over ranks. The replicated layout (each rank
its own 16 lines, all experts; weak scaling) and the NCCL all-gather exchange are reported beside it.

Extras at N = 1, one per BASELINE configuration (each with its roofline fraction and, where the reference has one,
its CPU path timed on the host cores): config 1 (int8 ConvRot, 1 line, and the reference's CPU int8 path); config 2
(fp8 block scales at 1, 4 and 16 lines with the reference's own kernels beside them, fp8c at 1 and 4 lines);
config 3 (W4A8 and the reference's W4 layout at 1 and 16 lines); config 4 (the 2048-row Zipf-skewed prompt pass);
config 5 (the whole 48-layer decoder step: attention over a 4096-token KV cache, router and MoE) and its host-offload
slot-cache mode (768 slots on one GPU: hit rate, PCIe GB/s, tokens/s); the end-to-end rate
through the drop-in module (FP8Experts) with host buffers in and out. `--impl reference` runs the reference's CPU
decode (rank 0) and prints its line.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "comfyui-drama3_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "MoE decode tokens/s (1 & 16 lines), expert GEMV HBM GB/s vs ~8 TB/s, 1-8 B200"
E, H, I, K_TOP = 128, 2048, 768, 8
LAYERS = 48
KINDS = ("fp8c", "fp8", "w4a8", "w6a8", "int8", "w4", "w6")
FORMAT_NAMES = {
    "fp8c": "e4m3 rows + fp32 per-output-channel scales (BASELINE configs[1])",
    "fp8": "e4m3 rows + fp32 128x128 block scales (the reference's fp8 layout)",
    "int8": "int8 rows + fp32 per-row scales in the ConvRot basis (the reference's int8 layout, BASELINE configs[0])",
    "w4a8": "int4 two per byte + bf16 group-128 scales, int8 per-row activations (BASELINE configs[2])",
    "w6a8": "int6 four per three bytes + bf16 group-128 scales, int8 per-row activations (BASELINE configs[3])",
    "w4": "4-bit codebook codes + e4m3 group-16 scales + s_channel, ConvRot (the reference's W4A8 layout)",
    "w6": "6-bit codes + e4m3 group-16 scales + s_channel, ConvRot (the reference's W6A8 layout)",
}
CODEBOOK4 = (-1.0, -0.6962, -0.5251, -0.3949, -0.2844, -0.1848, -0.0911, 0.0, 0.0796, 0.1609, 0.2461, 0.3379, 0.4407,
             0.5626, 0.7230, 1.0)
# dram bytes (read + write) per launch over algorithmic bytes per launch, from the ncu capture of the small case
# (bench.py --layers 4, the first 2 launches of the timed step: 86 and 87 routed experts); the full run's traffic is
# this ratio x its own bytes
TRAFFIC_RATIO = (407.196928 + 5.279488 + 411.930368 + 4.855552) / (407.164416 + 411.897344)
TRAFFIC_SOURCE = ("ncu capture of the 4-layer small case (bench.py --layers 4, moe_decode_tc_kernel, 2 launches): "
                  "DRAM read + write / algorithmic bytes of the same launches")
# the same for the one-line decode (bench.py --layers 4 --lines 1, moe_decode_gv_kernel, 2 launches of 37.87 MB)
TRAFFIC_RATIO_1 = (37.934848 + 0.035840 + 37.934592 + 0.027392) / (2 * 37.871712)
TRAFFIC_SOURCE_1 = ("ncu capture of the 4-layer one-line case (bench.py --layers 4 --lines 1, moe_decode_gv_kernel, "
                    "2 launches): DRAM read + write / algorithmic bytes of the same launches")


def kernel_of(kind, lines=16):
    """(kernel name, arithmetic) of the fused decode for `kind` banks at `lines` lines."""
    if kind == "fp8c" and lines == 1:
        return ("moe_decode_gv_kernel (mma.sync e4m3; one launch per layer: gate_up rows streamed by bulk copies, "
                "SwiGLU, per-pair counters, down by (pair, row block), rank-order combine by last arrival)",
                "e4m3 weights x e4m3 activation terms (two groups of three, the second scaled by 2^12: bf16 rows "
                "exact, fp32 rows ~24 significant bits), f32 accumulation")
    if kind == "fp8c":
        return ("moe_decode_tc_kernel (tcgen05 kind::f8f6f4; one persistent launch per layer: plan, gate_up + "
                "SwiGLU, down, combine)",
                "e4m3 weights x e4m3 activation terms on the tensor cores, f32 accumulation: bf16 rows exact as two "
                "terms, the fp32 SwiGLU rows of the down projection as four terms (16 significant bits)")
    if kind == "w4a8" and lines == 1:
        return ("moe_decode_gv_kernel (mma.sync s8; one launch per layer: int4 rows streamed by bulk copies and "
                "expanded in registers, per-pair counters, down by (pair, row block), rank-order combine by last "
                "arrival)", "int4 weights expanded to int8 x int8 per-row activations, s32 accumulation, bf16 group "
                "scales folded per 128 columns")
    if kind == "int8" and lines == 1:
        return ("moe_decode_gv_kernel (mma.sync s8; one launch per layer: ConvRot in registers, int8 rows streamed by "
                "bulk copies, per-pair counters, rank-order combine by last arrival)",
                "int8 weights x the rotated rows as three int8 terms (~21 significant bits), s32 accumulation")
    if kind == "fp8" and lines == 1:
        return ("moe_decode_gv_kernel (mma.sync e4m3; one launch per layer, block scales folded per 128 columns)",
                "e4m3 weights x e4m3 activation terms (two groups of three), f32 accumulation")
    if kind == "w4a8":
        return ("moe_decode_tc8_kernel (tcgen05 kind::i8; one persistent launch per layer)",
                "int4 weights expanded to int8 x int8 per-row activations on the tensor cores, s32 accumulation, "
                "bf16 group scales folded per 128 columns")
    return (f"moe_decode_kernel<{kind}> (mma.sync; one persistent launch per layer: plan, gate_up + SwiGLU, down, "
            f"combine)", "f16 MMA inputs (exact weight codes), f32 accumulation")


def rand_bank(kind, n, k, gen, device):
    """A flat bank [E * n, ...] of random valid codes in the layout of `kind`."""
    if kind in ("fp8", "fp8c"):
        w = torch.randint(0, 254, (E * n, k), generator=gen, device=device, dtype=torch.uint8)
        w = torch.where(w >= 0x7F, w + 1, w)  # no 0x7F / 0xFF (NaN codes)
        shape = (E * n // 128, k // 128) if kind == "fp8" else (E * n,)
        return {"weight": w, "scale": torch.rand(shape, generator=gen, device=device) * 1e-4 + 5e-5}
    if kind in ("w4a8", "w6a8"):
        q = torch.randint(0, 256, (E * n, k * int(kind[1]) // 8), generator=gen, device=device, dtype=torch.uint8)
        s = (torch.rand((E * n, k // 128), generator=gen, device=device) * 2e-3 + 1e-3).to(torch.bfloat16)
        return {"_qdata": q, "scale": s}
    if kind == "int8":
        q = torch.randint(-127, 128, (E * n, k), generator=gen, device=device, dtype=torch.int8)
        return {"_qdata": q, "scale": torch.rand((E * n,), generator=gen, device=device) * 2e-4 + 1e-4}
    bits = int(kind[1])
    q = torch.randint(0, 256, (E * n, k * bits // 8), generator=gen, device=device, dtype=torch.uint8)
    lo, hi = (0x50, 0x70) if bits == 4 else (0x30, 0x50)
    g = torch.randint(lo, hi, (E * n, k // 16), generator=gen, device=device, dtype=torch.uint8)
    c = torch.rand((E * n,), generator=gen, device=device) * 2e-4 + 1e-4
    return {"_qdata": q, "scale": g, "s_channel": c}


def codebooks(kind, device):
    if kind != "w4":
        return (None, None)
    cb = torch.tensor(CODEBOOK4, dtype=torch.float32, device=device)
    return (cb, cb.clone())


def expert_bytes(kind):
    """Algorithmic bytes of one expert of the BASELINE shape in `kind`'s layout (weight and scale bytes)."""
    total = 0
    for n, k in ((2 * I, H), (H, I)):
        total += n * {"fp8": k, "fp8c": k, "int8": k, "w4a8": k // 2, "w6a8": 3 * k // 4, "w4": k // 2,
                      "w6": 3 * k // 4}[kind]
        total += {"fp8": (n // 128) * (k // 128) * 4, "fp8c": n * 4, "int8": n * 4, "w4a8": n * (k // 128) * 2,
                  "w6a8": n * (k // 128) * 2, "w4": n * (k // 16 + 4), "w6": n * (k // 16 + 4)}[kind]
    return total


def make_routing(lines, n_layers, seed, device):
    """Per-layer seeded routing: distinct top-8 experts per row, renormalized bf16-valued weights."""
    cpu_gen = torch.Generator().manual_seed(seed)
    ids, weights = [], []
    for _ in range(n_layers):
        w, i = torch.softmax(torch.randn((lines, E), generator=cpu_gen), dim=-1).topk(K_TOP, dim=-1)
        ids.append(i)
        weights.append((w / w.sum(-1, keepdim=True)).to(torch.bfloat16).float())
    return torch.stack(ids).to(device), torch.stack(weights).to(device)


def make_layers(device, lines, kind="fp8c", seed=4, n_layers=LAYERS):
    """n_layers layers of banks (random valid codes, positive scales) and per-layer routing; layer l's routing does
    not depend on n_layers or the format."""
    gen = torch.Generator(device=device).manual_seed(seed)
    layers = [tuple(rand_bank(kind, n, k, gen, device) for n, k in ((2 * I, H), (H, I))) for _ in range(n_layers)]
    ids, weights = make_routing(lines, n_layers, seed + 1, device)
    return layers, ids, weights


def peaks():
    try:
        data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(data["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(self.rows[0][1]),
                "samples": len(self.rows), "reasons": reasons}


def unique_bytes(ids, kind, rows_bytes=True):
    """Algorithmic bytes of one step: each layer's unique experts, plus its rows in and out (bf16)."""
    per, total = expert_bytes(kind), 0
    lines = ids.shape[1]
    for layer in ids.cpu():
        total += len(set(layer.reshape(-1).tolist())) * per
        if rows_bytes:
            total += 2 * lines * H * 2 + lines * K_TOP * 12
    return total


def capture(fn, warmup, stream):
    """fn() run `warmup` times, then captured as one CUDA graph (replayed once)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    graph.replay()
    torch.cuda.synchronize()
    return graph


def time_replays(graph, steps, stream, before=None):
    """ms per replay of `graph`, CUDA events on `stream`; `before(i)` runs ahead of replay i (inside the timing)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        if before is not None:
            before(i)
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def replay_spread(graph, steps, stream):
    """{median, p90} ms of `steps` single replays of `graph`, each between its own CUDA events on `stream`."""
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for start, end in events:
        start.record(stream)
        graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    t = sorted(start.elapsed_time(end) for start, end in events)
    return {"steps": steps, "ms_median": t[len(t) // 2], "ms_p90": t[min(len(t) - 1, (9 * len(t)) // 10)]}


def decode_leg(kernels, device, kind, lines, steps, warmup, stream, n_layers, layers, cbs=(None, None)):
    """{tokens_per_s, ms_per_step, hbm_gbs, frac, ...} of the fused decode of `lines` rows through n_layers layers;
    layers = (banks, ids, weights), the first `lines` rows of the routing used."""
    hbm_peak, _ = peaks()
    banks, ids, weights = layers
    ids, weights = ids[:, :lines].contiguous(), weights[:, :lines].contiguous()
    x = torch.randn((lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)
    ws = kernels.decode_workspace(lines, K_TOP, I, device)
    outs = torch.empty((n_layers, lines, H), dtype=torch.bfloat16, device=device)

    def step():
        for l_ in range(n_layers):
            kernels.moe_decode(kind, x, ids[l_], weights[l_], banks[l_], cbs, workspace=ws, out=outs[l_])

    with torch.cuda.stream(stream):
        graph = capture(step, warmup, stream)
        ms = time_replays(graph, steps, stream)
    del graph
    b = unique_bytes(ids, kind)
    gbs = b / (ms * 1e-3) / 1e9
    return {"tokens_per_s": lines / (ms * 1e-3), "ms_per_step": ms, "us_per_layer": 1e3 * ms / n_layers,
            "hbm_gbs": gbs, "frac": gbs / hbm_peak, "bytes_per_step": b, "format": FORMAT_NAMES[kind],
            "lines": lines, "kernel": kernel_of(kind, lines)[0]}


def reference_gpu_leg(device, kind, lines, steps, stream, n_layers, layers, cbs=(None, None)):
    """The reference's own kernels (drama3/kernels.py compiled into oracle/_ref) on the same banks, rows and routing,
    driven as drama3/offload.py:108-123 drives them (gemv -> SwiGLU [+ rotation] -> gemv -> weighted_sum), one row at
    a time as drama3/model.py:111-113 runs lines, one CUDA graph per step."""
    from oracle import ref_gpu
    if not ref_gpu.available():
        return {"unavailable": "reference kernels not built (oracle/_ref)"}
    banks, ids, weights = layers
    x = torch.randn((lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)

    def ref_step():
        for l_ in range(n_layers):
            ref_gpu.lines_decode(x, ids[l_, :lines], weights[l_, :lines], banks[l_], (2 * I, H), kind, cbs)

    with torch.cuda.stream(stream):
        graph = capture(ref_step, 2, stream)
        ms = time_replays(graph, max(3, min(steps, 10)), stream)
    del graph
    return {"tokens_per_s": lines / (ms * 1e-3), "ms_per_step": ms, "us_per_layer": 1e3 * ms / n_layers,
            "what": "reference kernels (drama3/kernels.py, nvcc sm_100) driven as drama3/offload.py:108-123, one "
                    "row at a time"}


def layout_legs(kernels, device, kind, lines_list, args, stream, n_layers, seed, reference=False):
    """decode_leg at each line count of lines_list on one set of `kind` banks (and the reference's kernels)."""
    layers = make_layers(device, max(lines_list), kind, seed, n_layers)
    cbs = codebooks(kind, device)
    out = {}
    for lines in lines_list:
        leg = decode_leg(kernels, device, kind, lines, args.steps, args.warmup, stream, n_layers, layers, cbs)
        if reference:
            try:
                ref = reference_gpu_leg(device, kind, lines, args.steps, stream, n_layers, layers, cbs)
                leg["reference_gpu"] = ref
                if "ms_per_step" in ref:
                    leg["speedup_vs_reference_gpu"] = ref["ms_per_step"] / leg["ms_per_step"]
            except Exception as exc:  # the comparison must not sink the bench line
                leg["reference_gpu"] = {"error": repr(exc)[:200]}
        out[f"lines_{lines}"] = leg
    del layers
    torch.cuda.empty_cache()
    return out


def prefill_leg(device, steps, tokens=2048, seed=3):
    """one MoE layer's prompt pass of `tokens` rows, router logits biased so expert load is
    Zipf(1.1)-skewed (bias_e = -1.1 ln r_e, r a seeded permutation of ranks 1..128): W6A8 (the BASELINE layout),
    then the reference's W6 and fp8 layouts. Times the whole resident_prefill (sort, grouped GEMMs on the tensor
    cores, combine) with CUDA events, and for the reference layouts the reference's own grouped kernels
    (oracle/_ref) on the same inputs."""
    from drama3_b200 import offload
    gen = torch.Generator().manual_seed(seed)
    bias = -1.1 * torch.log(torch.randperm(E, generator=gen).float() + 1)
    w, ids = torch.softmax(torch.randn((tokens, E), generator=gen) + bias, -1).topk(K_TOP, dim=-1)
    w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)
    x = torch.randn((tokens, H), generator=gen).to(torch.bfloat16)
    counts = torch.bincount(ids.reshape(-1), minlength=E)
    x, ids, w = x.to(device), ids.to(device), w.to(device)
    flops = 2.0 * tokens * K_TOP * (2 * I * H + H * I)
    bf16_peak = 1590.0
    try:
        bf16_peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        pass
    dgen = torch.Generator(device=device).manual_seed(seed)
    out = {"tokens": tokens, "top_k": K_TOP, "largest_group": int(counts.max()), "median_group": int(counts.median()),
           "flops_per_layer": flops, "peak_tflops": bf16_peak,
           "note": "W6A8: tcgen05 kind::i8 (int6 codes expanded to int8, int8 activations, exact s32 sums per "
                   "128-column group); fp8 / W6: kind::f16 with f32 accumulation, activations as two f16 terms "
                   "(hi + lo); frac = algorithmic flops / time / measured dense bf16 peak (the int8 rate is twice it)"}
    for kind in ("w6a8", "w6", "fp8"):
        banks = (rand_bank(kind, 2 * I, H, dgen, device), rand_bank(kind, H, I, dgen, device))

        def run():
            return offload.resident_prefill(x, ids, w, banks, (2 * I, H), kind, (None, None), E)

        for _ in range(2):
            run()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(3, min(steps, 10))
        s0.record()
        for _ in range(n):
            run()
        s1.record()
        torch.cuda.synchronize()
        us = 1e3 * s0.elapsed_time(s1) / n
        leg = {"us_per_layer": us, "tflops": flops / us / 1e6, "frac": flops / us / 1e6 / bf16_peak,
               "tokens_per_s": tokens / us * 1e6, "format": FORMAT_NAMES[kind]}
        if kind == "w6a8":
            # the same pass sorted on the device (no host sync), captured once as a CUDA graph and replayed
            try:
                def run_free():
                    return offload.resident_prefill(x, ids, w, banks, (2 * I, H), kind, (None, None), E,
                                                    sync_free=True)

                side = torch.cuda.Stream(device)
                with torch.cuda.stream(side):
                    graph = capture(run_free, 2, side)
                    gus = 1e3 * time_replays(graph, n, side)
                del graph
                leg["sync_free_graph"] = {"us_per_layer": gus, "tflops": flops / gus / 1e6,
                                          "frac": flops / gus / 1e6 / bf16_peak, "tokens_per_s": tokens / gus * 1e6}
            except Exception as exc:  # the comparison must not sink the bench line
                leg["sync_free_graph"] = {"error": repr(exc)[:200]}
        if kind in ("w6", "fp8"):
            try:
                from oracle import ref_gpu
                if ref_gpu.available():
                    ref_gpu.resident_prefill(x, ids, w, banks, (2 * I, H), kind, (None, None), E)
                    torch.cuda.synchronize()
                    s0.record()
                    ref_gpu.resident_prefill(x, ids, w, banks, (2 * I, H), kind, (None, None), E)
                    s1.record()
                    torch.cuda.synchronize()
                    rus = 1e3 * s0.elapsed_time(s1)
                    leg["reference_gpu_us_per_layer"] = rus
                    leg["speedup_vs_reference_gpu"] = rus / us
            except Exception as exc:  # the comparison must not sink the bench line
                leg["reference_gpu"] = {"error": repr(exc)[:200]}
        out[kind] = leg
        del banks
    return out


def slot_cache_leg(device, args, stream, slots_per_layer=16, n_routings=8, seed=40):
    """BASELINE configs[4]'s host-offload mode on one GPU: every layer's fp8 experts (the reference's block-scaled
    layout, 29 GB at 48 layers) in pinned host memory behind one slot cache of 16 slots per layer (768 at 48
    layers), decoded through the drop-in ExpertStore / OffloadedExperts: per layer and row, resolve (slot lookup and
    least-used eviction on the GPU), gate_up, SwiGLU, down, weighted sum, with missed experts read from host memory
    over PCIe by the GEMVs themselves (and filled into their slot). Lines run one row at a time, as the store does
    for the reference. A step replays one CUDA graph; each step takes its routing from n_routings seeded routings in
    turn (copied in ahead of the replay, inside the timing). Reports the cache's hit rate, the PCIe bytes of the
    misses and tokens/s."""
    from drama3_b200 import offload
    n_layers, lines = args.layers, args.lines
    gen = torch.Generator(device=device).manual_seed(seed)
    per_expert = expert_bytes("fp8")
    # the cache budget is the configuration's slot count: the pool makes budget // expert bytes slots
    store = offload.ExpertStore(slots_per_layer * n_layers * per_expert, pin=True)
    modules = []
    for _ in range(n_layers):
        ex = offload.FP8Experts(E, H, I, device="meta")
        for name, n, k in (("gate_up", 2 * I, H), ("down", H, I)):
            bank = rand_bank("fp8", n, k, gen, device)
            w = torch.empty((E, n, k), dtype=torch.uint8, pin_memory=True)
            s = torch.empty((E, n // 128, k // 128), dtype=torch.float32, pin_memory=True)
            w.view(-1, k).copy_(bank["weight"])
            s.view(-1, k // 128).copy_(bank["scale"])
            setattr(ex, f"{name}_weight", torch.nn.Parameter(w.view(torch.float8_e4m3fn), requires_grad=False))
            setattr(ex, f"{name}_scale", torch.nn.Parameter(s, requires_grad=False))
        modules.append(store.add(ex))
    torch.cuda.synchronize()
    routings = [make_routing(lines, n_layers, seed + 1 + r, device) for r in range(n_routings)]
    ids_buf, w_buf = torch.empty_like(routings[0][0]), torch.empty_like(routings[0][1])
    x = torch.randn((lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)
    outs = torch.empty((n_layers, lines, H), dtype=torch.bfloat16, device=device)

    def step():
        for l_ in range(n_layers):
            for r in range(lines):
                outs[l_, r:r + 1] = modules[l_](x[r:r + 1], ids_buf[l_, r:r + 1], w_buf[l_, r:r + 1])

    def load(i):
        ids_buf.copy_(routings[i % n_routings][0], non_blocking=True)
        w_buf.copy_(routings[i % n_routings][1], non_blocking=True)

    with store.session(device, rows=lines):
        cache = store.cache
        with torch.cuda.stream(stream):
            load(0)
            step()  # first step eagerly: moves the cache state to the device
            torch.cuda.synchronize()
            graph = capture(step, 0, stream)
            for i in range(args.warmup):
                load(i)
                graph.replay()
            torch.cuda.synchronize()
            before = cache.reads.clone()
            n = max(3, min(args.steps, 8))
            ms = time_replays(graph, n, stream, before=load)
            reads = (cache.reads - before).tolist()
        del graph
        slots = cache.count
    total = sum(reads[:2])
    miss_bytes = reads[1] * per_expert / n
    del modules, store
    torch.cuda.empty_cache()
    return {"tokens_per_s": lines / (ms * 1e-3), "ms_per_step": ms, "us_per_layer": 1e3 * ms / n_layers,
            "slots": slots, "slots_per_layer": slots_per_layer, "layers": n_layers, "lines": lines,
            "hit_rate": reads[0] / total if total else None, "expert_reads_per_step": total / n,
            "misses_per_step": reads[1] / n, "pcie_gbs": miss_bytes / (ms * 1e-3) / 1e9,
            "format": FORMAT_NAMES["fp8"],
            "routing": f"{n_routings} seeded routings used in turn, one per step",
            "what": "ExpertStore (pinned host banks, 768-slot GPU cache): resolve + gemv_fp8 (slot or host "
                    "zero-copy, filling the slot) + SwiGLU + gemv_fp8 + weighted_sum per layer and row, one graph"}


def block_leg(kernels, device, args, stream, shared_i=512, seed=45):
    """The whole MoE block per layer (drama3/model.py:92-124) for 16 decode lines, 48 layers: router (bf16 linear
    2048 -> 128 and the decode routing), the routed experts (fp8c, the fused decode) and the sigmoid-gated shared
    expert (bf16, intermediate 512), fused (kernels.router: one launch; kernels.shared_expert: two) against the same
    block on torch's chain (cuBLAS linears, the route kernel, silu / sigmoid / mul / add). One graph per step each."""
    n_layers, lines = args.layers, args.lines
    gen = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape):
        return (torch.randn(shape, generator=gen, device=device) * 0.02).to(torch.bfloat16)

    layers = [{"router": randn(E, H), "gu": randn(2 * shared_i, H), "dn": randn(H, shared_i), "g": randn(1, H),
               "banks": tuple(rand_bank("fp8c", n, k, gen, device) for n, k in ((2 * I, H), (H, I)))}
              for _ in range(n_layers)]
    x = torch.randn((lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)
    ws = kernels.decode_workspace(lines, K_TOP, I, device)
    outs = torch.empty((n_layers, lines, H), dtype=torch.bfloat16, device=device)

    def fused():
        for l_, lay in enumerate(layers):
            ids, w = kernels.router(x, lay["router"], K_TOP)
            kernels.moe_decode("fp8c", x, ids, w, lay["banks"], workspace=ws, out=outs[l_])
            kernels.shared_expert(x, lay["gu"], lay["dn"], lay["g"], outs[l_])

    def eager():
        for l_, lay in enumerate(layers):
            ids, w = kernels.route(x @ lay["router"].T, K_TOP)
            moe = kernels.moe_decode("fp8c", x, ids, w, lay["banks"], workspace=ws, out=outs[l_])
            h = x @ lay["gu"].T
            sh = (torch.nn.functional.silu(h[:, :shared_i]) * h[:, shared_i:]) @ lay["dn"].T
            outs[l_].copy_(moe + torch.sigmoid(x @ lay["g"].T) * sh)

    res = {}
    for name, fn in (("fused", fused), ("torch_chain", eager)):
        with torch.cuda.stream(stream):
            graph = capture(fn, 2, stream)
            ms = time_replays(graph, max(3, min(args.steps, 20)), stream)
        del graph
        res[name] = {"tokens_per_s": lines / (ms * 1e-3), "ms_per_step": ms, "us_per_layer": 1e3 * ms / n_layers}
    del layers
    torch.cuda.empty_cache()
    res["what"] = ("per layer: router 2048 -> 128 bf16 + top-8 routing, fp8c routed experts (fused decode), shared "
                   "expert 2048 -> 2 x 512 -> 2048 bf16 with its sigmoid gate, 16 lines")
    return res


def full_stack_leg(kernels, device, args, stream, ctx=4096, q_heads=32, kv_heads=4, head_dim=128, seed=44):
    """the whole 48-layer decoder step of `lines` lines, each layer RMSNorm -> attention (QKV
    projection, 32 query / 4 KV heads of 128 over a 4096-token bf16 KV cache per line, the step's K / V written at
    its position, output projection) -> residual -> RMSNorm -> router (linear and routing in one launch) -> the fused
    MoE decode (fp8c) -> residual. Random-init weights from seed 44, one CUDA graph per step. The attention, the
    projections and the norms are torch (cuBLAS / SDPA): library calls around this library's MoE path; RoPE is left
    out (it moves no bytes that matter). Reports tokens/s and the HBM fraction of the step's bytes (routed experts,
    KV cache, attention and router weights)."""
    n_layers, lines = args.layers, args.lines
    hbm_peak, _ = peaks()
    gen = torch.Generator(device=device).manual_seed(seed)
    qkv_rows = (q_heads + 2 * kv_heads) * head_dim

    def randn(*shape, std=0.02):
        return (torch.randn(shape, generator=gen, device=device) * std).to(torch.bfloat16)

    layers = []
    for _ in range(n_layers):
        layers.append({
            "n1": torch.ones((H,), dtype=torch.bfloat16, device=device), "n2": torch.ones((H,), dtype=torch.bfloat16,
                                                                                            device=device),
            "wqkv": randn(qkv_rows, H), "wo": randn(H, q_heads * head_dim), "router": randn(E, H),
            "k": randn(lines, kv_heads, ctx, head_dim, std=1.0), "v": randn(lines, kv_heads, ctx, head_dim, std=1.0),
            "banks": tuple(rand_bank("fp8c", n, k, gen, device) for n, k in ((2 * I, H), (H, I)))})
    x = torch.randn((lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)
    h = torch.empty_like(x)
    ws = kernels.decode_workspace(lines, K_TOP, I, device)
    moe_out = torch.empty((lines, H), dtype=torch.bfloat16, device=device)
    ids_seen = []

    def rmsnorm(t, w):
        tf = t.float()
        return (tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16) * w

    def step(record=False):
        h.copy_(x)
        for lay in layers:
            a = rmsnorm(h, lay["n1"])
            qkv = a @ lay["wqkv"].T
            # query head h reads KV head h // (q_heads / kv_heads): a KV head's query heads act as its query rows
            q = qkv[:, :q_heads * head_dim].view(lines, kv_heads, q_heads // kv_heads, head_dim)
            kv = qkv[:, q_heads * head_dim:].view(lines, 2, kv_heads, 1, head_dim)
            lay["k"][:, :, ctx - 1:ctx].copy_(kv[:, 0])
            lay["v"][:, :, ctx - 1:ctx].copy_(kv[:, 1])
            o = torch.nn.functional.scaled_dot_product_attention(q, lay["k"], lay["v"])
            h.add_(o.reshape(lines, q_heads * head_dim) @ lay["wo"].T)
            m = rmsnorm(h, lay["n2"])
            ids, w = kernels.router(m, lay["router"], K_TOP)
            if record:
                ids_seen.append(ids)
            kernels.moe_decode("fp8c", m, ids, w, lay["banks"], workspace=ws, out=moe_out)
            h.add_(moe_out)

    with torch.cuda.stream(stream):
        step(record=True)
        torch.cuda.synchronize()
        graph = capture(step, 2, stream)
        ms = time_replays(graph, max(3, min(args.steps, 20)), stream)
    del graph
    expert_b = unique_bytes(torch.stack(ids_seen), "fp8c", rows_bytes=False)
    kv_b = n_layers * 2 * lines * kv_heads * ctx * head_dim * 2
    weight_b = n_layers * (qkv_rows * H + H * q_heads * head_dim + E * H) * 2
    step_b = expert_b + kv_b + weight_b
    gbs = step_b / (ms * 1e-3) / 1e9
    del layers
    torch.cuda.empty_cache()
    return {"tokens_per_s": lines / (ms * 1e-3), "ms_per_step": ms, "us_per_layer": 1e3 * ms / n_layers,
            "lines": lines, "layers": n_layers, "context": ctx, "bytes_per_step": step_b,
            "expert_bytes_per_step": expert_b, "kv_bytes_per_step": kv_b, "attention_router_weight_bytes": weight_b,
            "hbm_gbs": gbs, "frac": gbs / hbm_peak,
            "what": "RMSNorm, QKV / O projections (cuBLAS bf16), GQA attention over the KV cache (torch SDPA), "
                    "router (router_kernel: linear + routing), fused MoE decode (moe_decode_tc_kernel), one graph"}


# ---- CPU baselines: the reference's CPU paths (oracle/cpu_port.py), bounded samples on the host cores
def cpu_fp8(lines, n_layers=LAYERS, seed=4, seconds=10.0, min_layers=2):
    """The reference's CPU decode for fp8 experts (the FP8Experts CPU forward, block-scaled layout: the reference
    has no per-channel layout) of `lines` rows, one row at a time; at least min_layers layers and about `seconds`.
    Returns (tokens/s of an n_layers step, seconds timed, threads, layers timed, sample description)."""
    from oracle import cpu_port
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn((lines, H), generator=gen).to(torch.bfloat16)
    banks = []
    for _ in range(2):
        gu = torch.randint(0, 126, (E, 2 * I, H), generator=gen, dtype=torch.uint8)
        dn = torch.randint(0, 126, (E, H, I), generator=gen, dtype=torch.uint8)
        gs = torch.rand((E, 2 * I // 128, H // 128), generator=gen) * 1e-4
        ds = torch.rand((E, H // 128, I // 128), generator=gen) * 1e-4
        banks.append((gu, gs, dn, ds))
    total, done = 0.0, 0
    while done < n_layers and (done < min_layers or total < seconds):
        gu, gs, dn, ds = banks[done % 2]
        w, ids = torch.softmax(torch.randn((lines, E), generator=gen), -1).topk(K_TOP, dim=-1)
        w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)
        started = time.perf_counter()
        cpu_port.fp8_decode_lines(x, ids, w, gu, gs, dn, ds)
        total += time.perf_counter() - started
        done += 1
    sample = (f"{lines} rows x {done} layers timed ({total:.1f} s) of the reference's CPU decode (FP8Experts CPU "
              f"forward: bf16 dequantization + matmuls, one row at a time), tokens/s of a {n_layers}-layer step")
    return lines / (total / done * n_layers), total, torch.get_num_threads(), done, sample


def cpu_int8(n_layers=LAYERS, seed=0, seconds=8.0):
    """BASELINE configs[0]'s CPU baseline: the reference's own CPU int8 decode of one row (hadamard rotation,
    experts_on_cpu with torch._weight_int8pack_mm, routing-weighted sum; oracle/cpu_port.int8_decode_row, bit for
    bit the reference's output on config 1), over layers of random int8 banks."""
    from oracle import cpu_port
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(seed)
    rot = cpu_port.hadamard()
    banks = [(torch.randint(-127, 128, (E, 2 * I, H), generator=gen, dtype=torch.int8),
              torch.rand((E, 2 * I), generator=gen) * 1e-3,
              torch.randint(-127, 128, (E, H, I), generator=gen, dtype=torch.int8),
              torch.rand((E, H), generator=gen) * 1e-3) for _ in range(2)]
    x = torch.randn((1, H), generator=gen).to(torch.bfloat16)
    total, done = 0.0, 0
    while done < n_layers and (done < 3 or total < seconds):
        w, ids = torch.softmax(torch.randn((E,), generator=gen), -1).topk(K_TOP)
        started = time.perf_counter()
        cpu_port.int8_decode_row(x, ids, w / w.sum(), *banks[done % 2], rot)
        total += time.perf_counter() - started
        done += 1
    sample = (f"1 row x {done} layers timed ({total:.2f} s) of the reference's CPU int8 decode (experts_on_cpu), "
              f"tokens/s of a {n_layers}-layer step")
    return 1 / (total / done * n_layers), total, torch.get_num_threads(), done, sample


def cpu_codes(kind, lines, n_layers=LAYERS, seed=2, seconds=8.0):
    """Configs[2]/[3]'s CPU baseline for the reference's W4 / W6 code layouts: a RESTATEMENT (the reference's CPU
    matmuls for these layouts live in comfy_kitchen, absent): codes decoded as drama3/kernels.py:466-483 to bf16
    weights, then the decode's matmuls, one row at a time (oracle/cpu_port.codes_decode_row)."""
    from oracle import cpu_port
    torch.set_num_threads(os.cpu_count() or 1)
    bits = int(kind[1])
    gen = torch.Generator().manual_seed(seed)
    rot = cpu_port.hadamard()
    cbs = (torch.tensor(CODEBOOK4), torch.tensor(CODEBOOK4)) if bits == 4 else (None, None)

    def bank(n, k):
        return (torch.randint(0, 256, (E, n, k * bits // 8), generator=gen, dtype=torch.uint8),
                torch.randint(0x30, 0x50, (E, n, k // 16), generator=gen, dtype=torch.uint8),
                torch.rand((E, n), generator=gen) * 2e-4 + 1e-4)

    b13, b2 = bank(2 * I, H), bank(H, I)
    x = torch.randn((lines, H), generator=gen).to(torch.bfloat16)
    total, done = 0.0, 0
    while done < n_layers and (done < 2 or total < seconds):
        w, ids = torch.softmax(torch.randn((lines, E), generator=gen), -1).topk(K_TOP, dim=-1)
        started = time.perf_counter()
        for t in range(lines):
            cpu_port.codes_decode_row(x[t:t + 1], ids[t], w[t] / w[t].sum(), b13, b2, bits, cbs, rot)
        total += time.perf_counter() - started
        done += 1
    sample = (f"{lines} rows x {done} layers timed ({total:.1f} s), restatement of the reference's {kind} CPU "
              f"decode (codes decoded to bf16 weights, matmuls, one row at a time), tokens/s of a {n_layers}-layer "
              "step")
    return lines / (total / done * n_layers), total, torch.get_num_threads(), done, sample


def cpu_line(result):
    tps, secs, threads, done, sample = result
    return {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "layers_timed": done,
            "seconds": secs, "sample": sample}


def e2e_leg(device, layers, x, ids, weights, lines, steps):
    """End to end through the drop-in module: 48 FP8Experts modules (per-channel layout, parameters viewing the
    bench's banks), host buffers in (rows, routing) and out (the last layer's rows), every step, each copy
    included in the timing."""
    from drama3_b200 import offload
    mods = []
    for banks in layers:
        ex = offload.FP8Experts(E, H, I, device="meta", per_channel=True)
        for name, bank, n, k in (("gate_up", banks[0], 2 * I, H), ("down", banks[1], H, I)):
            setattr(ex, f"{name}_weight", torch.nn.Parameter(bank["weight"].view(E, n, k).view(torch.float8_e4m3fn),
                                                             requires_grad=False))
            setattr(ex, f"{name}_scale", torch.nn.Parameter(bank["scale"].view(E, n), requires_grad=False))
        mods.append(ex)
    xh = x.cpu().pin_memory()
    idh, wh = ids.cpu().pin_memory(), weights.cpu().pin_memory()
    outh = torch.empty((lines, H), dtype=torch.bfloat16).pin_memory()
    xd, idd, wd = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(weights)
    n_e2e = max(3, min(steps, 20))
    for it in range(n_e2e + 2):
        if it == 2:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            es.record()
        xd.copy_(xh, non_blocking=True)
        idd.copy_(idh, non_blocking=True)
        wd.copy_(wh, non_blocking=True)
        out = xd
        for l_, mod in enumerate(mods):
            out = mod(xd, idd[l_], wd[l_])
        outh.copy_(out, non_blocking=True)
    ee.record()
    torch.cuda.synchronize()
    ms = es.elapsed_time(ee) / n_e2e
    return {"value": lines / (ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": xh.nbytes + idh.nbytes + wh.nbytes,
            "d2h_bytes_per_step": outh.nbytes, "ms_per_step": ms,
            "wall_ms_per_step": 1e3 * (time.perf_counter() - t0) / n_e2e,
            "through": "drama3_b200.offload.FP8Experts(per_channel=True).forward, 48 modules, eager (no graph)"}


def ep_setup(device, kind, args, rank, world):
    """Rank r's expert-parallel banks (experts expert_range(E, r, N) of every layer, sliced from seeded whole banks),
    the shared rows and routing."""
    from drama3_b200 import ep
    n_layers = args.layers
    gen = torch.Generator(device=device).manual_seed(4)
    layers = []
    for _ in range(n_layers):
        full = tuple(rand_bank(kind, n, k, gen, device) for n, k in ((2 * I, H), (H, I)))
        layers.append(tuple({n: t.clone() for n, t in b.items()} for b in ep.local_banks(full, E, rank, world)))
        del full
    torch.cuda.empty_cache()
    ids, weights = make_routing(args.lines, n_layers, 5, device)
    x = torch.randn((args.lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)
    return layers, ids, weights, x


def config(args, world):
    if world > 1:
        parallelism = (f"expert parallelism over {world} GPUs (experts 128/{world} per rank, one {args.lines}-line "
                       "job; partials exchanged over NVLink by the decode kernel)")
    else:
        parallelism = "1 GPU"
    return {"workload": f"MoE decode, {args.lines} lines x {args.layers} layers per step, {args.kind} experts "
                        f"(BASELINE configs[1] layer shape; 48 layers as configs[4])",
            "layers": args.layers, "lines": args.lines, "experts": E, "top_k": K_TOP, "hidden": H, "intermediate": I,
            "format": FORMAT_NAMES[args.kind],
            "l2": f"inputs larger than L2: {args.layers * E * expert_bytes(args.kind) / 1e9:.1f} GB of expert banks, "
                  f"each layer's routed experts streamed per step",
            "parallelism": parallelism}


def run_reference_arm(args, world):
    """The reference's CPU decode on the host cores: each step is a bounded sample of the workload, `lines` rows
    through ONE MoE layer (about 0.5 s at 16 lines); `value` is tokens/s of a whole `layers`-layer step at that
    layer rate. The reference's CPU forward reads its only fp8 layout, 128x128 block scales (the per-channel layout
    of this bench's headline is not in the reference; the bytes differ by under 0.3 %)."""
    from oracle import cpu_port
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(4)
    x = torch.randn((args.lines, H), generator=gen).to(torch.bfloat16)
    gu = torch.randint(0, 126, (E, 2 * I, H), generator=gen, dtype=torch.uint8)
    dn = torch.randint(0, 126, (E, H, I), generator=gen, dtype=torch.uint8)
    gs = torch.rand((E, 2 * I // 128, H // 128), generator=gen) * 1e-4
    ds = torch.rand((E, H // 128, I // 128), generator=gen) * 1e-4
    routes = []
    for _ in range(4):
        w, ids = torch.softmax(torch.randn((args.lines, E), generator=gen), -1).topk(K_TOP, dim=-1)
        routes.append((ids, (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)))
    for i in range(args.warmup):
        cpu_port.fp8_decode_lines(x, *routes[i % 4], gu, gs, dn, ds)
    started = time.perf_counter()
    for i in range(args.steps):
        cpu_port.fp8_decode_lines(x, *routes[i % 4], gu, gs, dn, ds)
    secs = time.perf_counter() - started
    layer_s = secs / args.steps
    tps = args.lines / (layer_s * args.layers)
    cfg = config(args, world)
    cfg["format"] = FORMAT_NAMES["fp8"] + " (the reference's only fp8 layout)"
    cfg["sample_layers_per_step"] = 1
    sample = (f"each step: {args.lines} rows through 1 MoE layer of the reference's CPU decode (FP8Experts CPU "
              f"forward, one row at a time); {args.steps} steps timed ({secs:.1f} s); value = tokens/s of a "
              f"{args.layers}-layer step at that layer rate")
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * layer_s, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16 (CPU: e4m3 weights dequantized to bf16, bf16 matmuls)", "data": "synthetic",
            "config": cfg,
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def timed_region(graph, args, stream, pg, local):
    """The timed region: a barrier and syncs on both sides, `steps` replays between CUDA events, clocks sampled;
    returns (ms per step, max over ranks; clock summary)."""
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clocks:
        torch.cuda.profiler.start()
        ms = time_replays(graph, args.steps, stream)
        torch.cuda.profiler.stop()
    if pg:
        t = torch.tensor([ms], device=stream.device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    return ms, clocks.summary()


def ep_extras(kind, args, stream, pg, device, local_layers, mods, ids, weights, x, ms, outs):
    """Beside the expert-parallel headline: each rank's decode alone (no exchange) and the NCCL all-gather exchange
    of the same job, and the end-to-end rate through ExpertParallelDecode with host buffers."""
    from drama3_b200 import ep
    n_layers = args.layers
    plain = [ep.ExpertParallelDecode(kind, banks, E) for banks in local_layers]
    timed = {}
    for name, fn in (("decode_only", lambda l_: plain[l_].partial(x, ids[l_], weights[l_])),
                     ("nccl_all_gather", lambda l_: plain[l_](x, ids[l_], weights[l_]))):
        def alt(fn=fn):
            for l_ in range(n_layers):
                outs[l_] = fn(l_)

        with torch.cuda.stream(stream):
            graph = capture(alt, args.warmup, stream)
            pg.barrier()
            t_ms = time_replays(graph, max(3, min(args.steps, 20)), stream)
        del graph  # released before the process group is destroyed
        t = torch.tensor([t_ms], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        timed[name] = {"ms_per_step": float(t.item()), "us_per_layer": 1e3 * float(t.item()) / n_layers,
                       "tokens_per_s": args.lines / (float(t.item()) * 1e-3)}
    timed["exchange_us_per_layer"] = 1e3 * (ms - timed["decode_only"]["ms_per_step"]) / n_layers
    # end to end: host rows and routing in, the last layer's rows out, every step, eager
    xh, idh, wh = x.cpu().pin_memory(), ids.cpu().pin_memory(), weights.cpu().pin_memory()
    outh = torch.empty((args.lines, H), dtype=torch.bfloat16).pin_memory()
    xd, idd, wd = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(weights)
    n_e2e = max(3, min(args.steps, 10))
    with torch.cuda.stream(stream):
        for it in range(n_e2e + 2):
            if it == 2:
                torch.cuda.synchronize()
                pg.barrier()
                es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                es.record(stream)
            xd.copy_(xh, non_blocking=True)
            idd.copy_(idh, non_blocking=True)
            wd.copy_(wh, non_blocking=True)
            for l_ in range(n_layers):
                outs[l_] = mods[l_](xd, idd[l_], wd[l_])
            outh.copy_(outs[-1], non_blocking=True)
        ee.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([es.elapsed_time(ee) / n_e2e], device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    e2e = {"value": args.lines / (float(t.item()) * 1e-3), "unit": "tokens/s",
           "h2d_bytes_per_step": xh.nbytes + idh.nbytes + wh.nbytes, "d2h_bytes_per_step": outh.nbytes,
           "ms_per_step": float(t.item()),
           "through": "drama3_b200.ep.ExpertParallelDecode (peer exchange), eager, every rank"}
    return timed, e2e


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("mine", "reference"), default="mine")
    ap.add_argument("--lines", type=int, default=16)
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers per step (48: the benchmark; 4: small case)")
    ap.add_argument("--kind", choices=("fp8c", "fp8", "w4a8", "w6a8"), default="fp8c",
                    help="expert layout of the headline decode")
    ap.add_argument("--no-extras", action="store_true", help="skip every leg but the headline")
    ap.add_argument("--prefill-only", action="store_true", help="print only the prompt-pass leg (BASELINE configs[3])")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference_arm(args, world)
        return
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        pg = dist

    from drama3_b200 import kernels

    if args.prefill_only:
        if rank == 0:
            print(json.dumps({"prefill": prefill_leg(device, args.steps)}), flush=True)
        return
    n_layers, kind = args.layers, args.kind
    stream = torch.cuda.Stream(device)
    hbm_peak, peak_kind = peaks()
    extras = {}
    spread = None
    if world == 1:
        layers, ids, weights = make_layers(device, args.lines, kind, seed=4, n_layers=n_layers)
        x = torch.randn((args.lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)
        ws = kernels.decode_workspace(args.lines, K_TOP, I, device)
        outs = torch.empty((n_layers, args.lines, H), dtype=torch.bfloat16, device=device)

        def step():
            for l_ in range(n_layers):
                kernels.moe_decode(kind, x, ids[l_], weights[l_], layers[l_], workspace=ws, out=outs[l_])

        with torch.cuda.stream(stream):
            graph = capture(step, args.warmup, stream)
            ms, clocks = timed_region(graph, args, stream, pg, local)
            try:
                spread = replay_spread(graph, max(5, min(args.steps, 50)), stream)
            except Exception as exc:  # the spread must not sink the bench line
                spread = {"error": repr(exc)[:200]}
        del graph
        step_bytes = unique_bytes(ids, kind)
        launches = n_layers * args.steps
    else:
        # expert parallelism: the headline at N > 1
        from drama3_b200 import ep
        local_layers, ids, weights, x = ep_setup(device, kind, args, rank, world)
        peer = ep.PeerExchange(args.lines, H, device)
        mods = [ep.ExpertParallelDecode(kind, banks, E, peer=peer) for banks in local_layers]
        outs = [None] * n_layers

        def step():
            for l_ in range(n_layers):
                outs[l_] = mods[l_](x, ids[l_], weights[l_])

        with torch.cuda.stream(stream):
            graph = capture(step, args.warmup, stream)
            ms, clocks = timed_region(graph, args, stream, pg, local)
        del graph
        first, count = ep.expert_range(E, rank, world)
        per, step_bytes = expert_bytes(kind), 0
        for layer in ids.cpu():
            step_bytes += len({v for v in layer.reshape(-1).tolist() if first <= v < first + count}) * per
        launches = 2 * n_layers * args.steps  # the decode kernel and the reduce kernel per layer
        if not args.no_extras:
            extras["expert_parallel_detail"], extras["e2e"] = ep_extras(kind, args, stream, pg, device, local_layers,
                                                                        mods, ids, weights, x, ms, outs)
        peer.close()
        del mods, local_layers
        torch.cuda.empty_cache()
        if not args.no_extras:
            # replicas (weak scaling): each rank its own 16 lines, all 128 experts resident, no collective
            rl = make_layers(device, args.lines, kind, seed=4 + rank, n_layers=n_layers)
            rleg = decode_leg(kernels, device, kind, args.lines, max(3, min(args.steps, 20)), args.warmup, stream,
                              n_layers, rl)
            t = torch.tensor([rleg["ms_per_step"]], device=device)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            extras["replicas"] = {"tokens_per_s": world * args.lines / (float(t.item()) * 1e-3),
                                  "ms_per_step": float(t.item()), "scaling": "weak (each rank its own lines)"}
            del rl
            torch.cuda.empty_cache()
    value = args.lines / (ms * 1e-3)
    achieved = step_bytes / (ms * 1e-3) / 1e9

    if world == 1 and not args.no_extras:
        # the headline layout at fewer lines (same banks): 1 and 4 lines (config 2's M)
        for lines in (1, 4):
            extras[f"lines_{lines}"] = decode_leg(kernels, device, kind, lines, args.steps, args.warmup, stream,
                                                  n_layers, (layers, ids, weights))
        extras["e2e"] = e2e_leg(device, layers, x, ids, weights, args.lines, args.steps)
        del layers
        torch.cuda.empty_cache()
        # config 1: int8 ConvRot (the reference's layout) at 1 line (and 16), the reference's kernels beside
        c1 = layout_legs(kernels, device, "int8", (1, 16), args, stream, n_layers, 10, reference=True)
        c1["cpu_baseline"] = cpu_line(cpu_int8(n_layers))
        extras["config1_int8"] = c1
        # config 2: the reference's fp8 layout at 1, 4 and 16 lines, the reference's kernels beside
        c2 = layout_legs(kernels, device, "fp8", (1, 4, 16), args, stream, n_layers, 4, reference=True)
        c2["cpu_baseline_lines_1"] = cpu_line(cpu_fp8(1, n_layers, seconds=6.0, min_layers=3))
        extras["config2_fp8_reference_layout"] = c2
        # config 3: W4A8 (BASELINE layout) and the reference's W4 layout at 1 and 16 lines
        extras["config3_w4a8"] = layout_legs(kernels, device, "w4a8", (1, 16), args, stream, n_layers, 5)
        c3 = layout_legs(kernels, device, "w4", (1, 16), args, stream, n_layers, 6, reference=True)
        c3["cpu_baseline_lines_1"] = cpu_line(cpu_codes("w4", 1, n_layers))
        extras["config3_w4_reference_layout"] = c3
        # config 4: the prompt pass on the tensor cores
        try:
            extras["config4_prefill"] = prefill_leg(device, args.steps)
        except Exception as exc:
            extras["config4_prefill"] = {"error": repr(exc)[:200]}
        # the whole MoE block (router, experts, shared expert), fused against torch's chain
        try:
            extras["moe_block"] = block_leg(kernels, device, args, stream)
        except Exception as exc:
            extras["moe_block"] = {"error": repr(exc)[:300]}
        # config 5: the whole decoder step (attention + MoE), 48 layers
        try:
            extras["config5_full_stack"] = full_stack_leg(kernels, device, args, stream)
        except Exception as exc:
            extras["config5_full_stack"] = {"error": repr(exc)[:300]}
        # config 5's host-offload mode: 768-slot cache on one GPU
        try:
            extras["config5_slot_cache"] = slot_cache_leg(device, args, stream)
        except Exception as exc:
            extras["config5_slot_cache"] = {"error": repr(exc)[:300]}
        # the reference's CPU path for the headline (block-scaled fp8: its only fp8 layout), 16 lines
        extras["cpu_baseline"] = cpu_line(cpu_fp8(args.lines, n_layers))

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": kernel_of(kind, args.lines)[1],
                "data": "synthetic (seeded random banks)", "config": config(args, world),
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                             "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                             "traffic": (TRAFFIC_RATIO_1 if args.lines == 1 else TRAFFIC_RATIO) * step_bytes
                             / n_layers, "traffic_unit": "bytes per launch",
                             "traffic_source": TRAFFIC_SOURCE_1 if args.lines == 1 else TRAFFIC_SOURCE,
                             "kernel": kernel_of(kind, args.lines)[0],
                             "bytes_per_launch": step_bytes / n_layers, "us_per_layer": 1e3 * ms / n_layers,
                             "launch_time": "step time / layers: the launches run back to back in one graph",
                             "bytes_of": "rank 0's experts" if world > 1 else "all routed experts"},
                "gpu_launches": launches, "step_spread": spread, "clocks": clocks}
        for key in ("e2e", "cpu_baseline"):
            if key in extras:
                line[key] = extras.pop(key)
        line.update(extras)
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
