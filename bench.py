"""Benchmark: MoE decode tokens/s of the routed-expert path on B200 (FP8 experts with
per-output-channel scales).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference] [--lines 16] [--layers 48]
                    [--kind fp8c] [--no-extras] [--prefill-only]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

A step is one decode pass of `lines` rows (16: lines decoded together) through 48 MoE layers of the BASELINE shape
(hidden 2048, 128 experts, top-8, intermediate 768, SwiGLU), each layer with its own expert banks (default fp8c:
e4m3 rows + fp32 per-output-channel scales) and its own seeded routing: 29 GB of experts, far
larger than L2, so every step streams its experts from HBM (no flush needed). Inputs are resident in HBM; the timed
region replays one CUDA graph per step and is bracketed by cudaProfilerStart/Stop, so `ncu --profile-from-start off`
sees exactly its launches; `--layers 4` is the small case for multi-pass captures (the same banks and routing as the
first 4 layers of the full run). Multi-GPU: independent replicas (each rank decodes its own lines with all experts
resident; no collective), weak scaling. `value` = tokens/s of all ranks; timing = CUDA events, max over ranks.

Also reported at N = 1: the 1-line decode; W4A8 at 16 and 1 lines; the reference's fp8 layout
(128 x 128 block scales) at 16 lines beside the reference's own kernels (compiled from drama3/kernels.py into
oracle/_ref) on the same GPU; the end-to-end rate through the Python API with host buffers; a prompt-pass leg
(2048 tokens, Zipf-skewed routing; W6A8, and the reference's W6 and fp8 layouts beside the
reference's kernels); the reference's CPU path on the host cores. At N > 1: expert parallelism over the N GPUs
(each holds 128 / N experts of every layer, all decode the same 16 lines, fp32 partials all-gathered and summed in
rank order per layer). `--impl reference` runs only that CPU path (rank 0) and prints its line.
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
KINDS = ("fp8c", "fp8", "w4a8", "w6a8", "w6")
FORMAT_NAMES = {
    "fp8c": "e4m3 rows + fp32 per-output-channel scales (BASELINE configs[1])",
    "fp8": "e4m3 rows + fp32 128x128 block scales (the reference's layout)",
    "w4a8": "int4 two per byte + bf16 group-128 scales, int8 per-row activations (BASELINE configs[2])",
    "w6a8": "int6 four per three bytes + bf16 group-128 scales, int8 per-row activations (BASELINE configs[3])",
    "w6": "6-bit codes + e4m3 group-16 scales + s_channel, ConvRot (the reference's W6A8 layout)",
}
# dram bytes (read + write) per launch over algorithmic bytes per launch, from the ncu capture of the small case
# (bench.py --layers 4, the first 2 launches of the timed step: 86 and 87 routed experts); the full run's traffic is
# this ratio x its own bytes
TRAFFIC_RATIO = (407.196928 + 5.279488 + 411.930368 + 4.855552) / (407.164416 + 411.897344)
TRAFFIC_SOURCE = ("ncu capture of the 4-layer small case (bench.py --layers 4, moe_decode_tc_kernel, 2 launches): "
                  "DRAM read + write / algorithmic bytes of the same launches")


def kernel_of(kind, lines):
    """(kernel name, arithmetic) of the fused decode for `kind` banks and `lines` rows."""
    if kind == "fp8c":
        return ("moe_decode_tc_kernel (tcgen05 kind::f8f6f4; one persistent launch per layer: plan, gate_up + "
                "SwiGLU, down, combine)",
                "e4m3 x e4m3 tensor-core MMA: e4m3 weights as stored, bf16 activations as two exact e4m3 terms, "
                "f32 accumulation")
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
    q = torch.randint(0, 256, (E * n, 3 * k // 4), generator=gen, device=device, dtype=torch.uint8)
    g = torch.randint(0x30, 0x50, (E * n, k // 16), generator=gen, device=device, dtype=torch.uint8)
    c = torch.rand((E * n,), generator=gen, device=device) * 2e-4 + 1e-4
    return {"_qdata": q, "scale": g, "s_channel": c}


def expert_bytes(kind):
    """Algorithmic bytes of one expert of the BASELINE shape in `kind`'s layout (weight and scale bytes)."""
    total = 0
    for n, k in ((2 * I, H), (H, I)):
        total += n * {"fp8": k, "fp8c": k, "w4a8": k // 2, "w6a8": 3 * k // 4, "w6": 3 * k // 4}[kind]
        total += {"fp8": (n // 128) * (k // 128) * 4, "fp8c": n * 4, "w4a8": n * (k // 128) * 2,
                  "w6a8": n * (k // 128) * 2, "w6": n * (k // 16 + 4)}[kind]
    return total


def make_layers(device, lines, kind="fp8c", seed=4, n_layers=LAYERS):
    """n_layers layers of banks (random valid codes, positive scales) and per-layer routing; layer l's routing does
    not depend on n_layers or the format."""
    gen = torch.Generator(device=device).manual_seed(seed)
    layers = [tuple(rand_bank(kind, n, k, gen, device) for n, k in ((2 * I, H), (H, I))) for _ in range(n_layers)]
    cpu_gen = torch.Generator().manual_seed(seed + 1)
    ids, weights = [], []
    for _ in range(n_layers):
        w, i = torch.softmax(torch.randn((lines, E), generator=cpu_gen), dim=-1).topk(K_TOP, dim=-1)
        ids.append(i)
        weights.append((w / w.sum(-1, keepdim=True)).to(torch.bfloat16).float())
    return layers, torch.stack(ids).to(device), torch.stack(weights).to(device)


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


def unique_bytes(ids, kind):
    """Algorithmic bytes of one step: each layer's unique experts, plus its rows in and out (bf16)."""
    per, total = expert_bytes(kind), 0
    lines = ids.shape[1]
    for layer in ids.cpu():
        total += len(set(layer.reshape(-1).tolist())) * per + 2 * lines * H * 2 + lines * K_TOP * 12
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


def time_replays(graph, steps, stream):
    """ms per replay of `graph`, CUDA events on `stream`."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
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


def decode_leg(kernels, device, kind, lines, steps, warmup, stream, n_layers, layers):
    """{tokens_per_s, ms_per_step, hbm_gbs, frac, ...} of the fused decode of `lines` rows through n_layers layers;
    layers = (banks, ids, weights)."""
    hbm_peak, _ = peaks()
    banks, ids, weights = layers
    x = torch.randn((lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)
    ws = kernels.decode_workspace(lines, K_TOP, I, device)
    outs = torch.empty((n_layers, lines, H), dtype=torch.bfloat16, device=device)

    def step():
        for l_ in range(n_layers):
            kernels.moe_decode(kind, x, ids[l_], weights[l_], banks[l_], workspace=ws, out=outs[l_])

    with torch.cuda.stream(stream):
        graph = capture(step, warmup, stream)
        ms = time_replays(graph, steps, stream)
    del graph
    b = unique_bytes(ids, kind)
    gbs = b / (ms * 1e-3) / 1e9
    return {"tokens_per_s": lines / (ms * 1e-3), "ms_per_step": ms, "us_per_layer": 1e3 * ms / n_layers,
            "hbm_gbs": gbs, "frac": gbs / hbm_peak, "bytes_per_step": b, "format": FORMAT_NAMES[kind],
            "lines": lines}


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
           "note": "f16 MMAs with f32 accumulation; fp32 activations enter as two f16 terms (hi + lo), int8-quantized "
                   "ones (W6A8) as one exact term; frac = algorithmic flops / time / measured dense bf16 peak"}
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


def cpu_reference(lines, layers_sampled=2, seed=4, n_layers=LAYERS, seconds=10.0):
    """The reference's CPU decode (oracle/cpu_port.py, the FP8Experts CPU forward with its block-scaled layout) on
    the host cores: `lines` rows through at least `layers_sampled` layers and about `seconds` of work, scaled to
    n_layers layers. Returns (tokens/s, seconds, threads, sample description)."""
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
    while done < n_layers and (done < layers_sampled or total < seconds):
        gu, gs, dn, ds = banks[done % 2]
        w, ids = torch.softmax(torch.randn((lines, E), generator=gen), -1).topk(K_TOP, dim=-1)
        w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)
        started = time.perf_counter()
        cpu_port.fp8_decode_lines(x, ids, w, gu, gs, dn, ds)
        total += time.perf_counter() - started
        done += 1
    per_step = total / done * n_layers
    sample = (f"{lines} rows x {done} layers ({total:.1f} s) of the reference CPU path (bf16 dequant + matmuls, one "
              f"row at a time), scaled to {n_layers} layers")
    return lines / per_step, total, torch.get_num_threads(), sample


def ep_leg(kernels, device, kind, args, stream, pg):
    """Expert-parallel decode of `lines` rows through n_layers layers: rank r holds experts expert_range(E, r, N) of
    every layer (seeded whole banks, sliced), all ranks see the same rows and routing; per layer one fused decode of
    the local experts (fp32 partial) and one all-gather + rank-order sum, captured as one CUDA graph per step. Timed
    with CUDA events, max over ranks."""
    from drama3_b200 import ep
    rank, world = pg.get_rank(), pg.get_world_size()
    n_layers = args.layers
    gen = torch.Generator(device=device).manual_seed(4)
    layers = []
    for _ in range(n_layers):
        full = tuple(rand_bank(kind, n, k, gen, device) for n, k in ((2 * I, H), (H, I)))
        layers.append(ep.ExpertParallelDecode(kind, tuple({n: t.clone() for n, t in b.items()}
                                                          for b in ep.local_banks(full, E, rank, world)), E))
        del full
    torch.cuda.empty_cache()
    cpu_gen = torch.Generator().manual_seed(5)
    ids, weights = [], []
    for _ in range(n_layers):
        w, i = torch.softmax(torch.randn((args.lines, E), generator=cpu_gen), dim=-1).topk(K_TOP, dim=-1)
        ids.append(i.to(device))
        weights.append((w / w.sum(-1, keepdim=True)).to(torch.bfloat16).float().to(device))
    x = torch.randn((args.lines, H), generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(device)

    peer = ep.PeerExchange(args.lines, H, device)
    peer_layers = [ep.ExpertParallelDecode(kind, lay.banks, E, peer=peer) for lay in layers]
    outs = [None] * n_layers
    timed = {}
    for name, mods in (("local", layers), ("nccl", layers), ("peer", peer_layers)):
        def step(mods=mods, local=name == "local"):
            for l_ in range(n_layers):
                # "local": each rank's decode alone (its fp32 partial, no exchange), the floor of both exchanges
                outs[l_] = (mods[l_].partial if local else mods[l_])(x, ids[l_], weights[l_])

        with torch.cuda.stream(stream):
            graph = capture(step, args.warmup, stream)  # the exchanges are captured with the kernels
            torch.cuda.synchronize()
            pg.barrier()
            ms = time_replays(graph, max(3, min(args.steps, 20)), stream)
        del graph  # released before the process group is destroyed
        t = torch.tensor([ms], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        timed[name] = float(t.item())
    fault = kernels._lib.take_fault()
    peer.close()
    first, count = ep.expert_range(E, rank, world)
    ms = timed["peer"]
    return {"tokens_per_s": args.lines / (ms * 1e-3), "ms_per_step": ms, "us_per_layer": 1e3 * ms / n_layers,
            "experts_per_rank": count, "scaling": "strong (one job of `lines` rows over all ranks)",
            "exchange": "fused: each rank's decode kernel stores its fp32 partial into every rank's exchange area "
                        "over NVLink (P2P), flags with system-scope release, a small reduce kernel sums in rank order",
            "fault_bits": fault,
            "nccl_all_gather": {"tokens_per_s": args.lines / (timed["nccl"] * 1e-3), "ms_per_step": timed["nccl"],
                                "us_per_layer": 1e3 * timed["nccl"] / n_layers},
            "decode_only_us_per_layer": 1e3 * timed["local"] / n_layers,
            "resident_bytes_per_rank": sum(t.nbytes for lay in layers for b in lay.banks for t in b.values())}


def config(args):
    return {"workload": f"MoE decode, {args.lines} lines x {args.layers} layers per step, {args.kind} experts "
                        f"(BASELINE configs[1] layer shape; 48 layers as configs[4])",
            "layers": args.layers, "lines": args.lines, "experts": E, "top_k": K_TOP, "hidden": H, "intermediate": I,
            "format": FORMAT_NAMES[args.kind],
            "l2": f"inputs larger than L2: {args.layers * E * expert_bytes(args.kind) / 1e9:.1f} GB of expert banks, "
                  f"each layer's routed experts streamed per step",
            "parallelism": f"replicas x{args.gpus} (lines data-parallel)"}


def run_reference_arm(args, rank):
    if rank != 0:
        return
    tps, secs, threads, sample = cpu_reference(args.lines, layers_sampled=max(1, min(args.steps, 2)),
                                               n_layers=args.layers)
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * args.lines / tps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (CPU)",
            "data": "synthetic", "config": config(args),
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("mine", "reference"), default="mine")
    ap.add_argument("--lines", type=int, default=16)
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers per step (48: the benchmark; 4: small case)")
    ap.add_argument("--kind", choices=KINDS[:4], default="fp8c", help="expert layout of the headline decode")
    ap.add_argument("--no-extras", action="store_true", help="skip every leg but the headline")
    ap.add_argument("--prefill-only", action="store_true", help="print only the prompt-pass leg (BASELINE configs[3])")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
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
    layers, ids, weights = make_layers(device, args.lines, kind, seed=4 + rank, n_layers=n_layers)
    x = torch.randn((args.lines, H), generator=torch.Generator().manual_seed(7 + rank)).to(torch.bfloat16).to(device)
    ws = kernels.decode_workspace(args.lines, K_TOP, I, device)
    outs = torch.empty((n_layers, args.lines, H), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.Stream(device)

    def step(xin=x, ids_=ids, w_=weights, out_=outs):
        for l_ in range(n_layers):
            kernels.moe_decode(kind, xin, ids_[l_], w_[l_], layers[l_], workspace=ws, out=out_[l_])

    with torch.cuda.stream(stream):
        graph = capture(step, args.warmup, stream)
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
        # the spread of single steps, after the timed region (this rank's)
        try:
            spread = replay_spread(graph, max(5, min(args.steps, 50)), stream)
        except Exception as exc:  # the spread must not sink the bench line
            spread = {"error": repr(exc)[:200]}
    if pg:
        t = torch.tensor([ms], device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    step_bytes = unique_bytes(ids, kind)
    hbm_peak, peak_kind = peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    value = world * args.lines / (ms * 1e-3)
    del graph

    extras = {}
    if world > 1 and not args.no_extras:
        # expert parallelism (every rank): each rank holds 128 / N experts of one bank set, all ranks decode the same
        # 16 lines, partials gathered and summed in rank order (ep.py); strong scaling of one job
        extras["expert_parallel"] = ep_leg(kernels, device, kind, args, stream, pg)
    if not args.no_extras and world == 1:
        # the single-GPU legs (at N > 1 the other ranks would wait on them at the final barrier)
        # one line decoded at a time (M = 1), same banks
        extras["lines_1"] = decode_leg(kernels, device, kind, 1, args.steps, args.warmup, stream, n_layers,
                                       (layers, ids[:, :1].contiguous(), weights[:, :1].contiguous()))
        # end to end through the Python API: host inputs in, host output back, every step
        xh = x.cpu().pin_memory()
        idh, wh = ids.cpu().pin_memory(), weights.cpu().pin_memory()
        outh = torch.empty((args.lines, H), dtype=torch.bfloat16).pin_memory()
        xd, idd, wd = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(weights)
        n_e2e = max(3, min(args.steps, 20))
        for it in range(n_e2e + 2):
            if it == 2:
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                es.record()
            xd.copy_(xh, non_blocking=True)
            idd.copy_(idh, non_blocking=True)
            wd.copy_(wh, non_blocking=True)
            step(xd, idd, wd, outs)
            outh.copy_(outs[-1], non_blocking=True)
        ee.record()
        torch.cuda.synchronize()
        ms_e2e = es.elapsed_time(ee) / n_e2e
        extras["e2e"] = {"value": args.lines / (ms_e2e * 1e-3), "unit": "tokens/s",
                         "h2d_bytes_per_step": xh.nbytes + idh.nbytes + wh.nbytes, "d2h_bytes_per_step": outh.nbytes,
                         "ms_per_step": ms_e2e, "wall_ms_per_step": 1e3 * (time.perf_counter() - t0) / n_e2e}
        del layers
        torch.cuda.empty_cache()
        # W4A8 at 16 and 1 lines
        w4 = make_layers(device, args.lines, "w4a8", 5, n_layers)
        extras["w4a8"] = {
            "lines_16": decode_leg(kernels, device, "w4a8", args.lines, args.steps, args.warmup, stream, n_layers, w4),
            "lines_1": decode_leg(kernels, device, "w4a8", 1, args.steps, args.warmup, stream, n_layers,
                                  (w4[0], w4[1][:, :1].contiguous(), w4[2][:, :1].contiguous()))}
        del w4
        torch.cuda.empty_cache()
        # the reference's fp8 layout, and the reference's own kernels on it, one row at a time
        # (drama3/model.py:111-113), one CUDA graph per step
        ref_layers = make_layers(device, args.lines, "fp8", 4, n_layers)
        leg = decode_leg(kernels, device, "fp8", args.lines, args.steps, args.warmup, stream, n_layers, ref_layers)
        try:
            from oracle import ref_gpu
            if ref_gpu.available():
                banks_r, ids_r, w_r = ref_layers

                def ref_step():
                    for l_ in range(n_layers):
                        ref_gpu.lines_decode(x, ids_r[l_], w_r[l_], banks_r[l_], (2 * I, H), "fp8", (None, None))

                with torch.cuda.stream(stream):
                    gr = capture(ref_step, 2, stream)
                    rms = time_replays(gr, max(3, min(args.steps, 10)), stream)
                del gr
                leg["reference_gpu"] = {"tokens_per_s": args.lines / (rms * 1e-3), "ms_per_step": rms,
                                        "what": "reference kernels (drama3/kernels.py, nvcc sm_100) driven as "
                                                "drama3/offload.py:108-117, one row at a time"}
                leg["speedup_vs_reference_gpu"] = rms / leg["ms_per_step"]
        except Exception as exc:  # the comparison leg must not sink the bench line
            leg["reference_gpu"] = {"error": repr(exc)[:200]}
        extras["fp8_reference_layout"] = leg
        del ref_layers
        torch.cuda.empty_cache()
        # a prompt pass on the tensor cores (BASELINE configs[3] shape)
        try:
            extras["prefill"] = prefill_leg(device, args.steps)
        except Exception as exc:
            extras["prefill"] = {"error": repr(exc)[:200]}
        # the reference's CPU path on the host cores (bounded sample)
        tps, secs, threads, sample = cpu_reference(args.lines, n_layers=n_layers)
        extras["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                                  "sample": sample, "seconds": secs}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": kernel_of(kind, args.lines)[1],
                "data": "synthetic (seeded random banks)", "config": config(args),
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                             "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                             "traffic": TRAFFIC_RATIO * step_bytes / n_layers,
                             "traffic_unit": "bytes per launch", "traffic_source": TRAFFIC_SOURCE,
                             "kernel": kernel_of(kind, args.lines)[0],
                             "bytes_per_launch": step_bytes / n_layers, "us_per_layer": 1e3 * ms / n_layers,
                             "launch_time": "step time / layers: the launches run back to back in one graph"},
                "gpu_launches": n_layers * args.steps, "step_spread": spread,
                "clocks": clocks.summary()}
        line.update(extras)
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
