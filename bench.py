#!/usr/bin/env python3
"""Benchmark of the FlashMoE hot path on B200.

Default workload (the metric "MoE decode tok/s at
1/2/4/8 B200"): one full decode step of the synthetic 48-layer model — per
layer MLA latent attention (16 heads, nope 128, rope 64, latent 512) over an
8192-row cache and a 512-expert top-10 4-bit MoE FFN with a shared expert,
then the 151936-row vocabulary head and its top-64 candidates — for --batch
sequences (default 8). Random-init weights of that architecture (45 GB) and
random caches; every step reads all its weights and cache rows from HBM
(inputs larger than L2).

Reported (one JSON line on rank 0):
  value     tokens/s of the whole job (batch / step time), device-timed with
            CUDA events over exactly --steps graph-replayed steps (max over
            ranks), inputs resident.
  e2e       the same metric with host buffers: per step, the H2D copy of the
            step's input embeddings from pinned memory, the step, and the D2H
            of its candidate ids and values, all inside the timed region.
  roofline  the dominant kernel (largest share of the step in a per-call
            event-timed pass): its algorithmic bytes per launch / its mean
            launch time vs the measured HBM copy bandwidth; `step` gives the
            whole step's algorithmic bytes / step time.
  cpu_baseline  the C++ oracle chain (restatement of the reference's Rust CPU
            path) on this host's cores, one and all threads, on a bounded
            sample (tokens through 2 of the 48 layers plus the head), scaled to
            the 48-layer step.
`--impl reference` times that oracle chain alone on all host threads (the
reference cannot be built: Rust toolchain absent; its GPU path is Metal).

Multi-GPU (torchrun, N>1): expert and vocabulary parallelism. Rank r holds
experts [r*512/N, (r+1)*512/N) of every layer (the shared expert on rank 0)
and rows [r*V/N, (r+1)*V/N) of the head; attention, router and norms are
replicated, so every rank routes the same tokens and runs its own experts'
routes; each layer's output is the one-shot NVLink peer-memory combine of the
ranks' partials (pbmoe_ep_moe_layer), and the head's candidate lists are
all-gathered (NCCL) and merged (pbmoe_head_merge). The job processes the same
--batch tokens per step at every N ("strong" scaling).

Other lines (`--workload`, one GPU): moe (config 1: one MoE FFN decode layer
per step, 48 layers cycled), matvec (config 0, Q4 [4096x2048]), gemm
(config 2, tcgen05 prefill GEMM, dense and grouped), mla (config 3, absorbed
MLA decode), head (config 4's vocab head + top-64), mxfp4 (the config-0 shape
in MXFP4). Each prints the same keys as the headline line.

`--timeline` (step, one GPU) also prints to stderr each kernel's share of the
graph-replayed step's critical path from a CUPTI kernel timeline; it is
analysis only and changes nothing in the JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, EXPERTS, TOPK, INTER, GROUP = 2048, 512, 10, 512, 64
SLOT_BYTES = 1_769_472
GATE_UP_BYTES = 2 * (524_288 + 2 * 32_768)  # gate + up: nibbles + bf16 S + B
DOWN_BYTES = 524_288 + 2 * 32_768
ROUTER_BYTES = EXPERTS * HIDDEN * 2
SHARED_GATE_BYTES = HIDDEN * 2
METRIC = "MoE decode tok/s (config 1: one MoE FFN decode layer per step)"
# dram__bytes_read.sum + dram__bytes_write.sum per launch from one ncu --set
# full capture of each kernel (profiles/ holds the summaries and commands)
NCU_TRAFFIC = {"expert_gate_up": 95.2e6, "expert_down": 46.6e6, "router+topk": 2.2e6, "combine": 0.75e6}
NCU_TRAFFIC_SOURCE = "ncu --set full of each kernel, 4-layer config-1 case at B=8"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--layers", type=int, default=48)
    p.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    p.add_argument("--workload", default="step", choices=["step", "moe", "matvec", "gemm", "mla", "head", "mxfp4"],
                   help="step: config 4's full 48-layer decode step (the headline line); moe: config 1; "
                        "matvec: config 0; gemm: config 2; mla: config 3; head: config 4's vocab head + top-k; "
                        "mxfp4: the config-0 matvec in MXFP4")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--timeline", action="store_true",
                   help="step workload, one GPU: after the timed runs, print to stderr each kernel's share of the "
                        "graph-replayed step's critical path from a CUPTI kernel timeline (torch.profiler); "
                        "analysis only, never part of the JSON line")
    p.add_argument("--only-batch", action="store_true",
                   help="head / step workloads: run the --batch case alone (no batch 1/8/32 listing)")
    return p.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        return float(json.load(open(path))["bf16_tflops"]), "measured (bf16 burst)"
    return 1590.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        with open(self.file.name) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ CPU arm
def host_layer(seed: int):
    """One config-1 layer generated on the host (torch CPU generator)."""
    import numpy as np
    import torch

    from oracle import pb_oracle

    g = torch.Generator().manual_seed(seed)
    offs, nbytes = pb_oracle.fixed_q4_layout(HIDDEN, INTER, GROUP)

    def sb(rows, groups, n):
        s = torch.empty(n, rows, groups).uniform_(0.004, 0.02, generator=g).to(torch.bfloat16)
        b = (-8.0 * s.float() + torch.randn(n, rows, groups, generator=g) * 1e-3).to(torch.bfloat16)
        return s.view(torch.int16).numpy().view(np.uint8).reshape(n, -1), \
            b.view(torch.int16).numpy().view(np.uint8).reshape(n, -1)

    def table(n):
        t = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, generator=g).numpy()
        for p, (rows, cols) in enumerate([(INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)]):
            s, b = sb(rows, cols // GROUP, n)
            so, bo = int(offs[3 * p + 1]), int(offs[3 * p + 2])
            t[:, so:so + s.shape[1]] = s
            t[:, bo:bo + b.shape[1]] = b
        return t

    router = (torch.randn(EXPERTS, HIDDEN, generator=g) * 0.02).to(torch.bfloat16).view(torch.int16).numpy()
    experts = table(EXPERTS)
    shared = table(1)[0]
    gate = (torch.randn(HIDDEN, generator=g) * 0.02).to(torch.bfloat16).view(torch.int16).numpy()
    return dict(router=router.view(np.uint16), experts=experts, shared=shared, gate=gate.view(np.uint16), offs=offs,
                nbytes=nbytes)


def cpu_oracle_rate(batch: int, steps: int, warmup: int = 0, budget_s: float = 12.0, layer=None):
    """Tokens/s of the oracle MoE layer on this host's cores over `steps` timed
    steps (after `warmup`), each a bounded sample of the workload: the full
    batch when warm-up + steps fit `budget_s`, else fewer tokens per step, and
    if even one token per step does not fit, fewer steps (reported)."""
    import torch

    from oracle import pb_oracle

    threads = os.cpu_count() or 1
    L = layer if layer is not None else host_layer(99)
    g = torch.Generator().manual_seed(5)

    def run(tokens):
        x = torch.randn(tokens, HIDDEN, generator=g).to(torch.bfloat16).float().numpy()
        t0 = time.perf_counter()
        pb_oracle.moe_layer(x, L["router"], L["experts"], L["offs"], L["nbytes"], EXPERTS, TOPK, INTER, GROUP,
                            shared_slot=L["shared"], shared_gate_bits=L["gate"], threads=threads)
        return time.perf_counter() - t0

    run(min(batch, threads))  # warm the page cache / code
    per_token = run(batch) / batch
    total = max(1, steps + warmup)
    tokens = max(1, min(batch, int(budget_s / (total * per_token))))
    run_steps = steps if total * tokens * per_token <= 3 * budget_s else max(1, int(3 * budget_s / per_token) - warmup)
    for _ in range(warmup if run_steps == steps else 0):
        run(tokens)
    times = [run(tokens) for _ in range(run_steps)]
    secs = sum(times)
    return dict(value=tokens * run_steps / secs, unit="tok/s", cores=threads, kind="port",
                sample=(f"{run_steps} steps x {tokens} of the {batch} tokens through one config-1 layer "
                        f"(C++ oracle, {threads} threads)"),
                seconds=secs, per_step_s=secs / run_steps, steps_run=run_steps, tokens_per_step=tokens)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # the reference's CPU path on all host threads; the whole --steps/--warmup
    # run is bounded to a few minutes by the per-step sample size
    from oracle import pb_oracle

    pb_oracle.build()
    res = cpu_oracle_rate(args.batch, steps=args.steps, warmup=max(1, args.warmup), budget_s=150.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": args.gpus,
        "steps": res["steps_run"], "warmup": args.warmup, "ms_per_step": res["per_step_s"] * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, config-1 distributions)",
        "config": {"workload": "config1 MoE FFN decode layer", "batch": args.batch, "hidden": HIDDEN,
                   "experts": EXPERTS, "top_k": TOPK, "intermediate": INTER, "group": GROUP,
                   "tokens_per_step": res["tokens_per_step"]},
        "cpu_baseline": {"value": res["value"], "unit": "tok/s", "cores": res["cores"], "kind": "port",
                         "sample": res["sample"]},
        "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = C++ restatement of pb's Rust CPU path (Rust toolchain absent; Metal GPU path "
                "unavailable on this box)",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ CUDA arm
def main():
    args = parse()
    if args.impl == "reference":
        (run_reference_step if args.workload == "step" else run_reference)(args)
        return
    {"moe": run_moe, "matvec": run_matvec, "gemm": run_gemm, "mla": run_mla, "head": run_head,
     "step": run_step, "mxfp4": run_mxfp4}[args.workload](args)


def run_moe(args):
    """Config 1: one MoE FFN decode layer per step (48 seeded layers cycled)."""
    import numpy as np
    import torch

    from pb_b200 import capi, synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    B, NL = args.batch, args.layers
    ctx = capi.Context(local)
    ep_mode = world > 1
    e_begin, e_count = capi.ep_expert_range(EXPERTS, rank, world) if ep_mode else (0, EXPERTS)
    layers = []
    for i in range(NL):  # identical weights on every rank; each keeps its expert shard
        lw = synth.MoeLayerWeights(dev, seed=1000 + i)
        if ep_mode:
            lw.experts = lw.experts[e_begin:e_begin + e_count].clone()
            if rank != 0:
                lw.shared, lw.shared_gate = None, None
            torch.cuda.empty_cache()
        layers.append(lw)
    cfg = capi.moe_config(layers[0].layout, EXPERTS, TOPK)
    ctx.reserve(B, cfg)
    shard = capi.EpShard(e_begin, e_count, 0)
    if ep_mode:
        from pb_b200 import ep as ep_host

        ep_host.connect(ctx, max_tokens=B, hidden=HIDDEN)
    NIN = 2 * NL  # distinct inputs: step j uses layer j % NL and input j % NIN
    g = synth.gen(dev, 7)  # the same tokens on every rank (replicated activations)
    xs = [synth.normal_bf16((B, HIDDEN), 1.0, g, dev) for _ in range(NIN)]
    outs = [torch.empty(B, HIDDEN, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    weights = [lw.c_weights() for lw in layers]
    stream = torch.cuda.Stream(dev)

    def step(j, s=None, debug=None):
        if ep_mode:
            ctx.ep_moe_layer(cfg, weights[j % NL], shard, xs[j % NIN], outs[j % 2], B, stream=s)
        else:
            ctx.moe_layer(cfg, weights[j % NL], xs[j % NIN], outs[j % 2], B, debug=debug, stream=s)

    # -- unique experts of this rank per (layer, input) combination, from the
    #    routes (the layer's own on one GPU; a torch routing of the same
    #    logits for the byte count of a shard)
    ids = torch.empty(B, TOPK, dtype=torch.int32, device=dev)
    uniq = []
    with torch.cuda.stream(stream):
        for j in range(NIN):
            if ep_mode:
                logits = xs[j].float() @ layers[j % NL].router.float().t()
                sel = torch.unique(torch.topk(logits, TOPK, dim=1).indices)
                uniq.append(int(((sel >= e_begin) & (sel < e_begin + e_count)).sum().item()))
                step(j, stream)
                stream.synchronize()
            else:
                step(j, stream, capi.MoeDebug(None, ids.data_ptr(), None, None, None))
                stream.synchronize()
                uniq.append(int(torch.unique(ids).numel()))
    assert ctx.device_status(stream=stream) == 0

    # -- CUDA graphs: one per step slot, plus one holding a whole cycle of NIN
    #    slots so that the host launches one graph per NIN steps
    graphs = []
    with torch.cuda.stream(stream):
        for j in range(NIN):
            step(j, stream)  # warm the launch path for this slot
        stream.synchronize()
        for j in range(NIN):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                step(j, stream)
            graphs.append(gr)
        cycle = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cycle, stream=stream):
            for j in range(NIN):
                step(j, stream)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()

    def replay_steps(first, count):
        """Replay exactly `count` steps starting at slot `first` (mod NIN)."""
        slot, left = first % NIN, count
        while left and slot != 0:
            graphs[slot].replay()
            slot, left = (slot + 1) % NIN, left - 1
        while left >= NIN:
            cycle.replay()
            left -= NIN
        for j in range(left):
            graphs[j].replay()

    W, K = max(3, args.warmup), args.steps
    with torch.cuda.stream(stream):
        replay_steps(0, W)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            replay_steps(W, K)
            ev1.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clock_summary = clocks.summary()
    assert ctx.device_status(stream=stream) == 0
    value = K * B / (ms / 1e3)  # the job's tokens: replicated over the ranks, not multiplied
    steps_u = [uniq[(W + i) % NIN] for i in range(K)]
    mean_u = float(np.mean(steps_u))
    # bytes one GPU must read per step (its expert shard, replicated router; shared expert on rank 0)
    layer_bytes = (ROUTER_BYTES + SHARED_GATE_BYTES + SLOT_BYTES * (mean_u + (1 if rank == 0 else 0)) +
                   2 * B * HIDDEN * 2)

    # -- per-kernel durations (events between the four kernels; serialised, no PDL overlap)
    NPH = min(K, NIN) if not ep_mode else 0
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(NPH)]
    for row in evs:  # torch creates the CUDA event lazily, on first record
        for e in row:
            e.record(stream)
    stream.synchronize()
    handles = [(C_void_p_array(e)) for e in evs]
    # a device-side sleep first, so the host has queued every launch before
    # the GPU reaches them and host launch gaps stay out of the timings
    with torch.cuda.stream(stream):
        torch.cuda._sleep(50_000_000)
        for i in range(NPH):
            step(W + i, stream, capi.MoeDebug(None, None, None, None, handles[i][0]))
    stream.synchronize()
    names = ["router+topk", "expert_gate_up", "expert_down", "combine"]
    dur = {n: [] for n in names}
    for e in evs:
        for k, n in enumerate(names):
            dur[n].append(e[k].elapsed_time(e[k + 1]))
    mean_dur = {n: float(np.mean(v)) if v else 0.0 for n, v in dur.items()}
    u_ph = [uniq[(W + i) % NIN] for i in range(NPH)] or [mean_u]
    kbytes = {
        "router+topk": ROUTER_BYTES + SHARED_GATE_BYTES + B * HIDDEN * 2,
        "expert_gate_up": float(np.mean([(u + 1) * GATE_UP_BYTES for u in u_ph])) + B * HIDDEN * 2,
        "expert_down": float(np.mean([(u + 1) * DOWN_BYTES for u in u_ph])),
        "combine": B * HIDDEN * 2 * 2 + B * (TOPK + 1) * HIDDEN * 4,
    }
    peak, peak_kind = measured_peaks()
    if ep_mode:  # no per-kernel events through the EP call: the whole layer per GPU
        dominant = "layer (per GPU, expert shard)"
        kbytes[dominant] = layer_bytes
        mean_dur[dominant] = ms / K
    else:
        dominant = max(mean_dur, key=lambda n: mean_dur[n])
    achieved = kbytes[dominant] / (mean_dur[dominant] / 1e3) / 1e9
    serial_ms = sum(v for n, v in mean_dur.items() if n != dominant or not ep_mode)

    # -- end to end through the public C-ABI call with host buffers
    h_in = torch.empty(B, HIDDEN, dtype=torch.bfloat16).pin_memory()
    h_out = torch.empty(B, HIDDEN, dtype=torch.bfloat16).pin_memory()
    h_in.copy_(xs[0].cpu())
    d_in = torch.empty(B, HIDDEN, device=dev, dtype=torch.bfloat16)
    KE = min(K, 4 * NIN)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(KE):
            if ep_mode:
                d_in.copy_(h_in, non_blocking=True)
                ctx.ep_moe_layer(cfg, weights[i % NL], shard, d_in, outs[0], B, stream=stream)
                h_out.copy_(outs[0], non_blocking=True)
            else:
                # one C-ABI call: H2D of the tokens, the layer, D2H of its output
                ctx.moe_layer_host(cfg, weights[i % NL], h_in, h_out, B, stream=stream)
        e1.record(stream)
    stream.synchronize()
    ems = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ems], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e_value = KE * B / (ems / 1e3)
    assert ctx.device_status(stream=stream) == 0

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from oracle import pb_oracle

            pb_oracle.build()
            cpu = cpu_oracle_rate(B, steps=20, warmup=1, budget_s=12.0)
            cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "port", "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded; config-1 shapes and distributions)",
            "config": {"workload": "config1 MoE FFN decode layer", "batch": B, "hidden": HIDDEN,
                       "experts": EXPERTS, "top_k": TOPK, "intermediate": INTER, "group": GROUP,
                       "shared_expert": True, "layers_cycled": NL,
                       "l2": f"inputs larger than L2: {NL} distinct layers cycled ({NL * SLOT_BYTES * EXPERTS / 1e9:.1f} GB experts)",
                       "parallelism": (f"ep{world}: experts sharded {EXPERTS // world}/GPU, one-shot NVLink "
                                       "P2P combine" if ep_mode else "single GPU"),
                       "graph": f"CUDA graphs of {NIN} steps replayed back to back"},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": B * HIDDEN * 2,
                    "d2h_bytes_per_step": B * HIDDEN * 2, "steps": KE},
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         # DRAM read+write of one gate/up launch (ncu, config-1 shapes, B = 8)
                         "traffic": NCU_TRAFFIC.get(dominant), "traffic_source": NCU_TRAFFIC_SOURCE,
                         "algorithmic_bytes_per_launch": kbytes[dominant],
                         "launch_ms": mean_dur[dominant]},
            "layer": {"unique_experts_mean": mean_u, "algorithmic_bytes": layer_bytes,
                      "achieved_gbs": layer_bytes / (ms / K / 1e3) / 1e9,
                      "frac_of_peak": layer_bytes / (ms / K / 1e3) / 1e9 / peak,
                      "kernel_ms": mean_dur, "kernel_ms_serial_sum": serial_ms},
            "gpu_launches": 4 * K,
            "clocks": clock_summary,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()


# ------------------------------------------------------------------ other configs
# Single-GPU measurements of the other hot-path stages (BASELINE.json configs
# 0, 2 and 3), each one JSON line with the same keys as the headline.
def _graph_time(calls, stream, steps, warmup):
    """ms per call of `calls` (a list of no-arg launches) captured as one CUDA
    graph and replayed until `steps` calls ran, after `warmup` replays."""
    import torch

    with torch.cuda.stream(stream):
        for c in calls:
            c()
        stream.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for c in calls:
                c()
        for _ in range(max(3, warmup)):
            gr.replay()
        stream.synchronize()
        reps = max(1, (steps + len(calls) - 1) // len(calls))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(torch.cuda.current_device()) as clocks:
            e0.record(stream)
            for _ in range(reps):
                gr.replay()
            e1.record(stream)
            stream.synchronize()
    return e0.elapsed_time(e1) / (reps * len(calls)), reps * len(calls), clocks.summary()


def _e2e_time(call, stream, steps):
    import torch

    with torch.cuda.stream(stream):
        call()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            call()
        e1.record(stream)
        stream.synchronize()
    return e0.elapsed_time(e1) / steps


def _emit(line):
    print(json.dumps(line), flush=True)


QMV_R, QMV_C, QMV_G, QMV_N = 4096, 2048, 64, 64  # config 0, 64 distinct matrices cycled (303 MB > L2)
QMV_BYTES = QMV_R * QMV_C // 2 + 2 * QMV_R * (QMV_C // QMV_G) * 2 + QMV_C * 2 + QMV_R * 2  # 4,730,880 per launch


def qmatvec_rates(ctx, steps, warmup, seed=1):
    """Config 0 on the device: y = W x for 64 distinct Q4 [4096 x 2048]
    matrices cycled in one CUDA graph (ms per launch), and the same matrices
    as one resident projection batch on the input (pbmoe_q4_matvec_batch,
    resident_mmap_matvec_batch: 4 launches of 16)."""
    import torch

    from pb_b200 import synth

    R, Cc, G, NC = QMV_R, QMV_C, QMV_G, QMV_N
    g = synth.gen("cuda", seed)
    mats = [synth.q4_matrix(R, Cc, G, g, "cuda") for _ in range(NC)]
    x = synth.normal_bf16((1, Cc), 1.0, g, "cuda")
    y = torch.empty(1, R, device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.Stream()
    calls = [(lambda m=m: ctx.q4_matvec(m[0], m[1], m[2], R, Cc, G, x, y, stream=s)) for m in mats]
    ms, n, clocks = _graph_time(calls, s, steps, warmup)
    ys = [torch.empty(1, R, device="cuda", dtype=torch.bfloat16) for _ in range(NC)]
    spec = [(m[0], m[1], m[2], R, Cc, G) for m in mats]
    bms, _, _ = _graph_time([lambda: ctx.q4_matvec_batch(spec, x, ys, stream=s)], s, max(8, steps // NC), warmup)
    return dict(ms=ms, steps=n, clocks=clocks, gbs=QMV_BYTES / (ms / 1e3) / 1e9, batch_ms=bms,
                batch_gbs=NC * QMV_BYTES / (bms / 1e3) / 1e9, mats=mats, x=x, y=y, stream=s)


def run_matvec(args):
    """Config 0: y = W x for W Q4 [4096 x 2048] (group 64), x bf16 [1 x 2048],
    y bf16; 64 distinct weight matrices cycled (303 MB > L2)."""
    import torch

    from pb_b200 import capi

    R, Cc, G, NC, byts = QMV_R, QMV_C, QMV_G, QMV_N, QMV_BYTES
    ctx = capi.Context(0)
    q = qmatvec_rates(ctx, args.steps, args.warmup)
    ms, steps, clocks, gbs, bms, bgbs = q["ms"], q["steps"], q["clocks"], q["gbs"], q["batch_ms"], q["batch_gbs"]
    mats, x, y, s = q["mats"], q["x"], q["y"], q["stream"]
    hx = x.cpu().pin_memory()
    hy = torch.empty(1, R, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty_like(x)
    it = [0]

    def e2e():
        m = mats[it[0] % NC]
        it[0] += 1
        dx.copy_(hx, non_blocking=True)
        ctx.q4_matvec(m[0], m[1], m[2], R, Cc, G, dx, y, stream=s)
        hy.copy_(y, non_blocking=True)

    ems = _e2e_time(e2e, s, min(args.steps, 4 * NC))
    cpu = None
    try:
        import numpy as np

        from oracle import pb_oracle

        pb_oracle.build()
        p, sc, b = (t.cpu() for t in mats[0])
        pn = p.numpy().reshape(-1)
        sn, bn = (synth.bf16_bits(t).numpy().view(np.uint16).reshape(-1) for t in (sc, b))
        xn = x.float().cpu().numpy().reshape(-1)
        t0, n = time.perf_counter(), 0
        while time.perf_counter() - t0 < 5.0:
            pb_oracle.q4_fma_matvec_bf16(pn, xn, sn, bn, R, Cc, G)
            n += 1
        cpu = {"value": byts * n / (time.perf_counter() - t0) / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"{n} matvecs of one config-0 matrix (C++ oracle, 1 thread)"}
    except Exception as exc:
        cpu = {"value": None, "unit": "GB/s", "cores": None, "kind": "port", "sample": f"failed: {exc}"}
    peak, kind = measured_peaks()
    _emit({
        "metric": "qmatvec HBM GB/s (config 0: Q4 [4096x2048] x bf16 [1x2048] -> bf16)", "value": gbs,
        "unit": "GB/s", "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; config-0 distributions)",
        "config": {"workload": "config0 Q4 matvec", "rows": R, "cols": Cc, "group": G,
                   "l2": f"inputs larger than L2: {NC} distinct matrices cycled ({NC * byts / 1e6:.0f} MB)",
                   "graph": f"CUDA graph of {NC} launches"},
        "e2e": {"value": byts / (ems / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": Cc * 2,
                "d2h_bytes_per_step": R * 2, "steps": min(args.steps, 4 * NC)},
        "roofline": {"bound": "hbm", "kernel": "q4_matvec", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_kind": kind, "traffic": None,
                     "algorithmic_bytes_per_launch": byts, "launch_ms": ms},
        "projection_batch": {"value": bgbs, "unit": "GB/s", "frac": bgbs / peak, "matrices": NC,
                             "launches": (NC + 15) // 16, "ms_per_batch": bms,
                             "note": "the 64 config-0 matrices on one input through pbmoe_q4_matvec_batch"},
        "gpu_launches": steps, "clocks": clocks, "cpu_baseline": cpu,
    })
    ctx.close()


def run_gemm(args):
    """Config 2: dense X bf16 [2048 x 2048] . W^T, W Q4 [5120 x 2048]; and the
    grouped layer-major projection: 2048 tokens routed top-10 over 512
    experts, gate W [512 x 2048] per expert (plan + gather + GEMM)."""
    import torch

    from pb_b200 import capi, synth

    M, N, Kd, NC = 2048, 5120, 2048, 24
    flops = 2.0 * M * N * Kd
    ctx = capi.Context(0)
    ctx.prefill_reserve(20480, Kd)
    g = synth.gen("cuda", 2002)
    ws = [synth.q4_matrix(N, Kd, 64, g, "cuda") for _ in range(NC)]  # 142 MB of weights > L2
    x = synth.normal_bf16((M, Kd), 1.0, g, "cuda")
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.Stream()
    calls = [(lambda w=w: ctx.q4_gemm(w[0], w[1], w[2], N, Kd, 64, x, y, stream=s)) for w in ws]
    ms, steps, clocks = _graph_time(calls, s, args.steps, args.warmup)
    tflops = flops / (ms / 1e3) / 1e12
    hx = x.cpu().pin_memory()
    hy = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty_like(x)
    it = [0]

    def e2e():
        w = ws[it[0] % NC]
        it[0] += 1
        dx.copy_(hx, non_blocking=True)
        ctx.q4_gemm(w[0], w[1], w[2], N, Kd, 64, dx, y, stream=s)
        hy.copy_(y, non_blocking=True)

    ems = _e2e_time(e2e, s, min(args.steps, 2 * NC))
    # grouped
    E, TK, I = 512, 10, 512
    layout = capi.fixed_q4_layout(Kd, I, 64)
    table = synth.expert_table(E, layout, g, "cuda")
    ids = synth.random_routes(M, E, TK, g, "cuda")
    i32 = dict(device="cuda", dtype=torch.int32)
    R = M * TK
    se, un, sr, oi, gr_ = (torch.zeros(E, **i32), torch.zeros(1, **i32), torch.zeros(R, **i32),
                           torch.zeros(R, **i32), torch.zeros(E, 2, **i32))
    mat = capi.expert_matrix(table, layout, E, "gate")
    yg = torch.empty(R, I, device="cuda", dtype=torch.bfloat16)
    plan = lambda: ctx.prefill_group_plan(ids, M, TK, E, se, un, sr, oi, gr_, stream=s)
    gemm_g = lambda: ctx.q4_gemm_grouped(mat, se, un, gr_, sr, R, E, x, yg, stream=s)
    plan_ms, _, _ = _graph_time([plan], s, 200, 3)
    g_ms, _, _ = _graph_time([gemm_g], s, 50, 3)
    gflops = 2.0 * R * I * Kd
    wbytes = E * (I * Kd // 2 + 2 * I * (Kd // 64) * 2)
    peak, kind = measured_tensor_peak()
    hbm, _ = measured_peaks()
    cpu = None
    try:
        import numpy as np

        from oracle import pb_oracle

        pb_oracle.build()
        w0 = [t.cpu() for t in ws[0]]
        sn, bn = (synth.bf16_bits(t).numpy().view(np.uint16).reshape(-1) for t in (w0[1], w0[2]))
        rows = 16
        xs = x[:rows].float().cpu().numpy()
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        pb_oracle.q4_gemm(xs, w0[0].numpy().reshape(-1), sn, bn, N, Kd, 64, threads=threads)
        dt = time.perf_counter() - t0
        cpu = {"value": 2.0 * rows * N * Kd / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{rows} of the {M} token rows against the dense W (C++ oracle, {threads} threads)"}
    except Exception as exc:
        cpu = {"value": None, "unit": "TFLOP/s", "cores": None, "kind": "port", "sample": f"failed: {exc}"}
    _emit({
        "metric": "prefill Q4 GEMM TFLOP/s (config 2 dense: X bf16 [2048x2048] . W Q4 [5120x2048]^T)",
        "value": tflops, "unit": "TFLOP/s", "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded; config-2 distributions)",
        "config": {"workload": "config2 prefill qGEMM", "m": M, "n": N, "k": Kd, "group": 64,
                   "l2": f"inputs larger than L2: {NC} distinct weights cycled",
                   "operands": "fp16 (w = q*s+b rounded once; bf16 x converted exactly), fp32 accumulate"},
        "e2e": {"value": flops / (ems / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": M * Kd * 2,
                "d2h_bytes_per_step": M * N * 2, "steps": min(args.steps, 2 * NC)},
        "roofline": {"bound": "tensor", "kernel": "q4_umma_kernel (dense)", "achieved": tflops, "peak": peak,
                     "unit": "TFLOP/s", "frac": tflops / peak, "peak_kind": kind, "traffic": 17.6e6,
                     "traffic_source": "ncu --set full, one dense launch of the config-2 GEMM",
                     "algorithmic_flops_per_launch": flops, "launch_ms": ms},
        "grouped": {"routes": R, "experts": E, "projection": "gate [512x2048] per expert",
                    "plan_ms": plan_ms, "gather_gemm_ms": g_ms, "tflops": gflops / (g_ms / 1e3) / 1e12,
                    "weight_gbs": wbytes / (g_ms / 1e3) / 1e9, "weight_frac_of_hbm": wbytes / (g_ms / 1e3) / 1e9 / hbm},
        "gpu_launches": steps * 2, "clocks": clocks, "cpu_baseline": cpu,
    })
    ctx.close()


def run_mla(args):
    """Config 3: MLA absorbed decode attention, 16 heads, nope 128, rope 64,
    latent 512, v 128, bf16 cache; headline at L = 32768, batch 8 (two cache
    sets cycled, 604 MB > L2), with the four (L, batch) cases listed."""
    import torch

    from pb_b200 import capi, synth

    Hh, NOPE, ROPE, LAT, V = 16, 128, 64, 512, 128
    ctx = capi.Context(0)
    cfg = capi.mla_config()
    ctx.mla_reserve(cfg, 32)
    g = synth.gen("cuda", 3)
    wuk = synth.normal_bf16((Hh, NOPE, LAT), 0.02, g, "cuda")
    wuv = synth.normal_bf16((Hh, V, LAT), 0.02, g, "cuda")
    s = torch.cuda.Stream()
    cases, head = [], None
    for L, B in ((4096, 1), (4096, 8), (32768, 1), (32768, 8)):
        NC = max(2, min(16, (1 << 30) // (L * 1152 * B)))
        sets = [([synth.normal_bf16((L, LAT), 1.0, g, "cuda") for _ in range(B)],
                 [synth.normal_bf16((L, ROPE), 1.0, g, "cuda") for _ in range(B)]) for _ in range(NC)]
        q = synth.normal_bf16((B, Hh, NOPE + ROPE), 1.0, g, "cuda")
        out = torch.empty(B, Hh, V, device="cuda")
        calls = [(lambda st=st: ctx.mla_decode(cfg, q, st[0], st[1], wuk, wuv, out, stream=s)) for st in sets]
        steps = args.steps if (L, B) == (32768, 8) else 200
        ms, n, clocks = _graph_time(calls, s, steps, args.warmup)
        byts = B * L * (LAT + ROPE) * 2 + 2 * Hh * NOPE * LAT * 2
        case = {"L": L, "batch": B, "us": ms * 1e3, "gbs": byts / (ms / 1e3) / 1e9}
        cases.append(case)
        if (L, B) == (32768, 8):
            hq = q.cpu().pin_memory()
            ho = torch.empty(B, Hh, V).pin_memory()
            dq = torch.empty_like(q)

            def e2e():
                dq.copy_(hq, non_blocking=True)
                ctx.mla_decode(cfg, dq, sets[0][0], sets[0][1], wuk, wuv, out, stream=s)
                ho.copy_(out, non_blocking=True)

            ems = _e2e_time(e2e, s, 50)
            head = dict(ms=ms, steps=n, clocks=clocks, bytes=byts, e2e_ms=ems, B=B, L=L, NC=NC)
        del sets
        torch.cuda.empty_cache()
    peak, kind = measured_peaks()
    gbs = head["bytes"] / (head["ms"] / 1e3) / 1e9
    _emit({
        "metric": "MLA decode latent-cache GB/s (config 3: L=32768, batch 8)", "value": gbs, "unit": "GB/s",
        "n_gpus": 1, "steps": head["steps"], "warmup": max(3, args.warmup), "ms_per_step": head["ms"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; config-3 distributions)",
        "config": {"workload": "config3 MLA absorbed decode", "heads": Hh, "nope": NOPE, "rope": ROPE,
                   "latent": LAT, "v": V, "L": head["L"], "batch": head["B"],
                   "l2": f"inputs larger than L2: {head['NC']} cache sets cycled"},
        "e2e": {"value": head["bytes"] / (head["e2e_ms"] / 1e3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": head["B"] * Hh * (NOPE + ROPE) * 2, "d2h_bytes_per_step": head["B"] * Hh * V * 4,
                "steps": 50},
        "roofline": {"bound": "hbm", "kernel": "mla decode (4 kernels)", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_kind": kind, "traffic": None,
                     "algorithmic_bytes_per_launch": head["bytes"], "launch_ms": head["ms"]},
        "cases": cases, "gpu_launches": head["steps"] * 4, "clocks": head["clocks"], "cpu_baseline": None,
    })
    ctx.close()


def run_mxfp4(args):
    """The config-0 matvec shape in MXFP4 (survey row f4): W [4096 x 2048]
    E2M1 + E8M0 per 32 columns, x bf16 [1 x 2048], y bf16; 64 distinct
    matrices cycled (285 MB > L2)."""
    import torch

    from pb_b200 import capi, synth

    R, Cc, NC = 4096, 2048, 64
    byts = R * Cc // 2 + R * Cc // 32 + Cc * 2 + R * 2
    ctx = capi.Context(0)
    g = torch.Generator("cuda").manual_seed(5)
    mats = [(torch.randint(0, 256, (R, Cc // 2), dtype=torch.uint8, device="cuda", generator=g),
             torch.randint(118, 136, (R, Cc // 32), dtype=torch.uint8, device="cuda", generator=g)) for _ in range(NC)]
    x = synth.normal_bf16((1, Cc), 1.0, synth.gen("cuda", 6), "cuda")
    y = torch.empty(1, R, device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.Stream()
    calls = [(lambda m=m: ctx.mxfp4_matvec(m[0], m[1], R, Cc, x, y, stream=s)) for m in mats]
    ms, steps, clocks = _graph_time(calls, s, args.steps, args.warmup)
    gbs = byts / (ms / 1e3) / 1e9
    hx = x.cpu().pin_memory()
    hy = torch.empty(1, R, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty_like(x)
    it = [0]

    def e2e():
        m = mats[it[0] % NC]
        it[0] += 1
        dx.copy_(hx, non_blocking=True)
        ctx.mxfp4_matvec(m[0], m[1], R, Cc, dx, y, stream=s)
        hy.copy_(y, non_blocking=True)

    ems = _e2e_time(e2e, s, min(args.steps, 4 * NC))
    peak, kind = measured_peaks()
    _emit({
        "metric": "MXFP4 matvec HBM GB/s (W E2M1/E8M0 [4096x2048] x bf16 [1x2048] -> bf16)", "value": gbs,
        "unit": "GB/s", "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; uniform nibbles, E8M0 in [118, 136))",
        "config": {"workload": "MXFP4 matvec (config-0 shape)", "rows": R, "cols": Cc, "group": 32,
                   "l2": f"inputs larger than L2: {NC} distinct matrices cycled ({NC * byts / 1e6:.0f} MB)",
                   "graph": f"CUDA graph of {NC} launches"},
        "e2e": {"value": byts / (ems / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": Cc * 2,
                "d2h_bytes_per_step": R * 2, "steps": min(args.steps, 4 * NC)},
        "roofline": {"bound": "hbm", "kernel": "mxfp4_matvec", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_kind": kind, "traffic": None,
                     "algorithmic_bytes_per_launch": byts, "launch_ms": ms},
        "gpu_launches": steps, "clocks": clocks, "cpu_baseline": None,
    })
    ctx.close()


def run_head(args):
    """Config 4's vocab head: logits = W x for W bf16 [151936 x 2048] (622 MB
    > L2, read once per call) and top-64 candidates per token (topk_vocab
    order); headline at --batch tokens (1, 8 and 32 listed)."""
    import torch

    from pb_b200 import capi, synth

    V, H, K = 151936, 2048, 64
    ctx = capi.Context(0)
    ctx.head_reserve(32, V, K)
    w = synth.normal_bf16((V, H), 0.02, synth.gen("cuda", 4), "cuda")
    s = torch.cuda.Stream()
    cases, head = [], None
    for B in ([args.batch] if args.only_batch else (1, 8, 32)):
        x = synth.normal_bf16((B, H), 1.0, synth.gen("cuda", 40 + B), "cuda")
        ids = torch.empty(B, K, dtype=torch.int32, device="cuda")
        vals = torch.empty(B, K, device="cuda")
        call = lambda x=x, ids=ids, vals=vals: ctx.head_topk(w, x, ids, vals, stream=s)
        steps = args.steps if B == args.batch else 100
        ms, n, clocks = _graph_time([call], s, steps, args.warmup)
        byts = V * H * 2 + B * H * 2 + B * K * 8
        cases.append({"batch": B, "us": ms * 1e3, "gbs": byts / (ms / 1e3) / 1e9, "tok_s": B / (ms / 1e3)})
        if B == args.batch:
            hx = x.cpu().pin_memory()
            hi = torch.empty(B, K, dtype=torch.int32).pin_memory()
            hv = torch.empty(B, K).pin_memory()
            dx = torch.empty_like(x)

            def e2e():
                dx.copy_(hx, non_blocking=True)
                ctx.head_topk(w, dx, ids, vals, stream=s)
                hi.copy_(ids, non_blocking=True)
                hv.copy_(vals, non_blocking=True)

            ems = _e2e_time(e2e, s, 100)
            head = dict(ms=ms, steps=n, clocks=clocks, bytes=byts, e2e_ms=ems, B=B)
    peak, kind = measured_peaks()
    gbs = head["bytes"] / (head["ms"] / 1e3) / 1e9
    _emit({
        "metric": f"vocab head GB/s (config 4 LM head [151936x2048] bf16 + top-{K}, batch {head['B']})",
        "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": head["steps"], "warmup": max(3, args.warmup),
        "ms_per_step": head["ms"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded; head weight ~N(0,0.02), x ~N(0,1))",
        "config": {"workload": "config4 vocab head + topk_vocab", "vocab": V, "hidden": H, "top_k": K,
                   "batch": head["B"], "l2": "inputs larger than L2: the 622 MB head is read once per call"},
        "e2e": {"value": head["bytes"] / (head["e2e_ms"] / 1e3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": head["B"] * H * 2, "d2h_bytes_per_step": head["B"] * K * 8, "steps": 100},
        "roofline": {"bound": "hbm", "kernel": "head (memset + gemv + 2 select)", "achieved": gbs, "peak": peak,
                     "unit": "GB/s", "frac": gbs / peak, "peak_kind": kind, "traffic": None,
                     "algorithmic_bytes_per_launch": head["bytes"], "launch_ms": head["ms"]},
        "cases": cases, "gpu_launches": head["steps"] * 3, "clocks": head["clocks"], "cpu_baseline": None,
    })
    ctx.close()


# ------------------------------------------------------------------ config 4: the decode step
STEP_SAMPLE_LAYERS = 2  # layers of the CPU sample (scaled to the model's 48)


def host_step_model(cfg, layers: int, seed: int = 0):
    """Config-4 weights on the host (numpy) for the CPU baseline: `layers`
    layers at full shapes plus the vocabulary head, the synthetic
    distributions of the GPU model (not the same draws: a timing sample; the
    512 expert slots repeat 16 distinct ones and the head's rows a 4096-row
    block, which changes no operation count)."""
    import numpy as np

    from oracle import pb_oracle

    rng = np.random.default_rng(seed)

    def bf(a):  # f32 -> bf16 bits, round to nearest even (finite inputs), in u32 arithmetic
        u = np.ascontiguousarray(a, np.float32).view(np.uint32)
        return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)

    def q4(rows, cols):
        s = rng.uniform(0.004, 0.02, (rows, cols // cfg.group)).astype(np.float32)
        sb = bf(s)
        b = bf(-8.0 * pb_oracle.bf16_bits_to_f32(sb) + rng.normal(0, 1e-3, s.shape))
        return dict(packed=np.frombuffer(rng.bytes(rows * cols // 2), dtype=np.uint8).reshape(rows, cols // 2).copy(),
                    s=sb.reshape(-1),
                    b=b.reshape(-1), rows=rows, cols=cols)

    def table(n):
        offs, nbytes = pb_oracle.fixed_q4_layout(cfg.hidden, cfg.inter, cfg.group)
        m = min(n, 16)
        t = np.frombuffer(rng.bytes(m * nbytes), dtype=np.uint8).reshape(m, nbytes).copy()
        for p, (rows, cols) in enumerate([(cfg.inter, cfg.hidden), (cfg.inter, cfg.hidden), (cfg.hidden, cfg.inter)]):
            s = rng.uniform(0.004, 0.02, (m, rows * cols // cfg.group)).astype(np.float32)
            sb = bf(s)
            b = bf(-8.0 * pb_oracle.bf16_bits_to_f32(sb) + rng.normal(0, 1e-3, s.shape))
            so, bo = int(offs[3 * p + 1]), int(offs[3 * p + 2])
            t[:, so:so + sb.shape[1] * 2] = sb.view(np.uint8).reshape(m, -1)
            t[:, bo:bo + b.shape[1] * 2] = b.view(np.uint8).reshape(m, -1)
        return np.ascontiguousarray(np.tile(t, (n // m + 1, 1))[:n]), offs, nbytes

    norm = lambda n: (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    out = []
    for _ in range(layers):
        experts, offs, nbytes = table(cfg.experts)
        shared, _, _ = table(1)
        out.append(dict(
            q_a=q4(cfg.q_lora, cfg.hidden), kv_a=q4(cfg.latent + cfg.rope, cfg.hidden),
            q_b=q4(cfg.heads * (cfg.nope + cfg.rope), cfg.q_lora), o_proj=q4(cfg.hidden, cfg.heads * cfg.v_dim),
            q_a_norm=norm(cfg.q_lora), kv_a_norm=norm(cfg.latent), post_norm=norm(cfg.hidden),
            in_norm=norm(cfg.hidden), w_uk=bf(rng.normal(0, 0.02, cfg.heads * cfg.nope * cfg.latent)),
            w_uv=bf(rng.normal(0, 0.02, cfg.heads * cfg.v_dim * cfg.latent)),
            router=bf(rng.normal(0, 0.02, cfg.experts * cfg.hidden)), gate=bf(rng.normal(0, 0.02, cfg.hidden)),
            experts=experts, shared=shared[0], offs=offs, nbytes=nbytes,
            lat=pb_oracle.bf16_bits_to_f32(bf(rng.standard_normal((cfg.context, cfg.latent), dtype=np.float32))),
            rot=pb_oracle.bf16_bits_to_f32(bf(rng.standard_normal((cfg.context, cfg.rope), dtype=np.float32)))))
    block = bf(rng.standard_normal((4096, cfg.hidden), dtype=np.float32) * np.float32(0.02))
    head = np.ascontiguousarray(np.tile(block, (cfg.vocab // 4096 + 1, 1))[:cfg.vocab])
    return out, head


def cpu_step_chain(cfg, layers, head, x, position, threads):
    """One token through the sampled layers and the head on the CPU oracle,
    in the decode step's order (runtime/mod.rs:1432-2024, 2779-2940): returns
    (seconds in the layers, seconds in the head)."""
    import numpy as np

    from oracle import pb_oracle as o

    q4 = lambda P, v: o.q4_fma_matvec_bf16(P["packed"], np.ascontiguousarray(v, np.float32), P["s"], P["b"],
                                           P["rows"], P["cols"], cfg.group, threads=threads)
    bf = lambda a: o.bf16_bits_to_f32(o.f32_to_bf16_bits(np.asarray(a, np.float32)))
    t0 = time.perf_counter()
    xn = o.rms_norm(x, layers[0]["in_norm"], cfg.eps)
    for L in layers:
        qa = o.rms_norm(q4(L["q_a"], xn), L["q_a_norm"], cfg.eps)
        kv = q4(L["kv_a"], xn)
        kv[:cfg.latent] = o.rms_norm(kv[:cfg.latent], L["kv_a_norm"], cfg.eps)
        q = q4(L["q_b"], qa).reshape(cfg.heads, cfg.nope + cfg.rope)
        for h in range(cfg.heads):
            q[h, cfg.nope:] = o.rope_interleaved_to_split_half(q[h, cfg.nope:], position, cfg.rope, cfg.theta)
        L["lat"][position] = bf(kv[:cfg.latent])
        L["rot"][position] = bf(o.rope_interleaved_to_split_half(kv[cfg.latent:], position, cfg.rope, cfg.theta))
        attn = o.mla_absorbed_attention(q.reshape(-1), L["lat"][:position + 1], L["rot"][:position + 1], L["w_uk"],
                                        L["w_uv"], cfg.heads, cfg.nope, cfg.rope, cfg.latent, cfg.v_dim)
        h_row = x + q4(L["o_proj"], attn)
        n = bf(o.rms_norm(h_row, L["post_norm"], cfg.eps))
        out, _, _, _ = o.moe_layer(n[None, :], L["router"], L["experts"], L["offs"], L["nbytes"], cfg.experts,
                                   cfg.top_k, cfg.inter, cfg.group, shared_slot=L["shared"], shared_gate_bits=L["gate"],
                                   residual=h_row[None, :], threads=threads)
        x = out[0]
        xn = o.rms_norm(x, L["in_norm"], cfg.eps)
    t1 = time.perf_counter()
    o.head_topk(head, xn[None, :], cfg.candidates)
    return t1 - t0, time.perf_counter() - t1


def cpu_step_rate(cfg, batch, threads, model=None, reps=1):
    """Tokens/s of the oracle chain for the 48-layer step: `threads` = 1 runs
    one token at a time on one thread; more threads run min(batch, threads)
    tokens concurrently (one token per thread, each oracle call on one
    thread). Layer time is scaled from the sampled layers to cfg.layers."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    layers, head = model if model is not None else host_step_model(cfg, STEP_SAMPLE_LAYERS)
    conc = 1 if threads <= 1 else max(1, min(batch, threads))
    rng = np.random.default_rng(3)
    xs = [rng.standard_normal(cfg.hidden).astype(np.float32) for _ in range(conc)]
    cpu_step_chain(cfg, layers, head, xs[0], cfg.context - 1, 1)  # warm caches and code
    walls = []
    for _ in range(reps):
        t0 = time.perf_counter()
        if conc == 1:
            tl, th = cpu_step_chain(cfg, layers, head, xs[0], cfg.context - 1, 1)
        else:
            with ThreadPoolExecutor(max_workers=conc) as pool:
                res = list(pool.map(lambda x: cpu_step_chain(cfg, layers, head, x, cfg.context - 1, 1), xs))
            tl, th = max(r[0] for r in res), max(r[1] for r in res)
        walls.append(time.perf_counter() - t0)
        per_step = tl * cfg.layers / len(layers) + th  # seconds for conc tokens through the whole model
    return dict(value=conc / per_step, unit="tok/s", cores=conc, kind="port", seconds=sum(walls), per_step_s=per_step,
                sample=(f"{conc} token(s) on {conc} thread(s) through {len(layers)} of the {cfg.layers} layers "
                        f"(context {cfg.context}) and the {cfg.vocab}-row head, layer time scaled x"
                        f"{cfg.layers // len(layers)} (C++ oracle chain)"))


def cpu_model_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference_step(args):
    """The reference arm for the config-4 step: the oracle chain on all host
    threads (one token per thread), each step a bounded sample."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import pb_oracle

    from pb_b200 import decode

    pb_oracle.build()
    cfg = decode.StepConfig()
    threads = os.cpu_count() or 1
    model = host_step_model(cfg, STEP_SAMPLE_LAYERS)
    cpu_step_rate(cfg, args.batch, threads, model=model, reps=max(1, min(args.warmup, 2)))  # warm-up samples
    res = cpu_step_rate(cfg, args.batch, threads, model=model, reps=args.steps)
    line = {
        "impl": "reference", "metric": STEP_METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["per_step_s"] * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; config-4 shapes and distributions)",
        "config": {"workload": "config4 decode step", "batch": args.batch, "layers": cfg.layers,
                   "context": cfg.context, "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k,
                   "vocab": cfg.vocab},
        "cpu_baseline": {"value": res["value"], "unit": "tok/s", "cores": res["cores"], "kind": "port",
                         "sample": res["sample"], "cpu": cpu_model_name()},
        "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = C++ restatement of pb's Rust CPU path (Rust toolchain absent; Metal GPU path "
                "unavailable on this box)",
    }
    print(json.dumps(line), flush=True)


STEP_METRIC = "MoE decode tok/s (config 4: 48-layer MLA + 512-expert top-10 MoE decode step, context 8192)"


def run_step(args):
    """Config 4: the full 48-layer decode step for --batch sequences at
    position 8191 of their 8192-row caches; expert and vocabulary parallel
    under torchrun."""
    import numpy as np
    import torch

    from pb_b200 import capi, decode

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    cfg = decode.StepConfig()
    B = args.batch
    ctx = capi.Context(local)
    model = decode.Model(cfg, seed=4, ep=(rank, world) if world > 1 else None)
    caches = decode.Caches(cfg, B, seed=B)
    step = decode.DecodeStep(ctx, model, caches, B, [cfg.context - 1] * B)
    x0 = torch.randn(B, cfg.hidden, generator=torch.Generator("cuda").manual_seed(11), device=dev)
    s = torch.cuda.Stream(dev)

    # one recorded step: the routes give the experts each layer reads on this rank
    with torch.cuda.stream(s):
        step.set_input(x0)
        step.launch(stream=s, record_routes=True)
        step.finish(stream=s)
    s.synchronize()
    assert ctx.device_status(stream=s) == 0
    routes = step.route_ids.cpu().numpy()
    lo, cnt = model.expert_range if model.expert_range is not None else (0, cfg.experts)
    uniq = [len({int(e) for e in routes[i].reshape(-1) if lo <= e < lo + cnt}) for i in range(cfg.layers)]
    mean_u = float(np.mean(uniq))
    slot = int(model.layers[0].moe.layout.expert_bytes)
    kv_bytes = cfg.layers * B * cfg.context * (cfg.latent + cfg.rope) * 2
    step_bytes = step.step_weight_bytes() + sum(uniq) * slot + kv_bytes + B * cfg.hidden * 4

    # the step as one CUDA graph (the head's cross-rank merge follows it)
    with torch.cuda.stream(s):
        step.launch(stream=s)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step.launch(stream=s)

    def one_step(copy_in=None):
        if copy_in is not None:
            step.x.copy_(copy_in, non_blocking=True)
        else:
            step.x.copy_(x0)
        graph.replay()
        step.finish(stream=s)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    W, K = max(3, args.warmup), args.steps
    with torch.cuda.stream(s):
        for _ in range(W):
            one_step()
    s.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(s):
            ev0.record(s)
            for _ in range(K):
                one_step()
            ev1.record(s)
        s.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / K)
    clock_summary = clocks.summary()
    assert ctx.device_status(stream=s) == 0
    value = B / (ms / 1e3)

    # end to end with host buffers: embeddings in, candidates out, every step
    hx = x0.cpu().pin_memory()
    hi = torch.empty(B, cfg.candidates, dtype=torch.int32).pin_memory()
    hv = torch.empty(B, cfg.candidates).pin_memory()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(K):
            one_step(copy_in=hx)
            hi.copy_(step.ids, non_blocking=True)
            hv.copy_(step.vals, non_blocking=True)
        e1.record(s)
    s.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / K)
    assert ctx.device_status(stream=s) == 0

    if args.timeline and world == 1:
        _print_timeline(graph, step, x0, s, cfg.layers)

    # per-call timing: one step launched call by call with events between the
    # calls (and the MoE layer's phase events on one GPU); serialised, so the
    # shares are the figure, not the sum
    names_ev = []

    def mark(name):
        e = torch.cuda.Event(enable_timing=True)
        e.record(s)
        names_ev.append((name, e))

    moe_ev = []
    if world == 1:
        moe_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(cfg.layers)]
        for row in moe_ev:
            for e in row:
                e.record(s)
        s.synchronize()
    handles = [C_void_p_array(r) for r in moe_ev]
    with torch.cuda.stream(s):
        step.x.copy_(x0)
        torch.cuda._sleep(20_000_000)
        step.launch(stream=s, mark=mark, moe_events=(lambda i: handles[i][0]) if moe_ev else None)
    s.synchronize()
    tot, cnt_l = {}, {}
    for (n0, a), (_, b) in zip(names_ev[:-1], names_ev[1:]):
        if n0 == "moe_layer" and moe_ev:
            continue
        tot[n0] = tot.get(n0, 0.0) + a.elapsed_time(b)
        cnt_l[n0] = cnt_l.get(n0, 0) + 1
    for row in moe_ev:
        for k, n in enumerate(["moe_router", "moe_gate_up", "moe_down", "moe_combine"]):
            tot[n] = tot.get(n, 0.0) + row[k].elapsed_time(row[k + 1])
            cnt_l[n] = cnt_l.get(n, 0) + 1
    L0 = model.layers[0]
    H, Bf = cfg.hidden, B * 4
    mla_bytes = B * cfg.context * (cfg.latent + cfg.rope) * 2 + 2 * cfg.heads * cfg.latent * (cfg.nope + cfg.v_dim)
    launch_bytes = {
        "q_a+kv_a": L0.q_a.nbytes() + L0.kv_a.nbytes() + Bf * H + Bf * (cfg.q_lora + cfg.latent + cfg.rope),
        "q_b": L0.q_b.nbytes() + Bf * cfg.q_lora + Bf * cfg.heads * (cfg.nope + cfg.rope),
        "mla_decode": mla_bytes + Bf * cfg.heads * (cfg.nope + cfg.rope + cfg.v_dim),
        "o_proj": L0.o_proj.nbytes() + Bf * (cfg.heads * cfg.v_dim + 2 * H),
        "moe_router": cfg.experts * H * 2 + H * 2 + Bf * H + B * H * 2,
        "moe_gate_up": (mean_u + 1) * 2 * (524_288 + 2 * 32_768) + B * H * 2,
        "moe_down": (mean_u + 1) * (524_288 + 2 * 32_768),
        "head": int(model.head.numel()) * 2 + Bf * H,
    }
    per_launch = {n: tot[n] / cnt_l[n] for n in tot}
    dominant = max((n for n in tot if n in launch_bytes), key=lambda n: tot[n])
    achieved = launch_bytes[dominant] / (per_launch[dominant] / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    serial = sum(tot.values())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from oracle import pb_oracle

            pb_oracle.build()
            hm = host_step_model(cfg, STEP_SAMPLE_LAYERS)
            one = cpu_step_rate(cfg, B, 1, model=hm)
            allt = cpu_step_rate(cfg, B, os.cpu_count() or 1, model=hm)
            cpu = {"value": allt["value"], "unit": "tok/s", "cores": allt["cores"], "kind": "port",
                   "sample": allt["sample"], "cpu": cpu_model_name(),
                   "single_thread": {"value": one["value"], "cores": 1, "sample": one["sample"]}}
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "port", "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": STEP_METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; random-init 48-layer MLA + MoE model of the config-4 architecture, "
                    "random bf16 caches)",
            "config": {"workload": "config4 decode step", "batch": B, "layers": cfg.layers, "hidden": cfg.hidden,
                       "experts": cfg.experts, "top_k": cfg.top_k, "q_lora": cfg.q_lora, "heads": cfg.heads,
                       "context": cfg.context, "vocab": cfg.vocab, "head_top_k": cfg.candidates,
                       "l2": "inputs larger than L2: 45 GB of weights and the caches read once per step",
                       "parallelism": (f"ep{world}: experts {cfg.experts // world}/GPU and the head {cfg.vocab // world}"
                                       " rows/GPU, NVLink P2P combine, NCCL candidate all-gather"
                                       if world > 1 else "single GPU"),
                       "graph": "one CUDA graph per step"},
            "e2e": {"value": B / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": B * cfg.hidden * 4,
                    "d2h_bytes_per_step": B * cfg.candidates * 8, "steps": K},
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": STEP_NCU_TRAFFIC.get(dominant),
                         "traffic_source": STEP_NCU_SOURCE.get(dominant),
                         "algorithmic_bytes_per_launch": launch_bytes[dominant],
                         "launch_ms": per_launch[dominant], "share_of_serial": tot[dominant] / serial,
                         "note": ("the call with the largest share in the per-call pass; the router is bound by "
                                  "its serial routing replay and plan (latency), not by its 2 MB of bytes"
                                  if dominant == "moe_router" else "the call with the largest share in the "
                                  "per-call pass"),
                         # the streaming calls (>= 10 MB per call) against the same peak
                         "streaming_calls": {n: {"algorithmic_bytes_per_launch": launch_bytes[n],
                                                 "launch_ms": per_launch[n],
                                                 "frac": launch_bytes[n] / (per_launch[n] / 1e3) / 1e9 / peak,
                                                 "traffic": STEP_NCU_TRAFFIC.get(n)}
                                             for n in launch_bytes if n in per_launch and launch_bytes[n] >= 1e7}},
            "step": {"algorithmic_bytes_per_gpu": step_bytes, "achieved_gbs": step_bytes / (ms / 1e3) / 1e9,
                     "frac_of_peak": step_bytes / (ms / 1e3) / 1e9 / peak, "unique_experts_per_layer": mean_u,
                     "kernel_ms_per_step": {n: round(v, 4) for n, v in sorted(tot.items(), key=lambda kv: -kv[1])},
                     "kernel_ms_serial_sum": serial},
            "gpu_launches": K * step.launches_per_step(),
            "clocks": clock_summary,
            "cpu_baseline": cpu,
        }
        if world == 1:
            # the other half of the headline metric: config 0's qmatvec GB/s
            # (the same figures as --workload matvec, after the step's timing)
            q = qmatvec_rates(ctx, 640, 3)
            line["qmatvec"] = {
                "value": q["gbs"], "unit": "GB/s", "frac": q["gbs"] / peak, "ms_per_launch": q["ms"],
                "launches": q["steps"], "config": "config 0: Q4 [4096x2048] group 64 x bf16 [1x2048] -> bf16, "
                "64 distinct matrices cycled in one CUDA graph (303 MB > L2)",
                "projection_batch": {"value": q["batch_gbs"], "unit": "GB/s", "frac": q["batch_gbs"] / peak,
                                     "ms_per_batch": q["batch_ms"],
                                     "note": "the 64 matrices on one input through pbmoe_q4_matvec_batch"},
                "clocks": q["clocks"]}
            del q
        print(json.dumps(line), flush=True)
    del graph
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()


# dram__bytes_read.sum + dram__bytes_write.sum per launch of the step's kernels
# from one ncu capture (config-4 shapes, batch 8); filled per kernel captured
# DRAM read + write bytes per call, summed over the call's kernels (ncu flushes
# the caches before each profiled kernel, so reads that hit L2 in a replayed
# step, e.g. the MLA split partials, count here)
STEP_NCU_TRAFFIC: dict = {
    "mla_decode": (2.218496 + 75.826176 + 2.808832 + 11.866368) * 1e6,  # absorb, attention (+ partials written), merge
    "moe_router": 2.25792e6,
    "moe_gate_up": (73.243648 + 3.973632) * 1e6,
    "moe_down": (36.826368 + 0.134144) * 1e6,
    "q_a+kv_a": 2.526464e6,
    "q_b": 2.74432e6,
}
_STEP_NCU_CMD = ("ncu --set full --clock-control none -k regex:<kernel> -s <n> -c 1 python bench.py --workload step "
                 "--layers 2 --steps 3 --warmup 3 --no-cpu-baseline (one launch per kernel, config-4 shapes, batch 8)")
STEP_NCU_SOURCE: dict = {k: _STEP_NCU_CMD for k in STEP_NCU_TRAFFIC}


def _print_timeline(graph, step, x0, s, layers):
    """Each kernel's contribution to the critical path of one graph-replayed
    step (how far it extends the timeline past every earlier kernel's end),
    from a CUPTI kernel timeline; written to stderr."""
    import json
    import tempfile

    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        with torch.cuda.stream(s):
            step.x.copy_(x0)
            graph.replay()
        s.synchronize()
    with tempfile.NamedTemporaryFile(suffix=".json") as fh:
        prof.export_chrome_trace(fh.name)
        ev = json.load(open(fh.name))["traceEvents"]
    ks = sorted((e for e in ev if e.get("cat") == "kernel"), key=lambda e: e["ts"])
    agg, prev_end = {}, None
    for e in ks:
        name = e["name"].split("(")[0].split("<")[0].replace("void ", "").replace("pbmoe::", "")
        st, end = e["ts"], e["ts"] + e["dur"]
        a = agg.setdefault(name, [0, 0.0, 0.0])
        a[0] += 1
        a[1] += e["dur"]
        a[2] += end - st if prev_end is None else max(0.0, end - max(prev_end, st))
        prev_end = end if prev_end is None else max(prev_end, end)
    span = (ks[-1]["ts"] + ks[-1]["dur"] - ks[0]["ts"]) if ks else 0.0
    print(f"timeline: {len(ks)} kernels, span {span / 1e3:.3f} ms (under the profiler)", file=sys.stderr)
    print(f"{'kernel':30s} {'launches':>8s} {'busy ms':>8s} {'critical ms':>11s} {'us/layer':>9s}", file=sys.stderr)
    for name, (n, busy, crit) in sorted(agg.items(), key=lambda kv: -kv[1][2]):
        print(f"{name:30s} {n:8d} {busy / 1e3:8.3f} {crit / 1e3:11.3f} {crit / layers:9.2f}", file=sys.stderr)


def C_void_p_array(events):
    """Host array of cudaEvent_t handles for pbmoe_moe_debug.phase_events."""
    import ctypes

    arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
    return ctypes.cast(arr, ctypes.c_void_p).value, arr


if __name__ == "__main__":
    main()
