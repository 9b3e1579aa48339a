"""Benchmark of the kadan_b200 quantized-weight linear path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (decode): the Llama-3-70B-shaped mixed
Q6_K/Q4_K stack (hidden 8192, 64 q / 8 kv heads of 128, ffn 28672, 80
layers; 46.46 GB of packed weights), T=1, tensor-parallel over the N ranks of
one node, N=1 included. q/k/v (by heads) and gate/up (by output columns) are
column shards; o and down are cut along K on super-block boundaries, and
their partial sums are added over NVLink by the GEMV epilogue's peer stores
plus a gather kernel (`--collective fused`, the default). A step is one
token through the whole stack, captured once in a CUDA graph; the weights
(46 GB, 5.8 GB per rank at N=8) are far larger than L2, so no flush is needed
between steps. Total work is fixed as N grows (strong scaling): value = the
stack's weight + activation bytes per step / device time per step (CUDA
events, max over ranks).

On the same line: `launches` (per dependency group, the time of one launch
of every layer, each group replayed alone), `roofline` (the group with the
largest share), `parity` (outputs of the timed graph against the CPU oracle),
`e2e`, and at N=1 on rank 0 `config2` (the config-2 Llama-3-8B Q4_K decode
stack), `moe` (the config-3 MXFP4 MoE layer at T=4096 and T=1), `h3_reference`
(the reference worker's own device GEMV rebuilt for sm_100a, on the config-2
stack) and `cpu_baseline`.

`--impl reference` times the reference's own CPU path (kadan::text::CpuMatvec
over ggml's AVX2 Q6_K / Q4_K dots, compiled from the reference sources into
oracle/_ref) on one layer of the same stack per step, with all host threads.
It loads nothing of this repository's CUDA library.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode GB/s (% HBM peak) & MXFP4 MoE tokens/s at 1/2/4/8 B200"
# Config 2: Llama-3-8B Q4_K stack.
HIDDEN, KV, FFN, LAYERS = 4096, 1024, 14336, 32
# (name, out, in) per layer; dependency groups of one decode step.
GROUPS = [[("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN)],
          [("o", HIDDEN, HIDDEN)],
          [("gate", FFN, HIDDEN), ("up", FFN, HIDDEN)],
          [("down", HIDDEN, FFN)]]
Q4K_BLOCK, Q4K_VALUES = 144, 256
# Config 4: Llama-3-70B, Q6_K attention and down, Q4_K gate/up. Encodings are
# kadan::gguf::Encoding values (Q4_K 1, Q6_K 3); GGML_TYPE ids 12 and 14.
Q4K, Q6K = 1, 3
GGML_TYPE = {Q4K: 12, Q6K: 14}
BLOCK = {Q4K: (144, 256), Q6K: (210, 256)}
C4_HIDDEN, C4_FFN, C4_LAYERS = 8192, 28672, 80
C4_GROUPS = [[("q", Q6K, 8192, 8192), ("k", Q6K, 1024, 8192), ("v", Q6K, 1024, 8192)],
             [("o", Q6K, 8192, 8192)],
             [("gate", Q4K, 28672, 8192), ("up", Q4K, 28672, 8192)],
             [("down", Q6K, 8192, 28672)]]
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
# DRAM bytes (read + write) of one [gate, up] launch of the config-2 stack,
# from an ncu capture of that launch (the profile summary of
# gemv_q4k_mma_kernel holds the command).
GATE_UP_TRAFFIC = 66922496  # 66,164,224 read + 758,272 written
# DRAM bytes (read + write) per launch of config-4 groups at N=1, keyed by
# group, from ncu captures of a 2-layer stack (a launch has the same size at
# any layer count; the profile summaries give the commands).
C4_TRAFFIC: dict = {"down": 194910464 + 4431872,  # gemv_q6k_pair_kernel<3, 4, staged>
                    "gate,up": 270300928 + 4588800}  # gemv_q4k_mma_kernel<1, staged>


def weight_bytes(out: int, in_: int) -> int:
    return out * in_ // Q4K_VALUES * Q4K_BLOCK


def packed_bytes(enc: int, out: int, in_: int) -> int:
    bb, bv = BLOCK[enc]
    return out * (in_ // bv) * bb


def layer_weight_bytes() -> int:
    return sum(weight_bytes(o, i) for g in GROUPS for _, o, i in g)


def c4_layer_bytes() -> int:
    return sum(packed_bytes(e, o, i) for g in C4_GROUPS for _, e, o, i in g)


def step_bytes() -> tuple[int, int]:
    """(weight bytes, activation bytes) streamed per config-2 step."""
    w = LAYERS * layer_weight_bytes()
    act = 0
    for g in GROUPS:
        act += g[0][2] * 4  # shared fp32 input of the group
        act += sum(o * 4 for _, o, _ in g)  # fp32 outputs
    return w, LAYERS * act


def c4_step_bytes(layers: int, tokens: int) -> tuple[int, int]:
    """(weight bytes, activation bytes) of one config-4 step (whole stack)."""
    act = sum(tokens * 4 * (g[0][3] + sum(o for _, _, o, _ in g)) for g in C4_GROUPS)
    return layers * c4_layer_bytes(), layers * act


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    out = {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
           "bf16_tflops_sustained": FALLBACK_BF16_TFLOPS, "source": "fallback"}
    if p.exists():
        try:
            d = json.loads(p.read_text())
            out = {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                   "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                   "source": "measured"}
        except Exception:
            pass
    return out


def rel_err(got, want) -> float:
    """max|got - want| / max(max|want|, 1): the reference's own GEMV check
    (IW/tests/gguf_text.cpp:247-250)."""
    import numpy as np

    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(float(np.max(np.abs(want))), 1.0))


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        # nvidia-smi needs a moment before its first sample.
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.file.flush()

    def summary(self) -> dict:
        rows = []
        try:
            for line in Path(self.file.name).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        finally:
            os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3] not in ("", "[N/A]"))}


def max_over_ranks(dist, value: float, device) -> float:
    if not dist:
        return value
    import torch

    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------ config 2 stack
def build_stack(torch, kb, device, seed: int = 0):
    from kadan_b200 import synth

    layers = []
    for layer in range(LAYERS):
        mats = {}
        for g in GROUPS:
            for i, (name, out, in_) in enumerate(g):
                mats[name] = synth.device_gguf(kb.Q4_K, out, in_, seed * 1000 + layer * 16 + len(mats), device)
        layers.append(mats)
    gen = torch.Generator(device=device).manual_seed(seed + 7)
    acts = {n: torch.randn(1, k, device=device, generator=gen).half().float()
            for n, k in (("x", HIDDEN), ("attn", HIDDEN), ("h", HIDDEN), ("g", FFN))}
    outs = {name: torch.empty(1, out, device=device) for g in GROUPS for name, out, _ in g}
    return layers, acts, outs


def step_jobs(kb, layers, acts, outs):
    """Per layer, per group: a ctypes job array ready for kb200_gguf_gemv_batch."""
    inputs = ["x", "attn", "h", "g"]
    calls = []
    for mats in layers:
        for gi, g in enumerate(GROUPS):
            jobs = [kb.gemv_job(kb.Q4_K, mats[name], acts[inputs[gi]], outs[name], in_=in_, columns=out, rows=1)
                    for name, out, in_ in g]
            arr = (kb.GemvJob * len(jobs))(*jobs)
            calls.append((gi, arr, len(jobs)))
    return calls


def graph_of(torch, stream, fn):
    """fn() once outside capture (kernel attributes, per-stream buffers), then
    captured into a CUDA graph on `stream`."""
    with torch.cuda.stream(stream):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    torch.cuda.synchronize()
    return graph


def launches_of(kb, torch, stream, fn) -> dict:
    """The library's kernel launches of one eager call of fn() on `stream`,
    by kernel name (telemetry phase: every launch is counted)."""
    with kb.Phase() as phase:
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        snap = phase.snapshot()
    phase.close()
    return {k: v["calls"] for k, v in snap["kernels"].items()}


def time_graph(torch, stream, graph, reps: int, warm: int = 1) -> float:
    """ms per replay of `graph` on `stream` (CUDA events on that stream)."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(warm):
            graph.replay()
        a.record(stream)
        for _ in range(reps):
            graph.replay()
        b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def config2_object(args, torch, kb, device, pk) -> tuple[dict, tuple]:
    """The config-2 decode stack (Llama-3-8B Q4_K, 32 layers, T=1), one CUDA
    graph per token, and each dependency group's launches replayed alone."""
    layers, acts, outs = build_stack(torch, kb, device)
    calls = step_jobs(kb, layers, acts, outs)
    stream = torch.cuda.Stream(device)
    sptr = ctypes.c_void_p(stream.cuda_stream)

    def launch(group=None):
        for gi, arr, n in calls:
            if group is None or gi == group:
                kb.check(kb.lib.kb200_gguf_gemv_batch(arr, n, sptr))

    graph = graph_of(torch, stream, launch)
    time_graph(torch, stream, graph, max(3, args.warmup), warm=0)
    steps = max(args.steps, 20)
    ms = time_graph(torch, stream, graph, steps)
    wbytes, abytes = step_bytes()
    names = ["q,k,v", "o", "gate,up", "down"]
    launches = []
    per_layer = 0
    for gi, g in enumerate(GROUPS):
        gg = graph_of(torch, stream, lambda gi=gi: launch(gi))
        us = time_graph(torch, stream, gg, max(3, steps // 4)) / LAYERS * 1e3
        nbytes = sum(weight_bytes(o, i) for _, o, i in g)
        kernels = launches_of(kb, torch, stream, lambda gi=gi: launch(gi))
        per_layer += sum(kernels.values()) // LAYERS
        launches.append({"launch": names[gi], "kernel": " + ".join(sorted(kernels, key=lambda k: (k.startswith("gemv"), k))),
                         "bytes": nbytes,
                         "us": round(us, 2), "gbps": round(nbytes / us / 1e3, 1),
                         "frac": round(nbytes / us / 1e3 / pk["hbm_gbs"], 4)})
        del gg
    value = (wbytes + abytes) / (ms * 1e-3) / 1e9
    gu = launches[2]
    out = {"workload": "BASELINE config 2 decode: Llama-3-8B Q4_K linear stack, 32 layers, T=1",
           "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms, 5), "steps": steps,
           "hbm_frac": round(value / pk["hbm_gbs"], 4), "weight_bytes_per_step": wbytes,
           "launch": f"one CUDA graph per step, {per_layer} dependent launches per layer", "launches": launches,
           "roofline": {"bound": "hbm", "kernel": f"{gu['kernel']} ([gate, up] launch)",
                        "achieved": gu["gbps"], "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gu["frac"],
                        "traffic": GATE_UP_TRAFFIC, "algorithmic_bytes_per_launch": gu["bytes"]}}
    graph = None
    return out, (layers, acts, outs)


# --------------------------------------------------------- headline: config 4
def tp_parity(torch, kb, stack, groups, world: int, rank: int, dist, device, cols: int = 256) -> dict:
    """Outputs the timed graph left behind (the last layer's) against the CPU
    oracle (decode, then a float64 dot), on the first `cols` output columns:
    gate (column shard: this rank's slice) and down (row shards: every rank's
    oracle partial sum over its K slice, added over the ranks, against the
    all-reduced device output). Tolerance 1e-3 (fp32 outputs)."""
    import numpy as np

    from kadan_b200 import tensor_parallel as tp
    from oracle.pyoracle import Oracle

    orc = Oracle()
    proj = {p.name: p for g in groups for p in g}
    first_of = {p.name: g[0].name for g in groups for p in g}
    res = {}
    for name in ("gate", "down"):
        p = proj[name]
        s = tp.shard(p, world, rank)
        n = min(cols, s.out_count)
        rb = kb.row_bytes(p.encoding, s.in_count)
        w = np.ascontiguousarray(stack.weights[-1][name][:n].cpu().numpy()[:, :rb])
        x = stack.local_inputs[first_of[name]]
        want = torch.from_numpy(orc.gemv_f64(p.encoding, w, x.cpu().numpy(), s.in_count, n)).to(device)
        if p.mode == "row" and dist:
            dist.all_reduce(want)
        got = stack.outputs[name][:, :n].double()
        res[name] = rel_err(got.cpu().numpy(), want.cpu().numpy())
    return {"ok": all(v <= 1e-3 for v in res.values()), "max_rel_err": res, "tolerance": 1e-3,
            "columns_checked": cols,
            "what": "last layer's gate (this rank's column shard) and down (all-reduced over the ranks) outputs "
                    "of the graph-replayed stack vs the oracle (decode + float64 dot)"}


def run_default(args, rank, world, local_rank):
    import datetime

    import numpy as np
    import torch

    import kadan_b200 as kb
    from kadan_b200 import tensor_parallel as tp

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    pk = peaks()
    tokens = args.tokens if args.tokens and args.tokens <= 32 else 1
    layers = args.layers or C4_LAYERS
    groups = tp.llama3_70b_projections()
    assert [[(p.name, p.encoding, p.out, p.in_) for p in g] for g in groups] == C4_GROUPS_T
    weights = tp.synth_shards(groups, layers, world, rank, device)
    reducer = None
    if dist and args.collective in ("fused", "peer"):
        from kadan_b200.collectives import PeerAllReduce

        reducer = PeerAllReduce(tokens * C4_HIDDEN, fused=args.collective == "fused")
    stack = tp.DecodeStack(groups, weights, tokens, world, rank, device, collective=reducer)
    stream = torch.cuda.Stream(device)
    graph = graph_of(torch, stream, lambda: stack.launch(stream))
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    names = [",".join(p.name for p in g) for g in groups]
    group_graphs = [graph_of(torch, stream, lambda gi=gi: stack.launch(stream, gi)) for gi in range(len(groups))]
    group_kernels = [launches_of(kb, torch, stream, lambda gi=gi: stack.launch(stream, gi)) for gi in range(len(groups))]
    launches_per_step = sum(sum(k.values()) for k in group_kernels)
    if dist:
        dist.barrier()
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
        # Each dependency group alone (one launch per layer, captured), in the
        # same clocks window: per-launch device time of the kernels of a step.
        group_ms = [time_graph(torch, stream, gg, max(3, args.steps // 4)) for gg in group_graphs]
    ms = max_over_ranks(dist, start.elapsed_time(end) / args.steps, device)
    group_ms = [max_over_ranks(dist, v, device) for v in group_ms]
    clock = clocks.summary()
    group_graphs = None

    launches = []
    for gi, g in enumerate(groups):
        nbytes = sum(tp.shard(p, world, rank).out_count * tp.shard_pitch(p, tp.shard(p, world, rank)) for p in g)
        us = group_ms[gi] / layers * 1e3
        kernel = " + ".join(sorted(group_kernels[gi], key=lambda k: (k.startswith("gemv"), k)))
        launches.append({"launch": names[gi], "kernel": kernel, "bytes": nbytes, "us": round(us, 2),
                         "kernel_launches_per_layer": {k: v // layers for k, v in group_kernels[gi].items()},
                         "gbps": round(nbytes / us / 1e3, 1), "frac": round(nbytes / us / 1e3 / pk["hbm_gbs"], 4),
                         "share": round(group_ms[gi] / sum(group_ms), 4)})
    top = max(range(len(groups)), key=lambda i: group_ms[i])
    dom = launches[top]
    parity = tp_parity(torch, kb, stack, groups, world, rank, dist, device)

    # End to end with host buffers.
    h2d = tokens * C4_HIDDEN * 4
    d2h = tokens * C4_HIDDEN * 4
    e2e_steps = max(3, min(args.steps, 10))
    pin_in = torch.empty(tokens, C4_HIDDEN, pin_memory=True)
    pin_out = torch.empty(tokens, C4_HIDDEN, pin_memory=True)
    dev_in = stack.local_inputs["q"]  # column group: the whole input row
    pin_in.copy_(dev_in.cpu())
    dev_out = stack.outputs["down"]

    def graph_e2e():
        with torch.cuda.stream(stream):
            dev_in.copy_(pin_in, non_blocking=True)
            graph.replay()
            pin_out.copy_(dev_out, non_blocking=True)
        stream.synchronize()

    graph_e2e()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        graph_e2e()
    graph_s = max_over_ranks(dist, (time.perf_counter() - t0) / e2e_steps, device)
    wbytes, abytes = c4_step_bytes(layers, tokens)
    graph_path = {"value": round((wbytes + abytes) / graph_s / 1e9, 2), "unit": "GB/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(graph_s * 1e3, 4),
                  "timing": "host wall clock per step: pinned upload of the step's input, the step's CUDA graph "
                            "(the library's launches), download of the last projection's output, stream sync"}
    if world == 1:
        # The reference-facing call (DenseCompute::dense_gguf_batch): one
        # synchronous kb200_dense_gguf_batch per dependency group with host
        # spans (upload, launch, download, sync inside each call).
        ctx = kb.Context(local_rank)
        host_in = {g[0].name: stack.inputs[g[0].name].cpu().numpy().copy() for g in groups}
        host_out = {p.name: np.empty((tokens, p.out), dtype=np.float32) for g in groups for p in g}
        host_calls = []
        for mats in stack.weights:
            for g in groups:
                jobs = [kb.host_job(p.encoding, mats[p.name].data_ptr(), host_in[g[0].name], host_out[p.name],
                                    in_=p.in_, out=p.out, validated=True, row_bytes_=tp.shard_pitch(p, tp.shard(p, 1, 0)))
                        for p in g]
                host_calls.append((kb.HostJob * len(jobs))(*jobs))
        result = ctypes.c_int(0)

        def host_step():
            for arr in host_calls:
                kb.check(kb.lib.kb200_dense_gguf_batch(ctx.handle, arr, len(arr), None, ctypes.byref(result)))

        host_step()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            host_step()
        host_s = (time.perf_counter() - t0) / e2e_steps
        # The library's own view of one step (telemetry phase): launches per
        # kernel, host seconds inside the launch calls, device seconds.
        with kb.Phase() as phase:
            host_step()
            torch.cuda.synchronize()
            tel = phase.snapshot()
        phase.close()
        telemetry = {k: {"calls": v["calls"], "launch_host_ms": round(v["host_seconds"] * 1e3, 3),
                         "gpu_ms": round(v["gpu_seconds"] * 1e3, 3)} for k, v in tel["kernels"].items()}
        # The Python side of those calls alone: the same number of ctypes
        # calls of kb200_dense_gguf_batch with an empty batch (it returns
        # KB200_UNSUPPORTED at once, before touching anything).
        empty = (kb.HostJob * 1)()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            for _arr in host_calls:
                kb.lib.kb200_dense_gguf_batch(ctx.handle, empty, 0, None, ctypes.byref(result))
        ctypes_s = (time.perf_counter() - t0) / e2e_steps
        ctx.close()
        e2e = {"value": round((wbytes + abytes) / host_s / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": layers * sum(tokens * g[0].in_ * 4 for g in groups),
               "d2h_bytes_per_step": layers * sum(tokens * p.out * 4 for g in groups for p in g),
               "calls_per_step": len(host_calls), "ms_per_step": round(host_s * 1e3, 4),
               "python_call_ms_per_step": round(ctypes_s * 1e3, 4),
               "library_ms_per_step": round((host_s - ctypes_s) * 1e3, 4),
               "telemetry_one_step": telemetry,
               "timing": "host wall clock around synchronous kb200_dense_gguf_batch calls (host spans), one per "
                         "dependency group", "graph_path": graph_path}
    else:
        e2e = dict(graph_path)

    graph = None
    if dist:
        if reducer:
            reducer.close()
        dist.barrier()
        dist.destroy_process_group()
    local_bytes = stack.weight_bytes()
    del stack, weights
    torch.cuda.empty_cache()
    value = (wbytes + abytes) / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q6_k/q4_k weights; activations quantised per 256-value super-block and token to two int8 levels "
                 "(x ~ s*(h + l/254)); exact int32 sub-block sums on the integer tensor pipe, fp32 scale "
                 "combination and accumulation; fp32 outputs",
        "data": "synthetic (seeded Q6_K/Q4_K shards drawn on each device, bf16-representable N(0,1) activations)",
        "config": c4_config(layers, tokens, world),
        "setup": {"weight_bytes_per_rank": local_bytes,
                  "collective": ("none (one rank)" if world == 1 else
                                 "GEMV epilogue stores to peers + gather kernel (fp32, NVLink)" if reducer and
                                 reducer.fused else "peer-memory all-reduce kernel (fp32)" if reducer else
                                 "NCCL all-reduce (fp32)") + (" after o and down" if world > 1 else ""),
                  "launch": f"one CUDA graph per step, {launches_per_step // layers} launches per layer"},
        "hbm_frac_per_gpu": round(local_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        "gpu_launches": args.steps * launches_per_step,
        "gpu_launches_note": "the library's kernel launches of the timed graph replays: per step, the launches "
                             "telemetry counts for one eager call of the captured work (GEMV, Q6_K activation "
                             "quantisation, and the gather kernel of a row-parallel group at N > 1)",
        "launches": launches,
        "roofline": {"bound": "hbm", "kernel": f"{dom['kernel']} ([{dom['launch']}] launch)",
                     "achieved": dom["gbps"], "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": dom["frac"],
                     "peak_source": f"{pk['source']} hbm_gbs",
                     "traffic": C4_TRAFFIC.get(dom["launch"]) if world == 1 else None,
                     "algorithmic_bytes_per_launch": dom["bytes"],
                     "timing": "CUDA events around the group's launches of all layers replayed alone (a captured "
                               "graph), same clocks window as the timed steps"},
        "parity": parity,
        "parity_ok": parity["ok"],
        "e2e": e2e,
        "clocks": clock,
    }
    if rank == 0 and world == 1 and not args.no_extras:
        extras(args, torch, kb, device, pk, line)
    if rank != 0:
        return
    print(json.dumps(line), flush=True)


C4_GROUPS_T = [[tuple(x) for x in g] for g in C4_GROUPS]


def c4_config(layers: int, tokens: int, world: int) -> dict:
    """The headline workload's config, identical on both arms."""
    wbytes, abytes = c4_step_bytes(layers, tokens)
    return {"workload": f"BASELINE config 4 decode: Llama-3-70B Q6_K/Q4_K linear stack, {layers} layers, T={tokens}",
            "weight_bytes_per_step": wbytes, "activation_bytes_per_step": abytes, "parallelism": f"tp{world}",
            "l2": "inputs larger than L2 (46.5 GB of weights per step; 5.8 GB per rank at N=8)"}


def extras(args, torch, kb, device, pk, line):
    """N=1, rank 0: config 2, the config-3 MoE layer, the reference's device
    GEMV, and the CPU baselines. A failure here is reported, not raised."""
    def guarded(name, fn):
        try:
            return fn()
        except Exception as e:  # an extra must not cost the headline line
            return {"error": f"{type(e).__name__}: {e}"}

    c2 = guarded("config2", lambda: config2_object(args, torch, kb, device, pk))
    if isinstance(c2, tuple):
        line["config2"], stack2 = c2
        line["h3_reference"] = guarded("h3", lambda: h3_reference_object(args, torch, kb, *stack2))
        del stack2
    else:
        line["config2"] = c2
    torch.cuda.empty_cache()
    line["moe"] = guarded("moe", lambda: moe_object(args, torch, kb, device, pk))
    torch.cuda.empty_cache()
    line["layer_math"] = guarded("layer_math", lambda: layer_math_object(args, torch, kb, device, pk))
    torch.cuda.empty_cache()
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = guarded("cpu", lambda: cpu_baseline(budget_s=args.cpu_seconds))


def layer_math_object(args, torch, kb, device, pk) -> dict:
    """The layer math around the path on the device: Llama-3-70B decode
    attention (64 query / 8 KV heads of 128, one query row) over a 4k and a
    32k-position fp32 KV cache (HBM bound: the K and V bytes per call against
    the measured copy bandwidth; the 32k cache, 256 MB, exceeds L2), parity of
    the 4k case against the oracle; and one gated delta-net step (16 key / 32
    value heads of 128, kernel 4, one row) with its state read and written."""
    import numpy as np

    from oracle.pyoracle import Oracle

    res = {}
    heads, kv_heads, dim = 64, 8, 128
    gen = torch.Generator(device=device).manual_seed(0)
    for ctx in (4096, 32768):
        q = torch.randn(heads * dim, device=device, generator=gen)
        k = torch.randn(ctx * kv_heads * dim, device=device, generator=gen)
        v = torch.randn(ctx * kv_heads * dim, device=device, generator=gen)
        out = torch.empty(1, heads, dim, device=device)
        ws = torch.empty(kb.lib.kb200_attend_workspace_bytes(1, ctx - 1, heads, dim), dtype=torch.uint8,
                         device=device)
        stream = torch.cuda.current_stream()

        def call():
            kb.check(kb.lib.kb200_attend_cached(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, ctx - 1, heads,
                                                kv_heads, dim, 1.0 / dim ** 0.5, None, None, out.data_ptr(),
                                                ws.data_ptr(), ws.numel(), stream.cuda_stream))

        for _ in range(5):
            call()
        torch.cuda.synchronize()
        reps = 50
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            call()
        b.record(stream)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) / reps * 1e3
        kv_bytes = 2 * ctx * kv_heads * dim * 4
        gbps = kv_bytes / (us * 1e-6) / 1e9
        entry = {"us_per_call": round(us, 2), "kv_bytes": kv_bytes,
                 "roofline": {"bound": "hbm", "kernel": "attend_kernel + attend_combine_kernel",
                              "achieved": round(gbps, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                              "frac": round(gbps / pk["hbm_gbs"], 4), "peak_source": f"{pk['source']} hbm_gbs"}}
        if ctx == 4096:
            want = Oracle().attend_cached(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), rows=1,
                                          position=ctx - 1, heads=heads, kv_heads=kv_heads, dim=dim,
                                          scale=1.0 / dim ** 0.5)
            err = rel_err(out.cpu().numpy(), want)
            entry["parity"] = {"ok": err <= 1e-4, "max_rel_err": err, "tolerance": 1e-4}
        res[f"attention_ctx{ctx}"] = entry
        del q, k, v, ws
    kh, vh, dd, kern = 16, 32, 128, 4
    channels = (2 * kh + vh) * dd
    t = {n: torch.randn(sz, device=device, generator=gen) for n, sz in
         (("qkv", channels), ("z", vh * dd), ("alpha", vh), ("beta", vh), ("conv", channels * kern), ("dt", vh),
          ("norm", dd))}
    t["a"] = -torch.rand(vh, device=device, generator=gen)
    hist = torch.zeros((kern - 1) * channels, device=device)
    state = torch.zeros(vh * dd * dd, device=device)
    y = torch.empty(vh * dd, device=device)

    def step():
        kb.delta_step(history=hist, state=state, output=y, rows=1, key_heads=kh, value_heads=vh, dim=dd,
                      kernel=kern, eps=1e-6, sigmoid_gate=True, **t)

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(50):
        step()
    b.record()
    torch.cuda.synchronize()
    res["delta_step"] = {"us_per_step": round(a.elapsed_time(b) / 50 * 1e3, 2), "rows": 1, "key_heads": kh,
                         "value_heads": vh, "dim": dd, "kernel": kern, "state_bytes": vh * dd * dd * 4,
                         "note": "includes the step workspace allocation of the Python binding"}
    return res


def c4_host_layer(synth):
    """One config-4 layer's packed matrices and activations, host side
    (the same generators as the tests; seeded)."""
    mats = {}
    for gi, g in enumerate(C4_GROUPS):
        for i, (name, enc, out, in_) in enumerate(g):
            gen = synth.q6_k if enc == Q6K else synth.q4_k
            mats[name] = gen(out, in_, seed=gi * 4 + i)
    x = {C4_HIDDEN: synth.activations(C4_HIDDEN, seed=1, dtype="bf16"),
         C4_FFN: synth.activations(C4_FFN, seed=2, dtype="bf16")}
    return mats, x


def load_synth():
    """kadan_b200/synth.py by file path: its host generators need numpy only,
    and importing the package would load the CUDA library."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("kb200_synth_host", ROOT / "kadan_b200" / "synth.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cpu_baseline(budget_s: float = 10.0) -> dict:
    """The reference's CpuMatvec (oracle/_ref) on one config-4 layer (seven
    matrices, 580.8 MB of Q6_K/Q4_K), all host cores, repeated for about
    `budget_s` seconds; plus the same on one core and the scalar restatement."""
    from oracle.pyoracle import REF_LIB, Oracle, Reference

    threads = os.cpu_count() or 1
    mats, x = c4_host_layer(load_synth())
    if REF_LIB.exists():
        ref = Reference()
        kind = "reference"

        def one_layer():
            for g in C4_GROUPS:
                for n, e, o, i in g:
                    ref.cpu_matvec(GGML_TYPE[e], mats[n], x[i], i, o, threads=threads)
        nbytes = c4_layer_bytes()
    else:
        orc = Oracle()
        kind, threads = "port", 1

        def one_layer():
            for g in C4_GROUPS:
                for n, e, o, i in g:
                    orc.gemv_f64(e, mats[n][:64], x[i], i, 64)
        nbytes = sum(packed_bytes(e, 64, i) for g in C4_GROUPS for _, e, _, i in g)
    dt, n = timed_repeats(one_layer, budget_s)
    out = {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": kind,
           "sample": f"one layer of the config-4 stack (7 matrices, {nbytes} weight bytes) x {n} repetitions, "
                     f"{round(dt * n, 1)} s; kadan::text::CpuMatvec 64-column units, activations quantized to Q8_K "
                     f"once per input as the reference does"}
    if kind == "reference":
        out["single_core"] = single_core_baselines(ref, Oracle(), mats, x)
    return out


def timed_repeats(fn, budget_s: float):
    """Seconds per call of `fn` (one untimed call first), repeated for at least `budget_s`."""
    fn()
    t0, n = time.perf_counter(), 0
    while n == 0 or time.perf_counter() - t0 < budget_s:
        fn()
        n += 1
    return (time.perf_counter() - t0) / n, n


def single_core_baselines(ref, oracle, mats, x, budget_s: float = 3.0) -> dict:
    """The other host figures of the decode path, each on one core, GB/s of
    packed weight bytes: the reference's CpuMatvec with one worker over the
    layer (its production host path), and the scalar restatement (decode each
    block, fp64 dot: the oracle's gemv) over the first 256 columns of each
    matrix."""
    def cpu_matvec_one():
        for g in C4_GROUPS:
            for n, e, o, i in g:
                ref.cpu_matvec(GGML_TYPE[e], mats[n], x[i], i, o, threads=1)

    cols = 256

    def scalar():
        for g in C4_GROUPS:
            for n, e, o, i in g:
                oracle.gemv_f64(e, mats[n][:cols], x[i], i, cols)

    dt1, n1 = timed_repeats(cpu_matvec_one, budget_s)
    dt2, n2 = timed_repeats(scalar, budget_s)
    scalar_bytes = sum(packed_bytes(e, cols, i) for g in C4_GROUPS for _, e, _, i in g)
    return {"cpu_matvec_1_core_gbps": round(c4_layer_bytes() / dt1 / 1e9, 3),
            "cpu_matvec_1_core_sample": f"one layer x {n1}",
            "scalar_restatement_1_core_gbps": round(scalar_bytes / dt2 / 1e9, 3),
            "scalar_restatement_1_core_sample": f"first {cols} columns of each matrix x {n2} "
                                                "(oracle decode + fp64 dot)"}


def run_reference(args, rank, world):
    """Reference arm: the reference's CPU path on the box's host cores, one
    config-4 layer per step (rank 0 only; other ranks exit at once)."""
    if rank != 0:
        return
    from oracle.pyoracle import REF_LIB, Oracle, Reference

    threads = os.cpu_count() or 1
    mats, x = c4_host_layer(load_synth())
    if REF_LIB.exists():
        ref = Reference()
        kind = "reference"

        def sample():
            for g in C4_GROUPS:
                for n, e, o, i in g:
                    ref.cpu_matvec(GGML_TYPE[e], mats[n], x[i], i, o, threads=threads)
        sample_bytes = c4_layer_bytes()
    else:
        orc = Oracle()
        kind, threads = "port", 1

        def sample():
            for g in C4_GROUPS:
                for n, e, o, i in g:
                    orc.gemv_f64(e, mats[n][:64], x[i], i, 64)
        sample_bytes = sum(packed_bytes(e, 64, i) for g in C4_GROUPS for _, e, _, i in g)
    for _ in range(args.warmup):
        sample()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sample()
    dt = (time.perf_counter() - t0) / args.steps
    value = sample_bytes / dt / 1e9
    layers = args.layers or C4_LAYERS
    maps = Path("/proc/self/maps").read_text() if Path("/proc/self/maps").exists() else ""
    assert "libkadan_b200" not in maps, "the reference arm must not load this repository's CUDA library"
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q6_k/q4_k weights, Q8_K-quantized activations (reference CPU dot)",
        "data": "synthetic", "impl": "reference",
        "config": c4_config(layers, 1, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"one layer of the stack ({sample_bytes} weight bytes) per step"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_case(args):
    """Small single-kernel cases for profiling (not the headline number):
    gemv-q4k: one batched launch of four 14336x4096 Q4_K GEMVs (132 MB of
    weights, more than L2), T=1, repeated --steps times after --warmup."""
    import torch

    import kadan_b200 as kb
    from kadan_b200 import synth

    dev = torch.device("cuda:0")
    enc = {"gemv-q4k": kb.Q4_K, "gemv-q6k": kb.Q6_K, "gemv-q8": kb.Q8_0}[args.case]
    mats = [synth.device_gguf(enc, FFN, HIDDEN, 100 + i, dev) for i in range(4)]
    x = torch.randn(1, HIDDEN, device=dev).half().float()
    ys = [torch.empty(1, FFN, device=dev) for _ in mats]
    jobs = [kb.gemv_job(enc, w, x, y, in_=HIDDEN, columns=FFN, rows=1) for w, y in zip(mats, ys)]
    for _ in range(args.warmup):
        kb.gguf_gemv_batch(jobs)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        kb.gguf_gemv_batch(jobs)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    nbytes = sum(w.numel() for w in mats)
    print(json.dumps({"case": args.case, "ms_per_launch": round(ms, 5),
                      "gbps": round(nbytes / (ms * 1e-3) / 1e9, 1), "weight_bytes": nbytes}), flush=True)


def moe_layer_inputs(torch, kb, dev, tokens, seed=0):
    """BASELINE config 3 (gpt-oss-20b MoE layer: H=2880, 32 experts, top-4,
    I=2880, SwiGLU clamp 7): MXFP4 codes uniform over 16, E8M0 uniform in
    118..126, bf16 N(0,1) activations and N(0,1) router logits, on `dev`."""
    E, H, I, K = 32, 2880, 2880, 4
    gen = torch.Generator(device=dev).manual_seed(seed)

    def mx(rows, cols):
        blocks = torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device=dev, generator=gen)
        scales = torch.randint(118, 127, (rows, cols // 32), dtype=torch.uint8, device=dev, generator=gen)
        return blocks, scales

    gu_w, gu_s = mx(E * 2 * I, H)
    dn_w, dn_s = mx(E * H, I)
    w = kb.moe_weights(gu_w, gu_s, dn_w, dn_s, hidden=H, inter=I, experts=E, top_k=K)
    x = torch.randn(tokens, H, device=dev, generator=gen).to(torch.bfloat16)
    logits = torch.randn(tokens, E, device=dev, generator=gen)
    weight_bytes = gu_w.numel() + gu_s.numel() + dn_w.numel() + dn_s.numel()
    return w, (gu_w, gu_s, dn_w, dn_s), x, logits, weight_bytes


def mxfp4_to_ggml(blocks, scales, rows: int, cols: int):
    """Exact repack of checkpoint MXFP4 rows (codes [rows, cols/2], value 2j in
    the low nibble of byte j; E8M0 [rows, cols/32], value = e2m1 * 2^(E-127))
    into ggml block_mxfp4 rows (GGML_TYPE_MXFP4 = 39: per 32 values the E8M0
    byte, then 16 bytes whose low nibbles hold values 0..15 and high nibbles
    16..31; ggml's doubled code table with its halved scale gives the same
    value). Returns uint8 [rows, cols/32*17]."""
    import numpy as np

    b = np.asarray(blocks, dtype=np.uint8).reshape(rows, cols // 32, 16)
    codes = np.stack([b & 15, b >> 4], axis=-1).reshape(rows, cols // 32, 32)
    out = np.empty((rows, cols // 32, 17), dtype=np.uint8)
    out[..., 0] = np.asarray(scales, dtype=np.uint8).reshape(rows, cols // 32)
    out[..., 1:] = codes[..., :16] | (codes[..., 16:] << 4)
    return out.reshape(rows, -1)


def moe_cpu_layer(ref, oracle, x, logits, gu_ggml, dn_ggml, *, hidden: int, inter: int, experts: int, top_k: int,
                  threads: int, limit: float = 7.0, alpha: float = 1.702):
    """The MoE layer on the reference's host path: routing with the reference's
    MoeLayer::forward semantics (oracle restatement, qwen_layers.cpp:397-491),
    each expert's gathered rows through kadan::text::CpuMatvec on MXFP4 rows
    (activations quantised to Q8_0 as the reference does, 64-column units on
    `threads` workers), the gpt-oss SwiGLU on interleaved gate/up, and the
    weighted sum in selection order. x: float32 [T, H]."""
    import numpy as np

    chosen, weight = oracle.moe_route(logits, top_k)
    tokens = x.shape[0]
    per_slot = np.zeros((tokens, top_k, hidden), dtype=np.float32)
    for e in range(experts):
        toks, slots = np.nonzero(chosen == e)
        if not len(toks):
            continue
        gu = ref.cpu_matvec(39, gu_ggml[e * 2 * inter:(e + 1) * 2 * inter], x[toks], hidden, 2 * inter, threads)
        gate = np.minimum(gu[:, 0::2], limit).astype(np.float64)
        up = np.clip(gu[:, 1::2], -limit, limit)
        act = (gate / (1.0 + np.exp(np.minimum(-alpha * gate, 700.0))) * (up + 1.0)).astype(np.float32)
        per_slot[toks, slots] = ref.cpu_matvec(39, dn_ggml[e * hidden:(e + 1) * hidden], act, inter, hidden, threads)
    out = np.zeros((tokens, hidden), dtype=np.float32)
    for k in range(top_k):
        out += weight[:, k:k + 1].astype(np.float32) * per_slot[:, k]
    return out


def run_attention(args):
    """--case attention: the layer math around the path (decode attention at
    4k and 32k cached positions, one delta-net step), as in the default
    line's `layer_math`, as its own JSON line."""
    import torch

    import kadan_b200 as kb

    dev = torch.device("cuda:0")
    res = layer_math_object(args, torch, kb, dev, peaks())
    a32 = res["attention_ctx32768"]
    print(json.dumps({"metric": "decode attention GB/s (64 query / 8 KV heads of 128, 32k fp32 positions)",
                      "value": a32["roofline"]["achieved"], "unit": "GB/s", "n_gpus": 1, "steps": 50,
                      "warmup": 5, "higher_is_better": True, "data": "synthetic", "dtype": "f32",
                      "config": {"workload": "Llama-3-70B decode attention, one query row"}, "layer_math": res}),
          flush=True)


def run_moe(args):
    """--case moe: the config-3 MoE layer at --tokens T (tokens/s, TFLOP/s),
    with the reference's host path (moe_cpu_layer on all host threads) timed
    on a bounded sample of the same tokens as cpu_baseline."""
    import torch

    import kadan_b200 as kb

    dev = torch.device("cuda:0")
    T, H, I, K = args.tokens, 2880, 2880, 4
    w, keep, x, logits, weight_bytes = moe_layer_inputs(torch, kb, dev, T)
    out = torch.empty(T, H, device=dev)
    ws = torch.empty(kb.moe_workspace_bytes(w, T), dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        kb.moe_forward(w, x, logits, out=out, workspace=ws)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        kb.moe_forward(w, x, logits, out=out, workspace=ws)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    flops = 2.0 * T * K * (2 * I * H + H * I)
    line = {"case": "moe-config3", "tokens": T, "ms_per_layer": round(ms, 4),
            "tokens_per_s": round(T / (ms * 1e-3), 1), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "all_expert_weight_gbps": round(weight_bytes / (ms * 1e-3) / 1e9, 1)}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = moe_cpu_baseline(keep, x, logits, T, min_seconds=min(args.cpu_seconds, 5.0))
    print(json.dumps(line), flush=True)


def moe_cpu_baseline(keep, x, logits, tokens: int, min_seconds: float = 5.0) -> dict:
    """The config-3 layer on the reference's host path (moe_cpu_layer), all host
    threads, over the first min(tokens, 64) tokens, repeated until at least
    `min_seconds` of host work has been timed."""
    from oracle.pyoracle import Oracle, Reference

    E, H, I, K = 32, 2880, 2880, 4
    sample = min(tokens, 64)
    gu_w, gu_s, dn_w, dn_s = (t.cpu().numpy() for t in keep)
    gu_g, dn_g = mxfp4_to_ggml(gu_w, gu_s, E * 2 * I, H), mxfp4_to_ggml(dn_w, dn_s, E * H, I)
    xs = x[:sample].float().cpu().numpy()
    ls = logits[:sample].cpu().numpy()
    ref, oracle, threads = Reference(), Oracle(), os.cpu_count() or 1
    moe_cpu_layer(ref, oracle, xs[:1], ls[:1], gu_g, dn_g, hidden=H, inter=I, experts=E, top_k=K, threads=threads)
    reps, t0 = 0, time.perf_counter()
    while reps == 0 or time.perf_counter() - t0 < min_seconds:
        moe_cpu_layer(ref, oracle, xs, ls, gu_g, dn_g, hidden=H, inter=I, experts=E, top_k=K, threads=threads)
        reps += 1
    s = time.perf_counter() - t0
    return {"value": round(reps * sample / s, 1), "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"{sample} tokens of the layer x {reps} passes ({s:.1f} s): oracle routing, CpuMatvec "
                      "(ggml MXFP4, Q8_0 activations) experts from oracle/_ref, gpt-oss SwiGLU, selection-order combine",
            "single_core": mxfp4_single_core(ref, gu_w, gu_s, gu_g, xs[0], H, I)}


def mxfp4_single_core(ref, gu_w, gu_s, gu_g, x, hidden: int, inter: int, budget_s: float = 3.0) -> dict:
    """One expert's fused gate/up matrix (2*inter x hidden MXFP4) times one
    token on one core, GB/s of MXFP4 bytes: the reference's numerical path
    quantization::matvec (checkpoint layout, fp64 accumulation) and its
    production host path CpuMatvec on the repacked ggml rows."""
    rows = 2 * inter
    w, sc = gu_w[:rows], gu_s[:rows]
    nbytes = w.nbytes + sc.nbytes
    dt1, n1 = timed_repeats(lambda: ref.mxfp4_matvec(w, sc, rows, hidden, x), budget_s)
    dt2, n2 = timed_repeats(lambda: ref.cpu_matvec(39, gu_g[:rows], x, hidden, rows, 1), budget_s)
    return {"quantization_matvec_1_core_gbps": round(nbytes / dt1 / 1e9, 3),
            "cpu_matvec_mxfp4_1_core_gbps": round(nbytes / dt2 / 1e9, 3),
            "sample": f"expert 0 gate/up ({rows}x{hidden}, {nbytes} bytes), one token, x {n1} and x {n2}"}


def run_prefill(args):
    """--case prefill: BASELINE config 2 prefill, the Llama-3-8B Q4_K stack at
    T = --tokens input rows through kb200_gguf_gemm (one launch per matrix,
    each with its activation-conversion kernel), 2*T*6.98 G FLOP per pass."""
    import torch

    import kadan_b200 as kb

    dev = torch.device("cuda:0")
    T = args.tokens
    layers, _, _ = build_stack(torch, kb, dev)
    gen = torch.Generator(device=dev).manual_seed(7)
    xs = {k: torch.randn(T, k, device=dev, generator=gen) for k in (HIDDEN, FFN)}
    ys = {name: torch.empty(T, out, device=dev) for g in GROUPS for name, out, _ in g}
    ws = torch.empty(kb.gemm_workspace_bytes(T, FFN), dtype=torch.uint8, device=dev)
    jobs = [kb.gemv_job(kb.Q4_K, mats[name], xs[in_], ys[name], in_=in_, columns=out, rows=T)
            for mats in layers for g in GROUPS for name, out, in_ in g]
    stream = torch.cuda.current_stream()

    def one_pass():
        for job in jobs:
            kb.gguf_gemm(job, ws, stream)

    for _ in range(args.warmup):
        one_pass()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, min(args.steps, 20))
    a.record()
    for _ in range(steps):
        one_pass()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    flops = 2.0 * T * LAYERS * sum(o * i for g in GROUPS for _, o, i in g)
    wbytes, _ = step_bytes()
    print(json.dumps({"case": "prefill-config2", "tokens": T, "ms_per_pass": round(ms, 4),
                      "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "weight_gbps": round(wbytes / (ms * 1e-3) / 1e9, 1),
                      "launches_per_pass": 2 * len(jobs)}), flush=True)


def run_tp(args, rank, world, local_rank):
    """--case tp70b: BASELINE config 4, the Llama-3-70B mixed Q6_K/Q4_K decode
    stack (80 layers, 46.46 GB of weights), tensor-parallel over the ranks of
    torchrun: q/k/v (by heads) and gate/up split by output columns, o and
    down split along K with an NCCL all-reduce of the partial sums (two per
    layer). --tokens T rows per step (1..32). A step is captured in one CUDA
    graph (GEMV launches and collectives). value = the whole stack's weight
    and activation bytes per step / step time (max over ranks): total work
    is fixed as N grows (strong scaling)."""
    import datetime

    import torch

    import kadan_b200 as kb
    from kadan_b200 import tensor_parallel as tp

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    group = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    tokens = args.tokens if 1 <= args.tokens <= 32 else 1
    layers = args.layers or 80
    groups = tp.llama3_70b_projections()
    weights = tp.synth_shards(groups, layers, world, rank, device)
    reducer = None
    if dist and args.collective in ("fused", "peer"):
        from kadan_b200.collectives import PeerAllReduce

        reducer = PeerAllReduce(tokens * 8192, fused=args.collective == "fused")
    stack = tp.DecodeStack(groups, weights, tokens, world, rank, device, group=group, collective=reducer)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        stack.launch(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        stack.launch(stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = min(args.steps, 200)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(steps):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    ar_us = None
    if dist:
        # The collective alone (same sizes, same count per step), for the
        # breakdown; not part of the value.
        t = torch.zeros(tokens, 8192, device=device)
        cur = torch.cuda.current_stream()

        def one():
            if reducer:
                reducer(t, cur)
            else:
                dist.all_reduce(t)

        side = torch.cuda.Stream(device)
        for _ in range(20):
            one()
        torch.cuda.synchronize()
        # 2 * layers collectives back to back in one CUDA graph: device time
        # per collective without host launch cost.
        ar_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ar_graph, stream=side):
            cur = side
            for _ in range(2 * layers):
                one()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(side):
            for _ in range(3):
                ar_graph.replay()
            a.record(side)
            for _ in range(10):
                ar_graph.replay()
            b.record(side)
        torch.cuda.synchronize()
        ar_us = a.elapsed_time(b) / (10 * 2 * layers) * 1e3
        ar_graph = None
        m = torch.tensor([ms], device=device)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    wbytes = tp.full_weight_bytes(groups, layers)
    local_bytes = stack.weight_bytes()
    abytes = layers * tokens * 4 * sum(g[0].in_ + sum(p.out for p in g) for g in groups)
    clock = clocks.summary()
    peak, peak_kind = peaks()
    graph = None
    if dist:
        if reducer:
            reducer.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank:
        return
    value = (wbytes + abytes) / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": METRIC, "case": "tp70b", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong", "dtype": "q6_k/q4_k weights, bf16-valued fp32 activations, fp32 accumulation",
        "data": "synthetic (seeded shards drawn on each device)",
        "config": {"workload": f"BASELINE config 4 decode: Llama-3-70B Q6_K/Q4_K, {layers} layers, T={tokens}",
                   "weight_bytes_per_step": wbytes, "weight_bytes_per_rank": local_bytes,
                   "parallelism": f"tp{world}",
                   "collective": ("GEMV epilogue stores to peers + gather-sum kernel (fp32, NVLink)"
                                  if reducer and reducer.fused else
                                  "peer-memory all-reduce kernel (fp32, NVLink stores)" if reducer else
                                  "NCCL all-reduce (fp32)") + " after o and down",
                   "l2": "inputs larger than L2"},
        "hbm_frac_per_gpu": round(local_bytes / (ms * 1e-3) / 1e9 / peak, 4), "peak_gbs": peak,
        "peak_source": f"{peak_kind} hbm_gbs",
        "allreduce_us_alone": None if ar_us is None else round(ar_us, 2),
        "allreduces_per_step": 2 * layers if world > 1 else 0,
        "gpu_launches": steps * len(stack.calls), "clocks": clock}), flush=True)


def run_ep(args, rank, world, local_rank):
    """--case ep120b: BASELINE config 5, the gpt-oss-120b MoE stack (36
    layers, H=I=2880, 128 experts, top-4, SwiGLU clamp 7, MXFP4 experts)
    with 8192 bf16 tokens per step, expert-parallel over the torchrun ranks:
    each rank holds 128/N experts of every layer and routes 8192/N of the
    tokens; rows travel to their expert's rank and back with NCCL
    all-to-alls. value = 8192 tokens / step time (max over ranks); total
    work fixed as N grows (strong scaling)."""
    import datetime

    import torch

    import kadan_b200 as kb
    from kadan_b200 import expert_parallel as ep

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1 or args.exchange == "peer":
        import socket

        import torch.distributed as dist

        if world == 1:  # the peer buffers are set up over a (one-rank) process group
            with socket.socket() as sk:
                sk.bind(("127.0.0.1", 0))
                os.environ.setdefault("MASTER_PORT", str(sk.getsockname()[1]))
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("RANK", "0")
            os.environ.setdefault("WORLD_SIZE", "1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    E, H, I, K, T = 128, 2880, 2880, 4, 8192
    layers = args.layers or 36
    tokens = T // world
    first, end = ep.expert_range(E, world, rank)
    el = end - first
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    stack = []
    for _ in range(layers):
        gu_w = torch.randint(0, 256, (el, 2 * I, H // 2), dtype=torch.uint8, device=device, generator=gen)
        gu_s = torch.randint(118, 127, (el, 2 * I, H // 32), dtype=torch.uint8, device=device, generator=gen)
        dn_w = torch.randint(0, 256, (el, H, I // 2), dtype=torch.uint8, device=device, generator=gen)
        dn_s = torch.randint(118, 127, (el, H, I // 32), dtype=torch.uint8, device=device, generator=gen)
        w = kb.moe_weights(gu_w, gu_s, dn_w, dn_s, hidden=H, inter=I, experts=el, top_k=K)
        stack.append((ep.ExpertParallelMoE(w, E, world, rank, exchange=args.exchange, max_tokens=tokens,
                                           device=device), (gu_w, gu_s, dn_w, dn_s)))
    tgen = torch.Generator(device=device).manual_seed(7 + rank)
    x = torch.randn(tokens, H, device=device, generator=tgen).to(torch.bfloat16)
    logits = [torch.randn(tokens, E, device=device, generator=tgen) for _ in range(layers)]
    out = torch.empty(tokens, H, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)

    def step():
        for (layer, _), lg in zip(stack, logits):
            layer.forward(x, lg, out=out, status=status)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    steps = max(1, min(args.steps, 10))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    watchdog = kb.take_device_error()
    if dist:
        m = torch.tensor([ms], device=device)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
        for layer, _ in stack:
            layer.close()
        dist.barrier()
        dist.destroy_process_group()
    clock = clocks.summary()
    if rank:
        return
    flops = 2.0 * T * K * (2 * I * H + H * I) * layers
    tflops = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": METRIC, "case": "ep120b", "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong",
        "dtype": "mxfp4 weights, fp16 tensor-core operands, fp32 accumulation",
        "data": "synthetic (MXFP4 codes uniform, E8M0 118..126, bf16 N(0,1) tokens, N(0,1) logits)",
        "config": {"workload": f"BASELINE config 5: gpt-oss-120b MoE, {layers} layers, E=128, top-4, "
                               f"{T} tokens per step", "parallelism": f"ep{world}",
                   "tokens_per_rank": tokens, "experts_per_rank": el,
                   "collective": ("peer-memory exchange kernels (counts, fp16 rows out, fp32 rows back; no host sync)"
                                  if args.exchange == "peer" else
                                  "NCCL all-to-all (counts, fp16 rows out, fp32 rows back)")},
        "watchdog": watchdog,
        "tflops": round(tflops, 1), "tflops_per_gpu": round(tflops / world, 1),
        "status": int(status.item()) if world == 1 else None, "clocks": clock}), flush=True)


def run_source(args):
    """--case source-batch: the config-2 stack (--layers, default 4 layers =
    491 MB of Q4_K, more than L2) through kb200_dense_gguf_source_batch, one
    call per dependency group with host fp32 inputs and outputs. "cold": no
    bank, every chunk is read from its host source, staged, uploaded and
    multiplied; "admit": the first pass into an empty bank (streams and admits
    every chunk); "warm": every chunk is a bank hit. Host wall clock around
    the synchronous calls; GB/s counts packed weight bytes. The cold pass is
    also timed with 1, 8 and 16 source-read lanes (default 4). --source
    python reads rows through Python callbacks over host arrays; --source gguf
    writes the stack to a GGUF file in a temporary directory and reads it
    with the library's own packed-row source (kb200_gguf_rows_source)."""
    import numpy as np
    import torch

    import kadan_b200 as kb
    from kadan_b200 import synth
    from kadan_b200.weight_bank import SourceJob, WeightBank, WeightIdentity, dense_gguf_source_batch

    dev = torch.device("cuda:0")
    n_layers = args.layers or 4
    host_in = {n: torch.randn(1, k).half().float().numpy() for n, k in (("x", HIDDEN), ("attn", HIDDEN),
                                                                        ("h", HIDDEN), ("g", FFN))}
    inputs = ["x", "attn", "h", "g"]
    mats, total = [], 0
    for layer in range(n_layers):
        for gi, g in enumerate(GROUPS):
            group = []
            for name, out, in_ in g:
                w = synth.device_gguf(kb.Q4_K, out, in_, layer * 16 + gi * 4 + len(group), dev).cpu().numpy()
                total += w.nbytes
                group.append((f"blk.{layer}.{name}.weight", out, in_, w))
            mats.append((gi, group))
    ckpt = tmpdir = None
    if args.source == "gguf":
        # The stack as one GGUF file on local disk, read by the library itself.
        from kadan_b200 import gguf_write
        from kadan_b200.gguf_file import GgufCheckpoint

        tmpdir = Path(tempfile.mkdtemp(prefix="kb200_ckpt_"))
        gguf_write.write_arrays(tmpdir / "stack.gguf", [("general.architecture", gguf_write.STRING, "llama")],
                                [(n, [in_, out], 12, w) for _, group in mats for n, out, in_, w in group])
        ckpt = GgufCheckpoint(tmpdir)
    calls = []
    for gi, group in mats:
        jobs = []
        for n, out, in_, w in group:
            if ckpt is not None:
                ident, read = ckpt.identity(n), ckpt.rows(n)
            else:
                ident = WeightIdentity(device=1, inode=1000 + len(calls), payload_begin=len(jobs),
                                       payload_end=len(jobs) + 1)
                read = (lambda first, nb, w=w, rb=w.shape[1]: w[first:first + nb // rb])
            jobs.append(SourceJob(ident, read, host_in[inputs[gi]], np.empty((1, out), dtype=np.float32), in_, out,
                                  kb.Q4_K))
        calls.append(jobs)
    ctx = kb.Context(0)
    bank = WeightBank.cuda(0, 2 * total)

    def step(b):
        for jobs in calls:
            for j in jobs:
                j.reads.clear()
            dense_gguf_source_batch(ctx, b, jobs)

    def timed(b, steps):
        t0 = time.perf_counter()
        for _ in range(steps):
            step(b)
        return (time.perf_counter() - t0) / steps

    steps = max(1, min(args.steps, 10))
    cold_by_lanes = {}
    for lanes in (1, 8, 16, 4):  # the default, 4, last: admit and warm run with it
        ctx.set_read_lanes(lanes)
        step(None)
        cold_by_lanes[lanes] = timed(None, steps)
    cold = cold_by_lanes[4]
    admit = timed(bank, 1)
    reads_after_admit = sum(len(j.reads) for jobs in calls for j in jobs)
    warm = timed(bank, steps)
    warm_reads = sum(len(j.reads) for jobs in calls for j in jobs)
    line = {"case": "source-batch", "source": args.source, "layers": n_layers, "calls_per_step": len(calls),
            "weight_bytes_per_step": total, "bank_entries": bank.entries(),
            "cold": {"ms_per_step": round(cold * 1e3, 3), "gbps": round(total / cold / 1e9, 2), "read_lanes": 4,
                     "gbps_by_read_lanes": {k: round(total / v / 1e9, 2) for k, v in sorted(cold_by_lanes.items())}},
            "admit": {"ms_per_step": round(admit * 1e3, 3), "gbps": round(total / admit / 1e9, 2),
                      "source_reads": reads_after_admit},
            "warm": {"ms_per_step": round(warm * 1e3, 3), "gbps": round(total / warm / 1e9, 2),
                     "source_reads": warm_reads},
            "timing": "host wall clock around synchronous calls"}
    bank.close()
    ctx.close()
    if ckpt is not None:
        ckpt.close()
        shutil.rmtree(tmpdir, ignore_errors=True)
    print(json.dumps(line), flush=True)


def h3_reference_object(args, torch, kb, layers, acts, outs) -> dict:
    """The reference worker's own device GEMV (IW/src/cuda/h3_compute.cu,
    built from the reference sources for sm_100a into oracle/_ref/libh3_ref.so
    by the oracle recipe) over the config-2 decode stack: per dependency
    group, its job table copied and one launch per encoding on the legacy
    stream, as dense_gguf_batch launches resident chunks. Device time per
    step (CUDA events), the headline's bytes; also the largest relative
    difference between its [gate, up] outputs of the last layer and this
    library's."""
    path = ROOT / "oracle" / "_ref" / "libh3_ref.so"
    try:
        L = ctypes.CDLL(str(path))
    except OSError as e:
        return {"unavailable": f"{path.name}: {e}"}
    vp, sz, u32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint
    L.h3ref_last_error.restype = ctypes.c_char_p
    L.h3ref_job_bytes.restype = sz
    L.h3ref_matvec_batch.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(sz),
                                     ctypes.POINTER(u32), ctypes.POINTER(u32), ctypes.POINTER(u32),
                                     ctypes.POINTER(ctypes.c_int), sz, vp]
    device = acts["x"].device
    inputs = ["x", "attn", "h", "g"]
    calls = []
    for mats in layers:
        for gi, g in enumerate(GROUPS):
            n = len(g)
            calls.append(((vp * n)(*[mats[name].data_ptr() for name, _, _ in g]),
                          (vp * n)(*[acts[inputs[gi]].data_ptr()] * n),
                          (vp * n)(*[outs[name].data_ptr() for name, _, _ in g]),
                          (sz * n)(*[weight_bytes(o, i) // o for _, o, i in g]),
                          (u32 * n)(*[i for _, _, i in g]), (u32 * n)(*[o for _, o, _ in g]), (u32 * n)(*[1] * n),
                          (ctypes.c_int * n)(*[kb.Q4_K] * n), n))
    table = torch.empty(int(L.h3ref_job_bytes()) * 8, dtype=torch.uint8, device=device)

    def step():
        for c in calls:
            if L.h3ref_matvec_batch(*c, table.data_ptr()):
                raise RuntimeError(L.h3ref_last_error().decode())

    # Parity of the baseline with this library on the last layer's [gate, up]
    # (the outputs a step leaves behind).
    step()
    torch.cuda.synchronize()
    theirs = {n: outs[n].clone() for n in ("gate", "up")}
    jobs = [kb.gemv_job(kb.Q4_K, layers[-1][n], acts["h"], outs[n], in_=HIDDEN, columns=FFN, rows=1)
            for n in ("gate", "up")]
    kb.gguf_gemv_batch(jobs, torch.cuda.default_stream(device))
    torch.cuda.synchronize()
    diff = max(float((outs[n] - theirs[n]).abs().max() / max(float(theirs[n].abs().max()), 1.0))
               for n in ("gate", "up"))
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 20))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    wbytes, abytes = step_bytes()
    return {"ms_per_step": round(ms, 3), "gbps": round((wbytes + abytes) / (ms * 1e-3) / 1e9, 1), "steps": steps,
            "max_rel_diff_vs_ours": diff,
            "what": "reference device GEMV (gguf_matvec_batch_kernel built for sm_100a, job table copied per group, "
                    "legacy stream) over the config-2 decode stack"}


def run_h3_reference(args):
    """--case h3-reference: h3_reference_object on its own line."""
    import torch

    import kadan_b200 as kb

    device = torch.device("cuda:0")
    layers, acts, outs = build_stack(torch, kb, device)
    print(json.dumps({"case": "h3-reference", **h3_reference_object(args, torch, kb, layers, acts, outs)}), flush=True)


def moe_graph_ms(torch, kb, keep, x, logits, dims, layers: int = 8, reps: int = 50) -> float:
    """Device ms per layer of the MoE layer replayed from one CUDA graph of
    `layers` consecutive calls, each over its own copy of the experts (the
    copies together far exceed L2, so every call streams its routed experts
    from HBM, as consecutive layers of a model do)."""
    E, H, I, K = dims
    copies = [keep] + [tuple(t.clone() for t in keep) for _ in range(layers - 1)]
    ws_list = [kb.moe_weights(*c, hidden=H, inter=I, experts=E, top_k=K) for c in copies]
    out = torch.empty(x.shape[0], H, device=x.device)
    ws = torch.empty(kb.moe_workspace_bytes(ws_list[0], x.shape[0]), dtype=torch.uint8, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    stream = torch.cuda.Stream(x.device)

    def run():
        for w in ws_list:
            kb.moe_forward(w, x, logits, out=out, workspace=ws, status=status, stream=stream)

    graph = graph_of(torch, stream, run)
    ms = time_graph(torch, stream, graph, reps, warm=3) / layers
    del graph
    if int(status.item()):
        raise RuntimeError(f"MoE status {int(status.item())} in the graph replays")
    return ms


def moe_object(args, torch, kb, device, pk) -> dict:
    """The config-3 MoE layer (gpt-oss-20b: H=2880, 32 experts, top-4, I=2880,
    SwiGLU clamp 7) through kb200_moe_forward at T=4096 (tensor bound: TFLOP/s
    against the measured sustained dense bf16 rate, the fp16 operands' rate)
    and T=1 (HBM bound: the four selected experts' MXFP4 bytes per layer
    against the measured copy bandwidth); outputs of sampled tokens against
    the unrounded oracle (1e-3); the reference's host path as cpu_baseline."""
    import numpy as np

    from oracle.pyoracle import Oracle

    E, H, I, K = 32, 2880, 2880, 4
    orc = Oracle()
    res = {"workload": "BASELINE config 3: gpt-oss-20b MoE layer, H=2880, E=32, top-4, I=2880, SwiGLU clamp 7"}
    for T in (4096, 1):
        w, keep, x, logits, wbytes = moe_layer_inputs(torch, kb, device, T)
        out = torch.empty(T, H, device=device)
        ws = torch.empty(kb.moe_workspace_bytes(w, T), dtype=torch.uint8, device=device)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        stream = torch.cuda.current_stream()
        for _ in range(max(3, args.warmup)):
            kb.moe_forward(w, x, logits, out=out, workspace=ws, status=status)
        torch.cuda.synchronize()
        steps = max(20, args.steps)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(device.index or 0) as clocks:
            a.record(stream)
            for _ in range(steps):
                kb.moe_forward(w, x, logits, out=out, workspace=ws, status=status)
            b.record(stream)
            torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        timing = "CUDA events around eager calls (host time per call included)"
        eager_ms = ms
        if T == 1:
            # At one token an eager call is bound by the host (the Python
            # call and the launches); the device time comes from graph
            # replays over distinct expert copies.
            try:
                ms = moe_graph_ms(torch, kb, keep, x, logits, (E, H, I, K))
                timing = ("device time per layer: one CUDA graph of 8 consecutive layer calls, each over its own "
                          "copy of the experts (3.4 GB in all, so every call streams its routed experts from HBM)")
            except RuntimeError as exc:
                timing += f" (graph replay unavailable: {exc})"
        flops = 2.0 * T * K * (2 * I * H + H * I)
        entry = {"tokens": T, "ms_per_layer": round(ms, 4), "tokens_per_s": round(T / (ms * 1e-3), 1),
                 "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "status": int(status.item()),
                 "timing": timing, "eager_ms_per_layer": round(eager_ms, 4), "clocks": clocks.summary()}
        if T >= 512:
            tf = flops / (ms * 1e-3) / 1e12
            entry["roofline"] = {"bound": "tensor", "kernel": "moe_gemm_kernel (tcgen05 kind::f16)",
                                 "achieved": round(tf, 1), "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                                 "frac": round(tf / pk["bf16_tflops_sustained"], 4),
                                 "peak_source": f"{pk['source']} bf16_tflops_sustained (whole layer timed)",
                                 "frac_of_nominal_mxf8f6f4_4500": round(tf / 4500.0, 4)}
        else:
            touched = K * (wbytes // E)
            gbps = touched / (ms * 1e-3) / 1e9
            entry["roofline"] = {"bound": "hbm", "kernel": "whole layer (route + grouped MXFP4 GEMV + combine)",
                                 "achieved": round(gbps, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                 "frac": round(gbps / pk["hbm_gbs"], 4), "algorithmic_bytes": touched,
                                 "peak_source": f"{pk['source']} hbm_gbs"}
        # Parity on sampled tokens against the unrounded oracle (fp32
        # intermediate, as the reference's MoeLayer keeps it).
        pick = np.unique(np.linspace(0, T - 1, min(T, 6)).astype(np.int64))
        host = [t.cpu().numpy() for t in keep]
        xs = x.float().cpu().numpy()[pick]
        ls = logits.cpu().numpy()[pick]
        want = orc.moe_forward(xs, ls, *host, hidden=H, inter=I, experts=E, top_k=K, round_act=0)
        err = rel_err(out.cpu().numpy()[pick], want)
        entry["parity"] = {"ok": err <= 1e-3, "max_rel_err": err, "tokens_checked": int(len(pick)),
                           "what": "unrounded oracle (routing, exact MXFP4 decode, fp64 dots, fp32 SwiGLU)"}
        res[f"T{T}"] = entry
        if T == 4096 and not args.no_cpu_baseline:
            res["cpu_baseline"] = moe_cpu_baseline(keep, x, logits, T, min_seconds=min(args.cpu_seconds, 5.0))
        del w, keep, x, logits, out, ws
        torch.cuda.empty_cache()
    big = res["T4096"]
    res.update({"value": big["tokens_per_s"], "unit": "tokens/s", "roofline": big["roofline"],
                "parity_ok": all(res[k]["parity"]["ok"] for k in ("T4096", "T1"))})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="profiling case instead of the headline workload")
    ap.add_argument("--tokens", type=int, default=0,
                    help="tokens per step (default: 1 for the headline and tp70b, 4096 for --case moe / prefill)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="host seconds for the default case's CPU baseline (the MoE layer uses at most 5)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="headline only: no config2 / moe / h3_reference / cpu_baseline objects")
    ap.add_argument("--collective", choices=["fused", "peer", "nccl"], default="fused",
                    help="all-reduce of --case tp70b at N > 1: GEMV+exchange fused, peer kernel after the GEMV, NCCL")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="nccl",
                    help="token exchange of --case ep120b")
    ap.add_argument("--layers", type=int, default=0, help="layers for --case tp70b / ep120b (default 80 / 36)")
    ap.add_argument("--source", choices=["python", "gguf"], default="python",
                    help="packed-row source for --case source-batch")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.case in ("moe", "prefill") and not args.tokens:
        args.tokens = 4096
    if args.case == "moe":
        run_moe(args)
    elif args.case == "prefill":
        run_prefill(args)
    elif args.case == "tp70b":
        run_tp(args, rank, world, local_rank)
    elif args.case == "ep120b":
        run_ep(args, rank, world, local_rank)
    elif args.case == "source-batch":
        run_source(args)
    elif args.case == "h3-reference":
        run_h3_reference(args)
    elif args.case == "attention":
        run_attention(args)
    elif args.case:
        run_case(args)
    elif args.impl == "reference":
        if args.steps > 200:
            args.steps = 20
        run_reference(args, rank, world)
    else:
        run_default(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
