"""Benchmark of the kadan_b200 quantized-weight linear path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (decode): the Llama-3-8B-shaped Q4_K linear stack,
32 layers x {q, o: 4096x4096; k, v: 1024x4096; gate, up: 14336x4096;
down: 4096x14336}, one input row (T=1). A step is one token through the whole
stack: per layer four dependent launches ([q,k,v], [o], [gate,up], [down]),
captured once in a CUDA graph. The weights (3.93 GB) are far larger than L2,
so no flush is needed between steps.

metric value = weight+activation bytes streamed per step / device time per
step, summed over ranks (each rank runs its own replica of the stack: the path
has no exchange step at this config, so scaling is weak).

`--impl reference` times the reference's own CPU path (kadan::text::CpuMatvec
over ggml's AVX2 Q4_K dot, compiled from the reference sources into
oracle/_ref) on a bounded sample of the same stack with all host threads.
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
HIDDEN, KV, FFN, LAYERS = 4096, 1024, 14336, 32
# (name, out, in) per layer; dependency groups of one decode step.
GROUPS = [[("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN)],
          [("o", HIDDEN, HIDDEN)],
          [("gate", FFN, HIDDEN), ("up", FFN, HIDDEN)],
          [("down", HIDDEN, FFN)]]
Q4K_BLOCK, Q4K_VALUES = 144, 256
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) of one [gate, up] launch, from an ncu capture of
# that launch (the profile summary of gemv_q4k_mma_kernel holds the command).
GATE_UP_TRAFFIC = 66922496  # 66,164,224 read + 758,272 written


def weight_bytes(out: int, in_: int) -> int:
    return out * in_ // Q4K_VALUES * Q4K_BLOCK


def layer_weight_bytes() -> int:
    return sum(weight_bytes(o, i) for g in GROUPS for _, o, i in g)


def step_bytes() -> tuple[int, int]:
    """(weight bytes, activation bytes) streamed per step."""
    w = LAYERS * layer_weight_bytes()
    act = 0
    for g in GROUPS:
        act += g[0][2] * 4  # shared fp32 input of the group
        act += sum(o * 4 for _, o, _ in g)  # fp32 outputs
    return w, LAYERS * act


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


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


# --------------------------------------------------------------------- ours
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


def run_ours(args, rank, world, local_rank):
    import torch

    import kadan_b200 as kb

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    layers, acts, outs = build_stack(torch, kb, device, seed=rank)
    calls = step_jobs(kb, layers, acts, outs)
    stream = torch.cuda.Stream(device)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    gate_up_bytes = 2 * weight_bytes(FFN, HIDDEN)

    def launch_step():
        for gi, arr, n in calls:
            kb.check(kb.lib.kb200_gguf_gemv_batch(arr, n, sptr))

    # First call per kernel sets attributes/occupancy outside capture.
    with torch.cuda.stream(stream):
        launch_step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch_step()
    torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gate_up = [(gi, arr, n) for gi, arr, n in calls if gi == 2]
    gu_start, gu_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gu_reps = max(1, args.steps // 20)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):  # replays run on the capture stream
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            end.record(stream)
        # The dominant launch ([gate, up] of every layer, 66 MB each) timed on
        # its own stream with events, back to back, same clocks window.
        gu_start.record(stream)
        for _ in range(gu_reps):
            for _, arr, n in gate_up:
                kb.check(kb.lib.kb200_gguf_gemv_batch(arr, n, sptr))
        gu_end.record(stream)
        torch.cuda.synchronize()
    gate_up_ms = [gu_start.elapsed_time(gu_end) / (gu_reps * len(gate_up))]
    ms = start.elapsed_time(end) / args.steps
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    wbytes, abytes = step_bytes()
    value = world * (wbytes + abytes) / (ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    achieved = gate_up_bytes / (statistics.mean(gate_up_ms) * 1e-3) / 1e9

    # End to end through the host-span C ABI: host inputs, one upload, the
    # launches, one download and a sync per dependency group (128 per token).
    import numpy as np

    ctx = kb.Context(local_rank)
    host_in = {n: a.cpu().numpy().copy() for n, a in acts.items()}
    host_out = {n: np.empty((1, o), dtype=np.float32) for g in GROUPS for n, o, _ in g}
    inputs = ["x", "attn", "h", "g"]
    host_calls = []
    for mats in layers:
        for gi, g in enumerate(GROUPS):
            jobs = [kb.host_job(kb.Q4_K, mats[n].data_ptr(), host_in[inputs[gi]], host_out[n], in_=i, out=o,
                                validated=True) for n, o, i in g]
            host_calls.append((kb.HostJob * len(jobs))(*jobs))
    result = ctypes.c_int(0)

    def e2e_step():
        for arr in host_calls:
            kb.check(kb.lib.kb200_dense_gguf_batch(ctx.handle, arr, len(arr), None, ctypes.byref(result)))

    e2e_step()
    e2e_steps = max(3, min(args.steps // 20, 50))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if dist:
        t = torch.tensor([e2e_s], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    h2d = LAYERS * sum(g[0][2] * 4 for g in GROUPS)
    d2h = LAYERS * sum(o * 4 for g in GROUPS for _, o, _ in g)
    e2e = {"value": round(world * (wbytes + abytes) / e2e_s / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "calls_per_step": len(host_calls), "ms_per_step": round(e2e_s * 1e3, 4),
           "timing": "host wall clock around synchronous kb200_dense_gguf_batch calls"}
    ctx.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(layers, kb, budget_s=args.cpu_seconds)

    clock = clocks.summary()
    if dist:
        graph = None
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4_k weights, fp32 activations and accumulation",
        "data": "synthetic (seeded Q4_K blocks and fp16-representable N(0,1) activations on the device)",
        "config": {"workload": "BASELINE config 2 decode: Llama-3-8B Q4_K linear stack, 32 layers, T=1",
                   "weight_bytes_per_step": wbytes, "activation_bytes_per_step": abytes,
                   "l2": "inputs larger than L2 (3.93 GB of weights per step)",
                   "launch": "one CUDA graph per step, 4 dependent launches per layer",
                   "parallelism": f"replicas x{world}"},
        "hbm_frac": round(value / world / peak, 4),
        "gpu_launches": len(calls) * args.steps,
        "gpu_launches_note": "kernel launches of the timed graph replays (one per encoding per group)",
        "roofline": {"bound": "hbm", "kernel": "gemv_q4k_mma_kernel<1> ([gate, up] launch, balanced split)",
                     "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": GATE_UP_TRAFFIC,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch "
                                       "(one-pass capture, bench.py --steps 3 --warmup 3)",
                     "algorithmic_bytes_per_launch": gate_up_bytes},
        "e2e": e2e,
        "clocks": clock,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def cpu_baseline(layers, kb, budget_s: float = 15.0):
    """The reference's CpuMatvec on the same bytes: one layer's seven matrices
    copied to the host, repeated for about `budget_s` seconds on all cores."""
    from oracle.pyoracle import REF_LIB, Oracle, Reference

    import numpy as np

    threads = os.cpu_count() or 1
    mats = {n: t.cpu().numpy() for n, t in layers[0].items()}
    x = {HIDDEN: np.random.default_rng(0).standard_normal(HIDDEN).astype(np.float16).astype(np.float32),
         FFN: np.random.default_rng(1).standard_normal(FFN).astype(np.float16).astype(np.float32)}
    if REF_LIB.exists():
        ref = Reference()
        kind = "reference"

        def one_layer():
            for g in GROUPS:
                for n, o, i in g:
                    ref.cpu_matvec(12, mats[n], x[i], i, o, threads=threads)
    else:
        orc = Oracle()
        kind, threads = "port", 1

        def one_layer():
            for g in GROUPS:
                for n, o, i in g:
                    orc.gemv_f64(1, mats[n][: max(1, o // 64)], x[i], i, max(1, o // 64))

    dt, n = timed_repeats(one_layer, budget_s)
    per_layer = layer_weight_bytes() if kind == "reference" else sum(
        weight_bytes(max(1, o // 64), i) for g in GROUPS for _, o, i in g)
    out = {"value": round(per_layer / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": kind,
           "sample": f"layer 0 of the stack (7 matrices, {per_layer} weight bytes) x {n} repetitions, "
                     f"{round(dt * n, 1)} s; kadan::text::CpuMatvec 64-column units, activations quantized "
                     f"to Q8_K once per input as the reference does"}
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
    Q4_K weight bytes: the reference's CpuMatvec with one worker over layer 0
    (its production host path), and the scalar restatement (decode each
    block, fp64 dot: the oracle's gemv) over the first 512 columns of each
    of layer 0's matrices."""
    def cpu_matvec_one():
        for g in GROUPS:
            for n, o, i in g:
                ref.cpu_matvec(12, mats[n], x[i], i, o, threads=1)

    cols = 512

    def scalar():
        for g in GROUPS:
            for n, o, i in g:
                oracle.gemv_f64(1, mats[n][:cols], x[i], i, cols)

    dt1, n1 = timed_repeats(cpu_matvec_one, budget_s)
    dt2, n2 = timed_repeats(scalar, budget_s)
    scalar_bytes = sum(weight_bytes(cols, i) for g in GROUPS for _, _, i in g)
    return {"cpu_matvec_1_core_gbps": round(layer_weight_bytes() / dt1 / 1e9, 3),
            "cpu_matvec_1_core_sample": f"layer 0 x {n1}",
            "scalar_restatement_1_core_gbps": round(scalar_bytes / dt2 / 1e9, 3),
            "scalar_restatement_1_core_sample": f"first {cols} columns of each layer-0 matrix x {n2} "
                                                "(oracle Q4_K decode + fp64 dot)"}


def run_reference(args, rank, world):
    """Reference arm: the reference's CPU path on the box's host cores."""
    if rank != 0:
        return
    import numpy as np

    from kadan_b200 import synth
    from oracle.pyoracle import REF_LIB, Oracle, Reference

    threads = os.cpu_count() or 1
    rng_x = {HIDDEN: synth.activations(HIDDEN, seed=1), FFN: synth.activations(FFN, seed=2)}
    # Bounded sample: one layer's matrices (122.7 MB) drawn host-side per step.
    mats = {}
    for g in GROUPS:
        for n, o, i in g:
            mats[n] = synth.q4_k(o, i, seed=len(mats))
    if REF_LIB.exists():
        ref = Reference()
        kind = "reference"

        def sample():
            for g in GROUPS:
                for n, o, i in g:
                    ref.cpu_matvec(12, mats[n], rng_x[i], i, o, threads=threads)
        sample_bytes = layer_weight_bytes()
    else:
        orc = Oracle()
        kind, threads = "port", 1

        def sample():
            for g in GROUPS:
                for n, o, i in g:
                    orc.gemv_f64(1, mats[n][:64], rng_x[i], i, 64)
        sample_bytes = sum(weight_bytes(64, i) for g in GROUPS for _, _, i in g)
    for _ in range(args.warmup):
        sample()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sample()
    dt = (time.perf_counter() - t0) / args.steps
    value = sample_bytes / dt / 1e9
    wbytes, abytes = step_bytes()
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_k weights, Q8_K-quantized activations (reference CPU dot)",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "BASELINE config 2 decode: Llama-3-8B Q4_K linear stack, 32 layers, T=1",
                   "sample": "one layer (7 matrices) per step", "full_step_weight_bytes": wbytes},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": "one layer of the stack per step"},
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
    tokens = args.tokens if args.tokens <= 32 else 1
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


def run_h3_reference(args):
    """--case h3-reference: the reference worker's own device GEMV
    (IW/src/cuda/h3_compute.cu, built from the reference sources for sm_100a
    into oracle/_ref/libh3_ref.so by the oracle recipe) over the config-2
    decode stack: per dependency group, its job table copied and one launch per
    encoding on the legacy stream, as dense_gguf_batch launches resident
    chunks. Device time per step (CUDA events), the headline's bytes; also the
    largest relative difference between its [gate, up] outputs of the last
    layer and this library's."""
    import torch

    import kadan_b200 as kb

    path = ROOT / "oracle" / "_ref" / "libh3_ref.so"
    try:
        L = ctypes.CDLL(str(path))
    except OSError as e:
        print(json.dumps({"case": "h3-reference", "unavailable": f"{path.name}: {e}"}), flush=True)
        return
    vp, sz, u32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint
    L.h3ref_last_error.restype = ctypes.c_char_p
    L.h3ref_job_bytes.restype = sz
    L.h3ref_matvec_batch.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(sz),
                                     ctypes.POINTER(u32), ctypes.POINTER(u32), ctypes.POINTER(u32),
                                     ctypes.POINTER(ctypes.c_int), sz, vp]
    device = torch.device("cuda:0")
    layers, acts, outs = build_stack(torch, kb, device)
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
    print(json.dumps({"case": "h3-reference", "ms_per_step": round(ms, 3),
                      "gbps": round((wbytes + abytes) / (ms * 1e-3) / 1e9, 1), "steps": steps,
                      "max_rel_diff_vs_ours": diff,
                      "what": "reference device GEMV (gguf_matvec_batch_kernel, job table copied per group, legacy "
                              "stream) over the config-2 decode stack"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="profiling case instead of the headline workload")
    ap.add_argument("--tokens", type=int, default=4096, help="tokens for --case moe / prefill")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="host seconds for the default case's CPU baseline (the MoE case uses at most 5)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    elif args.case:
        run_case(args)
    elif args.impl == "reference":
        if args.steps > 200:
            args.steps = 20
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
