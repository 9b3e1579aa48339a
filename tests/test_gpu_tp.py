"""Tensor-parallel decode on the GPU against the oracle's full projections.

One rank (always) and two NCCL ranks (when the machine shows two GPUs): a
two-layer stack with the Llama-3-70B block structure at reduced width
(hidden 1024, 8 q / 2 kv heads of 128, ffn 3584; Q6_K attention and down,
Q4_K gate/up). Every rank checks its outputs — its column slice of q/k/v and
gate/up, the all-reduced o and down — against the fp64 product of the oracle's
decode of the full matrices, within 1e-3 (max|y - ref| / max(max|ref|, 1)),
after an eager step and after a CUDA-graph replay of the step.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-3
TOKENS = 3


def small_groups():
    from kadan_b200 import Q4_K, Q6_K
    from kadan_b200.tensor_parallel import Projection

    h, kv, ffn, head = 1024, 256, 3584, 128
    return [[Projection("q", Q6_K, h, h, "column", head), Projection("k", Q6_K, kv, h, "column", head),
             Projection("v", Q6_K, kv, h, "column", head)],
            [Projection("o", Q6_K, h, h, "row")],
            [Projection("gate", Q4_K, ffn, h, "column"), Projection("up", Q4_K, ffn, h, "column")],
            [Projection("down", Q6_K, h, ffn, "row")]]


def run_rank(rank: int, world: int, port: int, collective: str = "nccl") -> dict:
    import torch

    from kadan_b200 import synth
    from kadan_b200 import tensor_parallel as tp
    from oracle.pyoracle import Oracle

    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                                timeout=datetime.timedelta(seconds=60))
    try:
        groups = small_groups()
        orc = Oracle()
        layers, full, weights = 2, [], []
        for layer in range(layers):
            mats, local = {}, {}
            for gi, g in enumerate(groups):
                for i, p in enumerate(g):
                    mats[p.name] = synth.gguf(p.encoding, p.out, p.in_, seed=100 * layer + 10 * gi + i)
                    local[p.name] = torch.from_numpy(tp.shard_packed(p, mats[p.name], world, rank)).to(device)
            full.append(mats)
            weights.append(local)
        xs = {g[0].name: synth.activations(TOKENS * g[0].in_, seed=7 + gi, dtype="bf16").reshape(TOKENS, g[0].in_)
              for gi, g in enumerate(groups)}
        reducer = None
        if world > 1 and collective in ("peer", "fused"):
            from kadan_b200.collectives import PeerAllReduce

            reducer = PeerAllReduce(TOKENS * 1024, fused=collective == "fused")
        stack = tp.DecodeStack(groups, weights, TOKENS, world, rank, device,
                               inputs={k: torch.from_numpy(v).to(device) for k, v in xs.items()},
                               collective=reducer)
        # The stack writes each projection's output once per layer; the last
        # layer's values remain.
        want = {}
        for g in groups:
            for p in g:
                w = orc.decode(p.encoding, full[-1][p.name], p.out * p.in_).reshape(p.out, p.in_)
                y = xs[g[0].name].astype(np.float64) @ w.astype(np.float64).T
                s = tp.shard(p, world, rank)
                want[p.name] = y[:, s.out_first:s.out_first + s.out_count]
        errs = {}
        stream = torch.cuda.Stream(device)
        with torch.cuda.stream(stream):
            stack.launch(stream)
        torch.cuda.synchronize()
        for name, y in want.items():
            errs[f"eager/{name}"] = _rel(stack.outputs[name].cpu().numpy(), y)
        for t in stack.outputs.values():
            t.fill_(float("nan"))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            stack.launch(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize()
        for name, y in want.items():
            errs[f"graph/{name}"] = _rel(stack.outputs[name].cpu().numpy(), y)
        graph = None
        if reducer is not None and reducer.fused:
            # The fused GEMV + exchange and the GEMV followed by the all-reduce
            # kernel add the same values in the same order: same bits.
            fused_out = {k: v.clone() for k, v in stack.outputs.items()}
            reducer.fused = False
            with torch.cuda.stream(stream):
                stack.launch(stream)
            torch.cuda.synchronize()
            for name in ("o", "down"):
                same = torch.equal(fused_out[name].view(torch.int32), stack.outputs[name].view(torch.int32))
                errs[f"bitwise/{name}"] = 0.0 if same else float("inf")
        if reducer:
            reducer.close()
        return errs
    finally:
        if dist:
            dist.destroy_process_group()


def _rel(got, want) -> float:
    if not np.isfinite(got).all():
        return float("inf")
    return float(np.max(np.abs(got - want)) / max(1.0, float(np.max(np.abs(want)))))


def _child(rank, world, port, collective, results):
    results[rank] = run_rank(rank, world, port, collective)


def allreduce_rank(rank: int, world: int, port: int) -> dict:
    """Peer all-reduce of seeded vectors, several sizes back to back (eager
    and replayed from a CUDA graph): each result must equal the fp32 sum in
    rank order computed on the host, bit for bit."""
    import datetime

    import torch
    import torch.distributed as dist

    from kadan_b200.collectives import PeerAllReduce

    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    res = {}
    try:
        sizes = [4, 8192, 1028, 262144, 8192, 96, 300000, 8192]
        red = PeerAllReduce(max(sizes))
        stream = torch.cuda.current_stream()

        def data(n, r, salt):
            g = np.random.default_rng(1000 * salt + 17 * r + n)
            return g.standard_normal(n).astype(np.float32)

        def want(n, salt):
            acc = data(n, 0, salt)
            for r in range(1, world):
                acc = acc + data(n, r, salt)
            return acc

        for i, n in enumerate(sizes):
            t = torch.from_numpy(data(n, rank, i)).to(device)
            red(t, stream)
            res[f"eager/{i}/{n}"] = bool(np.array_equal(t.cpu().numpy().view(np.uint32), want(n, i).view(np.uint32)))
        bufs = [torch.from_numpy(data(n, rank, 50 + i)).to(device) for i, n in enumerate(sizes[:3])]
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device)
        with torch.cuda.graph(graph, stream=side):
            for b in bufs:
                red(b, side)
        for rep in range(3):
            for i, n in enumerate(sizes[:3]):
                bufs[i].copy_(torch.from_numpy(data(n, rank, 100 * rep + i)).to(device))
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            for i, n in enumerate(sizes[:3]):
                ok = np.array_equal(bufs[i].cpu().numpy().view(np.uint32), want(n, 100 * rep + i).view(np.uint32))
                res[f"graph/{rep}/{n}"] = bool(ok)
        graph = None
        red.close()
    finally:
        dist.destroy_process_group()
    return res


def _ar_child(rank, world, port, results):
    results[rank] = allreduce_rank(rank, world, port)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp_one_rank_matches_oracle(cuda):
    errs = run_rank(0, 1, 0)
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, bad


def _spawn(target, args_of, world=2):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _port()
        procs = [ctx.Process(target=target, args=args_of(r, port) + (results,)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.exitcode is None:
                p.kill()
        assert codes == [0] * world, codes
        return dict(results)


def test_peer_allreduce_two_ranks_bitwise(cuda):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("two GPUs needed")
    results = _spawn(_ar_child, lambda r, port: (r, 2, port))
    for r in range(2):
        bad = [k for k, ok in results[r].items() if not ok]
        assert not bad, (r, bad)


def test_tp_two_ranks_peer_collective_match_oracle(cuda):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("two GPUs needed")
    results = _spawn(_child, lambda r, port: (r, 2, port, "peer"))
    for r in range(2):
        bad = {k: v for k, v in results[r].items() if not v < TOL}
        assert not bad, (r, bad)


def test_tp_two_ranks_fused_gemv_allreduce_match_oracle(cuda):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("two GPUs needed")
    results = _spawn(_child, lambda r, port: (r, 2, port, "fused"))
    for r in range(2):
        bad = {k: v for k, v in results[r].items() if not v < TOL}
        assert not bad, (r, bad)
        assert "bitwise/o" in results[r] and "bitwise/down" in results[r]


def test_tp_two_ranks_match_oracle(cuda):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("two GPUs needed")
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _port()
        procs = [ctx.Process(target=_child, args=(r, 2, port, "nccl", results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.exitcode is None:
                p.kill()
        assert codes == [0, 0], codes
        for r in range(2):
            bad = {k: v for k, v in results[r].items() if not v < TOL}
            assert not bad, (r, bad)


def test_peer_allreduce_wait_ends_with_status_when_no_peer_writes(kb, cuda):
    """A bounded wait, run out on purpose without any fault: the "peer" is a
    second buffer on this GPU that nothing writes, so the words the kernel
    waits for never arrive. It must give up after its time limit, report
    watchdog bit 16 to the host, leave the data as it was, and leave the
    context usable for the next launch."""
    import ctypes

    import torch

    from kadan_b200 import collectives  # noqa: F401  (argument types)

    count = 8192
    nbytes = int(kb.lib.kb200_peer_buffer_bytes(2, count))
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        kb.check(kb.lib.kb200_device_alloc(nbytes, ctypes.byref(p)))
        bufs.append(p.value)
    try:
        assert kb.take_device_error() == 0
        data = torch.arange(count, dtype=torch.float32, device=cuda)
        peers = (ctypes.c_void_p * 2)(*bufs)
        stream = torch.cuda.current_stream()
        kb.check(kb.lib.kb200_peer_allreduce_f32(data.data_ptr(), count, peers, 2, 0, count, 0.05,
                                                 ctypes.c_void_p(stream.cuda_stream)))
        torch.cuda.synchronize()
        assert kb.take_device_error() & 16
        assert torch.equal(data, torch.arange(count, dtype=torch.float32, device=cuda))
        # The context still runs kernels.
        from kadan_b200 import synth

        w = synth.gguf(kb.Q4_K, 64, 256, seed=1)
        x = synth.activations(256, seed=2).reshape(1, 256)
        y = kb.gguf_gemv(kb.Q4_K, torch.from_numpy(w).to(cuda), torch.from_numpy(x).to(cuda), in_=256, columns=64)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
        assert kb.take_device_error() == 0
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            kb.lib.kb200_device_free(b)
