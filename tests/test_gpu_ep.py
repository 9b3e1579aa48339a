"""Expert-parallel MoE on the GPU: one rank (always) and two NCCL ranks (when
the machine shows two GPUs).

Each rank routes its own tokens; the layer's output for them must match the
oracle's single-host layer (1e-3 against the fp16-activation oracle, 2e-2
against the unrounded one; max|y - ref| / max(max|ref|, 1)). One rank runs
the same stages as kb200_moe_forward and must equal it bit for bit.
Small token counts take the grouped-GEMV expert path, larger ones the GEMM.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
E, H, I, K = 8, 256, 128, 2


def run_rank(rank: int, world: int, port: int, tokens: int, exchange: str = "nccl") -> dict:
    import torch

    import kadan_b200 as kb
    from kadan_b200 import expert_parallel as ep
    from kadan_b200 import synth
    from oracle.pyoracle import Oracle

    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1 or exchange == "peer":
        import datetime

        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                                timeout=datetime.timedelta(seconds=60))
    try:
        gu_w, gu_s = synth.mxfp4(E * 2 * I, H, seed=3)
        dn_w, dn_s = synth.mxfp4(E * H, I, seed=4)
        full = [torch.from_numpy(np.ascontiguousarray(a)).to(device) for a in (gu_w, gu_s, dn_w, dn_s)]
        shaped = [full[0].view(E, 2 * I, H // 2), full[1].view(E, 2 * I, H // 32),
                  full[2].view(E, H, I // 2), full[3].view(E, H, I // 32)]
        local, keep = ep.local_weights(*shaped, hidden=H, inter=I, experts=E, top_k=K, world=world, rank=rank)
        layer = ep.ExpertParallelMoE(local, E, world, rank, exchange=exchange, max_tokens=tokens + 3 * (world - 1),
                                     device=device)
        # Rank r's tokens: its own seed, a different count per rank.
        t = tokens + 3 * rank
        x = synth.activations(t * H, seed=50 + rank, dtype="bf16").reshape(t, H)
        logits = synth.activations(t * E, seed=70 + rank, dtype="f32").reshape(t, E)
        xb = torch.from_numpy(x).to(device).to(torch.bfloat16)
        ld = torch.from_numpy(logits).to(device)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        out = layer.forward(xb, ld, status=status)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        orc = Oracle()
        args = dict(hidden=H, inter=I, experts=E, top_k=K, gu_bias=None, dn_bias=None, activation=0, interleaved=1)
        ref16 = orc.moe_forward(x, logits, gu_w, gu_s, dn_w, dn_s, round_act=2, **args)
        ref = orc.moe_forward(x, logits, gu_w, gu_s, dn_w, dn_s, round_act=0, **args)
        res = {"tight": rel_err(got, ref16), "loose": rel_err(got, ref), "status": int(status.item())}
        if exchange == "peer":
            # A second layer call on the same buffers (the next epoch and bank).
            again = layer.forward(xb, ld).cpu().numpy()
            res["repeat"] = bool(np.array_equal(again.view(np.uint32), got.view(np.uint32)))
            res["watchdog"] = kb.take_device_error()
            layer.close()
        if world == 1:
            wfull = kb.moe_weights(*full, hidden=H, inter=I, experts=E, top_k=K)
            single = kb.moe_forward(wfull, xb, ld).cpu().numpy()
            res["bitwise"] = bool(np.array_equal(single.view(np.uint32), got.view(np.uint32)))
        return res
    finally:
        if dist:
            dist.destroy_process_group()


def _child(rank, world, port, tokens, exchange, results):
    results[rank] = run_rank(rank, world, port, tokens, exchange)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _check(res):
    assert res["tight"] <= 1e-3 and res["loose"] <= 2e-2 and res["status"] == 0, res
    if "repeat" in res:
        assert res["repeat"] and res["watchdog"] == 0, res


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("tokens", [5, 300])
def test_ep_one_rank(cuda, tokens, exchange):
    res = run_rank(0, 1, _port(), tokens, exchange)
    _check(res)
    assert res["bitwise"], res


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("tokens", [5, 300])
def test_ep_two_ranks(cuda, tokens, exchange):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("two GPUs needed")
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _port()
        procs = [ctx.Process(target=_child, args=(r, 2, port, tokens, exchange, results)) for r in range(2)]
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
            _check(results[r])
