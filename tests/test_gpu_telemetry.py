"""Per-kernel telemetry on a B200: launches issued inside a phase are counted
under their stable ids and timed with device events read back without
waiting; launches captured into a CUDA graph are counted but not timed; the
counted launches are the ones the work needs (one GEMV launch per encoding of
a batch, the MoE layer's route/sort/gather/GEMM/GEMM/combine)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_gemv_and_moe_launches_are_counted_and_timed(kb, cuda):
    import torch

    from kadan_b200 import synth

    in_, out = 4096, 512
    w4 = torch.from_numpy(synth.gguf(kb.Q4_K, out, in_, seed=1)).to(cuda)
    w6 = torch.from_numpy(synth.gguf(kb.Q6_K, out, in_, seed=2)).to(cuda)
    x = torch.from_numpy(synth.activations(in_, seed=3).reshape(1, in_)).to(cuda)
    E, H, I, K, T = 8, 256, 128, 2, 512
    gu_w, gu_s = synth.mxfp4(E * 2 * I, H, seed=5)
    dn_w, dn_s = synth.mxfp4(E * H, I, seed=6)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (gu_w, gu_s, dn_w, dn_s)]
    mw = kb.moe_weights(*dev, hidden=H, inter=I, experts=E, top_k=K)
    xm = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    lg = torch.randn(T, E, device=cuda)
    torch.cuda.synchronize()

    with kb.Phase(shared_batch_size=2) as ph:
        for _ in range(3):
            kb.gguf_gemv(kb.Q4_K, w4, x, in_=in_, columns=out)
            kb.gguf_gemv(kb.Q6_K, w6, x, in_=in_, columns=out)
        kb.moe_forward(mw, xm, lg)
        torch.cuda.synchronize()
        snap = ph.snapshot()
    ks = snap["kernels"]
    assert ks["gemv_q4k_mma_kernel"]["calls"] == 3
    assert ks["gemv_q6k_pair_kernel"]["calls"] == 3
    assert ks["pair_quant_kernel"]["calls"] == 3  # the Q6_K launch's activations, quantised once
    for name in ("moe_route_kernel", "moe_sort_kernel", "moe_gather_kernel", "moe_combine_kernel"):
        assert ks[name]["calls"] == 1, name
    assert ks["moe_gemm_kernel"]["calls"] == 2  # gate/up, then down
    for name, k in ks.items():
        assert k["measured"] == k["calls"], name
        assert k["gpu_seconds"] > 0.0, name
        assert k["host_seconds"] > 0.0, name
    assert snap["dropped"] == 0 and snap["unavailable"] == 0
    assert snap["shared_batch_size"] == 2 and snap["observed"]
    ph.close()


def test_graph_capture_counts_without_timing(kb, cuda):
    import torch

    from kadan_b200 import synth

    in_, out = 4096, 256
    w = torch.from_numpy(synth.gguf(kb.Q4_K, out, in_, seed=7)).to(cuda)
    x = torch.from_numpy(synth.activations(in_, seed=8).reshape(1, in_)).to(cuda)
    y = torch.empty(1, out, device=cuda)
    job = kb.gemv_job(kb.Q4_K, w, x, y, in_=in_, columns=out, rows=1)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        kb.gguf_gemv_batch([job], stream=s)  # first use outside capture sets the stream up
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with kb.Phase() as ph:
            kb.gguf_gemv_batch([job], stream=s)  # eager: counted and timed
            with torch.cuda.graph(g, stream=s):
                kb.gguf_gemv_batch([job], stream=s)  # captured: counted only
            g.replay()
            s.synchronize()
            snap = ph.snapshot()
    k = snap["kernels"]["gemv_q4k_mma_kernel"]
    assert k["calls"] == 2 and k["measured"] == 1
    assert snap["unavailable"] == 0 and snap["dropped"] == 0
    del g
    ph.close()
