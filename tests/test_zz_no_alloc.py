"""kb200_moe_forward_noalloc: the MoE layer for callers that cannot allocate
device memory per call (workers whose device memory is fully admitted to a
budget ledger before use, and callers that must not let cudaMalloc/cudaFree
synchronise the device). It must give the same result as
kb200_moe_forward with a caller workspace, call after call, while sharing one
fixed 16 MiB device array. This file is collected last on purpose.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def build_layer(kb, cuda, E, H, I, K, seed):
    import torch

    from kadan_b200 import synth

    gu_w, gu_s = synth.mxfp4(E * 2 * I, H, seed=seed)
    dn_w, dn_s = synth.mxfp4(E * H, I, seed=seed + 1)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (gu_w, gu_s, dn_w, dn_s)]
    return kb.moe_weights(*dev, hidden=H, inter=I, experts=E, top_k=K), dev


def call_inputs(cuda, T, H, E, seed):
    import torch

    from kadan_b200 import synth

    x = torch.from_numpy(synth.activations(T * H, seed=seed, dtype="bf16").reshape(T, H)).to(cuda).to(torch.bfloat16)
    logits = torch.from_numpy(synth.activations(T * E, seed=seed + 1, dtype="f32").reshape(T, E)).to(cuda)
    return x, logits


@pytest.mark.parametrize("E,H,I,K,T", [(8, 256, 128, 2, 37), (32, 2880, 2880, 4, 16)])
def test_noalloc_matches_workspace_entry_point_twice(kb, cuda, E, H, I, K, T):
    import torch

    w, keep = build_layer(kb, cuda, E, H, I, K, seed=E)
    assert kb.moe_workspace_bytes(w, T) <= kb.STATIC_MOE_SCRATCH_BYTES
    for call in range(2):
        x, logits = call_inputs(cuda, T, H, E, seed=100 * call + T)
        want = kb.moe_forward(w, x, logits)
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        got = kb.moe_forward_noalloc(w, x, logits, status=status)
        torch.cuda.synchronize()
        assert rel_err(got.cpu().numpy(), want.cpu().numpy()) <= TOL
        assert status.item() == 0


def test_noalloc_rejects_more_than_the_fixed_scratch(kb, cuda):
    import torch

    E, H, I, K = 32, 2880, 2880, 4
    w, keep = build_layer(kb, cuda, E, H, I, K, seed=1)
    T = 1
    while kb.moe_workspace_bytes(w, T) <= kb.STATIC_MOE_SCRATCH_BYTES:
        T *= 2
    x, logits = call_inputs(cuda, T, H, E, seed=3)
    out = torch.full((T, H), -1.0, device=cuda)
    with pytest.raises(kb.KadanError) as err:
        kb.moe_forward_noalloc(w, x, logits, out=out)
    assert err.value.status == kb.NO_MEMORY
    assert "16 MiB" in str(err.value)
    torch.cuda.synchronize()
    assert bool((out == -1.0).all())
