"""The MoE layer's CPU baseline (bench.py moe_cpu_layer): the checkpoint
MXFP4 layout repacked exactly into ggml's block_mxfp4, and the layer on the
reference's host path (routing semantics of MoeLayer::forward, CpuMatvec
experts from oracle/_ref with Q8_0 activations) within 2e-2 of the oracle
layer. No GPU."""
from __future__ import annotations

import numpy as np

from conftest import rel_err


def test_mxfp4_repack_is_exact(oracle):
    import bench
    from kadan_b200 import synth

    rows, cols = 12, 256
    w, s = synth.mxfp4(rows, cols, seed=3)
    g = bench.mxfp4_to_ggml(w, s, rows, cols)
    assert g.shape == (rows, cols // 32 * 17)
    got = oracle.mxfp4_gguf_decode(g).reshape(rows, cols)
    want = oracle.mxfp4_decode_rows(w, s, rows, cols)
    # Equal values; only the sign of zero differs (ggml's integer code table
    # decodes code 8 to +0, the checkpoint decoder to -0).
    assert np.array_equal(got, want)
    differ = got.view(np.uint32) != want.view(np.uint32)
    assert np.all(want[differ] == 0)


def test_reference_path_layer_matches_oracle(ref, oracle):
    import os

    import bench
    from kadan_b200 import synth

    E, H, I, K, T = 8, 256, 128, 2, 9
    gu_w, gu_s = synth.mxfp4(E * 2 * I, H, seed=5)
    dn_w, dn_s = synth.mxfp4(E * H, I, seed=6)
    x = synth.activations(T * H, seed=7, dtype="bf16").reshape(T, H)
    logits = synth.activations(T * E, seed=8, dtype="f32").reshape(T, E)
    got = bench.moe_cpu_layer(ref, oracle, x, logits, bench.mxfp4_to_ggml(gu_w, gu_s, E * 2 * I, H),
                              bench.mxfp4_to_ggml(dn_w, dn_s, E * H, I), hidden=H, inter=I, experts=E, top_k=K,
                              threads=min(4, os.cpu_count() or 1))
    want = oracle.moe_forward(x, logits, gu_w, gu_s, dn_w, dn_s, hidden=H, inter=I, experts=E, top_k=K, round_act=0)
    assert rel_err(got, want) <= 2e-2
