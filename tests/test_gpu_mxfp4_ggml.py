"""GGUF MXFP4 (ggml type 39) on the device: kb200_mxfp4_ggml_dequant against
ggml's own dequantize_row_mxfp4 (the reference's vendored ggml, compiled into
oracle/_ref), bit for bit, over every scale byte; kb200_mxfp4_from_ggml into
the MoE layer's expert layout, checked by the oracle's decode of that layout;
and a gpt-oss-style MoE layer built from separate GGUF gate and up expert
tensors, equal bit for bit to the same layer from checkpoint-layout rows."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def ggml_blocks(n, seed, scales=None):
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(n, 17), dtype=np.uint8)
    if scales is not None:
        b[:, 0] = scales
    return b


def test_dequant_matches_ggml_bit_for_bit(kb, ref, cuda):
    import torch

    n = 256 * 24
    blocks = ggml_blocks(n, 1, scales=np.arange(n) % 256)  # every E8M0 byte, 0 and 255 included
    out = torch.empty(n * 32, dtype=torch.float32, device=cuda)
    kb.mxfp4_ggml_dequant(torch.from_numpy(blocks).to(cuda), n, out)
    torch.cuda.synchronize()
    want = ref.to_float(39, blocks.reshape(-1), n * 32)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_conversion_to_expert_layout(kb, ref, oracle, cuda):
    """Converted rows decode (checkpoint rules, the oracle) to ggml's values
    bit for bit, written into a row window of a larger destination."""
    import torch

    experts, rows, cols, dst_rows, first = 3, 10, 96, 16, 4
    nblk = cols // 32
    blocks = ggml_blocks(experts * rows * nblk, 2)
    blocks[:, 0] = np.random.default_rng(3).integers(100, 150, size=len(blocks))
    codes = torch.full((experts, dst_rows, cols // 2), 0xAB, dtype=torch.uint8, device=cuda)
    scales = torch.full((experts, dst_rows, nblk), 0xCD, dtype=torch.uint8, device=cuda)
    kb.mxfp4_from_ggml(torch.from_numpy(blocks).to(cuda), experts, rows, cols, codes, scales, dst_rows, first)
    torch.cuda.synchronize()
    c, s = codes.cpu().numpy(), scales.cpu().numpy()
    want = ref.to_float(39, blocks.reshape(-1), blocks.shape[0] * 32).reshape(experts, rows, cols)
    for x in range(experts):
        got = oracle.mxfp4_decode_rows(c[x], s[x], dst_rows, cols)[first:first + rows]
        assert np.array_equal(got.view(np.uint32), want[x].view(np.uint32))
    untouched = np.r_[0:first, first + rows:dst_rows]
    assert np.all(c[:, untouched] == 0xAB) and np.all(s[:, untouched] == 0xCD)


def test_moe_layer_from_gguf_gate_and_up(kb, cuda):
    """The MoE layer over experts converted from GGUF ffn_gate_exps /
    ffn_up_exps / ffn_down_exps (separate gate and up: interleaved = 0) equals
    the layer over the same values written directly in the checkpoint layout."""
    import torch

    from kadan_b200 import synth

    E, H, I, K, T = 8, 256, 128, 2, 40
    rng = np.random.default_rng(5)

    def gguf_tensor(rows, cols, seed):
        b = ggml_blocks(E * rows * (cols // 32), seed)
        b[:, 0] = rng.integers(118, 127, size=len(b))
        return b

    gate, up, down = gguf_tensor(I, H, 6), gguf_tensor(I, H, 7), gguf_tensor(H, I, 8)

    def to_layout(parts, rows_total, cols):
        codes = torch.empty(E, rows_total, cols // 2, dtype=torch.uint8, device=cuda)
        scales = torch.empty(E, rows_total, cols // 32, dtype=torch.uint8, device=cuda)
        first = 0
        for blocks, rows in parts:
            kb.mxfp4_from_ggml(torch.from_numpy(blocks).to(cuda), E, rows, cols, codes, scales, rows_total, first)
            first += rows
        return codes, scales

    gu_c, gu_s = to_layout([(gate, I), (up, I)], 2 * I, H)
    dn_c, dn_s = to_layout([(down, H)], H, I)

    # The same values, repacked on the host into the checkpoint layout.
    def host_layout(blocks, rows, cols):
        q = blocks[:, 1:].astype(np.uint16)
        vals = np.concatenate([q & 15, q >> 4], axis=1)  # ggml order: low nibbles, then high
        vals[vals == 8] = 0
        packed = (vals[:, 0::2] | (vals[:, 1::2] << 4)).astype(np.uint8)
        return packed.reshape(E, rows, cols // 2), blocks[:, 0].reshape(E, rows, cols // 32)

    g_c, g_s = host_layout(gate, I, H)
    u_c, u_s = host_layout(up, I, H)
    d_c, d_s = host_layout(down, H, I)
    assert np.array_equal(gu_c.cpu().numpy(), np.concatenate([g_c, u_c], axis=1))
    assert np.array_equal(gu_s.cpu().numpy(), np.concatenate([g_s, u_s], axis=1))
    assert np.array_equal(dn_c.cpu().numpy(), d_c) and np.array_equal(dn_s.cpu().numpy(), d_s)

    x = synth.activations(T * H, seed=9, dtype="bf16").reshape(T, H)
    logits = synth.activations(T * E, seed=10, dtype="f32").reshape(T, E)
    xb = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    ld = torch.from_numpy(logits).to(cuda)
    w = kb.moe_weights(gu_c, gu_s, dn_c, dn_s, hidden=H, inter=I, experts=E, top_k=K, interleaved=False)
    host = [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in
            (np.concatenate([g_c, u_c], axis=1), np.concatenate([g_s, u_s], axis=1), d_c, d_s)]
    w2 = kb.moe_weights(*host, hidden=H, inter=I, experts=E, top_k=K, interleaved=False)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    a = kb.moe_forward(w, xb, ld, status=status)
    b = kb.moe_forward(w2, xb, ld)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and status.item() == 0
