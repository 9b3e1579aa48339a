"""GPU parity of the MXFP4 MoE layer against the pinned oracle.

The device keeps the activation fed to the down projection in fp16. At the
gpt-oss-20b layer shape the layer is held to 1e-3
against the unrounded oracle, which keeps that activation in fp32 as the
reference's MoeLayer::forward does (IW/src/models/text/qwen_layers.cpp:460-476):
the fp16 rounding moves those outputs by ~6e-5 of their largest magnitude.
At toy shapes (outputs below 1, where the tolerance's denominator is 1 and
rounding is relatively larger) the unrounded check is 2e-2 and the tight one
is against the oracle with the same fp16 rounding. Tolerances use
max|y - ref| / max(max|ref|, 1) (IW/tests/gguf_text.cpp:247-250).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def layer(kb, cuda, *, E, H, I, K, seed=0, interleaved=True, activation=0, bias=False):
    import torch

    from kadan_b200 import synth

    gu_w, gu_s = synth.mxfp4(E * 2 * I, H, seed=seed)
    dn_w, dn_s = synth.mxfp4(E * H, I, seed=seed + 1)
    rng = np.random.default_rng(seed)
    gu_b = (rng.standard_normal(E * 2 * I) * 0.1).astype(np.float32) if bias else None
    dn_b = (rng.standard_normal(E * H) * 0.1).astype(np.float32) if bias else None
    dev = {k: (torch.from_numpy(np.ascontiguousarray(v)).to(cuda) if v is not None else None)
           for k, v in dict(gu_w=gu_w, gu_s=gu_s, dn_w=dn_w, dn_s=dn_s, gu_b=gu_b, dn_b=dn_b).items()}
    w = kb.moe_weights(dev["gu_w"], dev["gu_s"], dev["dn_w"], dev["dn_s"], hidden=H, inter=I, experts=E, top_k=K,
                       gu_bias=dev["gu_b"], dn_bias=dev["dn_b"], activation=activation, interleaved=interleaved)
    host = dict(gu_w=gu_w, gu_s=gu_s, dn_w=dn_w, dn_s=dn_s, gu_b=gu_b, dn_b=dn_b)
    return w, dev, host


def inputs(cuda, T, H, E, seed):
    import torch

    from kadan_b200 import synth

    x = synth.activations(T * H, seed=seed, dtype="bf16").reshape(T, H)
    logits = synth.activations(T * E, seed=seed + 1, dtype="f32").reshape(T, E)
    xb = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    assert torch.equal(xb.float().cpu(), torch.from_numpy(x))
    return x, logits, xb, torch.from_numpy(logits).to(cuda)


def test_route_matches_oracle(kb, oracle, cuda):
    import torch

    from kadan_b200 import synth

    for T, E, K in ((257, 32, 4), (64, 128, 4), (33, 8, 8), (5, 256, 2)):
        logits = synth.activations(T * E, seed=T, dtype="f32").reshape(T, E)
        c, w = kb.moe_route(torch.from_numpy(logits).to(cuda), K)
        torch.cuda.synchronize()
        oc, ow = oracle.moe_route(logits, K)
        assert np.array_equal(c.cpu().numpy(), oc)
        np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("T", [1, 5, 64, 300])
@pytest.mark.parametrize("interleaved,activation,bias", [(True, 0, False), (False, 0, True), (True, 1, True)])
def test_moe_small_shapes(kb, oracle, cuda, T, interleaved, activation, bias):
    import torch

    E, H, I, K = 8, 256, 128, 2
    w, dev, host = layer(kb, cuda, E=E, H=H, I=I, K=K, seed=T, interleaved=interleaved, activation=activation,
                         bias=bias)
    x, logits, xb, ld = inputs(cuda, T, H, E, seed=T + 7)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = kb.moe_forward(w, xb, ld, status=status)
    torch.cuda.synchronize()
    args = dict(hidden=H, inter=I, experts=E, top_k=K, gu_bias=host["gu_b"], dn_bias=host["dn_b"],
                activation=activation, interleaved=int(interleaved))
    ref16 = oracle.moe_forward(x, logits, host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"], round_act=2, **args)
    ref = oracle.moe_forward(x, logits, host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"], round_act=0, **args)
    got = out.cpu().numpy()
    assert rel_err(got, ref16) <= 1e-3
    assert rel_err(got, ref) <= 2e-2
    assert status.item() == 0


def test_moe_config3_shape_small_batch(kb, oracle, cuda):
    """gpt-oss-20b layer shape (H=2880, 32 experts, top-4, I=2880) at T=4."""
    import torch

    E, H, I, K, T = 32, 2880, 2880, 4, 4
    w, dev, host = layer(kb, cuda, E=E, H=H, I=I, K=K, seed=3)
    x, logits, xb, ld = inputs(cuda, T, H, E, seed=11)
    out = kb.moe_forward(w, xb, ld)
    torch.cuda.synchronize()
    ref16 = oracle.moe_forward(x, logits, host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"], hidden=H, inter=I,
                               experts=E, top_k=K, round_act=2)
    assert rel_err(out.cpu().numpy(), ref16) <= 1e-3


@pytest.fixture(scope="module")
def config3_layer(kb, cuda):
    E, H, I, K = 32, 2880, 2880, 4
    return layer(kb, cuda, E=E, H=H, I=I, K=K, seed=21)


@pytest.mark.parametrize("T", [1, 64, 512, 4096])
def test_moe_config3_vs_unrounded_oracle(kb, oracle, cuda, config3_layer, T):
    """BASELINE config 3 (H=2880, 32 experts, top-4, I=2880) at each of its
    token counts, against the unrounded oracle (fp32 SwiGLU output, float64
    dots) at 1e-3 on sampled tokens: every token's output depends only on
    its own row and logits, so a subset checks the full-size launch."""
    import torch

    E, H, I, K = 32, 2880, 2880, 4
    w, dev, host = config3_layer
    x, logits, xb, ld = inputs(cuda, T, H, E, seed=100 + T)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = kb.moe_forward(w, xb, ld, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    pick = np.unique(np.linspace(0, T - 1, min(T, 8)).astype(np.int64))
    want = oracle.moe_forward(x[pick], logits[pick], host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"], hidden=H,
                              inter=I, experts=E, top_k=K, round_act=0)
    assert rel_err(out.cpu().numpy()[pick], want) <= 1e-3


def decode_mxfp4_torch(blocks, scales, rows, cols):
    """Exact MXFP4 decode on the GPU (test reference): e2m1(code) * 2^(E-127)."""
    import torch

    lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=torch.float32,
                       device=blocks.device)
    b = blocks.reshape(rows, cols // 2).long()
    codes = torch.stack([b & 15, b >> 4], dim=-1).reshape(rows, cols)
    scale = torch.pow(2.0, scales.reshape(rows, cols // 32).float() - 127.0)
    return lut[codes] * scale.repeat_interleave(32, dim=1)


def test_moe_config3_full_batch_vs_torch_fp32(kb, oracle, cuda):
    """Config 3 at T=4096 tokens, every token: against a float64 torch
    evaluation of the same layer from exactly decoded weights (oracle
    routing, unrounded SwiGLU output)."""
    import torch

    E, H, I, K, T = 32, 2880, 2880, 4, 4096
    w, dev, host = layer(kb, cuda, E=E, H=H, I=I, K=K, seed=5)
    x, logits, xb, ld = inputs(cuda, T, H, E, seed=13)
    out = kb.moe_forward(w, xb, ld)
    chosen, weight = oracle.moe_route(logits, K)
    xt = torch.from_numpy(x).to(cuda)
    ref = torch.zeros(T, H, dtype=torch.float64, device=cuda)
    for e in range(E):
        rows = np.nonzero(chosen == e)
        if len(rows[0]) == 0:
            continue
        tok = torch.from_numpy(rows[0]).to(cuda)
        wt = torch.from_numpy(weight[rows]).to(cuda).double()
        gu = decode_mxfp4_torch(dev["gu_w"].view(E, -1)[e], dev["gu_s"].view(E, -1)[e], 2 * I, H)
        dn = decode_mxfp4_torch(dev["dn_w"].view(E, -1)[e], dev["dn_s"].view(E, -1)[e], H, I)
        h = xt[tok].double() @ gu.double().T
        g, u = h[:, 0::2].clamp(max=7.0), h[:, 1::2].clamp(-7.0, 7.0)
        a = g * torch.sigmoid(1.702 * g) * (u + 1)
        y = a @ dn.double().T
        ref.index_add_(0, tok, wt[:, None] * y)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-3


@pytest.mark.parametrize("T,E,H,I,K,interleaved,bias", [(3, 8, 256, 128, 2, True, True), (4, 32, 2880, 2880, 4, False, False),
                                                       (37, 16, 512, 192, 4, False, True)])
def test_moe_gemv_and_gemm_paths_agree(kb, oracle, cuda, monkeypatch, T, E, H, I, K, interleaved, bias):
    """The decode-size grouped GEMV and the tcgen05 grouped GEMM compute the
    same layer: both within 1e-3 of the oracle with fp16 activation rounding,
    and within 1e-3 of each other."""
    import torch

    w, dev, host = layer(kb, cuda, E=E, H=H, I=I, K=K, seed=T + E, interleaved=interleaved, bias=bias)
    x, logits, xb, ld = inputs(cuda, T, H, E, seed=T + 3)
    outs = {}
    for path in ("gemv", "gemm"):
        monkeypatch.setenv("KB200_MOE_PATH", path)
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        outs[path] = kb.moe_forward(w, xb, ld, status=status)
        torch.cuda.synchronize()
        assert status.item() == 0
    args = dict(hidden=H, inter=I, experts=E, top_k=K, gu_bias=host["gu_b"], dn_bias=host["dn_b"], activation=0,
                interleaved=int(interleaved))
    ref16 = oracle.moe_forward(x, logits, host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"], round_act=2, **args)
    for path in ("gemv", "gemm"):
        assert rel_err(outs[path].cpu().numpy(), ref16) <= 1e-3, path
    assert rel_err(outs["gemv"].cpu().numpy(), outs["gemm"].cpu().numpy()) <= 1e-3


def test_moe_layer_from_safetensors_shard(kb, oracle, cuda, tmp_path):
    """A gpt-oss MoE layer written as safetensors (MXFP4 experts, BF16 biases
    and router), loaded by kadan_b200.shard.load_moe_layer, runs through
    kb200_moe_forward within the layer tolerances."""
    import torch

    from kadan_b200 import shard as sh
    from kadan_b200 import synth
    from test_shard import gpt_oss_layer_tensors, write_shard

    E, H, I, K, T = 8, 256, 128, 2, 64
    prefix = "model.layers.0.mlp"
    tensors, _ = gpt_oss_layer_tensors(prefix, E, H, I, seed=9)
    write_shard(tmp_path / "model.safetensors", tensors)
    layer = sh.load_moe_layer(sh.Shard(tmp_path, "model.safetensors"), prefix)

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)

    gu_w, gu_s, dn_w, dn_s = map(dev, (layer.gate_up_blocks, layer.gate_up_scales, layer.down_blocks,
                                       layer.down_scales))
    gu_b, dn_b = dev(layer.gate_up_bias), dev(layer.down_bias)
    w = kb.moe_weights(gu_w, gu_s, dn_w, dn_s, hidden=H, inter=I, experts=E, top_k=K, gu_bias=gu_b, dn_bias=dn_b,
                       activation=kb.MOE_SILU, interleaved=True)
    x = synth.activations(T * H, seed=3, dtype="bf16").reshape(T, H)
    logits = (x @ layer.router_weight.T + layer.router_bias).astype(np.float32)
    xb = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = kb.moe_forward(w, xb, dev(logits), status=status)
    torch.cuda.synchronize()
    args = dict(hidden=H, inter=I, experts=E, top_k=K, gu_bias=layer.gate_up_bias, dn_bias=layer.down_bias,
                activation=kb.MOE_SILU, interleaved=1)
    ref16 = oracle.moe_forward(x, logits, layer.gate_up_blocks, layer.gate_up_scales, layer.down_blocks,
                               layer.down_scales, round_act=2, **args)
    assert rel_err(out.cpu().numpy(), ref16) <= 1e-3
    assert status.item() == 0


def test_moe_host_span_call(kb, oracle, cuda, config3_layer):
    """kb200_moe_forward_host: fp32 host rows through the layer (config 3, T =
    64) within 1e-3 of the unrounded oracle on sampled tokens, result
    certified finite; calls outside the contract or with scales the fp16
    operands cannot hold are unsupported and leave the output untouched;
    non-finite inputs are refused before any device work."""
    import torch

    from kadan_b200 import synth

    E, H, I, K, T = 32, 2880, 2880, 4, 64
    w, dev, host = config3_layer
    x = synth.activations(T * H, seed=71, dtype="f32").reshape(T, H)
    logits = synth.activations(T * E, seed=72, dtype="f32").reshape(T, E)
    ctx = kb.Context(0)
    try:
        out, result = kb.moe_forward_host(ctx, w, x, logits)
        assert result == kb.RESULT_FINITE
        pick = np.array([0, 9, 31, 63])
        want = oracle.moe_forward(x[pick], logits[pick], host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"],
                                  hidden=H, inter=I, experts=E, top_k=K, round_act=0)
        assert rel_err(out[pick], want) <= 1e-3
        # A scale byte outside 104..140: the caller's path must take the layer.
        bad_s = dev["gu_s"].clone()
        bad_s.view(-1)[5] = 200
        wb = kb.moe_weights(dev["gu_w"], bad_s, dev["dn_w"], dev["dn_s"], hidden=H, inter=I, experts=E, top_k=K)
        sentinel = np.full((T, H), np.nan, dtype=np.float32)
        routed_to_0 = bool((oracle.moe_route(logits, K)[0] == 0).any())
        if routed_to_0:
            with pytest.raises(kb.Unsupported):
                kb.moe_forward_host(ctx, wb, x, logits, out=sentinel)
            assert np.isnan(sentinel).all()
        with pytest.raises(kb.Unsupported):
            kb.moe_forward_host(ctx, w, x[:0], logits[:0])
        nan_x = x.copy()
        nan_x[3, 7] = np.nan
        with pytest.raises(kb.KadanError) as err:
            kb.moe_forward_host(ctx, w, nan_x, logits)
        assert err.value.status == kb.NONFINITE_INPUT
        torch.cuda.synchronize()
    finally:
        ctx.close()


def test_shared_expert_composition(kb, oracle, cuda):
    """The reference MoE layer with its sigmoid-gated shared expert
    (qwen_layers.cpp:383-396, :477-490): the shared FFN's Q8_0 gate/up
    projections on the GEMV, silu(gate) * up on the device, its down
    projection, the routed layer, then the gated add; against the oracle
    composed the same way (double dots for the projections, the unrounded
    routed layer). Outputs are fp32: 1e-3."""
    import torch

    from kadan_b200 import synth

    E, H, I, K, T, SF = 8, 256, 128, 2, 24, 512
    w, dev, host = layer(kb, cuda, E=E, H=H, I=I, K=K, seed=11, activation=1, interleaved=False)
    x, logits, xb, ld = inputs(cuda, T, H, E, seed=12)
    g_w = synth.gguf(kb.Q8_0, SF, H, seed=13)
    u_w = synth.gguf(kb.Q8_0, SF, H, seed=14)
    d_w = synth.gguf(kb.Q8_0, H, SF, seed=15)
    sg = (np.random.default_rng(16).standard_normal(H) * 0.05).astype(np.float32)
    xf = torch.from_numpy(x).to(cuda)
    gd = kb.gguf_gemv(kb.Q8_0, torch.from_numpy(g_w).to(cuda), xf, in_=H, columns=SF)
    ud = kb.gguf_gemv(kb.Q8_0, torch.from_numpy(u_w).to(cuda), xf, in_=H, columns=SF)
    sd = kb.silu_mul(gd, ud)
    dd = kb.gguf_gemv(kb.Q8_0, torch.from_numpy(d_w).to(cuda), sd, in_=SF, columns=H)
    y = kb.moe_forward(w, xb, ld)
    kb.moe_add_shared(xf, torch.from_numpy(sg).to(cuda), dd, y)
    torch.cuda.synchronize()

    g = oracle.gemv_f64(kb.Q8_0, g_w, x, H, SF)
    u = oracle.gemv_f64(kb.Q8_0, u_w, x, H, SF)
    s = oracle.silu_mul(g, u).reshape(T, SF)
    d = oracle.gemv_f64(kb.Q8_0, d_w, s, SF, H)
    routed = oracle.moe_forward(x, logits, host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"], hidden=H, inter=I,
                                experts=E, top_k=K, activation=1, interleaved=0, round_act=0)
    want = oracle.moe_add_shared(x, sg, d, routed, hidden=H)
    assert rel_err(y.cpu().numpy(), want) <= 1e-3
    # silu_mul alone is elementwise float arithmetic.
    assert rel_err(sd.cpu().numpy(), oracle.silu_mul(gd.cpu().numpy(), ud.cpu().numpy())) <= 1e-6


@pytest.mark.parametrize("T,E,H,I,K,interleaved,activation,bias", [
    (1, 8, 256, 128, 2, True, 0, False), (5, 8, 256, 128, 2, False, 0, True), (8, 8, 256, 128, 2, True, 1, True),
    (1, 32, 2880, 2880, 4, True, 0, False), (8, 32, 2880, 2880, 4, True, 0, False), (3, 64, 512, 256, 8, False, 1, False)])
def test_moe_decode_kernel_matches_staged_path(kb, oracle, cuda, monkeypatch, T, E, H, I, K, interleaved, activation,
                                               bias):
    """The fused decode kernel (one cooperative launch: routing in every CTA,
    gate/up, a grid barrier, down, a grid barrier, the combine; taken by
    default up to 2 tokens and, with KB200_MOE_DECODE=1, up to 8) runs the
    staged path's per-item arithmetic in the same order, so its outputs equal
    the staged path's (route, sort, gather, grouped GEMVs, combine) to the
    last bit, and both stay within the oracle's tolerance."""
    import torch

    w, dev, host = layer(kb, cuda, E=E, H=H, I=I, K=K, seed=T + E + K, interleaved=interleaved,
                         activation=activation, bias=bias)
    x, logits, xb, ld = inputs(cuda, T, H, E, seed=T + 11)
    outs = {}
    for name, flag in (("fused", "1"), ("staged", "0")):
        monkeypatch.setenv("KB200_MOE_DECODE", flag)
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        with kb.Phase() as ph:
            outs[name] = kb.moe_forward(w, xb, ld, status=status)
            torch.cuda.synchronize()
            ks = ph.snapshot()["kernels"]
        ph.close()
        assert status.item() == 0
        assert ("moe_decode_kernel" in ks) == (name == "fused"), ks.keys()
    assert torch.equal(outs["fused"], outs["staged"])
    args = dict(hidden=H, inter=I, experts=E, top_k=K, gu_bias=host["gu_b"], dn_bias=host["dn_b"],
                activation=activation, interleaved=int(interleaved))
    ref16 = oracle.moe_forward(x, logits, host["gu_w"], host["gu_s"], host["dn_w"], host["dn_s"], round_act=2, **args)
    assert rel_err(outs["fused"].cpu().numpy(), ref16) <= 1e-3
