"""Pin the CPU oracle (oracle/oracle.c) to the reference before trusting it.

Each case follows a reference test or fixture (IW = services/hikari/inference_worker):
  * literal codes        IW/tests/gguf_quantization.cpp:36-79
  * all fp16 patterns    IW/tests/gguf_quantization.cpp:81-91
  * 2048 random blocks   IW/tests/gguf_quantization.cpp:100-165 (golden digest)
  * CpuMatvec case       IW/tests/gguf_text.cpp:200-254 (golden fixture)
  * MXFP4 known answers  IW/tests/quantization.cpp:250-351
"""
from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN, rel_err

Q3_K, Q4_K, Q8_0, Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS, IQ2_S, IQ3_S, BF16 = 0, 1, 2, 3, 4, 5, 6, 7, 8, 9


def bits(v):
    return np.asarray(v, dtype=np.float32).view(np.uint32)


def same(actual, expected):
    actual = np.asarray(actual, dtype=np.float32)
    expected = np.asarray(expected, dtype=np.float32)
    nan = np.isnan(expected)
    assert np.array_equal(np.isnan(actual), nan)
    assert np.array_equal(bits(actual)[~nan], bits(expected)[~nan])


def test_literal_codes(oracle):
    block = np.zeros(210, dtype=np.uint8)
    block[0:2] = [0x00, 0x38]  # 0.5
    for i in range(32):
        block[2 + i] = i if i < 16 else 256 - i
    got = oracle.decode(Q8_0, block[:34], 32)
    same(got, [0.5 * (i if i < 16 else -i) for i in range(32)])

    block[:] = 0
    block[0:32] = 0x55
    block[32:96] = 0xE4
    block[96:104] = 0x11
    block[104:108] = 0xAA
    block[108:110] = [0x00, 0xC0]  # -2
    want = []
    for i in range(256):
        code = (i // 32) % 4 - (4 if (i // 32) % 2 else 0)
        want.append(-2.0 * code)
    same(oracle.decode(Q3_K, block[:110], 256), want)

    block[:] = 0
    block[0:2] = [0x00, 0x40]  # 2
    block[2:4] = [0x00, 0x38]  # 0.5
    block[4:16] = [1, 2, 3, 4, 8, 7, 6, 5, 0x45, 0x36, 0x27, 0x18]
    block[16:144] = 0xC3
    want = []
    for i in range(256):
        g = i // 32
        want.append(np.float32(2.0 * (g + 1) * (12.0 if g % 2 else 3.0) - 0.5 * (8 - g)))
    same(oracle.decode(Q4_K, block[:144], 256), want)


def test_all_half_patterns(oracle, ref):
    for b in range(65536):
        a, e = oracle.half(b), ref.L.ref_fp16_to_fp32(b)
        if np.isnan(e):
            assert np.isnan(a)
        else:
            assert bits(a) == bits(e), hex(b)


def _golden_blocks():
    return json.loads((GOLDEN / "gguf_blocks.json").read_text())["encodings"]


GRID_CODED = {"iq3_xxs": IQ3_XXS, "iq2_s": IQ2_S, "iq3_s": IQ3_S}


@pytest.mark.parametrize("name", ["q8_0", "q4_k", "q6_k", "q3_k", "iq4_nl", "iq4_xs", "bf16", *GRID_CODED])
def test_reference_blocks_digest(oracle, name, request):
    """The grid-coded formats decode through code grids that the caller
    supplies; here the reference's own, as the worker would pass them."""
    from golden.make_golden import canonical_digest, reference_blocks

    if name in GRID_CODED:
        oracle.set_iq_grids(request.getfixturevalue("ref").iq_grids())
    spec = _golden_blocks()[name]
    blocks = reference_blocks(spec["encoding"], spec["trials"])
    assert hashlib.sha256(blocks.tobytes()).hexdigest() == spec["sha256_blocks"]
    values = oracle.block_values(spec["encoding"])
    got = oracle.decode(spec["encoding"], blocks, blocks.shape[0] * values)
    assert canonical_digest(got) == spec["sha256_expected"]
    assert int(np.isnan(got).sum()) == spec["nan_count"]


@pytest.mark.parametrize("enc", [Q8_0, Q4_K, Q6_K, Q3_K, IQ4_NL, IQ4_XS, IQ3_XXS, IQ2_S, IQ3_S])
def test_oracle_equals_reference_decode_and_runs(oracle, ref, enc):
    from golden.make_golden import reference_blocks

    oracle.set_iq_grids(ref.iq_grids())
    blocks = reference_blocks(enc, 256)
    n = blocks.shape[0] * oracle.block_values(enc)
    mine = oracle.decode(enc, blocks, n)
    same(mine, ref.decode(enc, blocks, n))
    same(mine, ref.decode_runs(enc, blocks, n))


@pytest.mark.parametrize("name,enc", [("q8_0", Q8_0), ("q4_k", Q4_K), ("q6_k", Q6_K)])
def test_gemv_oracle_golden(oracle, name, enc):
    g = np.load(GOLDEN / "cpu_matvec.npz")
    x, packed = g["input"], g[f"{name}_packed"]
    y = oracle.gemv_f64(enc, packed, x, 512, 37)
    assert rel_err(y, g[f"{name}_f64"]) < 1e-12
    # The fixture's own CpuMatvec output meets the reference test's bound.
    assert rel_err(g[f"{name}_cpu_matvec"], g[f"{name}_f64"]) <= 2e-2


def test_config1_golden(oracle):
    from kadan_b200 import synth

    g = np.load(GOLDEN / "config1_q8_0.npz")
    w = synth.q8_0(4096, 4096, seed=0)
    assert hashlib.sha256(w.tobytes()).digest() == g["weights_sha256"].tobytes()
    x = synth.activations(4096, seed=0, dtype="f32")
    assert np.array_equal(x, g["x"])
    y = oracle.gemv_f64(Q8_0, w, x, 4096, 4096)[0]
    assert rel_err(y, g["y_f64"]) < 1e-12


def test_mxfp4_golden(oracle):
    g = np.load(GOLDEN / "mxfp4.npz")
    rows, cols = g["weights"].shape[0], g["weights"].shape[1] * 2
    dec = oracle.mxfp4_decode_rows(g["weights"], g["scales"], rows, cols)
    same(dec, g["decoded"])
    y = (dec.astype(np.float64) @ g["x"].astype(np.float64)).astype(np.float32)
    same(y, g["matvec"])


def test_mxfp4_known_answers(oracle):
    # IW/tests/quantization.cpp:250-291
    packed = np.full(64, 0xA2, dtype=np.uint8)
    packed[0] = 0x71
    scales = np.array([127, 128, 126, 129], dtype=np.uint8)
    want = np.empty(128, dtype=np.float32)
    for i in range(128):
        f = 1.0 if i < 32 else 2.0 if i < 64 else 0.5 if i < 96 else 4.0
        want[i] = -f if i % 2 else f
    want[0], want[1] = 0.5, 6.0
    same(oracle.mxfp4_decode_rows(packed, scales, 2, 64).reshape(-1), want)
    same(oracle.mxfp4_decode_rows(packed, scales, 2, 64, first=1).reshape(-1), want[64:])
    with pytest.raises(ValueError):
        oracle.mxfp4_decode_rows(packed, np.array([127, 128, 126, 255], dtype=np.uint8), 2, 64)
    # :293-317 extremes: E8M0 0 -> 2^-127, 254 -> 2^127, signed zero.
    p16 = np.full(16, 0xA2, dtype=np.uint8)
    d = oracle.mxfp4_decode_rows(p16, np.array([0], dtype=np.uint8), 1, 32)[0]
    assert d[0] == np.float32(2.0 ** -127) and d[1] == -np.float32(2.0 ** -127)
    d = oracle.mxfp4_decode_rows(p16, np.array([254], dtype=np.uint8), 1, 32)[0]
    assert d[0] == np.float32(2.0 ** 127) and d[1] == -np.float32(2.0 ** 127)
    p16[0] = 0x11
    assert oracle.mxfp4_decode_rows(p16, np.array([0], dtype=np.uint8), 1, 32)[0][0] == np.float32(2.0 ** -128)
    z = np.full(16, 0x80, dtype=np.uint8)
    for s in (0, 127, 254):
        d = oracle.mxfp4_decode_rows(z, np.array([s], dtype=np.uint8), 1, 32)[0]
        assert d[0] == 0 and not np.signbit(d[0]) and d[1] == 0 and np.signbit(d[1])
    # :319-351 caller output {2, 8}
    p32 = np.full(32, 0xA2, dtype=np.uint8)
    x = np.zeros(32, dtype=np.float32)
    x[0], x[1] = 3, 1
    dec = oracle.mxfp4_decode_rows(p32, np.array([127, 129], dtype=np.uint8), 2, 32)
    assert np.array_equal(dec @ x, np.array([2, 8], dtype=np.float32))


def test_mxfp4_gguf_blocks_equal_ggml(oracle, ref):
    rng = np.random.default_rng(3)
    blocks = rng.integers(0, 256, size=(64, 17), dtype=np.uint8)
    blocks[:, 0] = rng.integers(1, 250, size=64)
    got = oracle.mxfp4_gguf_decode(blocks)
    same(got, ref.to_float(39, blocks, 64 * 32))


def test_moe_route_semantics(oracle):
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((64, 32)).astype(np.float32)
    chosen, weight = oracle.moe_route(logits, 4)
    p = np.exp(logits - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    order = np.argsort(-p, axis=1, kind="stable")[:, :4]
    assert np.array_equal(chosen, order)
    np.testing.assert_allclose(weight.sum(1), 1.0, rtol=1e-6)
    assert np.all(np.diff(weight, axis=1) <= 0)
    # Ties go to the lower expert index.
    c, w = oracle.moe_route(np.zeros((1, 8), dtype=np.float32), 3)
    assert list(c[0]) == [0, 1, 2]
    np.testing.assert_allclose(w[0], 1.0 / 3.0, rtol=1e-6)
