"""The native safetensors shard reader (kb200_shard_*) against the reference's
own Shard (services/hikari/inference_worker/src/weights/checkpoint.cpp,
compiled into oracle/_ref): same tensor table, identities, bytes and gpt-oss
MXFP4 expert rows, and the same message for every malformed header. The
expert rows also decode, through the oracle, to the reference's
quantization::decode_rows values. No GPU."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest

WIDTH = {"U8": 1, "I8": 1, "F8_E4M3": 1, "BF16": 2, "F16": 2, "F32": 4, "U32": 4}


def header_json(entries: dict, metadata=None) -> str:
    body = {}
    if metadata is not None:
        body["__metadata__"] = metadata
    body.update(entries)
    return json.dumps(body)


def write_shard(path, tensors, *, metadata=None, header=None, pad=0, tail=b""):
    """tensors: [(name, dtype, shape, bytes)] laid out back to back. `header`
    replaces the JSON text (for malformed files)."""
    entries, payload, at = {}, b"", 0
    for name, dtype, shape, data in tensors:
        entries[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [at, at + len(data)]}
        payload += data
        at += len(data)
    text = (header if header is not None else header_json(entries, metadata)) + " " * pad
    raw = text.encode("latin-1")
    path.write_bytes(struct.pack("<Q", len(raw)) + raw + payload + tail)


def mxfp4_tensors(prefix, experts, rows, groups, seed, bad_scale=None):
    rng = np.random.default_rng(seed)
    blocks = rng.integers(0, 256, size=(experts, rows, groups, 16), dtype=np.uint8)
    scales = rng.integers(118, 127, size=(experts, rows, groups), dtype=np.uint8)
    if bad_scale is not None:
        scales[bad_scale] = 255
    return [(prefix + "_blocks", "U8", blocks.shape, blocks.tobytes()),
            (prefix + "_scales", "U8", scales.shape, scales.tobytes())], blocks, scales


@pytest.fixture(scope="module")
def sh():
    from kadan_b200 import shard

    return shard


def message(err) -> str:
    text = str(err)
    return text.split(": ", 1)[1] if ": " in text else text


def outcome(fn):
    from kadan_b200 import KadanError

    try:
        return fn()
    except KadanError as e:
        return message(e)


def test_mxfp4_shard_matches_reference(sh, ref, oracle, tmp_path):
    gu, gu_blocks, gu_scales = mxfp4_tensors("model.layers.0.mlp.experts.gate_up_proj", 4, 12, 3, seed=1)
    dn, dn_blocks, dn_scales = mxfp4_tensors("model.layers.0.mlp.experts.down_proj", 4, 6, 2, seed=2)
    other = [("model.layers.0.mlp.router.weight", "BF16", (4, 96), bytes(range(256)) * 3),
             ("model.layers.0.mlp.router.bias", "F32", (4,), struct.pack("<4f", 1, 2, 3, 4))]
    write_shard(tmp_path / "model-00001-of-00001.safetensors", gu + dn + other,
                metadata={"format": "pt", "note": "tab\\there"})
    name = "model-00001-of-00001.safetensors"
    ours = sh.Shard(tmp_path, name)
    h = ref.shard_open(tmp_path, name)
    assert not isinstance(h, str), h
    try:
        theirs = ref.shard_tensors(h)
        mine = ours.tensors()
        assert [t.name for t in mine] == list(theirs)
        for t in mine:
            dtype, rank, nbytes, shape = theirs[t.name]
            assert (sh.DTYPES.index(t.dtype), len(t.shape), t.bytes, t.shape) == (dtype, rank, nbytes, shape)
            assert tuple(vars(ours.tensor_identity(t.name)).values()) == ref.shard_identity(h, t.name)
            for off, n in ((0, t.bytes), (1, t.bytes - 1), (t.bytes, 0)):
                assert np.array_equal(ours.read_tensor(t.name, off, n), ref.shard_read_tensor(h, t.name, off, n))
            assert outcome(lambda: ours.read_tensor(t.name, 1, t.bytes)) == ref.shard_read_tensor(h, t.name, 1, t.bytes)
        budget = 1 << 20
        for prefix, blocks, scales in (("model.layers.0.mlp.experts.gate_up_proj", gu_blocks, gu_scales),
                                       ("model.layers.0.mlp.experts.down_proj", dn_blocks, dn_scales)):
            rows, groups = blocks.shape[1], blocks.shape[2]
            for expert in range(4):
                for first, count in ((0, rows), (2, rows - 3), (rows - 1, 1)):
                    w, s, cols = ours.load_mxfp4_expert_rows(prefix, expert, first, count, budget)
                    rw, rs, rrows, rcols = ref.shard_load_mxfp4_expert_rows(h, prefix, expert, first, count, budget)
                    assert (count, cols) == (rrows, rcols) == (count, groups * 32)
                    assert np.array_equal(w.reshape(-1), rw) and np.array_equal(s.reshape(-1), rs)
                    assert np.array_equal(w, blocks[expert, first:first + count].reshape(count, -1))
                    assert np.array_equal(s, scales[expert, first:first + count])
            # The loaded rows decode to the reference's own MXFP4 values.
            w, s, cols = ours.load_mxfp4_expert_rows(prefix, 1, 0, rows, budget)
            assert np.array_equal(oracle.mxfp4_decode_rows(w, s, rows, cols),
                                  ref.mxfp4_decode_rows(w, s, rows, cols))
        # Failures of the loader, in the reference's order.
        p = "model.layers.0.mlp.experts.gate_up_proj"
        for args in ((p, 4, 0, 1, budget), (p, 0, 10, 3, budget), (p, 0, 0, 0, budget), (p, 0, 0, 12, 100),
                     ("", 0, 0, 1, budget), ("model.layers.0.mlp.router", 0, 0, 1, budget),
                     ("missing", 0, 0, 1, budget), ("x" * 481, 0, 0, 1, budget)):
            want = ref.shard_load_mxfp4_expert_rows(h, *args)
            assert isinstance(want, str)
            assert outcome(lambda: ours.load_mxfp4_expert_rows(*args)) == want, args
        assert ours.check_unchanged() is None and ref.shard_check_unchanged(h) is None
    finally:
        ref.shard_close(h)


def test_invalid_block_scale_matches_reference(sh, ref, tmp_path):
    t, _, _ = mxfp4_tensors("e", 2, 4, 2, seed=3, bad_scale=(1, 2, 1))
    write_shard(tmp_path / "s.safetensors", t)
    ours = sh.Shard(tmp_path, "s.safetensors")
    h = ref.shard_open(tmp_path, "s.safetensors")
    try:
        want = ref.shard_load_mxfp4_expert_rows(h, "e", 1, 0, 4, 1 << 20)
        assert want == "invalid_block_scale"
        assert outcome(lambda: ours.load_mxfp4_expert_rows("e", 1, 0, 4, 1 << 20)) == want
        # Rows that avoid the bad scale load.
        assert ref.shard_load_mxfp4_expert_rows(h, "e", 1, 0, 2, 1 << 20)[2] == 2
        assert ours.load_mxfp4_expert_rows("e", 1, 0, 2, 1 << 20)[2] == 64
    finally:
        ref.shard_close(h)


U8_TENSOR = ("t", "U8", (4,), b"abcd")


def bad_headers():
    ok = '{"t":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'
    yield "not an object", dict(header=' {"t":1}'), [U8_TENSOR]
    yield "syntax", dict(header='{"t" {"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "trailing", dict(header=ok + "x"), [U8_TENSOR]
    yield "duplicate metadata", dict(header='{"__metadata__":{},"__metadata__":{}}'), []
    yield "metadata dup key", dict(header='{"__metadata__":{"a":"1","a":"2"}}'), []
    yield "metadata long value", dict(header='{"__metadata__":{"a":"' + "v" * 600 + '"}}'), []
    yield "empty name", dict(header='{"":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "dtype", dict(header='{"t":{"dtype":"F64","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "unknown field", dict(header='{"t":{"dtype":"U8","shape":[4],"data_offsets":[0,4],"x":1}}'), [U8_TENSOR]
    yield "duplicate field", dict(header='{"t":{"dtype":"U8","dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "missing field", dict(header='{"t":{"dtype":"U8","shape":[4]}}'), [U8_TENSOR]
    yield "byte size", dict(header='{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "rank limit", dict(header='{"t":{"dtype":"U8","shape":[1,1,1,1,1,1,1,1,4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "leading zero", dict(header='{"t":{"dtype":"U8","shape":[04],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "huge integer", dict(header='{"t":{"dtype":"U8","shape":[99999999999999999999],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "escape", dict(header='{"t\\q":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "unicode", dict(header='{"t\\u00e9":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "non ascii", dict(header='{"té":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "unterminated", dict(header='{"t'), [U8_TENSOR]
    yield "long name", dict(header='{"' + "n" * 513 + '":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]
    yield "gap", dict(header='{"t":{"dtype":"U8","shape":[4],"data_offsets":[1,5]}}', tail=b"x"), [U8_TENSOR]
    yield "coverage", dict(header=ok, tail=b"extra"), [U8_TENSOR]
    yield "duplicate tensor", dict(header='{"t":{"dtype":"U8","shape":[0],"data_offsets":[0,0]},'
                                          '"t":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}'), [U8_TENSOR]


@pytest.mark.parametrize("label,kw,tensors", list(bad_headers()), ids=[b[0] for b in bad_headers()])
def test_header_rejections_match_reference(sh, ref, tmp_path, label, kw, tensors):
    write_shard(tmp_path / "s.safetensors", tensors, **kw)
    want = ref.shard_open(tmp_path, "s.safetensors")
    assert isinstance(want, str), f"the reference accepted the {label} file"
    assert outcome(lambda: sh.Shard(tmp_path, "s.safetensors")) == want


def test_open_rules(sh, ref, tmp_path):
    write_shard(tmp_path / "s.safetensors", [U8_TENSOR])
    for name in ("", "..", "a/b", "x" * 256, "s.safetensorsé"):
        want = ref.shard_open(tmp_path, name)
        assert isinstance(want, str)
        assert outcome(lambda: sh.Shard(tmp_path, name)) == want
    (tmp_path / "tiny.safetensors").write_bytes(b"\x01\x00")
    assert outcome(lambda: sh.Shard(tmp_path, "tiny.safetensors")) == ref.shard_open(tmp_path, "tiny.safetensors")
    big = tmp_path / "big.safetensors"
    big.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    assert outcome(lambda: sh.Shard(tmp_path, "big.safetensors")) == ref.shard_open(tmp_path, "big.safetensors")
    # Header limits set by the caller.
    assert outcome(lambda: sh.Shard(tmp_path, "s.safetensors", header_bytes=8)) == "header_size"
    two = [("a", "U8", (1,), b"a"), ("b", "U8", (1,), b"b")]
    write_shard(tmp_path / "two.safetensors", two)
    assert outcome(lambda: sh.Shard(tmp_path, "two.safetensors", tensors=1)) == "tensor_limit_or_name"


def test_changed_shard(sh, ref, tmp_path):
    write_shard(tmp_path / "s.safetensors", [U8_TENSOR])
    ours = sh.Shard(tmp_path, "s.safetensors")
    h = ref.shard_open(tmp_path, "s.safetensors")
    try:
        with open(tmp_path / "s.safetensors", "ab") as f:
            f.write(b"!")
        assert outcome(ours.check_unchanged) == ref.shard_check_unchanged(h) == "checkpoint_changed"
        assert outcome(lambda: ours.read_tensor("t", 0, 4)) == ref.shard_read_tensor(h, "t", 0, 4)
    finally:
        ref.shard_close(h)


def gpt_oss_layer_tensors(prefix, E, H, I, seed):
    """A gpt-oss MoE layer as its safetensors tensors (MXFP4 experts with BF16
    biases and a BF16 router), and the arrays they hold."""
    rng = np.random.default_rng(seed)
    gu, gu_b, gu_s = mxfp4_tensors(prefix + ".experts.gate_up_proj", E, 2 * I, H // 32, seed)
    dn, dn_b, dn_s = mxfp4_tensors(prefix + ".experts.down_proj", E, H, I // 32, seed + 1)

    def bf16(shape):
        return (rng.standard_normal(shape).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)

    gu_bias, dn_bias, router_w, router_b = bf16((E, 2 * I)), bf16((E, H)), bf16((E, H)), bf16((E,))
    tensors = gu + dn + [(prefix + ".experts.gate_up_proj_bias", "BF16", gu_bias.shape, gu_bias.tobytes()),
                         (prefix + ".experts.down_proj_bias", "BF16", dn_bias.shape, dn_bias.tobytes()),
                         (prefix + ".router.weight", "BF16", router_w.shape, router_w.tobytes()),
                         (prefix + ".router.bias", "BF16", router_b.shape, router_b.tobytes())]
    widen = lambda a: (a.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    arrays = dict(gu_w=gu_b.reshape(E, 2 * I, H // 2), gu_s=gu_s, dn_w=dn_b.reshape(E, H, I // 2), dn_s=dn_s,
                  gu_bias=widen(gu_bias), dn_bias=widen(dn_bias), router_w=widen(router_w), router_b=widen(router_b))
    return tensors, arrays


def test_load_moe_layer(sh, oracle, tmp_path):
    E, H, I, K, T = 8, 256, 128, 2, 9
    prefix = "model.layers.3.mlp"
    tensors, want = gpt_oss_layer_tensors(prefix, E, H, I, seed=5)
    write_shard(tmp_path / "model-00002-of-00003.safetensors", tensors)
    shard = sh.Shard(tmp_path, "model-00002-of-00003.safetensors")
    layer = sh.load_moe_layer(shard, prefix)
    assert (layer.hidden, layer.inter, layer.first, layer.count) == (H, I, 0, E)
    for got, key in ((layer.gate_up_blocks, "gu_w"), (layer.gate_up_scales, "gu_s"), (layer.down_blocks, "dn_w"),
                     (layer.down_scales, "dn_s"), (layer.gate_up_bias, "gu_bias"), (layer.down_bias, "dn_bias"),
                     (layer.router_weight, "router_w"), (layer.router_bias, "router_b")):
        assert np.array_equal(got, want[key]), key
    # An expert-parallel slice is the matching slice of the whole layer.
    part = sh.load_moe_layer(shard, prefix, first=2, count=3)
    assert np.array_equal(part.gate_up_blocks, layer.gate_up_blocks[2:5])
    assert np.array_equal(part.down_scales, layer.down_scales[2:5])
    assert np.array_equal(part.down_bias, layer.down_bias[2:5])
    assert np.array_equal(part.router_weight, layer.router_weight)
    # The loaded layer runs through the oracle exactly as the arrays it came from.
    from kadan_b200 import synth

    x = synth.activations(T * H, seed=1, dtype="bf16").reshape(T, H)
    logits = (x @ layer.router_weight.T + layer.router_bias).astype(np.float32)
    args = dict(hidden=H, inter=I, experts=E, top_k=K, activation=1, interleaved=1)
    a = oracle.moe_forward(x, logits, layer.gate_up_blocks, layer.gate_up_scales, layer.down_blocks,
                           layer.down_scales, gu_bias=layer.gate_up_bias, dn_bias=layer.down_bias, **args)
    b = oracle.moe_forward(x, logits, want["gu_w"], want["gu_s"], want["dn_w"], want["dn_s"], gu_bias=want["gu_bias"],
                           dn_bias=want["dn_bias"], **args)
    assert np.array_equal(a, b)
