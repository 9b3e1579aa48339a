"""Differential fuzz of the checkpoint readers: seeded random mutations
(bit flips, byte overwrites, truncations, insertions, deletions) of valid GGUF
and safetensors files, each opened by the native reader and by the
reference's own reader (oracle/_ref). Both must accept the same files and
reject the others with the same message. No GPU."""
from __future__ import annotations

import random

from test_gguf_file import KVS, TENSORS
from test_shard import mxfp4_tensors, write_shard

CASES = 300


def mutate(rng, m: bytearray, head: int) -> bytearray:
    kind = rng.choice(["flip", "byte", "trunc", "insert", "delete"])
    p = rng.randrange(min(len(m), head))
    if kind == "flip":
        m[p] ^= 1 << rng.randrange(8)
    elif kind == "byte":
        m[p] = rng.randrange(256)
    elif kind == "trunc":
        m = m[:rng.randrange(len(m))]
    elif kind == "insert":
        m[p:p] = bytes(rng.randrange(256) for _ in range(rng.randrange(1, 9)))
    else:
        del m[p:p + rng.randrange(1, 9)]
    return m


def ours(open_fn):
    from kadan_b200 import KadanError

    try:
        open_fn().close()
        return "accepted"
    except KadanError as e:
        text = str(e)
        return text.split(": ", 1)[1] if ": " in text else text


def test_gguf_reader_agrees_with_reference(ref, tmp_path):
    from kadan_b200 import gguf_write as gw
    from kadan_b200.gguf_file import GgufCheckpoint

    base, _ = gw.build(KVS, TENSORS, alignment=64)
    rng = random.Random(2024)
    outcomes = set()
    for i in range(CASES):
        d = tmp_path / f"g{i}"
        d.mkdir()
        (d / "m.gguf").write_bytes(bytes(mutate(rng, bytearray(base), 1200)))
        want = ref.gguf_open(d)
        if not isinstance(want, str):
            ref.gguf_close(want)
            want = "accepted"
        assert ours(lambda: GgufCheckpoint(d)) == want, (i, want)
        outcomes.add(want)
    assert len(outcomes) >= 10  # the mutations reach many distinct checks


def test_shard_reader_agrees_with_reference(ref, tmp_path):
    from kadan_b200.shard import Shard

    seed = tmp_path / "seed"
    seed.mkdir()
    tensors, _, _ = mxfp4_tensors("model.layers.0.mlp.experts.gate_up_proj", 2, 4, 2, seed=1)
    write_shard(seed / "s.safetensors", tensors + [("b", "BF16", (3, 2), b"\x01" * 12)], metadata={"format": "pt"})
    base = (seed / "s.safetensors").read_bytes()
    rng = random.Random(2025)
    outcomes = set()
    for i in range(CASES):
        d = tmp_path / f"s{i}"
        d.mkdir()
        (d / "s.safetensors").write_bytes(bytes(mutate(rng, bytearray(base), 400)))
        want = ref.shard_open(d, "s.safetensors")
        if not isinstance(want, str):
            ref.shard_close(want)
            want = "accepted"
        assert ours(lambda: Shard(d, "s.safetensors")) == want, (i, want)
        outcomes.add(want)
    assert len(outcomes) >= 8
