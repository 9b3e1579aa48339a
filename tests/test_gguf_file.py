"""The native GGUF checkpoint reader (kb200_gguf_*) against the reference's
own GgufCheckpoint (services/hikari/inference_worker/src/weights/
gguf_checkpoint.cpp, compiled into oracle/_ref): the same files give the same
tensors, identities, packed bytes and metadata, and the same malformed files
fail with the same message. No GPU."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

from kadan_b200 import gguf_write as gw
from kadan_b200.gguf_write import ARRAY, BOOL, F32, F64, I8, I32, I64, STRING, U8, U16, U32, U64

Q8_0, Q3_K, Q4_K, Q6_K, BF16, F32T = 8, 11, 12, 14, 30, 0

KVS = [
    ("general.architecture", STRING, "llama"),
    ("general.alignment", U32, 64),
    ("llama.block_count", U32, 2),
    ("llama.context_length", U64, 8192),
    ("llama.embedding_length", I32, 4096),
    ("llama.rope.freq_base", F32, 500000.0),
    ("llama.attention.layer_norm_rms_epsilon", F64, 1e-5),
    ("llama.small", U8, 7),
    ("llama.medium", U16, 300),
    ("llama.negative", I64, -3),
    ("llama.signed_byte", I8, -1),
    ("llama.use_parallel_residual", BOOL, 1),
    ("llama.rope.dimension_sections", ARRAY, (I32, [16, 24, 24, 0])),
    ("llama.big", ARRAY, (U64, [1, 2, 2**62])),
    ("llama.scales", ARRAY, (F32, [0.5, 1.5, -2.0])),
    ("tokenizer.ggml.tokens", ARRAY, (STRING, ["a", "bb", "ccc"])),
]
TENSORS = [
    ("blk.0.attn_q.weight", [512, 6], Q4_K, None),
    ("blk.0.ffn_down_exps.weight", [64, 5, 3], Q8_0, None),
    ("blk.1.attn_k.weight", [256, 3], Q6_K, None),
    ("output_norm.weight", [16], F32T, None),
    ("token_embd.weight", [8, 4], BF16, None),
    ("blk.1.attn_v.weight", [256, 2], Q3_K, None),
]


@pytest.fixture(scope="module")
def gg():
    from kadan_b200 import gguf_file

    return gguf_file


def message(err) -> str:
    """The reference's message part of a kb200 error text."""
    text = str(err)
    return text.split(": ", 1)[1] if ": " in text else text


def our_error(gg, root):
    from kadan_b200 import KadanError

    with pytest.raises(KadanError) as e:
        gg.GgufCheckpoint(root)
    return message(e.value)


def single(tmp_path, kvs=KVS, tensors=TENSORS, name="model.gguf", **kw):
    root = tmp_path / "ckpt"
    root.mkdir(parents=True, exist_ok=True)
    kw.setdefault("alignment", 64 if any(k == "general.alignment" for k, _, _ in kvs) else 32)
    payloads = gw.write(root / name, kvs, tensors, **kw)
    return root, payloads


def test_single_file_matches_reference(gg, ref, tmp_path):
    root, payloads = single(tmp_path)
    ours = gg.GgufCheckpoint(root)
    h = ref.gguf_open(root)
    assert not isinstance(h, str), h
    try:
        theirs = ref.gguf_tensors(h)
        mine = ours.tensors()
        assert [t.name for t in mine] == list(theirs) == sorted(payloads)
        for t in mine:
            shape, rank, gtype, nbytes = theirs[t.name]
            assert (t.shape, t.rank, t.ggml_type, t.bytes) == (shape, rank, gtype, nbytes)
            assert t.offset % 64 == 0
            for expert in range(t.shape[2]):
                ident = ours.identity(t.name, expert)
                assert tuple(vars(ident).values()) == ref.gguf_identity(h, t.name, expert)
            assert message_of_call(lambda: ours.identity(t.name, t.shape[2])) == ref.gguf_identity(h, t.name, t.shape[2])
            if t.rank < 2:
                continue
            rows, rb = t.shape[1], t.row_bytes
            data = np.frombuffer(payloads[t.name], dtype=np.uint8)
            for expert in range(t.shape[2]):
                for first, count in ((0, rows), (1, rows - 1), (rows - 1, 1), (rows, 0)):
                    got = ours.read_packed_rows(t.name, expert, first, count * rb)
                    want = ref.gguf_read_packed_rows(h, t.name, expert, first, count * rb)
                    base = (expert * rows + first) * rb
                    assert np.array_equal(got, want)
                    assert np.array_equal(got, data[base:base + count * rb])
        # Row ranges and names the reference rejects.
        q = "blk.0.attn_q.weight"
        rb = ours.tensor(q).row_bytes
        for args in ((q, 0, 5, 2 * rb), (q, 0, 7, 0), (q, 1, 0, rb), (q, 0, 0, rb + 1), ("output_norm.weight", 0, 0, 4),
                     ("missing", 0, 0, 0)):
            want = ref.gguf_read_packed_rows(h, *args)
            assert isinstance(want, str)
            assert message_of_call(lambda: ours.read_packed_rows(*args)) == want
        # Metadata accessors: same value or same failure for every key and accessor.
        keys = [k for k, _, _ in KVS] + ["missing.key"]
        for key in keys:
            assert ours.has(key) == ref.gguf_has(h, key)
            for name in ("integer", "number", "boolean", "string"):
                want = getattr(ref, "gguf_" + name)(h, key)
                got = call_or_message(lambda: getattr(ours, name)(key))
                if isinstance(want, float) and isinstance(got, float):
                    assert got == pytest.approx(want, rel=0, abs=0) or got == want
                else:
                    assert got == want, (key, name)
        assert ours.integers("llama.rope.dimension_sections") == [16, 24, 24, 0]
        assert ours.integers("llama.big") == [1, 2, 2**62]
        assert ours.numbers("llama.scales") == [0.5, 1.5, -2.0]
        assert message_of_call(lambda: ours.integers("llama.scales")) == "gguf_metadata_integers"
        assert message_of_call(lambda: ours.numbers("tokenizer.ggml.tokens")) == "gguf_metadata_numbers"
        assert ours.check_unchanged() is None and ref.gguf_check_unchanged(h) is None
    finally:
        ref.gguf_close(h)
        ours.close()


def call_or_message(fn):
    from kadan_b200 import KadanError

    try:
        return fn()
    except KadanError as e:
        return message(e)


def message_of_call(fn):
    got = call_or_message(fn)
    assert isinstance(got, str), got
    return got


def test_split_set_matches_reference(gg, ref, tmp_path):
    root = tmp_path / "split"
    root.mkdir()
    parts = [TENSORS[:2], TENSORS[2:5], TENSORS[5:]]
    payloads = {}
    for i, part in enumerate(parts):
        kvs = [("split.no", U16, i), ("split.count", U16, 3), ("split.tensors.count", I32, len(TENSORS))]
        if i == 0:
            kvs = KVS[:1] + kvs
        payloads.update(gw.write(root / f"m-{i + 1:05d}-of-00003.gguf", kvs, part))
    ours = gg.GgufCheckpoint(root)
    h = ref.gguf_open(root)
    assert not isinstance(h, str), h
    try:
        theirs = ref.gguf_tensors(h)
        assert [t.name for t in ours.tensors()] == list(theirs)
        for t in ours.tensors():
            assert t.file == next(i for i, p in enumerate(parts) if any(n == t.name for n, *_ in p))
            assert tuple(vars(ours.identity(t.name)).values()) == ref.gguf_identity(h, t.name, 0)
            if t.rank >= 2:
                got = ours.read_packed_rows(t.name, 0, 0, t.shape[1] * t.row_bytes)
                assert got.tobytes() == payloads[t.name][:t.shape[1] * t.row_bytes]
        assert ours.string("general.architecture") == "llama"
        assert ours.integer("split.count") == 3
    finally:
        ref.gguf_close(h)


def bad_files():
    """(label, kwargs for single(), optional file name) of files the reference rejects."""
    q = [("w", [256, 2], Q4_K, None)]
    yield "magic", dict(tensors=q, magic=b"GGUE"), None
    yield "version", dict(tensors=q, version=2), None
    yield "tensor count", dict(tensors=q, tensor_count=200001), None
    yield "key count", dict(tensors=q, kv_count=16385), None
    yield "duplicate key", dict(kvs=[("a", U8, 1), ("a", U8, 2)], tensors=q), None
    yield "alignment type", dict(kvs=[("general.alignment", U64, 32)], tensors=q), None
    yield "alignment value", dict(kvs=[("general.alignment", U32, 48)], tensors=q), None
    yield "alignment zero", dict(kvs=[("general.alignment", U32, 0)], tensors=q), None
    yield "long key", dict(kvs=[("k" * 257, U8, 1)], tensors=q), None
    yield "nul key", dict(kvs=[("a\0b", U8, 1)], tensors=q), None
    yield "empty key", dict(kvs=[("", U8, 1)], tensors=q), None
    yield "nested array", dict(kvs=[("a", ARRAY, (ARRAY, []))], tensors=q), None
    yield "long array", dict(kvs=[("a", ARRAY, (U8, [0] * 524289))], tensors=q), None
    yield "metadata type", dict(kvs=[("a", 13, 0)], tensors=[]), None
    yield "empty tensor name", dict(tensors=[("", [256, 2], Q4_K, None)]), None
    yield "duplicate tensor", dict(tensors=q + q), None
    yield "long tensor name", dict(tensors=[("t" * 64, [256, 2], Q4_K, None)]), None
    yield "rank 4", dict(tensors=[("w", [256, 2, 1, 1], Q4_K, None)]), None
    yield "zero dim", dict(tensors=[("w", [256, 0], Q4_K, None)]), None
    yield "f16 type", dict(tensors=[("w", [256, 2], 1, None)]), None
    yield "block alignment", dict(tensors=[("w", [128, 2], Q4_K, None)]), None
    yield "offset gap", dict(tensors=[("a", [32, 1], Q8_0, None), ("b", [32, 1], Q8_0, None)], offsets=[0, 128]), None
    yield "offset unaligned", dict(tensors=[("a", [32, 1], Q8_0, None)], offsets=[8]), None
    yield "truncated payload", dict(tensors=q, truncate=200), None
    yield "tiny file", dict(tensors=[], truncate=20), None
    yield "split name", dict(tensors=q), "m-00002-of-00002.gguf"
    yield "split metadata", dict(tensors=q), "m-00001-of-00001.gguf"


@pytest.mark.parametrize("label,kw,name", list(bad_files()), ids=[b[0] for b in bad_files()])
def test_rejections_match_reference(gg, ref, tmp_path, label, kw, name):
    kvs = kw.pop("kvs", [])
    tensors = kw.pop("tensors")
    root, _ = single(tmp_path, kvs=kvs, tensors=tensors, name=name or "model.gguf", **kw)
    want = ref.gguf_open(root)
    assert isinstance(want, str), f"the reference accepted the {label} file"
    assert our_error(gg, root) == want


def test_directory_rules(gg, ref, tmp_path):
    empty = tmp_path / "empty"
    empty.mkdir()
    assert our_error(gg, empty) == ref.gguf_open(empty) == "gguf_missing_files"
    # A split set with a file missing from the numbering.
    root = tmp_path / "gap"
    root.mkdir()
    for i in (1, 3):
        kvs = [("split.no", U16, i - 1), ("split.count", U16, 3), ("split.tensors.count", I32, 2)]
        gw.write(root / f"m-{i:05d}-of-00003.gguf", kvs, [(f"t{i}", [32, 1], Q8_0, None)])
    assert our_error(gg, root) == ref.gguf_open(root) == "gguf_split_name"
    # Split metadata that disagrees with the file names.
    root = tmp_path / "meta"
    root.mkdir()
    for i in (1, 2):
        kvs = [("split.no", U16, 0), ("split.count", U16, 2), ("split.tensors.count", I32, 2)]
        gw.write(root / f"m-{i:05d}-of-00002.gguf", kvs, [(f"t{i}", [32, 1], Q8_0, None)])
    assert our_error(gg, root) == ref.gguf_open(root) == "gguf_split_metadata"


def test_changed_file_and_cancel(gg, ref, tmp_path):
    from kadan_b200 import CANCELLED, KadanError

    root, _ = single(tmp_path)
    ours = gg.GgufCheckpoint(root)
    h = ref.gguf_open(root)
    try:
        path = root / "model.gguf"
        with open(path, "ab") as f:
            f.write(b"\0")
        assert message_of_call(ours.check_unchanged) == ref.gguf_check_unchanged(h) == "gguf_checkpoint_changed"
        q = "blk.0.attn_q.weight"
        assert message_of_call(lambda: ours.read_packed_rows(q, 0, 0, 0)) == "gguf_checkpoint_changed"
    finally:
        ref.gguf_close(h)
        ours.close()
    root2, _ = single(tmp_path / "x")
    with pytest.raises(KadanError) as e:
        gg.GgufCheckpoint(root2, cancel=ctypes.c_ubyte(1))
    assert e.value.status == CANCELLED and message(e.value) == "gguf_cancelled"
    ours = gg.GgufCheckpoint(root2)
    with pytest.raises(KadanError) as e:
        ours.read_packed_rows("blk.0.attn_q.weight", 0, 0, ours.tensor("blk.0.attn_q.weight").row_bytes,
                              cancel=ctypes.c_ubyte(1))
    assert e.value.status == CANCELLED


def test_native_row_source_reads_whole_rows(gg, tmp_path):
    """kb200_gguf_rows_source (the packed-row source a source batch calls)
    returns the tensor's rows of the bound expert; out-of-range reads fail."""
    from kadan_b200 import lib

    root, payloads = single(tmp_path)
    ours = gg.GgufCheckpoint(root)
    name = "blk.0.ffn_down_exps.weight"
    t = ours.tensor(name)
    rb, rows = t.row_bytes, t.shape[1]
    for expert in range(3):
        src = ours.rows(name, expert)
        buf = (ctypes.c_ubyte * (2 * rb))()
        assert lib.kb200_gguf_rows_source(src.user, 2, buf, 2 * rb) == 0
        base = (expert * rows + 2) * rb
        assert bytes(buf) == payloads[name][base:base + 2 * rb]
        assert lib.kb200_gguf_rows_source(src.user, rows - 1, buf, 2 * rb) != 0
    from kadan_b200 import KadanError

    with pytest.raises(KadanError):
        ours.rows(name, 3)
    with pytest.raises(KadanError):
        ours.rows("output_norm.weight", 0)


def test_reader_without_reference(gg, tmp_path):
    """Checks that need no reference build: bytes and layout of what was written."""
    root, payloads = single(tmp_path)
    ours = gg.GgufCheckpoint(root)
    assert ours.tensor_count() == len(TENSORS)
    st = os.stat(root / "model.gguf")
    for t in ours.tensors():
        assert t.bytes == len(payloads[t.name])
        ident = ours.identity(t.name)
        assert (ident.inode, ident.file_size, ident.payload_begin) == (st.st_ino, st.st_size, t.offset)
        if t.rank >= 2:
            got = ours.read_packed_rows(t.name, 0, 0, t.shape[1] * t.row_bytes)
            assert got.tobytes() == payloads[t.name][:t.shape[1] * t.row_bytes]
    assert ours.integer("llama.context_length") == 8192
    assert ours.number("llama.rope.freq_base") == 500000.0
    assert ours.boolean("llama.use_parallel_residual") is True


def test_source_pointer_the_batch_receives(gg, tmp_path):
    """The kb200_row_source pointer that weight_bank.dense_gguf_source_batch
    hands the library for a bound GgufRows reads the same rows when called."""
    from kadan_b200.weight_bank import _ROW_SOURCE

    root, payloads = single(tmp_path)
    ours = gg.GgufCheckpoint(root)
    name = "blk.0.attn_q.weight"
    t = ours.tensor(name)
    src = ours.rows(name)
    fn = _ROW_SOURCE(gg.ROWS_SOURCE_ADDRESS)
    buf = (ctypes.c_ubyte * (3 * t.row_bytes))()
    assert fn(src.user, 2, ctypes.addressof(buf), 3 * t.row_bytes) == 0
    assert bytes(buf) == payloads[name][2 * t.row_bytes:5 * t.row_bytes]
    assert fn(src.user, t.shape[1] - 1, ctypes.addressof(buf), 3 * t.row_bytes) != 0


def test_read_vector_matches_reference(gg, ref, tmp_path):
    vec = np.arange(24, dtype=np.float32).reshape(2, 3, 4) * 0.5
    bad = np.array([1.0, np.nan, 3.0, 4.0], dtype=np.float32)
    root = tmp_path / "v"
    root.mkdir()
    gw.write_arrays(root / "m.gguf", [("general.architecture", STRING, "x")],
                    [("norm", [4, 3, 2], F32T, vec), ("bad", [4], F32T, bad),
                     ("q", [256, 2], Q4_K, np.zeros((2, 144), np.uint8))])
    ours = gg.GgufCheckpoint(root)
    h = ref.gguf_open(root)
    try:
        got = ours.read_vector("norm", 24)
        assert np.array_equal(got, vec.reshape(-1)) and np.array_equal(got, ref.gguf_read_vector(h, "norm", 24))
        for name, count in (("norm", 23), ("bad", 4), ("q", 512), ("missing", 1)):
            want = ref.gguf_read_vector(h, name, count)
            assert isinstance(want, str)
            assert message_of_call(lambda: ours.read_vector(name, count)) == want, (name, want)
    finally:
        ref.gguf_close(h)


def test_mxfp4_tensors_opt_in(gg, ref, tmp_path):
    """GGUF MXFP4 (ggml type 39): refused by default with the reference's own
    message (its reader has no MXFP4 encoding); opened with ACCEPT_MXFP4, the
    tensor reports 17-byte blocks of 32 values and reads back byte for byte."""
    rng = np.random.default_rng(3)
    gate = rng.integers(0, 256, size=4 * 6 * (64 // 32) * 17, dtype=np.uint8)
    tensors = TENSORS + [("blk.0.ffn_gate_exps.weight", [64, 6, 4], 39, gate.tobytes())]
    root, payloads = single(tmp_path, tensors=tensors)
    want = ref.gguf_open(root)
    assert want == "gguf_tensor_type"
    assert our_error(gg, root) == want
    ours = gg.GgufCheckpoint(root, flags=gg.ACCEPT_MXFP4)
    try:
        t = ours.tensor("blk.0.ffn_gate_exps.weight")
        assert (t.shape, t.ggml_type, t.encoding, t.row_bytes, t.bytes) == ((64, 6, 4), 39, gg.MXFP4, 34, 4 * 6 * 34)
        for expert in range(4):
            got = ours.read_packed_rows(t.name, expert, 1, 5 * 34)
            assert np.array_equal(got, gate[(expert * 6 + 1) * 34:(expert * 6 + 6) * 34])
        # The other tensors are unchanged by the option.
        assert [x.name for x in ours.tensors()] == sorted(payloads)
    finally:
        ours.close()
