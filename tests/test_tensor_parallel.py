"""Tensor-parallel shard geometry and the partial-sum all-reduce, on CPU.

The geometry checks cover the Llama-3-70B stack at 1, 2,
4 and 8 ranks. The two-rank test runs real `gloo` ranks: each decodes its own
shards with the oracle, multiplies in fp64 and the ranks combine the results
with the collectives the GPU path uses (all-reduce of row-parallel partial
sums; column slices gathered), which must reproduce the full projection.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from kadan_b200 import Q4_K, Q6_K, Q8_0, block_bytes, block_values, row_bytes, synth
from kadan_b200 import tensor_parallel as tp


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_llama70b_shards_cover_each_projection_once(world):
    for g in tp.llama3_70b_projections():
        for p in g:
            shards = [tp.shard(p, world, r) for r in range(world)]
            if p.mode == "column":
                assert [s.out_first for s in shards] == [sum(t.out_count for t in shards[:r]) for r in range(world)]
                assert sum(s.out_count for s in shards) == p.out
                assert all(s.out_count % p.granule == 0 and s.in_count == p.in_ for s in shards)
                assert len({s.out_count for s in shards}) == 1  # heads divide evenly at 1..8 ranks
            else:
                assert [s.in_first for s in shards] == [sum(t.in_count for t in shards[:r]) for r in range(world)]
                assert sum(s.in_count for s in shards) == p.in_
                assert all(s.in_count % block_values(p.encoding) == 0 and s.out_count == p.out for s in shards)
                assert len({s.in_count for s in shards}) == 1
            for s in shards:
                pitch = tp.shard_pitch(p, s)
                assert pitch % 16 == 0 and 0 <= pitch - row_bytes(p.encoding, s.in_count) < 16


def test_shard_split_follows_the_reference_boundary(kb):
    p = tp.Projection("odd", Q6_K, 40, 256 * 7, "row")
    firsts = [tp.shard(p, 3, r).in_first // 256 for r in range(3)]
    assert firsts == [kb.weight_boundary(7, [1, 1, 1], r) for r in range(3)] == [0, 2, 4]
    c = tp.Projection("c", Q4_K, 5 * 128, 256, "column", 128)
    assert [tp.shard(c, 2, r).out_count for r in range(2)] == [256, 384]
    with pytest.raises(ValueError):
        tp.shard(tp.Projection("bad", Q4_K, 100, 256, "column", 128), 2, 0)
    with pytest.raises(ValueError):
        tp.shard(tp.Projection("bad", Q6_K, 8, 300, "row"), 2, 0)
    with pytest.raises(ValueError):
        tp.shard(p, 2, 2)


@pytest.mark.parametrize("enc", [Q4_K, Q6_K, Q8_0])
@pytest.mark.parametrize("world", [2, 3, 4])
def test_shard_packed_reassembles_the_matrix(enc, world):
    out, in_ = 48, 7 * 256
    full = synth.gguf(enc, out, in_, seed=5)
    bb, bv = block_bytes(enc), block_values(enc)
    row = tp.Projection("r", enc, out, in_, "row")
    parts = []
    for r in range(world):
        s = tp.shard(row, world, r)
        part = tp.shard_packed(row, full, world, r)
        assert part.shape == (out, tp.shard_pitch(row, s))
        assert not part[:, row_bytes(enc, s.in_count):].any()
        parts.append(part[:, :row_bytes(enc, s.in_count)])
    assert np.array_equal(np.concatenate(parts, axis=1), full)
    col = tp.Projection("c", enc, out, in_, "column", 8)
    cols = [tp.shard_packed(col, full, world, r)[:, :row_bytes(enc, in_)] for r in range(world)]
    assert np.array_equal(np.concatenate(cols, axis=0), full)
    assert full.shape[1] == in_ // bv * bb


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import torch
    import torch.distributed as dist

    from oracle.pyoracle import Oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc = Oracle()
        tokens, hidden, ffn = 3, 512, 768
        groups = [[tp.Projection("q", Q6_K, 256, hidden, "column", 128)],
                  [tp.Projection("o", Q6_K, hidden, 256, "row")],
                  [tp.Projection("up", Q4_K, ffn, hidden, "column")],
                  [tp.Projection("down", Q6_K, hidden, ffn, "row")]]
        out = {}
        for gi, g in enumerate(groups):
            p = g[0]
            full = synth.gguf(p.encoding, p.out, p.in_, seed=40 + gi)
            x = synth.activations(tokens * p.in_, seed=60 + gi, dtype="bf16").reshape(tokens, p.in_)
            s = tp.shard(p, world, rank)
            local = tp.shard_packed(p, full, world, rank)[:, :row_bytes(p.encoding, s.in_count)]
            w = orc.decode(p.encoding, np.ascontiguousarray(local), s.out_count * s.in_count)
            w = w.reshape(s.out_count, s.in_count).astype(np.float64)
            y = x[:, s.in_first:s.in_first + s.in_count].astype(np.float64) @ w.T
            t = torch.from_numpy(np.ascontiguousarray(y))
            if p.mode == "row":
                dist.all_reduce(t)
                got = t.numpy()
            else:
                parts = [torch.empty(tokens, tp.shard(p, world, r).out_count, dtype=torch.float64)
                         for r in range(world)]
                dist.all_gather(parts, t)
                got = torch.cat(parts, dim=1).numpy()
            want = x.astype(np.float64) @ orc.decode(p.encoding, full, p.out * p.in_).reshape(
                p.out, p.in_).astype(np.float64).T
            out[p.name] = float(np.max(np.abs(got - want)) / max(1.0, float(np.max(np.abs(want)))))
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reproduce_the_full_projections():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
        for pr in procs:
            pr.start()
        for pr in procs:
            pr.join(120)
        assert all(pr.exitcode == 0 for pr in procs), [pr.exitcode for pr in procs]
        for r in range(world):
            for name, err in results[r].items():
                assert err < 1e-12, (r, name, err)
