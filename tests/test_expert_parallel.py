"""Expert-parallel bookkeeping on CPU: send counts, the regroup segments, and
a two-rank `gloo` round trip of labelled rows through the same all-to-alls
and segment permutations the GPU layer issues."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from kadan_b200 import expert_parallel as ep


def apply_segments(src: np.ndarray, segs: np.ndarray) -> np.ndarray:
    dst = np.full_like(src, -1)
    for s, d, n in segs:
        dst[d:d + n] = src[s:s + n]
    return dst


def test_expert_range_and_send_counts():
    assert [ep.expert_range(128, 8, r) for r in (0, 7)] == [(0, 16), (112, 128)]
    with pytest.raises(ValueError):
        ep.expert_range(10, 4, 0)
    counts = np.arange(8)
    assert ep.send_counts(counts, 2).tolist() == [6, 22]
    assert ep.send_counts(counts, 4).tolist() == [1, 5, 9, 13]


@pytest.mark.parametrize("world,local", [(1, 4), (2, 3), (4, 16), (8, 16)])
def test_regroup_segments_make_expert_major_order(world, local):
    rng = np.random.default_rng(world * 100 + local)
    recv = rng.integers(0, 5, size=(world, local))
    recv[0, 0] = 0
    # Rows as (source, expert, index) labels in arrival (source-major) order.
    labels = np.array([(s, e, i) for s in range(world) for e in range(local) for i in range(recv[s, e])],
                      dtype=np.int64).reshape(-1, 3)
    segs, offsets = ep.regroup_segments(recv)
    grouped = apply_segments(labels, segs)
    want = np.array(sorted(map(tuple, labels), key=lambda r: (r[1], r[0], r[2])), dtype=np.int64).reshape(-1, 3)
    assert np.array_equal(grouped, want)
    assert offsets.tolist() == [0] + np.cumsum(recv.sum(axis=0)).tolist()
    assert all(n > 0 for _, _, n in segs)
    back = apply_segments(grouped, segs[:, [1, 0, 2]])
    assert np.array_equal(back, labels)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, experts, results):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        local = experts // world
        rng = np.random.default_rng(rank)
        chosen = rng.integers(0, experts, size=40 + 7 * rank)  # expert of each slot
        order = np.argsort(chosen, kind="stable")  # dispatch: expert-major, stable
        counts = np.bincount(chosen, minlength=experts).astype(np.int64)
        # Row payload: (origin rank, slot, expert) — the "expert" doubles the
        # slot id so the round trip can be checked.
        rows = np.stack([np.full(len(order), rank), order, chosen[order]], axis=1).astype(np.int64)
        recv = torch.empty(experts, dtype=torch.int64)
        dist.all_to_all_single(recv, torch.from_numpy(counts))
        recv_counts = recv.numpy().reshape(world, local)
        sends = ep.send_counts(counts, world).tolist()
        recvs = recv_counts.sum(axis=1).tolist()
        arrived = torch.empty(sum(recvs), 3, dtype=torch.int64)
        dist.all_to_all_single(arrived, torch.from_numpy(rows), output_split_sizes=recvs, input_split_sizes=sends)
        segs, offsets = ep.regroup_segments(recv_counts)
        grouped = apply_segments(arrived.numpy(), segs)
        ok = True
        for e in range(local):  # every grouped row belongs to the expert of its range
            ok &= bool(np.all(grouped[offsets[e]:offsets[e + 1], 2] == rank * local + e))
        y = grouped.copy()
        y[:, 2] = y[:, 1] * 2  # "expert output"
        back = apply_segments(y, segs[:, [1, 0, 2]])
        returned = torch.empty(len(order), 3, dtype=torch.int64)
        dist.all_to_all_single(returned, torch.from_numpy(back), output_split_sizes=sends, input_split_sizes=recvs)
        r = returned.numpy()
        ok &= bool(np.all(r[:, 0] == rank)) and bool(np.array_equal(r[:, 1], order))
        ok &= bool(np.array_equal(r[:, 2], 2 * order))
        results[rank] = ok
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,experts", [(2, 8), (3, 6)])
def test_gloo_round_trip_returns_every_row_to_its_slot(world, experts):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, experts, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert [p.exitcode for p in procs] == [0] * world
        assert all(results[r] for r in range(world))
