"""Tensor-parallel GGUF decode across the GPUs of one node.

The reference spreads one projection's output columns over its devices in
proportion to their weight capacity and gathers the slices on the host
(weight_boundary, IW/include/kadan/device_placement.hpp:341-357;
gguf_batch_partition, IW/include/kadan/gguf_batch_partition.hpp:62-83; the
host scatter at :48-59). On one B200 node every GPU runs one rank of a
process group instead, and the split follows the transformer block:

* column-parallel projections (q, k, v by heads; gate, up) take a contiguous
  slice of output columns: packed GGUF rows are whole, so a slice is a row
  range of the packed matrix;
* row-parallel projections (o, down) take a contiguous slice of the K
  (input) axis. The slice is cut on super-block boundaries (256 values for
  the K-quants), so every rank holds whole blocks: each packed row is cut at
  a byte offset of whole blocks and no block straddles two ranks. Each rank
  produces a partial sum of the full output and the ranks add them with one
  all-reduce over NVLink — two per layer: the peer-memory kernel of
  collectives.PeerAllReduce, or NCCL through torch.distributed.

Column and block splits use the same proportional boundary as the reference
(kb200_weight_boundary, equal capacities here), so N ranks of one projection
cover it exactly once, in rank order.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

from . import Q4_K, Q6_K, block_bytes, block_values, check, gemv_job, lib, row_bytes, weight_boundary


@dataclass(frozen=True)
class Projection:
    """One GGUF projection of a decoder block: y[T, out] = x[T, in] . W[out, in]^T."""

    name: str
    encoding: int
    out: int
    in_: int
    mode: str  # "column" (split out) or "row" (split in, partial sums all-reduced)
    granule: int = 1  # columns that must stay on one rank (a head), column mode only


def llama3_70b_projections() -> List[List[Projection]]:
    """Dependency groups of one Llama-3-70B decode layer (hidden 8192, 64 q /
    8 kv heads of 128, ffn 28672): Q6_K attention and down, Q4_K gate/up."""
    h, kv, ffn, head = 8192, 1024, 28672, 128
    return [[Projection("q", Q6_K, h, h, "column", head), Projection("k", Q6_K, kv, h, "column", head),
             Projection("v", Q6_K, kv, h, "column", head)],
            [Projection("o", Q6_K, h, h, "row")],
            [Projection("gate", Q4_K, ffn, h, "column"), Projection("up", Q4_K, ffn, h, "column")],
            [Projection("down", Q6_K, h, ffn, "row")]]


@dataclass(frozen=True)
class Shard:
    """The part of a projection that rank `rank` of `world` holds.

    out_first/out_count: output columns (packed rows) of the shard;
    in_first/in_count: input values (K) of the shard. Column shards keep all
    of K; row shards keep all output columns."""

    out_first: int
    out_count: int
    in_first: int
    in_count: int


def shard(p: Projection, world: int, rank: int) -> Shard:
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank outside the group")
    equal = [1] * world
    if p.mode == "column":
        if p.out % p.granule:
            raise ValueError(f"{p.name}: {p.out} columns are not whole granules of {p.granule}")
        units = p.out // p.granule
        first = weight_boundary(units, equal, rank) * p.granule
        end = weight_boundary(units, equal, rank + 1) * p.granule
        return Shard(first, end - first, 0, p.in_)
    if p.mode == "row":
        values = block_values(p.encoding)
        if p.in_ % values:
            raise ValueError(f"{p.name}: K = {p.in_} is not whole blocks of {values}")
        blocks = p.in_ // values
        first = weight_boundary(blocks, equal, rank) * values
        end = weight_boundary(blocks, equal, rank + 1) * values
        return Shard(0, p.out, first, end - first)
    raise ValueError(f"unknown split mode {p.mode!r}")


def shard_pitch(p: Projection, s: Shard) -> int:
    """Row pitch of a shard's packed rows: the whole blocks of its K slice,
    padded to 16 bytes so the bulk-copy and TMA kernels take every shard
    (a Q6_K row of 3584 values is 2940 bytes; padded, 2944)."""
    return (row_bytes(p.encoding, s.in_count) + 15) // 16 * 16


def pad_rows(packed, pitch: int):
    """[rows, row_bytes] packed rows copied into [rows, pitch] (zero padding)."""
    rows, width = packed.shape
    if width == pitch:
        return packed.copy() if hasattr(packed, "flags") else packed.contiguous()
    if hasattr(packed, "flags"):
        import numpy as np

        out = np.zeros((rows, pitch), dtype=packed.dtype)
    else:
        import torch

        out = torch.zeros((rows, pitch), dtype=packed.dtype, device=packed.device)
    out[:, :width] = packed
    return out


def shard_packed(p: Projection, packed, world: int, rank: int):
    """This rank's packed rows [out_count, shard_pitch], cut from the full
    packed matrix [out, row_bytes] (numpy array or torch tensor)."""
    s = shard(p, world, rank)
    rows = packed[s.out_first:s.out_first + s.out_count]
    if p.mode == "row":
        bb, bv = block_bytes(p.encoding), block_values(p.encoding)
        rows = rows[:, s.in_first // bv * bb:(s.in_first + s.in_count) // bv * bb]
    return pad_rows(rows, shard_pitch(p, s))


class DecodeStack:
    """Per-rank tensor-parallel decode through a stack of layers.

    weights[layer][name] are this rank's packed shards (device tensors, as
    shard_packed cuts them); inputs are the full activations a column group
    reads (x[T, in]) and this rank's K slice of what a row projection reads.
    One step enqueues, per layer and dependency group, one GEMV batch launch
    and, after a row-parallel group, the all-reduce of its partial sums on
    `group` (torch.distributed, NCCL). Every rank enqueues the same
    collectives in the same order. The whole step can be captured in a CUDA
    graph (NCCL collectives are capturable)."""

    def __init__(self, groups: Sequence[Sequence[Projection]], weights: Sequence[Dict[str, object]], tokens: int,
                 world: int, rank: int, device, group=None, seed: int = 0, inputs: Optional[Dict[str, object]] = None,
                 collective=None):
        """inputs: full fp32 activations [tokens, in] per group, keyed by the
        group's first projection; by default bf16-representable N(0,1) drawn
        from `seed` (the same on every rank). collective: a callable
        (tensor, stream) that sums a tensor over the ranks in place, such as
        collectives.PeerAllReduce; None uses torch.distributed.all_reduce."""
        import torch

        self.groups, self.world, self.rank, self.group, self.tokens = groups, world, rank, group, tokens
        self.collective = collective
        self.weights = weights
        gen = torch.Generator(device=device).manual_seed(seed + 7)
        self.inputs: Dict[str, object] = dict(inputs or {})
        self.outputs: Dict[str, object] = {}
        for g in groups:
            for p in g:
                s = shard(p, world, rank)
                if g[0].name not in self.inputs:
                    full = torch.randn(tokens, p.in_, device=device, generator=gen).bfloat16().float()
                    self.inputs[g[0].name] = full
                self.outputs[p.name] = torch.empty(tokens, s.out_count, device=device)
        # Row projections read their rank's K slice of the full activations.
        self.local_inputs = {}
        for g in groups:
            p = g[0]
            s = shard(p, world, rank)
            full = self.inputs[p.name]
            self.local_inputs[p.name] = full[:, s.in_first:s.in_first + s.in_count].contiguous()
        self.calls = []
        for mats in weights:
            for g in groups:
                x = self.local_inputs[g[0].name]
                jobs = []
                for p in g:
                    s = shard(p, world, rank)
                    jobs.append(gemv_job(p.encoding, mats[p.name], x, self.outputs[p.name], in_=s.in_count,
                                         columns=s.out_count, rows=tokens, row_bytes_=shard_pitch(p, s)))
                arr = (type(jobs[0]) * len(jobs))(*jobs)
                reduce = [self.outputs[p.name] for p in g if p.mode == "row"] if world > 1 else []
                self.calls.append((arr, len(jobs), reduce))

    def launch(self, stream, group_index: Optional[int] = None) -> None:
        """Enqueue one step on `stream` (must be torch's current stream, so
        that the collectives order after the GEMVs). group_index: only that
        dependency group of every layer (a per-launch timing; every rank must
        pass the same)."""
        import torch.distributed as dist

        sptr = ctypes.c_void_p(stream.cuda_stream)
        fused = getattr(self.collective, "fused", False)
        for i, (arr, n, reduce) in enumerate(self.calls):
            if group_index is not None and i % len(self.groups) != group_index:
                continue
            if fused and reduce and n == 1:
                self.collective.gemv_allreduce(arr[0], stream)
                continue
            check(lib.kb200_gguf_gemv_batch(arr, n, sptr))
            for t in reduce:
                if self.collective is not None:
                    self.collective(t, stream)
                else:
                    dist.all_reduce(t, group=self.group)

    def weight_bytes(self) -> int:
        """Packed weight bytes this rank streams per step."""
        total = 0
        for _ in self.weights:
            for g in self.groups:
                for p in g:
                    s = shard(p, self.world, self.rank)
                    total += s.out_count * shard_pitch(p, s)
        return total


def full_weight_bytes(groups: Sequence[Sequence[Projection]], layers: int) -> int:
    return layers * sum(p.out * row_bytes(p.encoding, p.in_) for g in groups for p in g)


def synth_shards(groups, layers: int, world: int, rank: int, device, seed: int = 0) -> List[Dict[str, object]]:
    """Random shards with the config distributions, drawn directly on the device
    (the bench: a 46 GB stack is never built whole on one GPU)."""
    from . import synth

    out = []
    for layer in range(layers):
        mats = {}
        for gi, g in enumerate(groups):
            for i, p in enumerate(g):
                s = shard(p, world, rank)
                packed = synth.device_gguf(p.encoding, s.out_count, s.in_count,
                                           ((seed * 1000 + layer) * 16 + gi * 4 + i) * 64 + rank, device)
                mats[p.name] = pad_rows(packed, shard_pitch(p, s))
        out.append(mats)
    return out
