"""Expert-parallel MXFP4 MoE layer across the GPUs of one node.

The reference runs the whole MoE layer on one host (MoeLayer::forward,
IW/src/models/text/qwen_layers.cpp:378-492) and has no multi-device split of
its experts. Here the experts are split evenly and contiguously over the ranks
of a process group (rank r holds experts [r*E/N, (r+1)*E/N)); every rank
routes its own tokens and the rows travel to the rank of their expert and
back:

  1. dispatch (kb200_moe_dispatch_rows): route, stable sort of the
     (token, choice) slots by expert, gather fp16 rows in expert-major order.
     Experts are contiguous per rank, so the rows for rank r are one range.
  2. exchange counts (all-to-all of the per-expert counts) and rows
     (all-to-all of the fp16 rows; NCCL over NVLink).
  3. regroup the received rows from source-major to expert-major order
     (kb200_rows_regroup), run the local experts (kb200_moe_experts), and
     put the fp32 results back in source-major order.
  4. all-to-all the results back; combine in selection order
     (kb200_moe_combine).

Each rank's output equals the single-device layer on the same tokens: the
same routing, the same expert arithmetic per row, the same combine order.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np

from . import MoeWeights, check, lib, moe_combine, moe_dispatch_rows, moe_experts, moe_weights, rows_regroup


def expert_range(experts: int, world: int, rank: int) -> Tuple[int, int]:
    """[first, end) of the experts rank `rank` holds (even split)."""
    if experts % world:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    per = experts // world
    return rank * per, (rank + 1) * per


def send_counts(expert_counts: np.ndarray, world: int) -> np.ndarray:
    """Rows this rank sends to each rank: its per-expert counts summed per owner."""
    return expert_counts.reshape(world, -1).sum(axis=1)


def regroup_segments(recv_counts: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Segments {src_row, dst_row, rows} that turn rows received source-major
    (for each source rank, its rows of local experts 0..E_l-1 in order) into
    expert-major order (for each local expert, the rows of source 0..N-1),
    and the local expert offsets [E_l + 1] of the result.

    recv_counts[s, e]: rows of local expert e received from rank s."""
    world, local = recv_counts.shape
    src_start = np.zeros((world, local), dtype=np.int64)
    flat = recv_counts.reshape(-1).astype(np.int64)
    src_start.reshape(-1)[1:] = np.cumsum(flat)[:-1]
    segs = []
    offsets = np.zeros(local + 1, dtype=np.int32)
    dst = 0
    for e in range(local):
        offsets[e] = dst
        for s in range(world):
            n = int(recv_counts[s, e])
            if n:
                segs.append((int(src_start[s, e]), dst, n))
            dst += n
    offsets[local] = dst
    return np.array(segs, dtype=np.int64).reshape(-1, 3), offsets


class ExpertParallelMoE:
    """One MoE layer whose experts are split over the ranks of `group`.

    weights: kb200 MoeWeights of the experts this rank holds (experts = E/N,
    top_k = the model's k), built over device tensors the caller keeps
    alive. experts: the model's total expert count E."""

    def __init__(self, local: MoeWeights, experts: int, world: int, rank: int, group=None, exchange: str = "nccl",
                 max_tokens: int = 0, device=None, timeout_s: float = 2.0):
        """exchange: "nccl" (all-to-alls sized by a count read-back on the
        host) or "peer" (kb200_ep_dispatch / kb200_ep_return over buffers
        mapped by CUDA IPC; no host synchronisation; needs max_tokens, the
        most tokens any rank routes per call, and a process group even for
        one rank)."""
        import torch
        import torch.distributed as dist

        self.w, self.experts, self.world, self.rank, self.group = local, experts, world, rank, group
        self.top_k = local.top_k
        self.local = experts // world
        if local.experts != self.local:
            raise ValueError("local weights must hold experts / world experts")
        self.dist = dist if world > 1 else None
        self._buffers = {}
        self.exchange = exchange
        if exchange == "peer":
            from .collectives import PeerBuffers

            if max_tokens <= 0:
                raise ValueError("the peer exchange needs max_tokens")
            hidden = local.hidden
            self.max_tokens = int(max_tokens)
            self.capacity = world * self.max_tokens * self.top_k
            self.local_capacity = self.max_tokens * self.top_k
            nbytes = int(lib.kb200_ep_buffer_bytes(world, experts, hidden, self.capacity, self.local_capacity))
            if not nbytes:
                raise ValueError("shape outside the peer exchange (at most 8 ranks, 256 experts)")
            self.timeout_s = float(timeout_s)
            self.peer = PeerBuffers(nbytes, group)
            self.rows_area = int(lib.kb200_ep_rows_area(self.peer.own))
            self.return_area = int(lib.kb200_ep_return_area(self.peer.own, self.capacity, hidden))
            self.local_offsets = torch.zeros(self.local + 1, dtype=torch.int32, device=device)
            self.zero_offsets = torch.zeros(experts + 1, dtype=torch.int32, device=device)
            self.results = torch.empty(self.capacity, hidden, dtype=torch.float32, device=device)
        elif exchange != "nccl":
            raise ValueError(f"unknown exchange {exchange!r}")

    def _buffer(self, name: str, nbytes: int, device):
        import torch

        buf = self._buffers.get(name)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._buffers[name] = buf
        return buf

    def forward(self, x_bf16, logits, out=None, status=None):
        """out[T, H] fp32 for this rank's tokens x (bf16 [T, H]) routed by
        fp32 logits [T, E]. Collective: every rank calls it for the layer."""
        import torch

        if self.exchange == "peer":
            return self._forward_peer(x_bf16, logits, out, status)

        dev = x_bf16.device
        tokens, hidden = x_bf16.shape
        k, world = self.top_k, self.world
        if out is None:
            out = torch.empty(tokens, hidden, dtype=torch.float32, device=dev)
        need = int(lib.kb200_moe_dispatch_workspace_bytes(tokens, hidden, self.experts, k))
        dws = self._buffer("dispatch", need, dev)
        d = moe_dispatch_rows(logits, x_bf16, k, dws, status)
        n = tokens * k
        base = dws.data_ptr()

        def view(ptr, count, dtype, elem):
            off = ptr - base
            return dws[off:off + count * elem].view(dtype)

        offsets = view(d.offsets, self.experts + 1, torch.int32, 4) if n else torch.zeros(
            self.experts + 1, dtype=torch.int32, device=dev)
        rows = view(d.rows, n * hidden, torch.float16, 2).view(n, hidden) if n else torch.empty(
            0, hidden, dtype=torch.float16, device=dev)
        counts = (offsets[1:] - offsets[:-1]).to(torch.int64)
        if self.dist:
            recv = torch.empty_like(counts)
            self.dist.all_to_all_single(recv, counts, group=self.group)
            host = torch.cat([counts, recv]).cpu().numpy()
            mine, recv_counts = host[:self.experts], host[self.experts:].reshape(world, self.local)
        else:
            mine = counts.cpu().numpy()
            recv_counts = mine.reshape(1, self.local)
        sends = send_counts(mine, world).tolist()
        recvs = recv_counts.sum(axis=1).tolist()
        r_total = int(sum(recvs))
        if self.dist:
            arrived = torch.empty(r_total, hidden, dtype=torch.float16, device=dev)
            self.dist.all_to_all_single(arrived, rows, output_split_sizes=recvs, input_split_sizes=sends,
                                        group=self.group)
        else:
            arrived = rows
        segs, local_offsets = regroup_segments(recv_counts)
        max_rows = int(segs[:, 2].max()) if len(segs) else 0
        grouped = torch.empty(r_total, hidden, dtype=torch.float16, device=dev)
        y_grouped = torch.empty(r_total, hidden, dtype=torch.float32, device=dev)
        if r_total:
            seg_dev, back_dev, off_dev = self._tables(segs, local_offsets, dev)
            rows_regroup(arrived, grouped, seg_dev, max_rows)
            ews = self._buffer("experts", int(lib.kb200_moe_experts_workspace_bytes(
                self._wref(), r_total)), dev)
            moe_experts(self.w, grouped, off_dev, y_grouped, ews, status)
            y_arrived = torch.empty(r_total, hidden, dtype=torch.float32, device=dev)
            rows_regroup(y_grouped, y_arrived, back_dev, max_rows)
        else:
            y_arrived = y_grouped
        if self.dist:
            y_sent = torch.empty(n, hidden, dtype=torch.float32, device=dev)
            self.dist.all_to_all_single(y_sent, y_arrived, output_split_sizes=sends, input_split_sizes=recvs,
                                        group=self.group)
        else:
            y_sent = y_arrived
        if tokens:
            moe_combine(y_sent, d.weight, d.pos, tokens, k, out)
        return out

    def _forward_peer(self, x_bf16, logits, out, status):
        """Dispatch, exchange, experts, return and combine, all enqueued on the
        current stream: nothing waits on the host."""
        import ctypes

        import torch

        dev = x_bf16.device
        tokens, hidden = x_bf16.shape
        k = self.top_k
        if tokens > self.max_tokens:
            raise ValueError("more tokens than the exchange buffers were sized for")
        if out is None:
            out = torch.empty(tokens, hidden, dtype=torch.float32, device=dev)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        sptr = None if status is None else status.data_ptr()
        if tokens:
            need = int(lib.kb200_moe_dispatch_workspace_bytes(tokens, hidden, self.experts, k))
            dws = self._buffer("dispatch", need, dev)
            d = moe_dispatch_rows(logits, x_bf16, k, dws, status)
            offsets, rows = d.offsets, d.rows
        else:  # a rank without tokens still takes part in the exchange
            d, offsets, rows = None, self.zero_offsets.data_ptr(), self.rows_area
        check(lib.kb200_ep_dispatch(offsets, rows, hidden, self.experts, self.world, self.rank, self.peer.peers,
                                    self.capacity, self.local_capacity, self.local_offsets.data_ptr(),
                                    self.timeout_s, stream))
        ews = self._buffer("experts", int(lib.kb200_moe_experts_workspace_bytes(self._wref(), self.capacity)), dev)
        check(lib.kb200_moe_experts(self._wref(), self.rows_area, self.local_offsets.data_ptr(), self.capacity,
                                    self.results.data_ptr(), ews.data_ptr(), ews.numel(), sptr, stream))
        check(lib.kb200_ep_return(self.results.data_ptr(), hidden, self.experts, self.world, self.rank,
                                  self.peer.peers, self.capacity, self.local_capacity, self.timeout_s, stream))
        if tokens:
            check(lib.kb200_moe_combine(self.return_area, d.weight, d.pos, tokens, k, hidden, out.data_ptr(), stream))
        return out

    def close(self) -> None:
        """Collective (peer exchange): release the mapped buffers."""
        if self.exchange == "peer" and self.peer is not None:
            self.peer.close()
            self.peer = None

    def _tables(self, segs, offsets, device):
        """Regroup segments (forward and back) and local expert offsets on the
        device, staged through one pinned buffer and copied asynchronously
        (a pageable copy would synchronise the stream). The staging buffer is
        rewritten only by the next call, after its count read-back, which
        waits for this copy."""
        import numpy as np
        import torch

        cap = self.world * self.local
        nbytes = 2 * cap * 24 + (self.local + 1) * 4
        if getattr(self, "_staging", None) is None:
            self._staging = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            self._tables_dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
        host = self._staging.numpy()
        fwd = host[:cap * 24].view(np.int64).reshape(cap, 3)
        back = host[cap * 24:2 * cap * 24].view(np.int64).reshape(cap, 3)
        count = len(segs)
        fwd[:count] = segs
        back[:count] = segs[:, [1, 0, 2]]
        host[2 * cap * 24:].view(np.int32)[:] = offsets
        self._tables_dev.copy_(self._staging, non_blocking=True)
        d = self._tables_dev
        return (d[:cap * 24].view(torch.int64).view(cap, 3)[:count],
                d[cap * 24:2 * cap * 24].view(torch.int64).view(cap, 3)[:count],
                d[2 * cap * 24:].view(torch.int32))

    def _wref(self):
        import ctypes

        return ctypes.byref(self.w)


def local_weights(gu_blocks, gu_scales, dn_blocks, dn_scales, *, hidden: int, inter: int, experts: int, top_k: int,
                  world: int, rank: int, gu_bias=None, dn_bias=None, **kw) -> Tuple[MoeWeights, List[object]]:
    """MoeWeights over this rank's experts, cut from full device tensors
    [E, ...] (views, no copy). Returns the struct and the views to keep alive."""
    first, end = expert_range(experts, world, rank)
    parts = [t[first:end] if t is not None else None for t in (gu_blocks, gu_scales, dn_blocks, dn_scales,
                                                               gu_bias, dn_bias)]
    for t in parts:
        if t is not None and not t.is_contiguous():
            raise ValueError("expert tensors must be contiguous")
    w = moe_weights(parts[0], parts[1], parts[2], parts[3], hidden=hidden, inter=inter, experts=end - first,
                    top_k=top_k, gu_bias=parts[4], dn_bias=parts[5], **kw)
    return w, parts
