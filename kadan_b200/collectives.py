"""Collectives of the tensor-parallel path over NVLink peer memory.

PeerBuffers maps one buffer per rank into every other rank (CUDA IPC handles,
swapped once over the process group). PeerAllReduce adds fp32 vectors over
them with one kernel per call (kb200_peer_allreduce_f32, or fused into a
row-parallel GEMV); the expert-parallel layer exchanges rows over them
(kadan_b200.expert_parallel). No library collective runs on the data path:
the process group is only used at setup and teardown.
"""
from __future__ import annotations

import ctypes

from . import check, lib

lib.kb200_peer_buffer_bytes.restype = ctypes.c_size_t
lib.kb200_peer_buffer_bytes.argtypes = [ctypes.c_int, ctypes.c_size_t]
lib.kb200_device_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]
lib.kb200_device_free.argtypes = [ctypes.c_void_p]
lib.kb200_ipc_handle.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
lib.kb200_ipc_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
lib.kb200_ipc_close.argtypes = [ctypes.c_void_p]
lib.kb200_peer_allreduce_f32.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_size_t, ctypes.c_double, ctypes.c_void_p]
lib.kb200_gguf_gemv_allreduce.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_size_t,
                                          ctypes.c_double, ctypes.c_void_p]
lib.kb200_ep_buffer_bytes.restype = ctypes.c_size_t
lib.kb200_ep_buffer_bytes.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t]
lib.kb200_ep_rows_area.restype = ctypes.c_void_p
lib.kb200_ep_rows_area.argtypes = [ctypes.c_void_p]
lib.kb200_ep_return_area.restype = ctypes.c_void_p
lib.kb200_ep_return_area.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
lib.kb200_ep_dispatch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                  ctypes.c_double, ctypes.c_void_p]
lib.kb200_ep_return.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_double, ctypes.c_void_p]
IPC_HANDLE_BYTES = 64


class PeerBuffers:
    """One device buffer per rank, mapped into every other rank of `group`
    (allocated zeroed, handles swapped once over the process group).
    `peers` is the ctypes array of every rank's address, this rank's at [rank]."""

    def __init__(self, nbytes: int, group=None):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        own = ctypes.c_void_p()
        check(lib.kb200_device_alloc(int(nbytes), ctypes.byref(own)))
        self.own = own.value
        handle = (ctypes.c_char * IPC_HANDLE_BYTES)()
        check(lib.kb200_ipc_handle(self.own, handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self.own)
                continue
            buf = (ctypes.c_char * IPC_HANDLE_BYTES).from_buffer_copy(h)
            p = ctypes.c_void_p()
            check(lib.kb200_ipc_open(buf, ctypes.byref(p)))
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.peers = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)

    def close(self) -> None:
        """Collective: every rank's kernels are done before any buffer goes."""
        if self.own is None:
            return
        import torch

        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)
        for p in self.opened:
            check(lib.kb200_ipc_close(p))
        self.opened = []
        self.dist.barrier(group=self.group)
        check(lib.kb200_device_free(self.own))
        self.own = None


class PeerAllReduce:
    """Sum fp32 device tensors of up to `max_count` elements over the ranks of
    `group` (every rank calls with the same sizes in the same order)."""

    def __init__(self, max_count: int, group=None, timeout_s: float = 2.0, fused: bool = True):
        """fused: row-parallel projections run as kb200_gguf_gemv_allreduce
        (the GEMV pushes its outputs to the peers itself) instead of a GEMV
        launch followed by the all-reduce."""
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_count = int(max_count)
        self.timeout_s = float(timeout_s)
        self.fused = bool(fused)
        nbytes = int(lib.kb200_peer_buffer_bytes(self.world, self.max_count))
        if not nbytes:
            raise ValueError("peer all-reduce supports 1..8 ranks")
        self.buffers = PeerBuffers(nbytes, group)
        self.peers = self.buffers.peers

    def __call__(self, tensor, stream) -> None:
        """In place on `tensor` (fp32, contiguous), enqueued on `stream`."""
        check(lib.kb200_peer_allreduce_f32(tensor.data_ptr(), tensor.numel(), self.peers, self.world, self.rank,
                                           self.max_count, self.timeout_s, ctypes.c_void_p(stream.cuda_stream)))

    def gemv_allreduce(self, job, stream) -> None:
        """One row-parallel GEMV job (kadan_b200.GemvJob) whose output is then
        summed over the ranks, enqueued on `stream`."""
        check(lib.kb200_gguf_gemv_allreduce(ctypes.byref(job), self.peers, self.world, self.rank, self.max_count,
                                            self.timeout_s, ctypes.c_void_p(stream.cuda_stream)))

    def close(self) -> None:
        """Collective: every rank's kernels are done before any buffer goes."""
        self.buffers.close()
