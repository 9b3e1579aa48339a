"""Resident weight bank: the worker's kadan::DeviceWeights over the C ABI.

Mirrors services/hikari/inference_worker/include/kadan/device_weights.hpp:35-486
(`find`, `retain`, `retain_device`, `release_sources`, `release`, `bound`,
`capacity`, `maximum_capacity`, `allocated`, `reserved`, `quarantined`).
A bank either owns CUDA memory of one device (`WeightBank.cuda`) or runs over
caller-supplied operations (`WeightBank(limit, ops)`, where `ops` implements
the reference's WeightDeviceOperations: available / allocate / copy_host /
copy_device / free / synchronize). Operations report failure by raising; the
bank then rolls back, or quarantines itself when the rollback fails, exactly
as the reference does with exceptions.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Iterable, Optional

import numpy as np

from . import CANCELLED, CUDA, OK, KadanError, check, lib

c_u64, vp, c_int, c_u8 = ctypes.c_uint64, ctypes.c_void_p, ctypes.c_int, ctypes.c_ubyte

ADMITTED, EMPTY, ENVELOPE, PHYSICAL, ALLOCATION = range(5)
REFUSAL_NAMES = {EMPTY: "empty", ENVELOPE: "envelope", PHYSICAL: "physical", ALLOCATION: "allocation"}


class WeightIdentityC(ctypes.Structure):
    _fields_ = [(name, c_u64) for name in (
        "device", "inode", "file_size", "modified_seconds", "modified_nanoseconds",
        "changed_seconds", "changed_nanoseconds", "payload_begin", "payload_end")]


class WeightKeyC(ctypes.Structure):
    _fields_ = [("source", WeightIdentityC), ("first", c_u64), ("count", c_u64), ("width", c_u64)]


_AVAILABLE = ctypes.CFUNCTYPE(c_int, vp, ctypes.POINTER(c_u64))
_ALLOCATE = ctypes.CFUNCTYPE(c_int, vp, c_u64, ctypes.POINTER(vp))
_COPY = ctypes.CFUNCTYPE(c_int, vp, vp, c_u64, vp, c_u64)
_RELEASE = ctypes.CFUNCTYPE(c_int, vp, vp)
_SYNC = ctypes.CFUNCTYPE(c_int, vp)


class WeightOpsC(ctypes.Structure):
    _fields_ = [("user", vp), ("available", _AVAILABLE), ("allocate", _ALLOCATE), ("copy_host", _COPY),
                ("copy_device", _COPY), ("release", _RELEASE), ("synchronize", _SYNC)]


class BankStateC(ctypes.Structure):
    _fields_ = [("capacity", c_u64), ("maximum_capacity", c_u64), ("allocated", c_u64), ("reserved", c_u64),
                ("entries", c_u64), ("quarantined", ctypes.c_int32)]


lib.kb200_bank_create.argtypes = [c_u64, ctypes.POINTER(WeightOpsC), ctypes.POINTER(vp)]
lib.kb200_bank_create_cuda.argtypes = [c_int, c_u64, c_u64, ctypes.POINTER(vp)]
lib.kb200_bank_destroy.argtypes = [vp]
lib.kb200_bank_destroy.restype = None
lib.kb200_bank_state_get.argtypes = [vp, ctypes.POINTER(BankStateC)]
lib.kb200_bank_find.argtypes = [vp, ctypes.POINTER(WeightKeyC), ctypes.POINTER(vp)]
for _fn in (lib.kb200_bank_retain, lib.kb200_bank_retain_device):
    _fn.argtypes = [vp, ctypes.POINTER(WeightKeyC), vp, c_u64, ctypes.POINTER(c_u8), ctypes.POINTER(vp),
                    ctypes.POINTER(c_int)]
lib.kb200_bank_release_sources.argtypes = [vp, ctypes.POINTER(WeightIdentityC), ctypes.c_size_t,
                                           ctypes.POINTER(c_u64)]
lib.kb200_bank_release.argtypes = [vp]
lib.kb200_bank_bound.argtypes = [vp, c_u64]


@dataclass(frozen=True)
class WeightIdentity:
    """kadan::WeightIdentity (IW/include/kadan/weight_identity.hpp:7-19)."""

    device: int = 0
    inode: int = 0
    file_size: int = 0
    modified_seconds: int = 0
    modified_nanoseconds: int = 0
    changed_seconds: int = 0
    changed_nanoseconds: int = 0
    payload_begin: int = 0
    payload_end: int = 0

    def c(self) -> WeightIdentityC:
        return WeightIdentityC(self.device, self.inode, self.file_size, self.modified_seconds,
                               self.modified_nanoseconds, self.changed_seconds, self.changed_nanoseconds,
                               self.payload_begin, self.payload_end)


@dataclass(frozen=True)
class WeightKey:
    """DeviceWeights::Key: `count` blocks of `width` bytes from block `first`."""

    source: WeightIdentity = field(default_factory=WeightIdentity)
    first: int = 0
    count: int = 0
    width: int = 0

    def c(self) -> WeightKeyC:
        return WeightKeyC(self.source.c(), self.first, self.count, self.width)


class WeightBank:
    """One device's bank of immutable packed tiles (DeviceWeights)."""

    def __init__(self, limit: int, ops=None, *, _handle: Optional[int] = None):
        self._ops = ops
        self._ops_c = None
        self.last_refusal = ADMITTED
        if _handle is not None:
            self._h = _handle
            return
        if ops is None:
            raise ValueError("WeightBank needs operations; use WeightBank.cuda(device, limit) for CUDA memory")
        self._ops_c = self._wrap(ops)
        h = vp()
        check(lib.kb200_bank_create(limit, ctypes.byref(self._ops_c), ctypes.byref(h)))
        self._h = h.value

    @classmethod
    def cuda(cls, device: int, limit: int, scratch: int = 0) -> "WeightBank":
        """A bank of cudaMalloc'd entries on `device`; `scratch` bytes of free
        memory stay reserved for projection workspaces."""
        h = vp()
        check(lib.kb200_bank_create_cuda(device, limit, scratch, ctypes.byref(h)))
        return cls(limit, _handle=h.value)

    @staticmethod
    def _wrap(ops) -> WeightOpsC:
        # Each callback turns a Python exception into a failed status, the way
        # the reference's operations throw.
        def guard(fn):
            def run(*args):
                try:
                    fn(*args)
                    return OK
                except Exception:  # noqa: BLE001 - any failure of the fake is an operation failure
                    return CUDA
            return run

        def available(_user, out):
            out[0] = int(ops.available_weight_bytes())

        def allocate(_user, nbytes, out):
            p = ops.allocate_weight(int(nbytes))
            out[0] = None if p is None else int(p)

        def copy_host(_user, dst, offset, src, nbytes):
            ops.copy_weight(int(dst), int(offset), int(src or 0), int(nbytes))

        def copy_device(_user, dst, offset, src, nbytes):
            ops.copy_weight_device(int(dst), int(offset), int(src or 0), int(nbytes))

        def release(_user, p):
            ops.free_weight(int(p))

        def synchronize(_user):
            ops.synchronize_weights()

        return WeightOpsC(None, _AVAILABLE(guard(available)), _ALLOCATE(guard(allocate)),
                          _COPY(guard(copy_host)), _COPY(guard(copy_device)), _RELEASE(guard(release)),
                          _SYNC(guard(synchronize)))

    # -- queries -----------------------------------------------------------
    def _state(self) -> BankStateC:
        s = BankStateC()
        check(lib.kb200_bank_state_get(self._h, ctypes.byref(s)))
        return s

    def capacity(self) -> int:
        return int(self._state().capacity)

    def maximum_capacity(self) -> int:
        return int(self._state().maximum_capacity)

    def allocated(self) -> int:
        return int(self._state().allocated)

    def reserved(self) -> int:
        return int(self._state().reserved)

    def entries(self) -> int:
        return int(self._state().entries)

    def quarantined(self) -> bool:
        return bool(self._state().quarantined)

    # -- operations --------------------------------------------------------
    def find(self, key: WeightKey) -> Optional[int]:
        p = vp()
        check(lib.kb200_bank_find(self._h, ctypes.byref(key.c()), ctypes.byref(p)))
        return p.value

    def _retain(self, fn, key: WeightKey, src: Optional[int], nbytes: int, cancel) -> Optional[int]:
        p, why = vp(), c_int(0)
        cancel_ptr = None if cancel is None else ctypes.pointer(cancel)
        check(fn(self._h, ctypes.byref(key.c()), src, nbytes, cancel_ptr, ctypes.byref(p), ctypes.byref(why)))
        self.last_refusal = why.value
        return p.value

    def retain(self, key: WeightKey, src: Optional[int], nbytes: int, cancel: Optional[ctypes.c_ubyte] = None):
        """Admit `nbytes` of host memory at address `src` (or return the hit);
        None when the bank refuses (reason in `last_refusal`)."""
        return self._retain(lib.kb200_bank_retain, key, src, nbytes, cancel)

    def retain_device(self, key: WeightKey, src: Optional[int], nbytes: int,
                      cancel: Optional[ctypes.c_ubyte] = None):
        """As `retain`, copying from device memory at `src`."""
        return self._retain(lib.kb200_bank_retain_device, key, src, nbytes, cancel)

    def release_sources(self, sources: Iterable[WeightIdentity]) -> int:
        srcs = list(sources)
        arr = (WeightIdentityC * max(1, len(srcs)))(*[s.c() for s in srcs])
        out = c_u64()
        check(lib.kb200_bank_release_sources(self._h, arr, len(srcs), ctypes.byref(out)))
        return int(out.value)

    def release(self) -> None:
        check(lib.kb200_bank_release(self._h))

    def bound(self, nbytes: int) -> None:
        check(lib.kb200_bank_bound(self._h, nbytes))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.kb200_bank_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


# --------------------------------------------------------------------------
# Host-span batch over packed-row sources (kb200_dense_gguf_source_batch).

_ROW_SOURCE = ctypes.CFUNCTYPE(c_int, vp, c_u64, vp, c_u64)


class SourceJobC(ctypes.Structure):
    _fields_ = [("identity", ctypes.POINTER(WeightIdentityC)), ("source", _ROW_SOURCE), ("source_user", vp),
                ("input", vp), ("output", vp), ("in_", ctypes.c_uint32), ("out", ctypes.c_uint32),
                ("rows", ctypes.c_uint32), ("encoding", ctypes.c_int32), ("retain_misses", ctypes.c_int32)]


lib.kb200_dense_gguf_source_batch.argtypes = [vp, vp, ctypes.POINTER(SourceJobC), ctypes.c_size_t, c_u64,
                                              ctypes.POINTER(c_u8), ctypes.POINTER(c_int)]
lib.kb200_dense_gguf_source.argtypes = [vp, vp, ctypes.POINTER(SourceJobC), vp, c_u64, c_int, ctypes.POINTER(c_u8),
                                        ctypes.POINTER(c_int)]
SOURCE_STAGING_HALF = 16 << 20


@dataclass
class SourceJob:
    """DenseCompute::GgufBatchJob with its GgufWeightSource: `read(first_row,
    nbytes)` returns `nbytes` bytes of whole packed rows from `first_row`
    (anything exposing the buffer protocol), or `read` is a native source
    from gguf_file.GgufCheckpoint.rows(...) (read by the C library with no
    Python call; `reads` then stays empty). x: float32 numpy [rows, in];
    y: float32 numpy [rows, out], written."""

    identity: WeightIdentity
    read: object
    x: object
    y: object
    in_: int
    out: int
    encoding: int
    retain_misses: bool = True
    reads: list = field(default_factory=list)  # (first_row, nbytes) of every source call


def _source_jobs_c(jobs):
    """The kb200_source_job array for `jobs` and the objects it points into."""
    from .gguf_file import ROWS_SOURCE_ADDRESS, GgufRows

    keep = []
    arr = (SourceJobC * len(jobs))()
    for i, job in enumerate(jobs):
        def read(_user, first_row, dst, nbytes, job=job):
            try:
                data = np.ascontiguousarray(np.frombuffer(job.read(int(first_row), int(nbytes)), dtype=np.uint8))
                if data.nbytes != nbytes:
                    return CUDA
                ctypes.memmove(dst, data.ctypes.data, nbytes)
                job.reads.append((int(first_row), int(nbytes)))
                return OK
            except Exception:  # noqa: BLE001 - a failing source fails the call
                return CUDA

        ident = job.identity.c()
        if isinstance(job.read, GgufRows):
            cb, user = _ROW_SOURCE(ROWS_SOURCE_ADDRESS), job.read.user
        else:
            cb, user = _ROW_SOURCE(read), None
        keep += [ident, cb, job.read]
        rows = job.x.size // job.in_
        arr[i] = SourceJobC(ctypes.pointer(ident), cb, user, job.x.ctypes.data, job.y.ctypes.data, job.in_, job.out,
                            rows, job.encoding, int(job.retain_misses))
    return arr, keep


def dense_gguf_source_batch(ctx, bank: Optional[WeightBank], jobs, scratch_limit: int = 0,
                            cancel: Optional[ctypes.c_ubyte] = None) -> int:
    """Run the jobs (kb200_dense_gguf_source_batch); returns the ProjectionResult code."""
    arr, keep = _source_jobs_c(jobs)
    result = c_int(0)
    check(lib.kb200_dense_gguf_source_batch(ctx.handle, None if bank is None else bank._h, arr, len(jobs),
                                            scratch_limit, None if cancel is None else ctypes.pointer(cancel),
                                            ctypes.byref(result)))
    del keep
    return int(result.value)


def dense_gguf_source(ctx, bank: Optional[WeightBank], job: SourceJob, bias=None, scratch_limit: int = 0,
                      precise: bool = False, cancel: Optional[ctypes.c_ubyte] = None) -> int:
    """DenseCompute::dense_gguf_source (kb200_dense_gguf_source): one job plus
    an optional float32 bias [out]; returns RESULT_FINITE."""
    arr, keep = _source_jobs_c([job])
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    result = c_int(0)
    check(lib.kb200_dense_gguf_source(ctx.handle, None if bank is None else bank._h, arr,
                                      None if b is None else b.ctypes.data, scratch_limit, int(precise),
                                      None if cancel is None else ctypes.pointer(cancel), ctypes.byref(result)))
    del keep
    return int(result.value)


__all__ = ["WeightBank", "SourceJob", "dense_gguf_source_batch", "dense_gguf_source", "WeightKey", "WeightIdentity", "KadanError", "CANCELLED", "ADMITTED", "EMPTY",
           "ENVELOPE", "PHYSICAL", "ALLOCATION", "REFUSAL_NAMES"]
