"""GGUF checkpoint reader over the C ABI (kb200_gguf_*): the worker's
kadan::checkpoint::GgufCheckpoint (services/hikari/inference_worker/include/
kadan/gguf_checkpoint.hpp:53-103) with the same method names. Failures raise
KadanError carrying the reference's message ("gguf_version",
"gguf_missing_tensor", "gguf_row_range", ...).

    ckpt = GgufCheckpoint(directory)
    ckpt.tensor("blk.0.ffn_up.weight")           -> TensorInfo
    ckpt.read_packed_rows(name, expert, first_row, nbytes) -> numpy uint8
    ckpt.rows(name, expert)                      -> a native packed-row source
                                                    for weight_bank.SourceJob
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import check, lib
from .weight_bank import WeightIdentity, WeightIdentityC

c_u64, vp, c_u8 = ctypes.c_uint64, ctypes.c_void_p, ctypes.c_ubyte


class GgufTensorC(ctypes.Structure):
    _fields_ = [("shape", c_u64 * 3), ("rank", ctypes.c_uint32), ("ggml_type", ctypes.c_uint32),
                ("encoding", ctypes.c_int32), ("file", ctypes.c_uint32), ("bytes", c_u64), ("row_bytes", c_u64),
                ("offset", c_u64)]


class GgufRowsC(ctypes.Structure):
    _fields_ = [("file", vp), ("tensor", c_u64), ("expert", c_u64)]


lib.kb200_gguf_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(c_u8), ctypes.POINTER(vp)]
lib.kb200_gguf_open_flags.argtypes = [ctypes.c_char_p, ctypes.POINTER(c_u8), ctypes.c_uint32, ctypes.POINTER(vp)]
ACCEPT_MXFP4 = 1  # KB200_GGUF_ACCEPT_MXFP4
MXFP4 = -3        # KB200_GGUF_MXFP4: the encoding an accepted ggml type-39 tensor reports
lib.kb200_gguf_close.argtypes = [vp]
lib.kb200_gguf_close.restype = None
lib.kb200_gguf_tensor_count.argtypes = [vp]
lib.kb200_gguf_tensor_count.restype = ctypes.c_size_t
lib.kb200_gguf_tensor_at.argtypes = [vp, ctypes.c_size_t, ctypes.POINTER(GgufTensorC), ctypes.POINTER(ctypes.c_char_p)]
lib.kb200_gguf_find_tensor.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(GgufTensorC)]
lib.kb200_gguf_identity.argtypes = [vp, ctypes.c_char_p, c_u64, ctypes.POINTER(WeightIdentityC)]
lib.kb200_gguf_check_unchanged.argtypes = [vp]
lib.kb200_gguf_read_packed_rows.argtypes = [vp, ctypes.c_char_p, c_u64, c_u64, vp, c_u64, ctypes.POINTER(c_u8)]
lib.kb200_gguf_has.argtypes = [vp, ctypes.c_char_p]
lib.kb200_gguf_read_vector.argtypes = [vp, ctypes.c_char_p, vp, c_u64, ctypes.POINTER(c_u8)]
lib.kb200_gguf_integer.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(c_u64)]
lib.kb200_gguf_number.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]
lib.kb200_gguf_boolean.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]
lib.kb200_gguf_string.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_size_t)]
lib.kb200_gguf_integers.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_size_t,
                                    ctypes.POINTER(ctypes.c_size_t)]
lib.kb200_gguf_numbers.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.c_size_t,
                                   ctypes.POINTER(ctypes.c_size_t)]
lib.kb200_gguf_rows_bind.argtypes = [vp, ctypes.c_char_p, c_u64, ctypes.POINTER(GgufRowsC)]
lib.kb200_gguf_rows_source.argtypes = [vp, c_u64, vp, c_u64]

# The C function kb200_gguf_rows_source as a kb200_row_source pointer.
ROWS_SOURCE_ADDRESS = ctypes.cast(lib.kb200_gguf_rows_source, vp).value


@dataclass(frozen=True)
class TensorInfo:
    """kadan::checkpoint::GgufTensor plus where its payload lies."""

    name: str
    shape: tuple  # ggml order: values per row, rows, experts
    rank: int
    ggml_type: int
    encoding: int
    file: int
    bytes: int
    row_bytes: int
    offset: int


def _info(name: str, t: GgufTensorC) -> TensorInfo:
    return TensorInfo(name, tuple(int(v) for v in t.shape), int(t.rank), int(t.ggml_type), int(t.encoding),
                      int(t.file), int(t.bytes), int(t.row_bytes), int(t.offset))


class GgufRows:
    """A bound packed-row source (kb200_gguf_rows) for one tensor and expert;
    keeps its checkpoint open while alive."""

    def __init__(self, ckpt: "GgufCheckpoint", name: str, expert: int):
        self.ckpt = ckpt
        self.c = GgufRowsC()
        check(lib.kb200_gguf_rows_bind(ckpt._h, name.encode(), expert, ctypes.byref(self.c)))

    @property
    def user(self) -> int:
        return ctypes.addressof(self.c)


class GgufCheckpoint:
    def __init__(self, root, cancel: Optional[ctypes.c_ubyte] = None, flags: int = 0):
        """flags: ACCEPT_MXFP4 also opens files with GGUF MXFP4 tensors, which
        the reference's reader (and this one by default) refuses."""
        h = vp()
        self._h = None
        check(lib.kb200_gguf_open_flags(str(root).encode(), None if cancel is None else ctypes.pointer(cancel), flags,
                                        ctypes.byref(h)))
        self._h = h.value

    def close(self) -> None:
        if self._h:
            lib.kb200_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def tensor_count(self) -> int:
        return int(lib.kb200_gguf_tensor_count(self._h))

    def tensor_at(self, index: int) -> TensorInfo:
        t, name = GgufTensorC(), ctypes.c_char_p()
        check(lib.kb200_gguf_tensor_at(self._h, index, ctypes.byref(t), ctypes.byref(name)))
        return _info(name.value.decode(), t)

    def tensors(self) -> list:
        return [self.tensor_at(i) for i in range(self.tensor_count())]

    def tensor(self, name: str) -> TensorInfo:
        t = GgufTensorC()
        check(lib.kb200_gguf_find_tensor(self._h, name.encode(), ctypes.byref(t)))
        return _info(name, t)

    def identity(self, name: str, expert: int = 0) -> WeightIdentity:
        c = WeightIdentityC()
        check(lib.kb200_gguf_identity(self._h, name.encode(), expert, ctypes.byref(c)))
        return WeightIdentity(*(int(getattr(c, f)) for f, _ in WeightIdentityC._fields_))

    def check_unchanged(self) -> None:
        check(lib.kb200_gguf_check_unchanged(self._h))

    def read_packed_rows(self, name: str, expert: int, first_row: int, nbytes: int,
                         cancel: Optional[ctypes.c_ubyte] = None) -> np.ndarray:
        out = np.empty(nbytes, dtype=np.uint8)
        check(lib.kb200_gguf_read_packed_rows(self._h, name.encode(), expert, first_row,
                                              out.ctypes.data if nbytes else None, nbytes,
                                              None if cancel is None else ctypes.pointer(cancel)))
        return out

    def read_vector(self, name: str, count: int, cancel: Optional[ctypes.c_ubyte] = None) -> np.ndarray:
        out = np.empty(max(1, count), dtype=np.float32)
        check(lib.kb200_gguf_read_vector(self._h, name.encode(), out.ctypes.data, count,
                                         None if cancel is None else ctypes.pointer(cancel)))
        return out[:count]

    def rows(self, name: str, expert: int = 0) -> GgufRows:
        return GgufRows(self, name, expert)

    # -- metadata ----------------------------------------------------------
    def has(self, key: str) -> bool:
        return bool(lib.kb200_gguf_has(self._h, key.encode()))

    def integer(self, key: str) -> int:
        v = c_u64()
        check(lib.kb200_gguf_integer(self._h, key.encode(), ctypes.byref(v)))
        return int(v.value)

    def number(self, key: str) -> float:
        v = ctypes.c_double()
        check(lib.kb200_gguf_number(self._h, key.encode(), ctypes.byref(v)))
        return float(v.value)

    def boolean(self, key: str) -> bool:
        v = ctypes.c_int()
        check(lib.kb200_gguf_boolean(self._h, key.encode(), ctypes.byref(v)))
        return bool(v.value)

    def string(self, key: str) -> str:
        p, n = ctypes.c_char_p(), ctypes.c_size_t()
        check(lib.kb200_gguf_string(self._h, key.encode(), ctypes.byref(p), ctypes.byref(n)))
        return ctypes.string_at(p, n.value).decode()

    def integers(self, key: str) -> list:
        n = ctypes.c_size_t()
        check(lib.kb200_gguf_integers(self._h, key.encode(), None, 0, ctypes.byref(n)))
        buf = (ctypes.c_int64 * max(1, n.value))()
        check(lib.kb200_gguf_integers(self._h, key.encode(), buf, n.value, ctypes.byref(n)))
        return [int(v) for v in buf[:n.value]]

    def numbers(self, key: str) -> list:
        n = ctypes.c_size_t()
        check(lib.kb200_gguf_numbers(self._h, key.encode(), None, 0, ctypes.byref(n)))
        buf = (ctypes.c_double * max(1, n.value))()
        check(lib.kb200_gguf_numbers(self._h, key.encode(), buf, n.value, ctypes.byref(n)))
        return [float(v) for v in buf[:n.value]]


__all__ = ["GgufCheckpoint", "GgufRows", "TensorInfo", "ROWS_SOURCE_ADDRESS"]
