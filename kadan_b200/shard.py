"""Safetensors shard reader over the C ABI (kb200_shard_*): the worker's
kadan::checkpoint::Shard (services/hikari/inference_worker/include/kadan/
checkpoint.hpp:91-178) for the gpt-oss MXFP4 expert tensors. Failures raise
KadanError carrying the reference's message.

    shard = Shard(directory, "model-00001-of-00003.safetensors")
    codes, scales, columns = shard.load_mxfp4_expert_rows(
        "model.layers.0.mlp.experts.gate_up_proj", expert, first, count, budget)
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import check, lib
from .weight_bank import WeightIdentity, WeightIdentityC

c_u64, vp = ctypes.c_uint64, ctypes.c_void_p
DTYPES = ("U8", "F8_E4M3", "F32", "BF16", "F16", "I8", "U32")  # checkpoint::Dtype order


class ShardLimitsC(ctypes.Structure):
    _fields_ = [("header_bytes", c_u64), ("tensors", c_u64), ("metadata_value_bytes", c_u64)]


class ShardTensorC(ctypes.Structure):
    _fields_ = [("shape", c_u64 * 8), ("rank", ctypes.c_uint32), ("dtype", ctypes.c_int32), ("bytes", c_u64),
                ("offset", c_u64)]


lib.kb200_shard_open.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ShardLimitsC), ctypes.POINTER(vp)]
lib.kb200_shard_close.argtypes = [vp]
lib.kb200_shard_close.restype = None
lib.kb200_shard_tensor_count.argtypes = [vp]
lib.kb200_shard_tensor_count.restype = ctypes.c_size_t
lib.kb200_shard_tensor_at.argtypes = [vp, ctypes.c_size_t, ctypes.POINTER(ShardTensorC), ctypes.POINTER(ctypes.c_char_p)]
lib.kb200_shard_find_tensor.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ShardTensorC)]
lib.kb200_shard_identity.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(WeightIdentityC)]
lib.kb200_shard_check_unchanged.argtypes = [vp]
lib.kb200_shard_read_tensor.argtypes = [vp, ctypes.c_char_p, c_u64, vp, c_u64]
lib.kb200_shard_load_mxfp4_expert_rows.argtypes = [vp, ctypes.c_char_p, c_u64, c_u64, c_u64, c_u64, vp, c_u64, vp,
                                                   c_u64, ctypes.POINTER(c_u64)]


@dataclass(frozen=True)
class ShardTensor:
    """checkpoint::TensorInfo plus the payload's absolute file offset."""

    name: str
    dtype: str
    shape: tuple
    bytes: int
    offset: int


class Shard:
    def __init__(self, root, name: str, *, header_bytes: int = 0, tensors: int = 0, metadata_value_bytes: int = 0):
        limits = None
        if header_bytes or tensors or metadata_value_bytes:
            limits = ShardLimitsC(header_bytes or 16 << 20, tensors or 65536, metadata_value_bytes or 512)
        h = vp()
        self._h = None
        check(lib.kb200_shard_open(str(root).encode(), name.encode(),
                                   None if limits is None else ctypes.byref(limits), ctypes.byref(h)))
        self._h = h.value

    def close(self) -> None:
        if self._h:
            lib.kb200_shard_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    @staticmethod
    def _info(name: str, t: ShardTensorC) -> ShardTensor:
        return ShardTensor(name, DTYPES[t.dtype], tuple(int(v) for v in t.shape[:t.rank]), int(t.bytes),
                           int(t.offset))

    def tensor_count(self) -> int:
        return int(lib.kb200_shard_tensor_count(self._h))

    def tensor_at(self, index: int) -> ShardTensor:
        t, name = ShardTensorC(), ctypes.c_char_p()
        check(lib.kb200_shard_tensor_at(self._h, index, ctypes.byref(t), ctypes.byref(name)))
        return self._info(name.value.decode(), t)

    def tensors(self) -> list:
        return [self.tensor_at(i) for i in range(self.tensor_count())]

    def tensor(self, name: str) -> ShardTensor:
        t = ShardTensorC()
        check(lib.kb200_shard_find_tensor(self._h, name.encode(), ctypes.byref(t)))
        return self._info(name, t)

    def tensor_identity(self, name: str) -> WeightIdentity:
        c = WeightIdentityC()
        check(lib.kb200_shard_identity(self._h, name.encode(), ctypes.byref(c)))
        return WeightIdentity(*(int(getattr(c, f)) for f, _ in WeightIdentityC._fields_))

    def check_unchanged(self) -> None:
        check(lib.kb200_shard_check_unchanged(self._h))

    def read_tensor(self, name: str, offset: int, nbytes: int) -> np.ndarray:
        out = np.empty(max(1, nbytes), dtype=np.uint8)
        check(lib.kb200_shard_read_tensor(self._h, name.encode(), offset, out.ctypes.data, nbytes))
        return out[:nbytes]

    def load_mxfp4_expert_rows(self, prefix: str, expert: int, first: int, count: int, payload_budget: int,
                               weights: Optional[np.ndarray] = None, scales: Optional[np.ndarray] = None):
        """(codes uint8 [count, columns/2], scales uint8 [count, columns/32], columns)."""
        if weights is None or scales is None:
            # Size the outputs from the blocks tensor; any problem with it is
            # left for the C call to report, in the reference's order.
            from . import KadanError

            try:
                shape = self.tensor(prefix + "_blocks").shape
                groups, rows = (shape[2], min(count, shape[1])) if len(shape) == 4 else (0, 0)
            except KadanError:
                groups = rows = 0
            weights = np.empty(max(1, rows * groups * 16), dtype=np.uint8)
            scales = np.empty(max(1, rows * groups), dtype=np.uint8)
        cols = c_u64()
        check(lib.kb200_shard_load_mxfp4_expert_rows(self._h, prefix.encode(), expert, first, count, payload_budget,
                                                     weights.ctypes.data, weights.nbytes, scales.ctypes.data,
                                                     scales.nbytes, ctypes.byref(cols)))
        c = int(cols.value)
        return weights[:count * c // 2].reshape(count, c // 2), scales[:count * c // 32].reshape(count, c // 32), c


def _bf16_to_f32(raw: np.ndarray) -> np.ndarray:
    """BF16 bytes -> float32, exactly (the 16 bits become the high half)."""
    return (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)


def _float_tensor(shard: Shard, name: str) -> np.ndarray:
    t = shard.tensor(name)
    raw = shard.read_tensor(name, 0, t.bytes)
    if t.dtype == "BF16":
        return _bf16_to_f32(raw).reshape(t.shape)
    if t.dtype == "F32":
        return raw.view("<f4").reshape(t.shape).copy()
    if t.dtype == "F16":
        return raw.view("<f2").astype(np.float32).reshape(t.shape)
    raise ValueError(f"{name}: {t.dtype} is not a float tensor")


@dataclass
class MoeLayerArrays:
    """One gpt-oss MoE layer in the layout kb200_moe_weights takes (interleaved
    gate/up rows), for experts [first, first + count) of the layer."""

    gate_up_blocks: np.ndarray  # uint8 [E, 2I, H/2]
    gate_up_scales: np.ndarray  # uint8 [E, 2I, H/32]
    down_blocks: np.ndarray     # uint8 [E, H, I/2]
    down_scales: np.ndarray     # uint8 [E, H, I/32]
    gate_up_bias: Optional[np.ndarray]  # float32 [E, 2I]
    down_bias: Optional[np.ndarray]     # float32 [E, H]
    router_weight: Optional[np.ndarray]  # float32 [all experts, H]
    router_bias: Optional[np.ndarray]    # float32 [all experts]
    hidden: int
    inter: int
    first: int
    count: int


def load_moe_layer(shard: Shard, prefix: str, first: int = 0, count: Optional[int] = None,
                   payload_budget: int = 1 << 40) -> MoeLayerArrays:
    """Experts [first, first + count) of the MoE layer under `prefix` (e.g.
    "model.layers.0.mlp"): <prefix>.experts.gate_up_proj_{blocks,scales,bias},
    <prefix>.experts.down_proj_{blocks,scales,bias} and, when present,
    <prefix>.router.{weight,bias}. Each expert's rows are loaded in place by
    kb200_shard_load_mxfp4_expert_rows; biases and the router are widened to
    float32 exactly."""
    gu, dn = prefix + ".experts.gate_up_proj", prefix + ".experts.down_proj"
    gu_shape, dn_shape = shard.tensor(gu + "_blocks").shape, shard.tensor(dn + "_blocks").shape
    if len(gu_shape) != 4 or len(dn_shape) != 4:
        raise ValueError("MXFP4 expert blocks must be [experts, rows, groups, 16]")
    experts, two_i, hidden = gu_shape[0], gu_shape[1], gu_shape[2] * 32
    inter = dn_shape[2] * 32
    if two_i != 2 * inter or dn_shape[:2] != (experts, hidden):
        raise ValueError("gate/up and down expert shapes disagree")
    count = experts - first if count is None else count
    arrays = {}
    for name, rows, cols in ((gu, two_i, hidden), (dn, hidden, inter)):
        blocks = np.empty((count, rows, cols // 2), dtype=np.uint8)
        scales = np.empty((count, rows, cols // 32), dtype=np.uint8)
        for e in range(count):
            shard.load_mxfp4_expert_rows(name, first + e, 0, rows, payload_budget, weights=blocks[e], scales=scales[e])
        arrays[name] = (blocks, scales)

    from . import KadanError

    def optional(name, sl=None):
        try:
            shard.tensor(name)
        except KadanError:  # absent
            return None
        v = _float_tensor(shard, name)
        return v if sl is None else np.ascontiguousarray(v[sl])

    experts_slice = slice(first, first + count)
    return MoeLayerArrays(arrays[gu][0], arrays[gu][1], arrays[dn][0], arrays[dn][1],
                          optional(gu + "_bias", experts_slice), optional(dn + "_bias", experts_slice),
                          optional(prefix + ".router.weight"), optional(prefix + ".router.bias"),
                          hidden, inter, first, count)


__all__ = ["Shard", "ShardTensor", "DTYPES", "MoeLayerArrays", "load_moe_layer"]
