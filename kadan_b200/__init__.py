"""kadan_b200: the B200 (sm_100a) quantized-weight linear path.

Python host mirror of the C ABI in include/kadan_b200.h. It exposes the
operations of the Hikari worker's DenseCompute path
(services/hikari/inference_worker/include/kadan/dense_compute.hpp) over
device tensors:

    gguf_dequant(encoding, packed, count, out)      gguf_decode_kernel
    gguf_gemv_batch([GemvJob, ...])                  dense_gguf_batch's launch
    Context.dense_gguf_batch(jobs)                   host-span batch (sync)
    gguf_gemm(job, workspace)                        prefill projection
    moe_forward(weights, x, logits)                  MXFP4 MoE layer

and, in submodules: weight_bank (DeviceWeights and the packed-source batch),
gguf_file (GgufCheckpoint), shard (the safetensors Shard with MXFP4 expert
rows), tensor_parallel / expert_parallel / collectives (one process per GPU).

Every call goes through libkadan_b200.so. There is no CPU or PyTorch
fallback: if the library cannot be loaded the import fails.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libkadan_b200.so"

# kadan::gguf::Encoding numbering (gguf_quantization.hpp:16-27); F32 = no encoding.
F32, Q3_K, Q4_K, Q8_0, Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS, IQ2_S, IQ3_S, BF16 = -1, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9
ENCODING_NAMES = {F32: "f32", Q3_K: "q3_k", Q4_K: "q4_k", Q8_0: "q8_0", Q6_K: "q6_k",
                  IQ4_NL: "iq4_nl", IQ4_XS: "iq4_xs", BF16: "bf16"}
# ggml type ids of the same encodings (gguf_quantization.hpp:30-55).
GGML_TYPE = {Q8_0: 8, Q3_K: 11, Q4_K: 12, Q6_K: 14, IQ4_NL: 20, IQ4_XS: 23, BF16: 30, F32: 0}

(OK, UNSUPPORTED, INVALID, CUDA, NONFINITE_WEIGHT, NONFINITE_INPUT, ALIAS, CANCELLED, TIMEOUT, NO_MEMORY,
 QUARANTINED, IO, NONFINITE_BIAS, NONFINITE_OUTPUT) = range(14)
BATCH_ROWS = 8
BATCH_MAX_ROWS = 4096


class KadanError(RuntimeError):
    """A failed kb200 call. `status` is the kb200_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Unsupported(KadanError):
    """ProjectionResult::unsupported: nothing was read or written."""


class GemvJob(ctypes.Structure):
    """kb200_gemv_job (the reference's MatvecJob, h3_compute.cu:110-121)."""

    _fields_ = [
        ("weights", ctypes.c_void_p),
        ("input", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("row_bytes", ctypes.c_size_t),
        ("stride", ctypes.c_size_t),
        ("in_", ctypes.c_uint32),
        ("columns", ctypes.c_uint32),
        ("rows", ctypes.c_uint32),
        ("encoding", ctypes.c_int32),
    ]


class HostJob(ctypes.Structure):
    """kb200_host_job (DenseCompute::GgufBatchJob over resident weights)."""

    _fields_ = [
        ("weights", ctypes.c_void_p),
        ("input", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("row_bytes", ctypes.c_size_t),
        ("in_", ctypes.c_uint32),
        ("out", ctypes.c_uint32),
        ("rows", ctypes.c_uint32),
        ("encoding", ctypes.c_int32),
        ("validated", ctypes.c_int32),
    ]


class ContextCounters(ctypes.Structure):
    """kb200_context_counters: work a context's calls issued (cumulative)."""

    _fields_ = [("calls", ctypes.c_uint64), ("gemm_launches", ctypes.c_uint64), ("gemv_batches", ctypes.c_uint64),
                ("gemm_fallbacks", ctypes.c_uint64)]


KERNEL_COUNT = 32


class KernelMetrics(ctypes.Structure):
    """kb200_kernel_metrics: one kernel id's launches in a phase."""

    _fields_ = [("calls", ctypes.c_uint64), ("host_seconds", ctypes.c_double), ("measured", ctypes.c_uint64),
                ("gpu_seconds", ctypes.c_double)]


class PhaseMetrics(ctypes.Structure):
    """kb200_phase_metrics."""

    _fields_ = [("kernels", KernelMetrics * KERNEL_COUNT), ("dropped", ctypes.c_uint64),
                ("unavailable", ctypes.c_uint64), ("shared_batch_size", ctypes.c_uint64), ("observed", ctypes.c_int32)]


class DeltaArgs(ctypes.Structure):
    """kb200_delta_args (device pointers)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("qkv", "z", "alpha", "beta", "conv", "dt", "a", "norm", "history",
                                               "state", "output")] + \
               [(n, ctypes.c_uint32) for n in ("rows", "key_heads", "value_heads", "dim", "kernel")] + \
               [("eps", ctypes.c_float), ("sigmoid_gate", ctypes.c_int32)]


RESULT_UNSUPPORTED, RESULT_UNVALIDATED, RESULT_FINITE = 0, 1, 2
MOE_SWIGLU_OAI, MOE_SILU = 0, 1


class MoeWeights(ctypes.Structure):
    """kb200_moe_weights (device pointers to MXFP4 expert tensors)."""

    _fields_ = [
        ("gate_up_blocks", ctypes.c_void_p),
        ("gate_up_scales", ctypes.c_void_p),
        ("gate_up_bias", ctypes.c_void_p),
        ("down_blocks", ctypes.c_void_p),
        ("down_scales", ctypes.c_void_p),
        ("down_bias", ctypes.c_void_p),
        ("hidden", ctypes.c_int32),
        ("inter", ctypes.c_int32),
        ("experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("interleaved", ctypes.c_int32),
        ("limit", ctypes.c_float),
        ("alpha", ctypes.c_float),
    ]


def _load() -> ctypes.CDLL:
    if os.environ.get("KADAN_B200_NO_BUILD") != "1":
        from . import build as _build

        if _build.stale():
            _build.build()
    if not LIB_PATH.exists():
        raise ImportError(f"kadan_b200: CUDA library missing at {LIB_PATH}")
    lib = ctypes.CDLL(str(LIB_PATH))
    c_int, c_size, vp = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p
    lib.kb200_status_name.restype = ctypes.c_char_p
    lib.kb200_status_name.argtypes = [c_int]
    lib.kb200_last_error.restype = ctypes.c_char_p
    lib.kb200_last_error.argtypes = []
    lib.kb200_version.restype = c_int
    lib.kb200_encoding_supported.argtypes = [c_int]
    lib.kb200_block_values.restype = c_size
    lib.kb200_block_values.argtypes = [c_int]
    lib.kb200_block_bytes.restype = c_size
    lib.kb200_block_bytes.argtypes = [c_int]
    lib.kb200_gguf_dequant.argtypes = [c_int, vp, c_size, vp, vp, vp]
    lib.kb200_set_iq_grids.argtypes = [vp, vp, vp]
    lib.kb200_gguf_gemv_batch.argtypes = [ctypes.POINTER(GemvJob), c_size, vp]
    lib.kb200_gemv_path.argtypes = [ctypes.POINTER(GemvJob)]
    lib.kb200_gguf_gemm_workspace_bytes.restype = c_size
    lib.kb200_gguf_gemm_workspace_bytes.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    lib.kb200_gguf_gemm.argtypes = [ctypes.POINTER(GemvJob), vp, c_size, vp]
    lib.kb200_gguf_gemm_supported.argtypes = [ctypes.POINTER(GemvJob)]
    lib.kb200_gguf_gemm_range_offset.restype = c_size
    lib.kb200_gguf_gemm_range_offset.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    lib.kb200_context_counters_get.argtypes = [vp, ctypes.POINTER(ContextCounters)]
    lib.kb200_rms_norm.argtypes = [vp, vp, c_size, c_size, ctypes.c_float, vp, vp, vp]
    lib.kb200_l2_norm.argtypes = [vp, c_size, c_size, ctypes.c_float, vp, vp]
    lib.kb200_rope.argtypes = [vp, c_size, c_size, c_size, c_size, c_size, ctypes.c_float, vp]
    lib.kb200_attend_supported.argtypes = [c_size, c_size, c_size]
    lib.kb200_attend_workspace_bytes.restype = c_size
    lib.kb200_attend_workspace_bytes.argtypes = [c_size, c_size, c_size, c_size]
    lib.kb200_attend_cached.argtypes = [vp, vp, vp, c_size, c_size, c_size, c_size, c_size, ctypes.c_float, vp, vp,
                                        vp, vp, c_size, vp]
    lib.kb200_delta_supported.argtypes = [ctypes.c_uint32] * 4
    lib.kb200_delta_workspace_bytes.restype = c_size
    lib.kb200_delta_workspace_bytes.argtypes = [ctypes.POINTER(DeltaArgs)]
    lib.kb200_delta_step.argtypes = [ctypes.POINTER(DeltaArgs), vp, c_size, vp]
    lib.kb200_phase_create.argtypes = [ctypes.c_uint64, ctypes.POINTER(vp)]
    lib.kb200_phase_enter.argtypes = [vp, ctypes.POINTER(vp)]
    lib.kb200_phase_snapshot.argtypes = [vp, ctypes.POINTER(PhaseMetrics)]
    lib.kb200_phase_release.restype = None
    lib.kb200_phase_release.argtypes = [vp]
    lib.kb200_kernel_name.restype = ctypes.c_char_p
    lib.kb200_kernel_name.argtypes = [c_int]
    lib.kb200_weight_boundary.restype = c_size
    lib.kb200_weight_boundary.argtypes = [c_size, ctypes.POINTER(ctypes.c_uint64), c_size, c_size]
    lib.kb200_gguf_batch_partition.argtypes = [c_size, c_size, c_int, ctypes.POINTER(ctypes.c_uint64), c_size,
                                               c_size, ctypes.c_uint64, vp]
    lib.kb200_partition_scatter.restype = None
    lib.kb200_partition_scatter.argtypes = [vp, vp, c_size, vp, c_size]
    lib.kb200_take_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    lib.kb200_context_create.argtypes = [c_int, ctypes.POINTER(vp)]
    lib.kb200_context_destroy.argtypes = [vp]
    lib.kb200_context_destroy.restype = None
    lib.kb200_context_stream.argtypes = [vp]
    lib.kb200_context_stream.restype = vp
    lib.kb200_context_set_read_lanes.argtypes = [vp, c_int]
    lib.kb200_weights_upload.argtypes = [vp, vp, c_size, ctypes.POINTER(vp)]
    lib.kb200_weights_free.argtypes = [vp, vp]
    lib.kb200_dense_gguf_batch.argtypes = [vp, ctypes.POINTER(HostJob), c_size, ctypes.POINTER(ctypes.c_ubyte),
                                           ctypes.POINTER(c_int)]
    lib.kb200_moe_workspace_bytes.restype = c_size
    lib.kb200_moe_workspace_bytes.argtypes = [ctypes.POINTER(MoeWeights), c_size]
    lib.kb200_moe_forward.argtypes = [ctypes.POINTER(MoeWeights), vp, vp, c_size, vp, vp, c_size, vp, vp]
    lib.kb200_moe_route.argtypes = [vp, c_size, ctypes.c_int32, ctypes.c_int32, vp, vp, vp]
    return lib


lib = _load()


def check(status: int) -> None:
    if status == OK:
        return
    message = lib.kb200_last_error().decode(errors="replace")
    if status == UNSUPPORTED:
        raise Unsupported(status, message)
    raise KadanError(status, message)


def block_values(encoding: int) -> int:
    return int(lib.kb200_block_values(encoding))


def block_bytes(encoding: int) -> int:
    return int(lib.kb200_block_bytes(encoding))


def row_bytes(encoding: int, in_: int) -> int:
    return in_ // block_values(encoding) * block_bytes(encoding)


def _stream_ptr(stream) -> Optional[int]:
    import torch

    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def set_iq_grids(iq3xxs, iq2s, iq3s) -> None:
    """kb200_set_iq_grids: the IQ3_XXS, IQ2_S and IQ3_S code grids (host
    arrays of uint32[256], uint64[1024], uint32[512]), after which those
    encodings decode on the device."""
    import numpy as np

    a, b, c = (np.ascontiguousarray(g) for g in (iq3xxs, iq2s, iq3s))
    if not (a.dtype == np.uint32 and a.size == 256 and b.dtype == np.uint64 and b.size == 1024
            and c.dtype == np.uint32 and c.size == 512):
        raise ValueError("IQ code grids: uint32[256], uint64[1024], uint32[512]")
    check(lib.kb200_set_iq_grids(a.ctypes.data, b.ctypes.data, c.ctypes.data))


def gguf_dequant(encoding: int, packed, count: int, out, status=None, stream=None) -> None:
    """out[:count] = exact decode of `packed` (device tensors)."""
    check(lib.kb200_gguf_dequant(encoding, _ptr(packed), count, _ptr(out), _ptr(status), _stream_ptr(stream)))


def gemv_job(encoding: int, weights, x, y, *, in_: int, columns: int, rows: int,
             row_bytes_: Optional[int] = None, stride: Optional[int] = None, status=None) -> GemvJob:
    rb = row_bytes_ if row_bytes_ is not None else (in_ * 4 if encoding == F32 else row_bytes(encoding, in_))
    job = GemvJob(_ptr(weights), _ptr(x), _ptr(y), _ptr(status), rb,
                  columns if stride is None else stride, in_, columns, rows, encoding)
    job._keep = (weights, x, y, status)  # the job holds raw pointers: keep the tensors alive with it
    return job


def gguf_gemv_batch(jobs: Sequence[GemvJob], stream=None) -> None:
    arr = (GemvJob * len(jobs))(*jobs)
    check(lib.kb200_gguf_gemv_batch(arr, len(jobs), _stream_ptr(stream)))


def gemm_workspace_bytes(rows: int, in_: int) -> int:
    return int(lib.kb200_gguf_gemm_workspace_bytes(rows, in_))


def gemm_supported(job: GemvJob) -> bool:
    """kb200_gguf_gemm_supported: the prefill GEMM takes the job's weights."""
    return bool(lib.kb200_gguf_gemm_supported(ctypes.byref(job)))


def gemm_range_offset(rows: int, in_: int) -> int:
    """Byte offset in the GEMM workspace of its fp16-range word."""
    return int(lib.kb200_gguf_gemm_range_offset(rows, in_))


def gguf_gemm(job: GemvJob, workspace, stream=None) -> None:
    """Prefill GEMM of one Q4_K, Q6_K or Q8_0 job (all of job.rows at once) on the tensor cores."""
    check(lib.kb200_gguf_gemm(ctypes.byref(job), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                              _stream_ptr(stream)))


class Partition(ctypes.Structure):
    _fields_ = [("first", ctypes.c_size_t), ("count", ctypes.c_size_t), ("chunk_columns", ctypes.c_size_t)]


def weight_boundary(units: int, capacities, index: int) -> int:
    caps = (ctypes.c_uint64 * max(1, len(capacities)))(*capacities)
    return int(lib.kb200_weight_boundary(units, caps, len(capacities), index))


def gguf_batch_partition(in_: int, out: int, encoding: int, capacities, device: int, scratch_limit: int) -> Partition:
    """Column slice and chunk width of device `device` (the worker's multi-device split)."""
    caps = (ctypes.c_uint64 * max(1, len(capacities)))(*capacities)
    p = Partition()
    check(lib.kb200_gguf_batch_partition(in_, out, encoding, caps, len(capacities), device, scratch_limit,
                                         ctypes.byref(p)))
    return p


def partition_scatter(p: Partition, local, rows: int, output, out: int) -> None:
    """Host fp32 arrays (numpy): output[r, first + c] = local[r, c]."""
    lib.kb200_partition_scatter(ctypes.byref(p), local.ctypes.data, rows, output.ctypes.data, out)


def gemv_path(job: GemvJob) -> int:
    return int(lib.kb200_gemv_path(ctypes.byref(job)))


def take_device_error() -> int:
    v = ctypes.c_uint(0)
    lib.kb200_take_device_error(ctypes.byref(v))
    return int(v.value)


def gguf_gemv(encoding: int, weights, x, *, in_: int, columns: int, out=None, status=None, stream=None):
    """y[rows, columns] = x[rows, in] @ decode(W[columns, in])^T on the device."""
    import torch

    rows = x.numel() // in_
    if out is None:
        out = torch.empty(rows, columns, dtype=torch.float32, device=x.device)
    gguf_gemv_batch([gemv_job(encoding, weights, x, out, in_=in_, columns=columns, rows=rows, status=status)], stream)
    return out


class Context:
    """kb200_context: the synchronous host-span boundary on one device."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib.kb200_context_create(device, ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self) -> None:
        if self.handle:
            lib.kb200_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream_ptr(self) -> int:
        return int(lib.kb200_context_stream(self.handle))

    def counters(self) -> dict:
        """kb200_context_counters_get: calls, GEMM launches, GEMV batches, GEMM fallbacks so far."""
        c = ContextCounters()
        check(lib.kb200_context_counters_get(self.handle, ctypes.byref(c)))
        return {name: int(getattr(c, name)) for name, _ in ContextCounters._fields_}

    def set_read_lanes(self, lanes: int) -> None:
        """Host threads (caller included) that read packed-row sources."""
        check(lib.kb200_context_set_read_lanes(self.handle, lanes))

    def upload(self, host_bytes) -> int:
        """Copy a host numpy array into a new device allocation; returns its address."""
        import numpy as np

        a = np.ascontiguousarray(host_bytes)
        p = ctypes.c_void_p()
        check(lib.kb200_weights_upload(self.handle, a.ctypes.data, a.nbytes, ctypes.byref(p)))
        return int(p.value)

    def free(self, ptr: int) -> None:
        check(lib.kb200_weights_free(self.handle, ptr))

    def dense_gguf_batch(self, jobs: Sequence[HostJob], cancel: Optional[ctypes.c_ubyte] = None) -> int:
        """Returns RESULT_UNVALIDATED; raises Unsupported / KadanError like the reference throws.
        `cancel`: a ctypes.c_ubyte another thread may set (the worker's atomic_bool)."""
        arr = (HostJob * len(jobs))(*jobs)
        result = ctypes.c_int(0)
        check(lib.kb200_dense_gguf_batch(self.handle, arr, len(jobs),
                                         None if cancel is None else ctypes.byref(cancel), ctypes.byref(result)))
        return int(result.value)


def host_job(encoding: int, weights_ptr: int, x, y, *, in_: int, out: int, validated: bool = False,
             row_bytes_: Optional[int] = None) -> HostJob:
    """x: float32 numpy [rows, in]; y: float32 numpy [rows, out] (written)."""
    rows = x.size // in_
    rb = row_bytes_ if row_bytes_ is not None else (in_ * 4 if encoding == F32 else row_bytes(encoding, in_))
    return HostJob(weights_ptr, x.ctypes.data, y.ctypes.data, rb, in_, out, rows, encoding, int(validated))


def moe_weights(gu_blocks, gu_scales, dn_blocks, dn_scales, *, hidden: int, inter: int, experts: int, top_k: int,
                gu_bias=None, dn_bias=None, activation: int = MOE_SWIGLU_OAI, interleaved: bool = True,
                limit: float = 7.0, alpha: float = 1.702) -> MoeWeights:
    """Device tensors in the MXFP4 expert layout (blocks [E, rows, cols/2], scales [E, rows, cols/32])."""
    return MoeWeights(_ptr(gu_blocks), _ptr(gu_scales), _ptr(gu_bias), _ptr(dn_blocks), _ptr(dn_scales),
                      _ptr(dn_bias), hidden, inter, experts, top_k, activation, int(interleaved), limit, alpha)


def moe_workspace_bytes(w: MoeWeights, tokens: int) -> int:
    return int(lib.kb200_moe_workspace_bytes(ctypes.byref(w), tokens))


def moe_forward(w: MoeWeights, x_bf16, logits, out=None, workspace=None, status=None, stream=None):
    """out[T, hidden] fp32 = MXFP4 MoE layer of bf16 x [T, hidden] routed by fp32 logits [T, experts]."""
    import torch

    tokens = x_bf16.shape[0]
    if out is None:
        out = torch.empty(tokens, w.hidden, dtype=torch.float32, device=x_bf16.device)
    need = moe_workspace_bytes(w, tokens)
    if workspace is None:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=x_bf16.device)
    check(lib.kb200_moe_forward(ctypes.byref(w), _ptr(x_bf16), _ptr(logits), tokens, _ptr(out), _ptr(workspace),
                                workspace.numel(), _ptr(status), _stream_ptr(stream)))
    return out


def moe_route(logits, top_k: int, stream=None):
    import torch

    tokens, experts = logits.shape
    chosen = torch.empty(tokens, top_k, dtype=torch.int32, device=logits.device)
    weight = torch.empty(tokens, top_k, dtype=torch.float32, device=logits.device)
    check(lib.kb200_moe_route(_ptr(logits), tokens, experts, top_k, _ptr(chosen), _ptr(weight), _stream_ptr(stream)))
    return chosen, weight


def moe_forward_noalloc(w: MoeWeights, x_bf16, logits, out=None, status=None, stream=None):
    """kb200_moe_forward_noalloc: the MoE layer on the library's fixed 16 MiB
    device scratch, for callers that cannot allocate per call."""
    import torch

    tokens = x_bf16.shape[0]
    if out is None:
        out = torch.empty(tokens, w.hidden, dtype=torch.float32, device=x_bf16.device)
    check(lib.kb200_moe_forward_noalloc(ctypes.byref(w), _ptr(x_bf16), _ptr(logits), tokens, _ptr(out), _ptr(status),
                                        _stream_ptr(stream)))
    return out


class MoeDispatch(ctypes.Structure):
    """kb200_moe_dispatch: device pointers into the dispatch workspace."""

    _fields_ = [("offsets", ctypes.c_void_p), ("pos", ctypes.c_void_p), ("weight", ctypes.c_void_p),
                ("rows", ctypes.c_void_p), ("count", ctypes.c_size_t)]


lib.kb200_moe_dispatch_workspace_bytes.restype = ctypes.c_size_t
lib.kb200_moe_dispatch_workspace_bytes.argtypes = [ctypes.c_size_t, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
lib.kb200_moe_dispatch_rows.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.POINTER(MoeDispatch), ctypes.c_void_p, ctypes.c_void_p]
lib.kb200_moe_experts_workspace_bytes.restype = ctypes.c_size_t
lib.kb200_moe_experts_workspace_bytes.argtypes = [ctypes.POINTER(MoeWeights), ctypes.c_size_t]
lib.kb200_moe_experts.argtypes = [ctypes.POINTER(MoeWeights), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
lib.kb200_moe_combine.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32,
                                  ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
lib.kb200_rows_regroup.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                   ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]


def moe_dispatch_rows(logits, x_bf16, top_k: int, workspace, status=None, stream=None) -> MoeDispatch:
    """Route, sort by expert and gather fp16 rows (kb200_moe_dispatch_rows)."""
    tokens, experts = logits.shape
    d = MoeDispatch()
    check(lib.kb200_moe_dispatch_rows(_ptr(logits), _ptr(x_bf16), tokens, x_bf16.shape[1], experts, top_k,
                                      _ptr(workspace), workspace.numel(), ctypes.byref(d), _ptr(status),
                                      _stream_ptr(stream)))
    return d


def moe_experts(w: MoeWeights, rows_f16, offsets, y, workspace, status=None, stream=None) -> None:
    """y[r] = expert FFN of rows grouped by expert (kb200_moe_experts)."""
    check(lib.kb200_moe_experts(ctypes.byref(w), _ptr(rows_f16), _ptr(offsets), rows_f16.shape[0], _ptr(y),
                                _ptr(workspace), workspace.numel(), _ptr(status), _stream_ptr(stream)))


def moe_combine(y, weight_ptr: int, pos_ptr: int, tokens: int, top_k: int, out, stream=None) -> None:
    check(lib.kb200_moe_combine(_ptr(y), weight_ptr, pos_ptr, tokens, top_k, out.shape[1], _ptr(out),
                                _stream_ptr(stream)))


def rows_regroup(src, dst, segments, max_rows: int, stream=None) -> None:
    """dst rows [d, d+n) = src rows [s, s+n) per segment row {s, d, n} (device int64 [count, 3])."""
    row_bytes = src.shape[1] * src.element_size()
    check(lib.kb200_rows_regroup(_ptr(src), _ptr(dst), row_bytes, _ptr(segments), segments.shape[0], max_rows,
                                 _stream_ptr(stream)))


lib.kb200_mxfp4_ggml_dequant.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
lib.kb200_mxfp4_from_ggml.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]
MXFP4_GGML_BLOCK_BYTES = 17


def mxfp4_ggml_dequant(blocks, count: int, out, stream=None) -> None:
    """out[:32 count] (fp32) = ggml's decode of `count` GGUF MXFP4 blocks (device tensors)."""
    check(lib.kb200_mxfp4_ggml_dequant(_ptr(blocks), count, _ptr(out), _stream_ptr(stream)))


def mxfp4_from_ggml(blocks, experts: int, rows: int, cols: int, codes, scales, dst_rows: int, first_row: int = 0,
                    stream=None) -> None:
    """GGUF MXFP4 rows [experts][rows][cols/32 blocks] into rows [first_row, first_row + rows)
    of the expert layout codes [experts][dst_rows][cols/2], scales [experts][dst_rows][cols/32]."""
    check(lib.kb200_mxfp4_from_ggml(_ptr(blocks), experts, rows, cols, _ptr(codes), _ptr(scales), dst_rows, first_row,
                                    _stream_ptr(stream)))


lib.kb200_moe_forward_f32.argtypes = [ctypes.POINTER(MoeWeights), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
lib.kb200_moe_forward_host.argtypes = [ctypes.c_void_p, ctypes.POINTER(MoeWeights), ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(ctypes.c_ubyte),
                                       ctypes.POINTER(ctypes.c_int)]


def rms_norm(x, weight, *, width: int, eps: float, out=None, status=None, stream=None):
    """kb200_rms_norm over rows of `width` (weight None: unweighted); out may be x."""
    import torch

    out = torch.empty_like(x) if out is None else out
    check(lib.kb200_rms_norm(x.data_ptr(), _ptr(weight), x.numel() // width, width, eps, out.data_ptr(),
                             _ptr(status), _stream_ptr(stream)))
    return out


def l2_norm(x, *, width: int, eps: float, out=None, stream=None):
    import torch

    out = torch.empty_like(x) if out is None else out
    check(lib.kb200_l2_norm(x.data_ptr(), x.numel() // width, width, eps, out.data_ptr(), _stream_ptr(stream)))
    return out


def rope(x, *, rows: int, width: int, rotary: int, position: int, base: float, stream=None):
    """kb200_rope in place on x ([rows][heads * width])."""
    check(lib.kb200_rope(x.data_ptr(), rows, x.numel() // rows, width, rotary, position, base, _stream_ptr(stream)))
    return x


def attend_cached(q, keys, values, *, rows: int, position: int, heads: int, kv_heads: int, dim: int, scale: float,
                  selected=None, offsets=None, out=None, stream=None):
    """kb200_attend_cached on device tensors; returns out [rows, heads, dim]."""
    import torch

    out = torch.empty(rows, heads, dim, device=q.device) if out is None else out
    ws = torch.empty(max(1, lib.kb200_attend_workspace_bytes(rows, position, heads, dim)), dtype=torch.uint8,
                     device=q.device)
    check(lib.kb200_attend_cached(q.data_ptr(), keys.data_ptr(), values.data_ptr(), rows, position, heads, kv_heads,
                                  dim, scale, _ptr(selected), _ptr(offsets), out.data_ptr(), ws.data_ptr(),
                                  ws.numel(), _stream_ptr(stream)))
    return out


def delta_step(*, qkv, z, alpha, beta, conv, dt, a, norm, history, state, output, rows: int, key_heads: int,
               value_heads: int, dim: int, kernel: int, eps: float, sigmoid_gate: bool, stream=None) -> None:
    """kb200_delta_step on device tensors (history and state updated in place)."""
    import torch

    args = DeltaArgs(qkv.data_ptr(), z.data_ptr(), alpha.data_ptr(), beta.data_ptr(), conv.data_ptr(), dt.data_ptr(),
                     a.data_ptr(), norm.data_ptr(), _ptr(history), state.data_ptr(), output.data_ptr(), rows,
                     key_heads, value_heads, dim, kernel, eps, int(bool(sigmoid_gate)))
    ws = torch.empty(max(1, lib.kb200_delta_workspace_bytes(ctypes.byref(args))), dtype=torch.uint8,
                     device=qkv.device)
    check(lib.kb200_delta_step(ctypes.byref(args), ws.data_ptr(), ws.numel(), _stream_ptr(stream)))


def kernel_name(kernel: int):
    """Stable name of a telemetry kernel id, or None."""
    name = lib.kb200_kernel_name(kernel)
    return name.decode() if name is not None else None


class Phase:
    """A telemetry phase (kb200_phase): while entered (a `with` block) every
    launch the library issues on this thread is counted and timed."""

    def __init__(self, shared_batch_size: int = 1):
        h = ctypes.c_void_p()
        check(lib.kb200_phase_create(shared_batch_size, ctypes.byref(h)))
        self.handle = h
        self._previous = []

    def __enter__(self):
        prev = ctypes.c_void_p()
        check(lib.kb200_phase_enter(self.handle, ctypes.byref(prev)))
        self._previous.append(prev)
        return self

    def __exit__(self, *exc):
        prev = self._previous.pop()
        check(lib.kb200_phase_enter(prev, None))
        if prev:
            lib.kb200_phase_release(prev)
        return False

    def snapshot(self) -> dict:
        """Counters by kernel name (only ids with calls), plus dropped,
        unavailable, shared_batch_size and observed."""
        m = PhaseMetrics()
        check(lib.kb200_phase_snapshot(self.handle, ctypes.byref(m)))
        kernels = {}
        for i in range(KERNEL_COUNT):
            k = m.kernels[i]
            if k.calls or k.measured:
                kernels[kernel_name(i)] = {"calls": int(k.calls), "host_seconds": float(k.host_seconds),
                                           "measured": int(k.measured), "gpu_seconds": float(k.gpu_seconds)}
        return {"kernels": kernels, "dropped": int(m.dropped), "unavailable": int(m.unavailable),
                "shared_batch_size": int(m.shared_batch_size), "observed": bool(m.observed)}

    def close(self) -> None:
        if self.handle:
            lib.kb200_phase_release(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def moe_forward_host(ctx: "Context", w: MoeWeights, x, logits, out=None, cancel=None) -> tuple:
    """kb200_moe_forward_host: the layer on host fp32 arrays (numpy x [T, H],
    logits [T, E]); returns (out, result). Raises Unsupported when the
    caller's own path must take the layer."""
    import numpy as np

    x = np.ascontiguousarray(x, dtype=np.float32)
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    tokens = x.shape[0]
    if out is None:
        out = np.empty((tokens, w.hidden), dtype=np.float32)
    result = ctypes.c_int(0)
    check(lib.kb200_moe_forward_host(ctx.handle, ctypes.byref(w), x.ctypes.data, logits.ctypes.data, tokens,
                                     out.ctypes.data, None if cancel is None else ctypes.byref(cancel),
                                     ctypes.byref(result)))
    return out, int(result.value)


lib.kb200_moe_forward_noalloc.argtypes = [ctypes.POINTER(MoeWeights), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
STATIC_MOE_SCRATCH_BYTES = 16 << 20


class DeltaHost(ctypes.Structure):
    """kb200_delta_host (host pointers)."""

    _fields_ = [("layer", ctypes.c_uint64), ("fresh", ctypes.c_int32)] + \
               [(n, ctypes.c_void_p) for n in ("qkv", "z", "alpha", "beta", "conv", "dt", "a", "norm")] + \
               [(n, ctypes.c_uint32) for n in ("rows", "key_heads", "value_heads", "dim", "kernel")] + \
               [("eps", ctypes.c_float), ("sigmoid_gate", ctypes.c_int32), ("output", ctypes.c_void_p),
                ("initial_state", ctypes.c_void_p), ("initial_history", ctypes.c_void_p)]


_vp = ctypes.c_void_p
lib.kb200_attend_cached_host.argtypes = [_vp, ctypes.c_uint64, _vp, _vp, _vp] + [ctypes.c_size_t] * 5 + \
    [ctypes.c_float, _vp, _vp, _vp, _vp]
lib.kb200_delta_step_host.argtypes = [_vp, ctypes.POINTER(DeltaHost), _vp]
lib.kb200_recurrent_state_get.argtypes = [_vp, ctypes.c_uint64, _vp, ctypes.c_size_t, _vp, ctypes.c_size_t]
lib.kb200_context_release_layers.argtypes = [_vp]


def _f32(a):
    import numpy as np

    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def attend_cached_host(ctx: "Context", layer: int, q, keys, values, *, rows: int, position: int, heads: int,
                       kv_heads: int, dim: int, scale: float, selected=None, offsets=None, cancel=None):
    """kb200_attend_cached_host on host arrays; returns out [rows, heads, dim]."""
    import numpy as np

    q, keys, values = _f32(q), _f32(keys), _f32(values)
    out = np.empty((rows, heads, dim), dtype=np.float32)
    sel = None if selected is None else np.ascontiguousarray(selected, dtype=np.uint32)
    off = None if offsets is None else np.ascontiguousarray(offsets, dtype=np.uint32)
    check(lib.kb200_attend_cached_host(ctx.handle, layer, q.ctypes.data, keys.ctypes.data, values.ctypes.data, rows,
                                       position, heads, kv_heads, dim, scale,
                                       None if sel is None else sel.ctypes.data,
                                       None if off is None else off.ctypes.data, out.ctypes.data,
                                       None if cancel is None else ctypes.byref(cancel)))
    return out


def delta_step_host(ctx: "Context", layer: int, *, fresh: bool, qkv, z, alpha, beta, conv, dt, a, norm, rows: int,
                    key_heads: int, value_heads: int, dim: int, kernel: int, eps: float, sigmoid_gate: bool,
                    initial_state=None, initial_history=None, cancel=None):
    """kb200_delta_step_host on host arrays; returns the output [rows, value_heads * dim]."""
    import numpy as np

    keep = [_f32(t) for t in (qkv, z, alpha, beta, conv, dt, a, norm)]
    init = [_f32(initial_state), _f32(initial_history)]
    out = np.empty((rows, value_heads * dim), dtype=np.float32)
    st = DeltaHost(layer, int(bool(fresh)), *[t.ctypes.data for t in keep], rows, key_heads, value_heads, dim,
                   kernel, eps, int(bool(sigmoid_gate)), out.ctypes.data,
                   *[None if t is None else t.ctypes.data for t in init])
    check(lib.kb200_delta_step_host(ctx.handle, ctypes.byref(st), None if cancel is None else ctypes.byref(cancel)))
    return out


def recurrent_state_get(ctx: "Context", layer: int, state_floats: int, history_floats: int):
    """kb200_recurrent_state_get: (state, history) of the layer as host arrays."""
    import numpy as np

    state = np.empty(state_floats, dtype=np.float32)
    history = np.empty(max(history_floats, 1), dtype=np.float32)
    check(lib.kb200_recurrent_state_get(ctx.handle, layer, state.ctypes.data, state_floats, history.ctypes.data,
                                        history_floats))
    return state, history[:history_floats]


def release_layers(ctx: "Context") -> None:
    """kb200_context_release_layers."""
    check(lib.kb200_context_release_layers(ctx.handle))


lib.kb200_silu_mul.argtypes = [_vp, _vp, ctypes.c_size_t, _vp, _vp]
lib.kb200_moe_add_shared.argtypes = [_vp, _vp, _vp, ctypes.c_size_t, ctypes.c_size_t, _vp, _vp]


def silu_mul(gate, up, out=None, stream=None):
    """kb200_silu_mul on device tensors: silu(gate) * up."""
    import torch

    out = torch.empty_like(gate) if out is None else out
    check(lib.kb200_silu_mul(gate.data_ptr(), up.data_ptr(), gate.numel(), out.data_ptr(), _stream_ptr(stream)))
    return out


def moe_add_shared(x, shared_gate, down, out, stream=None) -> None:
    """kb200_moe_add_shared: out += down * sigmoid(shared_gate . x) per token (device tensors, in place)."""
    hidden = shared_gate.numel()
    check(lib.kb200_moe_add_shared(x.data_ptr(), shared_gate.data_ptr(), down.data_ptr(), x.numel() // hidden, hidden,
                                   out.data_ptr(), _stream_ptr(stream)))
