"""Test infrastructure only: ctypes bindings of the CPU checkers.

  ORACLE  liboracle.so            this repository's C restatement (oracle.c)
  REF     _ref/libkadan_ref.so    the reference's own ggml / quantization /
                                  CpuMatvec code compiled in place (Makefile)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only to check or time against the CUDA path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libkadan_ref.so"
# The reference checkout the recipes build from: the `reference` directory
# beside this repository, unless KADAN_REFERENCE names another.
REFERENCE_TREE = Path(os.environ.get("KADAN_REFERENCE", HERE.parent.parent / "reference"))

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build(ref: bool = True) -> None:
    """make the oracle (and the reference build when its sources are present)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    if ref and REFERENCE_TREE.exists():
        subprocess.run(["make", "-s", "-j8", "-C", str(HERE), f"REF={REFERENCE_TREE}", "ref"], check=True)
        # The reference's device GEMV (a benchmark baseline only): best effort.
        r = subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REFERENCE_TREE}", "ref-gpu"], capture_output=True,
                           text=True)
        if r.returncode:
            print("oracle: reference GPU baseline not built:", r.stderr[-500:])


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class Oracle:
    def __init__(self, path: Path = ORACLE_LIB):
        if not path.exists():
            build(ref=False)
        L = ctypes.CDLL(str(path))
        L.orc_half.restype = ctypes.c_float
        L.orc_half.argtypes = [ctypes.c_uint16]
        L.orc_decode.restype = ctypes.c_float
        L.orc_decode.argtypes = [ctypes.c_int, _u8p, ctypes.c_size_t]
        L.orc_decode_stream.argtypes = [ctypes.c_int, _u8p, ctypes.c_size_t, _f32p]
        L.orc_block_values.restype = ctypes.c_size_t
        L.orc_block_bytes.restype = ctypes.c_size_t
        L.orc_gemv_f64.argtypes = [ctypes.c_int, _u8p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                   _f32p, ctypes.c_size_t, _f64p, ctypes.c_size_t]
        L.orc_e2m1.restype = ctypes.c_float
        L.orc_mxfp4_decode_rows.argtypes = [ctypes.c_size_t, ctypes.c_size_t, _u8p, _u8p,
                                            ctypes.c_size_t, ctypes.c_size_t, _f32p]
        L.orc_mxfp4_gguf_decode.argtypes = [_u8p, ctypes.c_size_t, _f32p]
        L.orc_moe_route.argtypes = [ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, _f32p, _i32p, _f32p]
        L.orc_moe_forward.argtypes = [ctypes.c_size_t] * 5 + [_f32p, _f32p, _u8p, _u8p, _f32p, _u8p, _u8p, _f32p,
                                                              ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                                              ctypes.c_float, ctypes.c_int, _f32p]
        L.orc_bf16_round.restype = ctypes.c_float
        L.orc_bf16_round.argtypes = [ctypes.c_float]
        L.orc_set_iq_grids.argtypes = [ctypes.c_void_p] * 3
        sz, f32 = ctypes.c_size_t, ctypes.c_float
        L.orc_rms_norm.argtypes = [_f32p, _f32p, sz, sz, f32]
        L.orc_l2_norm.restype = None
        L.orc_l2_norm.argtypes = [_f32p, sz, sz, f32]
        L.orc_rope.restype = None
        L.orc_rope.argtypes = [_f32p, sz, sz, sz, sz, sz, f32]
        _u32p = ctypes.POINTER(ctypes.c_uint32)
        L.orc_attend_cached.argtypes = [_f32p, _f32p, _f32p, sz, sz, sz, sz, sz, f32, _u32p, _u32p, _f32p]
        L.orc_silu_mul.restype = None
        L.orc_silu_mul.argtypes = [_f32p, _f32p, sz, _f32p]
        L.orc_moe_add_shared.restype = None
        L.orc_moe_add_shared.argtypes = [_f32p, _f32p, _f32p, sz, sz, _f32p]
        L.orc_delta_rule.restype = None
        L.orc_delta_rule.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, sz, f32, sz, _f32p]
        L.orc_delta_step.argtypes = [_f32p] * 8 + [sz] * 5 + [f32, ctypes.c_int, _f32p, _f32p, _f32p]
        self.L = L

    def set_iq_grids(self, grids) -> None:
        """Copy the (iq3xxs[256] u32, iq2s[1024] u64, iq3s[512] u32) grids in."""
        a, b, c = (np.ascontiguousarray(g) for g in grids)
        assert a.dtype == np.uint32 and a.size == 256 and b.dtype == np.uint64 and b.size == 1024
        assert c.dtype == np.uint32 and c.size == 512
        self.L.orc_set_iq_grids(a.ctypes.data, b.ctypes.data, c.ctypes.data)

    def half(self, bits: int) -> float:
        return self.L.orc_half(bits)

    def block_values(self, e: int) -> int:
        return int(self.L.orc_block_values(e))

    def block_bytes(self, e: int) -> int:
        return int(self.L.orc_block_bytes(e))

    def decode(self, e: int, packed: np.ndarray, count: int) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        out = np.empty(count, dtype=np.float32)
        self.L.orc_decode_stream(e, _p(packed, _u8p), count, _p(out, _f32p))
        return out

    def gemv_f64(self, e: int, weights: np.ndarray, x: np.ndarray, in_: int, out: int) -> np.ndarray:
        """y[rows, out] in float64 (decode then double dot)."""
        weights = np.ascontiguousarray(weights, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        rows = x.size // in_
        y = np.empty((rows, out), dtype=np.float64)
        row_bytes = weights.size // out
        self.L.orc_gemv_f64(e, _p(weights, _u8p), row_bytes, in_, out, _p(x, _f32p), rows, _p(y, _f64p), out)
        return y

    def mxfp4_decode_rows(self, weights, scales, rows, cols, first=0, count=None) -> np.ndarray:
        count = rows - first if count is None else count
        out = np.empty((count, cols), dtype=np.float32)
        w = np.ascontiguousarray(weights, dtype=np.uint8)
        s = np.ascontiguousarray(scales, dtype=np.uint8)
        rc = self.L.orc_mxfp4_decode_rows(rows, cols, _p(w, _u8p), _p(s, _u8p), first, count, _p(out, _f32p))
        if rc:
            raise ValueError(f"orc_mxfp4_decode_rows failed: {rc}")
        return out

    def mxfp4_gguf_decode(self, blocks: np.ndarray) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        n = blocks.size // 17
        out = np.empty(n * 32, dtype=np.float32)
        self.L.orc_mxfp4_gguf_decode(_p(blocks, _u8p), n, _p(out, _f32p))
        return out

    def moe_route(self, logits: np.ndarray, top_k: int):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        t, e = logits.shape
        chosen = np.empty((t, top_k), dtype=np.int32)
        weight = np.empty((t, top_k), dtype=np.float32)
        self.L.orc_moe_route(t, e, top_k, _p(logits, _f32p), _p(chosen, _i32p), _p(weight, _f32p))
        return chosen, weight

    def moe_forward(self, x, logits, gu_w, gu_s, dn_w, dn_s, *, hidden, inter, experts, top_k,
                    gu_bias=None, dn_bias=None, activation=0, interleaved=1, limit=7.0, alpha=1.702,
                    round_act=1) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        tokens = x.size // hidden
        out = np.empty((tokens, hidden), dtype=np.float32)
        arrs = [np.ascontiguousarray(a, dtype=np.uint8) for a in (gu_w, gu_s, dn_w, dn_s)]
        gb = None if gu_bias is None else np.ascontiguousarray(gu_bias, dtype=np.float32)
        db = None if dn_bias is None else np.ascontiguousarray(dn_bias, dtype=np.float32)
        rc = self.L.orc_moe_forward(
            tokens, hidden, inter, experts, top_k, _p(x, _f32p),
            _p(np.ascontiguousarray(logits, dtype=np.float32), _f32p),
            _p(arrs[0], _u8p), _p(arrs[1], _u8p), None if gb is None else _p(gb, _f32p),
            _p(arrs[2], _u8p), _p(arrs[3], _u8p), None if db is None else _p(db, _f32p),
            activation, interleaved, limit, alpha, round_act, _p(out, _f32p))
        if rc:
            raise ValueError(f"orc_moe_forward failed: {rc}")
        return out

    # ----------------------------------------------------------- layer math
    @staticmethod
    def _f(a) -> np.ndarray:
        return np.ascontiguousarray(a, dtype=np.float32)

    def rms_norm(self, x, weight=None, *, width: int, eps: float) -> np.ndarray:
        y = self._f(x).copy()
        w = None if weight is None else self._f(weight)
        rc = self.L.orc_rms_norm(_p(y, _f32p), None if w is None else _p(w, _f32p), y.size // width, width, eps)
        if rc:
            raise ValueError("gguf_text_norm_nonfinite")
        return y

    def l2_norm(self, x, *, width: int, eps: float) -> np.ndarray:
        y = self._f(x).copy()
        self.L.orc_l2_norm(_p(y, _f32p), y.size // width, width, eps)
        return y

    def rope(self, x, *, rows: int, width: int, rotary: int, position: int, base: float) -> np.ndarray:
        y = self._f(x).copy()
        self.L.orc_rope(_p(y, _f32p), rows, y.size // rows, width, rotary, position, base)
        return y

    def attend_cached(self, q, keys, values, *, rows, position, heads, kv_heads, dim, scale, selected=None,
                      offsets=None) -> np.ndarray:
        q, k, v = self._f(q), self._f(keys), self._f(values)
        out = np.empty(rows * heads * dim, dtype=np.float32)
        u32 = ctypes.POINTER(ctypes.c_uint32)
        sel = None if selected is None else np.ascontiguousarray(selected, dtype=np.uint32)
        off = None if offsets is None else np.ascontiguousarray(offsets, dtype=np.uint32)
        rc = self.L.orc_attend_cached(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), rows, position, heads, kv_heads,
                                      dim, scale, None if sel is None else _p(sel, u32),
                                      None if off is None else _p(off, u32), _p(out, _f32p))
        if rc:
            raise ValueError("gguf_text_attention_shape")
        return out.reshape(rows, heads, dim)

    def silu_mul(self, gate, up) -> np.ndarray:
        g, u = self._f(gate), self._f(up)
        out = np.empty_like(g)
        self.L.orc_silu_mul(_p(g, _f32p), _p(u, _f32p), g.size, _p(out, _f32p))
        return out

    def moe_add_shared(self, x, shared_gate, down, out, *, hidden: int) -> np.ndarray:
        """out + down * sigmoid(shared_gate . x) per token (a new array)."""
        xs, g, d = self._f(x), self._f(shared_gate), self._f(down)
        y = self._f(out).copy()
        self.L.orc_moe_add_shared(_p(xs, _f32p), _p(g, _f32p), _p(d, _f32p), xs.size // hidden, hidden, _p(y, _f32p))
        return y

    def delta_rule(self, state, q, k, v, decay, beta: float) -> np.ndarray:
        """One delta_rule step; `state` (float32, dim*dim) is updated in place."""
        dim = len(q)
        out = np.empty(dim, dtype=np.float32)
        d = self._f(decay)
        qs, ks, vs = self._f(q), self._f(k), self._f(v)
        self.L.orc_delta_rule(_p(state, _f32p), _p(qs, _f32p), _p(ks, _f32p), _p(vs, _f32p), _p(d, _f32p), d.size,
                              beta, dim, _p(out, _f32p))
        return out

    def delta_step(self, qkv, z, alpha, beta, conv, dt, a, norm, *, rows, key_heads, value_heads, dim, kernel, eps,
                   sigmoid_gate, history, state) -> np.ndarray:
        """`history` and `state` (float32 arrays) are updated in place."""
        ins = [self._f(t) for t in (qkv, z, alpha, beta, conv, dt, a, norm)]
        out = np.empty(rows * value_heads * dim, dtype=np.float32)
        rc = self.L.orc_delta_step(*[_p(t, _f32p) for t in ins], rows, key_heads, value_heads, dim, kernel, eps,
                                   int(bool(sigmoid_gate)), _p(history, _f32p), _p(state, _f32p), _p(out, _f32p))
        if rc:
            raise ValueError("gguf_text_delta_shape")
        return out


class Reference:
    """The reference's own CPU code (oracle/_ref/libkadan_ref.so)."""

    def __init__(self, path: Path = REF_LIB):
        if not path.exists():
            build(ref=True)
        if not path.exists():
            raise FileNotFoundError(f"reference build missing: {path}")
        L = ctypes.CDLL(str(path))
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_gguf_decode.restype = ctypes.c_float
        L.ref_gguf_decode.argtypes = [ctypes.c_int, _u8p, ctypes.c_size_t]
        L.ref_gguf_decode_stream.argtypes = [ctypes.c_int, _u8p, ctypes.c_size_t, _f32p]
        L.ref_gguf_decode_run_stream.argtypes = [ctypes.c_int, _u8p, ctypes.c_size_t, _f32p]
        L.ref_gguf_encoding.argtypes = [ctypes.c_uint32]
        L.ref_fp16_to_fp32.restype = ctypes.c_float
        L.ref_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.ref_ggml_row_size.restype = ctypes.c_size_t
        L.ref_ggml_row_size.argtypes = [ctypes.c_uint32, ctypes.c_int64]
        L.ref_ggml_blck_size.restype = ctypes.c_int64
        L.ref_ggml_type_size.restype = ctypes.c_size_t
        L.ref_ggml_to_float.argtypes = [ctypes.c_uint32, ctypes.c_void_p, _f32p, ctypes.c_int64]
        L.ref_ggml_quantize.restype = ctypes.c_size_t
        L.ref_ggml_quantize.argtypes = [ctypes.c_uint32, _f32p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64]
        L.ref_mxfp4_decode_rows.argtypes = [ctypes.c_size_t, ctypes.c_size_t, _u8p, _u8p,
                                            ctypes.c_size_t, ctypes.c_size_t, _f32p]
        L.ref_mxfp4_matvec.argtypes = [ctypes.c_size_t, ctypes.c_size_t, _u8p, _u8p, _f32p, _f32p]
        L.ref_cpu_matvec_supported.argtypes = [ctypes.c_uint32, ctypes.c_size_t]
        L.ref_cpu_matvec_create.restype = ctypes.c_void_p
        L.ref_cpu_matvec_create.argtypes = [ctypes.c_uint32, _f32p, ctypes.c_size_t, ctypes.c_size_t]
        L.ref_cpu_matvec_destroy.argtypes = [ctypes.c_void_p]
        L.ref_cpu_matvec_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                         ctypes.c_size_t, _f32p, ctypes.c_size_t]
        L.ref_cpu_matvec_parallel.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, _f32p,
                                              ctypes.c_size_t, ctypes.c_int]
        L.ref_weight_boundary.restype = ctypes.c_size_t
        L.ref_weight_boundary.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t,
                                          ctypes.c_size_t]
        L.ref_gguf_batch_partition.argtypes = [ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int,
                                               ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t, ctypes.c_size_t,
                                               ctypes.c_uint64, ctypes.POINTER(ctypes.c_size_t)]
        L.ref_gguf_batch_supported.argtypes = [ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int]
        vp, u64p = ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)
        L.ref_gguf_checkpoint_open.restype = vp
        L.ref_gguf_checkpoint_open.argtypes = [ctypes.c_char_p]
        L.ref_gguf_checkpoint_close.argtypes = [vp]
        L.ref_gguf_checkpoint_tensor_count.restype = ctypes.c_size_t
        L.ref_gguf_checkpoint_tensor_count.argtypes = [vp]
        L.ref_gguf_checkpoint_tensor.argtypes = [vp, ctypes.c_char_p, u64p]
        L.ref_gguf_checkpoint_tensor_name.restype = ctypes.c_char_p
        L.ref_gguf_checkpoint_tensor_name.argtypes = [vp, ctypes.c_size_t]
        L.ref_gguf_checkpoint_identity.argtypes = [vp, ctypes.c_char_p, ctypes.c_uint64, u64p]
        L.ref_gguf_checkpoint_read_packed_rows.argtypes = [vp, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_uint64,
                                                           vp, ctypes.c_size_t]
        L.ref_gguf_checkpoint_check_unchanged.argtypes = [vp]
        L.ref_gguf_checkpoint_read_vector.argtypes = [vp, ctypes.c_char_p, _f32p, ctypes.c_size_t]
        L.ref_gguf_checkpoint_integer.argtypes = [vp, ctypes.c_char_p, u64p]
        L.ref_gguf_checkpoint_number.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]
        L.ref_gguf_checkpoint_boolean.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]
        L.ref_gguf_checkpoint_string.restype = ctypes.c_int64
        L.ref_gguf_checkpoint_string.argtypes = [vp, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
        L.ref_gguf_checkpoint_has.argtypes = [vp, ctypes.c_char_p]
        L.ref_shard_open.restype = vp
        L.ref_shard_open.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
        L.ref_shard_close.argtypes = [vp]
        L.ref_shard_tensor_count.restype = ctypes.c_size_t
        L.ref_shard_tensor_count.argtypes = [vp]
        L.ref_shard_tensor_at.argtypes = [vp, ctypes.c_size_t, u64p, ctypes.POINTER(ctypes.c_void_p),
                                          ctypes.POINTER(ctypes.c_size_t)]
        L.ref_shard_identity.argtypes = [vp, ctypes.c_char_p, u64p]
        L.ref_shard_read_tensor.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t, vp, ctypes.c_size_t]
        L.ref_shard_check_unchanged.argtypes = [vp]
        L.ref_shard_load_mxfp4_expert_rows.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_size_t,
                                                       ctypes.c_size_t, ctypes.c_size_t, vp, ctypes.c_size_t, vp,
                                                       ctypes.c_size_t, u64p]
        self.L = L

    # -- kadan::checkpoint::Shard (IW/src/weights/checkpoint.cpp)
    def shard_open(self, root: str, name: str):
        h = self.L.ref_shard_open(str(root).encode(), name.encode())
        return h if h else self.error()

    def shard_close(self, h) -> None:
        self.L.ref_shard_close(h)

    def shard_tensors(self, h) -> dict:
        """name -> (dtype index, rank, bytes, shape tuple), in the reader's order."""
        out = {}
        for i in range(int(self.L.ref_shard_tensor_count(h))):
            info, name, n = (ctypes.c_uint64 * 11)(), ctypes.c_void_p(), ctypes.c_size_t()
            if self.L.ref_shard_tensor_at(h, i, info, ctypes.byref(name), ctypes.byref(n)):
                raise RuntimeError(self.error())
            key = ctypes.string_at(name, n.value).decode()
            rank = int(info[1])
            out[key] = (int(info[0]), rank, int(info[2]), tuple(int(v) for v in info[3:3 + rank]))
        return out

    def shard_identity(self, h, name: str):
        ident = (ctypes.c_uint64 * 9)()
        if self.L.ref_shard_identity(h, name.encode(), ident):
            return self.error()
        return tuple(int(v) for v in ident)

    def shard_read_tensor(self, h, name: str, offset: int, nbytes: int):
        buf = np.zeros(max(1, nbytes), dtype=np.uint8)
        if self.L.ref_shard_read_tensor(h, name.encode(), offset, buf.ctypes.data, nbytes):
            return self.error()
        return buf[:nbytes]

    def shard_check_unchanged(self, h):
        return None if self.L.ref_shard_check_unchanged(h) == 0 else self.error()

    def shard_load_mxfp4_expert_rows(self, h, prefix: str, expert: int, first: int, count: int, budget: int,
                                     capacity: int = 1 << 24):
        """(weights uint8, scales uint8, rows, columns), or the reference's exception text."""
        w, sc, shape = np.zeros(capacity, np.uint8), np.zeros(capacity, np.uint8), (ctypes.c_uint64 * 2)()
        if self.L.ref_shard_load_mxfp4_expert_rows(h, prefix.encode(), expert, first, count, budget,
                                                   w.ctypes.data, capacity, sc.ctypes.data, capacity, shape):
            return self.error()
        rows, cols = int(shape[0]), int(shape[1])
        return w[:rows * cols // 2], sc[:rows * cols // 32], rows, cols

    def gguf_batch_supported(self, in_: int, out: int, rows: int, encoding: int) -> bool:
        return bool(self.L.ref_gguf_batch_supported(in_, out, rows, encoding))

    # -- kadan::checkpoint::GgufCheckpoint (IW/src/weights/gguf_checkpoint.cpp)
    def gguf_open(self, root: str):
        """A checkpoint handle, or the reference's exception text (str)."""
        h = self.L.ref_gguf_checkpoint_open(str(root).encode())
        return h if h else self.error()

    def gguf_close(self, h) -> None:
        self.L.ref_gguf_checkpoint_close(h)

    def gguf_tensors(self, h) -> dict:
        """name -> (shape[3], rank, ggml type, bytes), in the reader's order."""
        out = {}
        for i in range(int(self.L.ref_gguf_checkpoint_tensor_count(h))):
            name = self.L.ref_gguf_checkpoint_tensor_name(h, i)
            info = (ctypes.c_uint64 * 6)()
            if self.L.ref_gguf_checkpoint_tensor(h, name, info):
                raise RuntimeError(self.error())
            out[name.decode()] = (tuple(int(v) for v in info[:3]), int(info[3]), int(info[4]), int(info[5]))
        return out

    def gguf_identity(self, h, name: str, expert: int = 0):
        ident = (ctypes.c_uint64 * 9)()
        if self.L.ref_gguf_checkpoint_identity(h, name.encode(), expert, ident):
            return self.error()
        return tuple(int(v) for v in ident)

    def gguf_read_packed_rows(self, h, name: str, expert: int, first_row: int, nbytes: int):
        buf = np.zeros(nbytes, dtype=np.uint8)
        if self.L.ref_gguf_checkpoint_read_packed_rows(h, name.encode(), expert, first_row,
                                                       buf.ctypes.data if nbytes else None, nbytes):
            return self.error()
        return buf

    def gguf_read_vector(self, h, name: str, count: int):
        out = np.zeros(max(1, count), dtype=np.float32)
        if self.L.ref_gguf_checkpoint_read_vector(h, name.encode(), _p(out, _f32p), count):
            return self.error()
        return out[:count]

    def gguf_check_unchanged(self, h):
        return None if self.L.ref_gguf_checkpoint_check_unchanged(h) == 0 else self.error()

    def gguf_integer(self, h, key: str):
        v = ctypes.c_uint64()
        return self.error() if self.L.ref_gguf_checkpoint_integer(h, key.encode(), ctypes.byref(v)) else int(v.value)

    def gguf_number(self, h, key: str):
        v = ctypes.c_double()
        return self.error() if self.L.ref_gguf_checkpoint_number(h, key.encode(), ctypes.byref(v)) else v.value

    def gguf_boolean(self, h, key: str):
        v = ctypes.c_int()
        return self.error() if self.L.ref_gguf_checkpoint_boolean(h, key.encode(), ctypes.byref(v)) else bool(v.value)

    def gguf_string(self, h, key: str):
        buf = ctypes.create_string_buffer(1 << 20)
        n = self.L.ref_gguf_checkpoint_string(h, key.encode(), buf, len(buf))
        return self.error() if n < 0 else buf.raw[:n].decode()

    def gguf_has(self, h, key: str) -> bool:
        return bool(self.L.ref_gguf_checkpoint_has(h, key.encode()))

    def error(self) -> str:
        return self.L.ref_last_error().decode(errors="replace")

    def weight_boundary(self, units: int, capacities, index: int) -> int:
        caps = (ctypes.c_uint64 * max(1, len(capacities)))(*capacities)
        return int(self.L.ref_weight_boundary(units, caps, len(capacities), index))

    def gguf_batch_partition(self, in_: int, out: int, encoding: int, capacities, device: int, scratch_limit: int):
        """(first, count, chunk_columns), or the reference's exception text."""
        caps = (ctypes.c_uint64 * max(1, len(capacities)))(*capacities)
        res = (ctypes.c_size_t * 3)()
        if self.L.ref_gguf_batch_partition(in_, out, encoding, caps, len(capacities), device, scratch_limit, res):
            return self.error()
        return tuple(int(v) for v in res)

    def decode(self, e: int, packed: np.ndarray, count: int) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        out = np.empty(count, dtype=np.float32)
        self.L.ref_gguf_decode_stream(e, _p(packed, _u8p), count, _p(out, _f32p))
        return out

    def iq_grids(self):
        """The reference's IQ3_XXS, IQ2_S and IQ3_S code grids, copied out:
        (uint32[256], uint64[1024], uint32[512])."""
        ptrs = [ctypes.c_void_p() for _ in range(3)]
        self.L.ref_iq_grids(*(ctypes.byref(p) for p in ptrs))
        out = []
        for p, n, t in zip(ptrs, (256, 1024, 512), (ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32)):
            out.append(np.ctypeslib.as_array((t * n).from_address(p.value)).copy())
        return tuple(out)

    def decode_runs(self, e: int, packed: np.ndarray, count: int) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        out = np.empty(count, dtype=np.float32)
        self.L.ref_gguf_decode_run_stream(e, _p(packed, _u8p), count, _p(out, _f32p))
        return out

    def to_float(self, ggml_type: int, packed: np.ndarray, count: int) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        out = np.empty(count, dtype=np.float32)
        self.L.ref_ggml_to_float(ggml_type, packed.ctypes.data, _p(out, _f32p), count)
        return out

    def quantize(self, ggml_type: int, values: np.ndarray, rows: int, per_row: int) -> np.ndarray:
        values = np.ascontiguousarray(values, dtype=np.float32)
        out = np.zeros(rows * self.L.ref_ggml_row_size(ggml_type, per_row), dtype=np.uint8)
        self.L.ref_ggml_quantize(ggml_type, _p(values, _f32p), out.ctypes.data, rows, per_row)
        return out.reshape(rows, -1)

    def row_size(self, ggml_type: int, n: int) -> int:
        return int(self.L.ref_ggml_row_size(ggml_type, n))

    def mxfp4_decode_rows(self, weights, scales, rows, cols, first=0, count=None) -> np.ndarray:
        count = rows - first if count is None else count
        out = np.empty((count, cols), dtype=np.float32)
        w = np.ascontiguousarray(weights, dtype=np.uint8)
        s = np.ascontiguousarray(scales, dtype=np.uint8)
        if self.L.ref_mxfp4_decode_rows(rows, cols, _p(w, _u8p), _p(s, _u8p), first, count, _p(out, _f32p)):
            raise ValueError(self.error())
        return out

    def mxfp4_matvec(self, weights, scales, rows, cols, x) -> np.ndarray:
        out = np.empty(rows, dtype=np.float32)
        w = np.ascontiguousarray(weights, dtype=np.uint8)
        s = np.ascontiguousarray(scales, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        if self.L.ref_mxfp4_matvec(rows, cols, _p(w, _u8p), _p(s, _u8p), _p(x, _f32p), _p(out, _f32p)):
            raise ValueError(self.error())
        return out

    def cpu_matvec(self, ggml_type: int, weights: np.ndarray, x: np.ndarray, in_: int, out: int,
                   threads: int = 1) -> np.ndarray:
        """kadan::text::CpuMatvec over 64-column units on `threads` workers."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        rows = x.size // in_
        h = self.L.ref_cpu_matvec_create(ggml_type, _p(x, _f32p), in_, rows)
        if not h:
            raise ValueError(self.error())
        try:
            y = np.empty((rows, out), dtype=np.float32)
            w = np.ascontiguousarray(weights, dtype=np.uint8)
            rc = self.L.ref_cpu_matvec_parallel(h, w.ctypes.data, w.size // out, _p(y, _f32p), out, threads)
            if rc:
                raise ValueError(self.error())
            return y
        finally:
            self.L.ref_cpu_matvec_destroy(h)


def xorshift32_stream(state: int, n: int) -> np.ndarray:
    """The reference tests' xorshift32 generator (tests/gguf_quantization.cpp:93-98)."""
    out = np.empty(n, dtype=np.uint32)
    s = state & 0xFFFFFFFF
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        out[i] = s
    return out
