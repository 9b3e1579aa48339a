"""Per-kernel telemetry on the host (no GPU needed): stable kernel ids and
names, phase scoping per thread, and a launch that cannot reach a device is
still counted (with its event pair unavailable), as the reference's
cuda_trace::kernel counts a launch whatever its timing outcome
(IW/src/cuda/cuda_telemetry.cuh:101-160)."""
from __future__ import annotations

import ctypes
import re
import threading

import pytest

from conftest import ROOT

NAMES = [
    "dequant_kernel", "gemv_staged_kernel", "gemv_generic_kernel", "gemv_q4k_mma_kernel", "gemv_q6k_mma_kernel",
    "gemv_q6k_pair_kernel", "prefill_rows_kernel", "gemm_gguf_kernel", "moe_route_kernel", "moe_sort_kernel",
    "moe_gather_kernel", "moe_mtile_kernel", "moe_gemm_kernel", "moe_gemv_kernel", "moe_combine_kernel",
    "rows_regroup_kernel", "mxfp4_ggml_dequant_kernel", "mxfp4_from_ggml_kernel", "peer_allreduce_kernel",
    "ep_exchange_kernel", "rms_norm_kernel", "rope_kernel", "attend_kernel", "attend_combine_kernel",
    "delta_conv_kernel", "delta_l2_kernel", "delta_heads_kernel", "silu_mul_kernel", "moe_shared_kernel",
    "moe_decode_kernel", "pair_quant_kernel", "q4k_quant_kernel",
]


def test_kernel_ids_are_a_fixed_protocol(kb):
    text = (ROOT / "include" / "kadan_b200.h").read_text()
    body = text[text.index("typedef enum kb200_kernel"):text.index("} kb200_kernel;")]
    ids = {name: int(v) for name, v in re.findall(r"(KB200_KERNEL_\w+)\s*=\s*(\d+)", body)}
    assert ids["KB200_KERNEL_COUNT"] == len(NAMES) == kb.KERNEL_COUNT
    assert sorted(v for k, v in ids.items() if k != "KB200_KERNEL_COUNT") == list(range(len(NAMES)))
    assert [kb.kernel_name(i) for i in range(len(NAMES))] == NAMES
    assert kb.kernel_name(len(NAMES)) is None and kb.kernel_name(-1) is None


def test_phase_scope_nests_and_restores(kb):
    outer, inner = kb.Phase(4), kb.Phase()
    with outer:
        with inner:
            pass
        # Back in the outer phase: the thread's current phase is `outer` again.
        prev = ctypes.c_void_p()
        kb.check(kb.lib.kb200_phase_enter(outer.handle, ctypes.byref(prev)))
        assert prev.value == outer.handle.value
        kb.lib.kb200_phase_release(prev)
    snap = outer.snapshot()
    assert snap == {"kernels": {}, "dropped": 0, "unavailable": 0, "shared_batch_size": 4, "observed": False}
    assert inner.snapshot()["shared_batch_size"] == 1
    outer.close()
    inner.close()


def test_phase_is_per_thread(kb):
    ph = kb.Phase()
    seen = []

    def other():
        prev = ctypes.c_void_p()
        kb.check(kb.lib.kb200_phase_enter(None, ctypes.byref(prev)))
        seen.append(prev.value)

    with ph:
        t = threading.Thread(target=other)
        t.start()
        t.join()
    assert seen == [None]


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the launch path without a device")
def test_launch_without_device_is_counted(kb):
    out = (ctypes.c_float * 256)()
    with kb.Phase() as ph:
        s = kb.lib.kb200_gguf_dequant(kb.Q8_0, ctypes.c_void_p(0x10000000), 256, out, None, None)
    assert s != kb.OK
    snap = ph.snapshot()
    k = snap["kernels"]["dequant_kernel"]
    assert k["calls"] == 1 and k["measured"] == 0 and k["host_seconds"] >= 0.0
    assert snap["unavailable"] >= 1 and snap["observed"]
    # Outside any phase nothing is counted.
    kb.lib.kb200_gguf_dequant(kb.Q8_0, ctypes.c_void_p(0x10000000), 256, out, None, None)
    assert ph.snapshot()["kernels"]["dequant_kernel"]["calls"] == 1
    ph.close()
