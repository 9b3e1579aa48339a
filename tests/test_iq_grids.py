"""The grid-coded GGUF formats IQ3_XXS, IQ2_S and IQ3_S on CPU.

The device decoder (kadan_b200/csrc/iq_decode.hpp, used by the dequant and
generic GEMV kernels) is written for host and device alike; here its host
build runs over the reference test's block recipe
(IW/tests/gguf_quantization.cpp:100-165, IW = services/hikari/inference_worker)
with the reference's own code grids, and must equal the reference's
gguf::decode bit for bit (NaN payloads aside) and the golden digests. The
registration rules of kb200_set_iq_grids run in a child process, so this
session's library keeps its unregistered state.
"""
from __future__ import annotations

import json
import shutil
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

IQ = {"iq3_xxs": (4, 98), "iq2_s": (7, 82), "iq3_s": (8, 110)}

HARNESS = r"""
#include <cstddef>
#include "iq_decode.hpp"
extern "C" void product_iq_decode(int e, const uint8_t* blocks, size_t count, float* out, const uint32_t* a,
                                  const unsigned long long* b, const uint32_t* c) {
    const kb200::IqGrids grids{a, b, c};
    const size_t bytes = size_t(kb200::block_bytes(e));
    for (size_t i = 0; i < count; ++i)
        out[i] = kb200::iq::value(e, blocks + i / 256 * bytes, unsigned(i % 256), grids);
}
"""


@pytest.fixture(scope="module")
def product_decode(tmp_path_factory):
    import ctypes

    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("needs a host C++ compiler")
    d = tmp_path_factory.mktemp("iq")
    (d / "harness.cpp").write_text(HARNESS)
    so = d / "libiq.so"
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC",
           f"-I{ROOT / 'kadan_b200' / 'csrc'}", f"-I{ROOT / 'include'}", str(d / "harness.cpp"), "-o", str(so)]
    run = subprocess.run(cmd, capture_output=True, text=True)
    assert run.returncode == 0, run.stderr
    lib = ctypes.CDLL(str(so))
    lib.product_iq_decode.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]

    def decode(e, blocks, grids):
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        out = np.empty(blocks.shape[0] * 256, dtype=np.float32)
        a, b, c = (np.ascontiguousarray(g) for g in grids)
        lib.product_iq_decode(e, blocks.ctypes.data, out.size, out.ctypes.data, a.ctypes.data, b.ctypes.data,
                              c.ctypes.data)
        return out

    return decode


def same_bits(a: np.ndarray, b: np.ndarray) -> None:
    nan = np.isnan(a)
    assert np.array_equal(nan, np.isnan(b))
    assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@pytest.mark.parametrize("name", list(IQ))
def test_device_decoder_source_equals_reference(product_decode, ref, name):
    from golden.make_golden import canonical_digest, reference_blocks

    enc, nbytes = IQ[name]
    grids = ref.iq_grids()
    blocks = reference_blocks(enc, 2048)
    assert blocks.shape[1] == nbytes
    got = product_decode(enc, blocks, grids)
    same_bits(got, ref.decode(enc, blocks, got.size))
    spec = json.loads((GOLDEN / "gguf_blocks.json").read_text())["encodings"][name]
    assert canonical_digest(got) == spec["sha256_expected"]
    assert int(np.isnan(got).sum()) == spec["nan_count"]
    # Every fp16 scale pattern, including subnormals, infinities and NaNs.
    rng = np.random.default_rng(enc)
    sweep = rng.integers(0, 256, (65536, nbytes), dtype=np.uint8)
    halves = np.arange(65536, dtype=np.uint32)
    sweep[:, 0] = halves & 255
    sweep[:, 1] = halves >> 8
    got = product_decode(enc, sweep, grids)
    same_bits(got, ref.decode(enc, sweep, got.size))


def test_registration_rules(kb):
    """Unsupported until registered; the same grids again are accepted, other
    values refused; geometry is reported once supported. In a child process."""
    script = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(ROOT)!r})
        import numpy as np
        import kadan_b200 as kb
        from oracle.pyoracle import REF_LIB, Reference
        grids = Reference().iq_grids() if REF_LIB.exists() else (
            np.arange(256, dtype=np.uint32), np.arange(1024, dtype=np.uint64), np.arange(512, dtype=np.uint32))
        iq = (kb.IQ3_XXS, kb.IQ2_S, kb.IQ3_S)
        assert not any(kb.lib.kb200_encoding_supported(e) for e in iq)
        assert kb.lib.kb200_set_iq_grids(None, None, None) == kb.INVALID
        kb.set_iq_grids(*grids)
        assert all(kb.lib.kb200_encoding_supported(e) for e in iq)
        assert [kb.lib.kb200_block_bytes(e) for e in iq] == [98, 82, 110]
        assert [kb.lib.kb200_block_values(e) for e in iq] == [256] * 3
        kb.set_iq_grids(*grids)
        # Registered, the support predicate agrees with the reference's
        # gguf_batch_supported for these encodings as for the others.
        if REF_LIB.exists():
            import ctypes
            from kadan_b200.weight_bank import SourceJobC, WeightIdentityC, _ROW_SOURCE
            ref = Reference()
            kb.lib.kb200_source_job_supported.argtypes = [ctypes.POINTER(SourceJobC)]
            ident, src, checked = WeightIdentityC(), _ROW_SOURCE(lambda *a: 0), 0
            for e in iq:
                for in_ in (8, 256, 264, 512, 4096, 14336, (16 << 20) // 110 * 256, ((16 << 20) // 82 + 1) * 256):
                    for out, rows in ((1, 1), (19, 3), (5, 4096), (5, 4097)):
                        if in_ * rows > (1 << 24):
                            continue
                        job = SourceJobC(ctypes.pointer(ident), src, None, 0x1000, 0x2000, in_, out, rows, e, 1)
                        got = bool(kb.lib.kb200_source_job_supported(ctypes.byref(job)))
                        assert got == ref.gguf_batch_supported(in_, out, rows, e), (e, in_, out, rows)
                        checked += got
            assert checked > 0
        other = grids[1].copy()
        other[5] ^= 1
        try:
            kb.set_iq_grids(grids[0], other, grids[2])
        except kb.KadanError as e:
            assert e.status == kb.INVALID and "other values" in str(e)
        else:
            raise AssertionError("different grids were accepted")
        print("ok")
    """)
    run = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stdout + run.stderr
