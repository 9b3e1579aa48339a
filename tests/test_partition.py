"""Multi-device column partition (host only) against the reference's own code.

The reference's kadan::gguf_batch_partition / weight_boundary
(IW/include/kadan/gguf_batch_partition.hpp:44-83, device_placement.hpp:76-142,
:341-357) are compiled from its headers into oracle/_ref; the library must
return the same geometry and fail in the same cases. The sweep follows the
reference's own test (IW/tests/gguf_batch_partition.cpp:102-187) and adds
larger capacities, widths and scratch limits.
"""
from __future__ import annotations

import itertools

import numpy as np
import pytest

ENCODINGS = [-1, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9]  # F32 rows, then kadan::gguf::Encoding
CAPACITIES = [[7], [1, 1], [1, 3], [0, 1, 0], [0, 0, 0], [183_359 << 20] * 8,
              [80 << 30, 80 << 30, 40 << 30], [1, 2, 3, 4, 5, 6, 7, 8]]


def test_weight_boundary_matches_reference(kb, ref):
    for caps in CAPACITIES:
        for units in (0, 1, 19, 100, 10003, 28672, 1 << 20, (1 << 40) + 7):
            for index in range(len(caps) + 2):
                assert kb.weight_boundary(units, caps, index) == ref.weight_boundary(units, caps, index)
    # The reference's worked values (IW/tests/worker_compute.cpp:699-704).
    assert kb.weight_boundary(100, [1, 3], 1) == 25 and kb.weight_boundary(100, [3, 1], 1) == 75
    assert kb.weight_boundary(100, [0, 0], 1) == 50 and kb.weight_boundary(100, [1, 3], 2) == 100


@pytest.mark.parametrize("caps", CAPACITIES)
def test_batch_partition_matches_reference(kb, ref, caps):
    limits = [64 << 20, 1 << 30, (16 << 20) + 300, (8 << 20) + 5000, 17 << 20]
    for in_, out, enc, limit in itertools.product([256, 4096, 14336], [1, 19, 10003, 28672], ENCODINGS, limits):
        for device in range(len(caps)):
            want = ref.gguf_batch_partition(in_, out, enc, caps, device, limit)
            if isinstance(want, str):
                with pytest.raises(kb.KadanError) as err:
                    kb.gguf_batch_partition(in_, out, enc, caps, device, limit)
                assert str(err.value).endswith(": " + want), (in_, out, enc, limit, caps, device)
                continue
            got = kb.gguf_batch_partition(in_, out, enc, caps, device, limit)
            assert (got.first, got.count, got.chunk_columns) == want, (in_, out, enc, limit, caps, device)


@pytest.mark.parametrize("caps", CAPACITIES[:5])
def test_partition_covers_every_column_once_and_scatters(kb, caps):
    """Slices are contiguous, in device order, cover [0, out) exactly once, and
    scatter puts each device's local rows back in place (the reference test's
    ownership and scatter checks)."""
    for rows, out in itertools.product([1, 8], [1, 19, 10003]):
        output = np.full((rows, out), -1.0, dtype=np.float32)
        owners = np.zeros(out, dtype=np.int64)
        previous = 0
        for device in range(len(caps)):
            p = kb.gguf_batch_partition(256, out, 1, caps, device, 64 << 20)
            assert p.first == previous == kb.weight_boundary(out, caps, device)
            previous += p.count
            if not p.count:
                assert p.chunk_columns == 0
                continue
            owners[p.first:p.first + p.count] += 1
            local = np.array([[r * out + p.first + c for c in range(p.count)] for r in range(rows)],
                             dtype=np.float32)
            kb.partition_scatter(p, np.ascontiguousarray(local), rows, output, out)
        assert previous == out
        assert np.all(owners == 1)
        assert np.array_equal(output.ravel(), np.arange(rows * out, dtype=np.float32))


def test_source_job_support_matches_reference(kb, ref):
    """kb200_source_job_supported agrees with the reference's
    gguf_batch_supported on every job shape, except for the encodings that
    have no device decoder until their code grids are registered (IQ3_XXS,
    IQ2_S, IQ3_S), which it declines here (registered, they agree too:
    tests/test_iq_grids.py)."""
    import ctypes

    from kadan_b200.weight_bank import SourceJobC, WeightIdentityC, _ROW_SOURCE

    kb.lib.kb200_source_job_supported.argtypes = [ctypes.POINTER(SourceJobC)]
    ident = WeightIdentityC()
    src = _ROW_SOURCE(lambda *a: 0)
    no_decoder = {kb.IQ3_XXS, kb.IQ2_S, kb.IQ3_S}
    checked = 0
    for enc in (kb.F32, kb.Q3_K, kb.Q4_K, kb.Q8_0, kb.Q6_K, kb.IQ3_XXS, kb.IQ4_NL, kb.IQ4_XS, kb.IQ2_S, kb.IQ3_S,
                kb.BF16):
        values = 1 if enc in (kb.F32, kb.BF16) else 32 if enc in (kb.Q8_0, kb.IQ4_NL) else 256
        ins = {8, 32, 40, 256, 264, 4096, 4100, 14336}
        if enc == kb.F32:
            ins |= {4 << 20, (4 << 20) + 8}
        elif values == 256:
            ins |= {(16 << 20) // 144 * 256, ((16 << 20) // 144 + 1) * 256}
        for in_ in sorted(ins):
            for out, rows in ((1, 1), (19, 3), (4096, 8), (5, 4096), (5, 4097)):
                if in_ * rows > (1 << 24):
                    continue
                want = ref.gguf_batch_supported(in_, out, rows, enc)
                job = SourceJobC(ctypes.pointer(ident), src, None, 0x1000, 0x2000, in_, out, rows, enc, 1)
                got = bool(kb.lib.kb200_source_job_supported(ctypes.byref(job)))
                if enc in no_decoder and not kb.lib.kb200_encoding_supported(enc):
                    # Grid-coded encodings before their grids are registered.
                    assert not got
                else:
                    assert got == want, (enc, in_, out, rows, want)
                checked += 1
    assert checked > 300
