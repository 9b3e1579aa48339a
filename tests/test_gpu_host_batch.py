"""GPU tests of the host-span boundary: kb200_dense_gguf_batch over resident
weights, the CUDA weight bank, and kb200_dense_gguf_source_batch (bank hits,
streamed misses through the two staging halves, admission after the finite
check), against the pinned oracle. Tolerance 1e-3 as max|y - ref| /
max(max|ref|, 1) (IW/tests/gguf_text.cpp:247-250)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


class DeviceBytes:
    """A uint8 view of `n` device bytes at `ptr` for torch.as_tensor."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def device_bytes(ptr, n):
    import torch

    return torch.as_tensor(DeviceBytes(ptr, n), device="cuda:0").cpu().numpy()


def weights(kb, enc, out, in_, seed):
    from kadan_b200 import synth

    if enc == kb.F32:
        rng = np.random.default_rng(seed)
        return (rng.standard_normal((out, in_)) * 0.05).astype(np.float32).view(np.uint8).reshape(out, -1)
    return synth.gguf(enc, out, in_, seed=seed)


def reference(kb, oracle, enc, w, x, in_, out):
    if enc == kb.F32:
        return x.astype(np.float64) @ w.view(np.float32).reshape(out, in_).astype(np.float64).T
    return oracle.gemv_f64(enc, w, x, in_, out)


def test_dense_gguf_batch_parity_and_errors(kb, oracle, cuda):
    from kadan_b200 import synth

    ctx = kb.Context(0)
    try:
        cases = [(kb.Q4_K, 4096, 1024, 1), (kb.Q6_K, 4096, 512, 2), (kb.Q8_0, 2048, 300, 3), (kb.F32, 256, 64, 1)]
        ptrs, jobs, want = [], [], []
        for i, (enc, in_, out, rows) in enumerate(cases):
            w = weights(kb, enc, out, in_, seed=10 + i)
            x = synth.activations(rows * in_, seed=20 + i, dtype="f32").reshape(rows, in_)
            y = np.full((rows, out), np.nan, dtype=np.float32)
            p = ctx.upload(w)
            ptrs.append(p)
            jobs.append((kb.host_job(enc, p, x, y, in_=in_, out=out), x, y))
            want.append(reference(kb, oracle, enc, w, x, in_, out))
        assert ctx.dense_gguf_batch([j for j, _, _ in jobs]) == kb.RESULT_UNVALIDATED
        for (_, _, y), ref in zip(jobs, want):
            assert rel_err(y, ref) < TOL
        # Errors: non-finite input, aliasing output, cancel, unsupported shape.
        j0, x0, y0 = jobs[0]
        x0[0, 5] = np.inf
        with pytest.raises(kb.KadanError) as e:
            ctx.dense_gguf_batch([j0])
        assert e.value.status == kb.NONFINITE_INPUT
        x0[0, 5] = 0.0
        alias = kb.HostJob(j0.weights, j0.input, j0.input, j0.row_bytes, j0.in_, 8, 1, j0.encoding, 0)
        with pytest.raises(kb.KadanError) as e:
            ctx.dense_gguf_batch([alias])
        assert e.value.status == kb.ALIAS
        with pytest.raises(kb.KadanError) as e:
            ctx.dense_gguf_batch([j0], cancel=ctypes.c_ubyte(1))
        assert e.value.status == kb.CANCELLED
        bad = kb.HostJob(j0.weights, j0.input, j0.output, j0.row_bytes, 100, j0.out, 1, j0.encoding, 0)
        with pytest.raises(kb.Unsupported):
            ctx.dense_gguf_batch([bad])
    finally:
        for p in ptrs:
            ctx.free(p)
        ctx.close()


def test_cuda_bank_round_trip(cuda):
    import torch

    from kadan_b200.weight_bank import ENVELOPE, WeightBank, WeightIdentity, WeightKey

    bank = WeightBank.cuda(0, 8 << 20)
    try:
        rng = np.random.default_rng(3)
        host = rng.integers(0, 256, size=3 * (1 << 20) + 100, dtype=np.uint8)
        k = WeightKey(WeightIdentity(inode=5), 0, host.size, 1)
        p = bank.retain(k, host.ctypes.data, host.size)
        assert p and bank.find(k) == p and p % 256 == 0
        assert np.array_equal(device_bytes(p, host.size), host)
        dev = torch.from_numpy(rng.integers(0, 256, size=(1 << 20) + 48, dtype=np.uint8)).to(cuda)
        kd = WeightKey(WeightIdentity(inode=6), 0, dev.numel() // 16, 16)
        q = bank.retain_device(kd, dev.data_ptr(), dev.numel())
        assert q and np.array_equal(device_bytes(q, dev.numel()), dev.cpu().numpy())
        assert bank.allocated() == host.size + dev.numel()
        big = WeightKey(WeightIdentity(inode=7), 0, 5 << 20, 1)
        assert bank.retain_device(big, dev.data_ptr(), 5 << 20) is None and bank.last_refusal == ENVELOPE
        assert bank.release_sources([WeightIdentity(inode=5)]) == host.size
        assert bank.find(k) is None and bank.find(kd) == q
        bank.release()
        assert bank.allocated() == 0 and bank.reserved() == 0
    finally:
        bank.close()


def source_jobs(kb, oracle, specs):
    """SourceJobs over numpy packed rows; returns (jobs, references)."""
    from kadan_b200 import synth
    from kadan_b200.weight_bank import SourceJob, WeightIdentity

    jobs, refs = [], []
    for i, (enc, in_, out, rows) in enumerate(specs):
        w = weights(kb, enc, out, in_, seed=40 + i)
        x = synth.activations(rows * in_, seed=50 + i, dtype="f32").reshape(rows, in_)
        y = np.full((rows, out), np.nan, dtype=np.float32)
        row_bytes = w.shape[1]

        def read(first_row, nbytes, w=w, row_bytes=row_bytes):
            assert nbytes % row_bytes == 0
            return w[first_row:first_row + nbytes // row_bytes]

        jobs.append(SourceJob(WeightIdentity(device=9, inode=100 + i, payload_end=w.nbytes), read, x, y, in_, out,
                              enc))
        refs.append(reference(kb, oracle, enc, w, x, in_, out))
    return jobs, refs


def rows_read(job):
    """How many times each packed row of the job was read from its source."""
    import kadan_b200 as kb

    rb = job.in_ * 4 if job.encoding == kb.F32 else kb.row_bytes(job.encoding, job.in_)
    counts = np.zeros(job.out, dtype=np.int64)
    for first, n in job.reads:
        assert n % rb == 0
        counts[first:first + n // rb] += 1
    return counts


# Q8_0 4096 x 8192: 4352-byte rows, chunks of 3855 columns (three chunks, each
# nearly a whole staging half: three groups over both halves); Q4_K 4096 x
# 14336: two chunks; Q6_K one chunk; F32 rows.
SPECS = [(2, 4096, 8192, 1), (1, 4096, 14336, 2), (3, 4096, 4096, 1), (-1, 512, 96, 3)]


def test_source_batch_streams_then_hits(kb, oracle, cuda):
    from kadan_b200.weight_bank import WeightBank, dense_gguf_source_batch

    jobs, refs = source_jobs(kb, oracle, SPECS)
    ctx = kb.Context(0)
    bank = WeightBank.cuda(0, 256 << 20)
    try:
        assert dense_gguf_source_batch(ctx, bank, jobs) == kb.RESULT_UNVALIDATED
        for job, ref in zip(jobs, refs):
            assert rel_err(job.y, ref) < TOL
        # Every packed row is read exactly once; with the default four read
        # lanes a chunk of 2 MiB or more is read in four row runs.
        assert all((rows_read(j) == 1).all() for j in jobs)
        assert [len(j.reads) for j in jobs] == [12, 8, 4, 1]
        total = sum(j.y.shape[1] * (j.in_ * 4 if j.encoding == kb.F32 else kb.row_bytes(j.encoding, j.in_))
                    for j in jobs)
        assert bank.entries() == 7 and bank.allocated() == total
        # Second call: every chunk is a bank hit, no source is read.
        for j in jobs:
            j.reads.clear()
            j.y[:] = np.nan
        assert dense_gguf_source_batch(ctx, bank, jobs) == kb.RESULT_UNVALIDATED
        assert all(not j.reads for j in jobs)
        for job, ref in zip(jobs, refs):
            assert rel_err(job.y, ref) < TOL
    finally:
        bank.close()
        ctx.close()


def test_source_batch_without_retention(kb, oracle, cuda):
    from kadan_b200.weight_bank import WeightBank, dense_gguf_source_batch

    jobs, refs = source_jobs(kb, oracle, SPECS[:2])
    jobs[1].retain_misses = False
    ctx = kb.Context(0)
    small = WeightBank.cuda(0, 20 << 20)
    try:
        for bank in (None, small):
            for j in jobs:
                j.reads.clear()
                j.y[:] = np.nan
            dense_gguf_source_batch(ctx, bank, jobs)
            for job, ref in zip(jobs, refs):
                assert rel_err(job.y, ref) < TOL
            assert all((rows_read(j) == 1).all() for j in jobs)
        # Q8_0 chunks 1 (16.8 MB) and 3 (2.1 MB) fit the envelope, chunk 2 is
        # refused; the Q4_K job keeps nothing.
        assert small.entries() == 2 and small.allocated() == (3855 + 482) * 4352
        # The next call hits those two chunks and streams the rest.
        for j in jobs:
            j.reads.clear()
        dense_gguf_source_batch(ctx, small, jobs)
        q8 = rows_read(jobs[0])
        assert (q8[3855:7710] == 1).all() and q8[:3855].sum() == 0 and q8[7710:].sum() == 0
        assert (rows_read(jobs[1]) == 1).all()
        for job, ref in zip(jobs, refs):
            assert rel_err(job.y, ref) < TOL
    finally:
        small.close()
        ctx.close()


def test_source_batch_failures_keep_nothing(kb, oracle, cuda):
    from kadan_b200.weight_bank import WeightBank, dense_gguf_source_batch

    jobs, _ = source_jobs(kb, oracle, [SPECS[0]])
    job = jobs[0]
    ctx = kb.Context(0)
    bank = WeightBank.cuda(0, 256 << 20)
    try:
        # A non-finite scale in the second chunk: the call fails, the first
        # chunk (finite, finished before it) may be kept, the bad one never is.
        w = job.read(0, 8192 * 4352).copy()
        w[5000, 0:2] = np.frombuffer(np.float16(np.inf).tobytes(), dtype=np.uint8)
        job.read = lambda first, n: w[first:first + n // 4352]
        y_before = job.y.copy()
        with pytest.raises(kb.KadanError) as e:
            dense_gguf_source_batch(ctx, bank, jobs)
        assert e.value.status == kb.NONFINITE_WEIGHT
        assert np.array_equal(np.isnan(job.y), np.isnan(y_before))
        assert bank.entries() <= 1
        from kadan_b200.weight_bank import WeightKey

        second = WeightKey(job.identity, 3855 * 128, 3855 * 128, 34)
        assert bank.find(second) is None
        # Cancellation raised while a source is read.
        cancel = ctypes.c_ubyte(0)

        def cancelling(first, n):
            cancel.value = 1
            return w[first:first + n // 4352]

        job.read = cancelling
        with pytest.raises(kb.KadanError) as e:
            dense_gguf_source_batch(ctx, bank, jobs, cancel=cancel)
        assert e.value.status == kb.CANCELLED
        # A failing source fails the call.
        job.read = lambda first, n: b"short"
        with pytest.raises(kb.KadanError):
            dense_gguf_source_batch(ctx, None, jobs)
    finally:
        bank.close()
        ctx.close()


def test_source_batch_read_lanes(kb, oracle, cuda):
    from kadan_b200.weight_bank import dense_gguf_source_batch

    jobs, refs = source_jobs(kb, oracle, [SPECS[0]])
    job = jobs[0]
    ctx = kb.Context(0)
    try:
        for bad in (0, 65):
            with pytest.raises(kb.KadanError) as e:
                ctx.set_read_lanes(bad)
            assert e.value.status == kb.INVALID
        for lanes, pieces in ((1, 3), (8, 24), (4, 12)):
            ctx.set_read_lanes(lanes)
            job.reads.clear()
            job.y[:] = np.nan
            dense_gguf_source_batch(ctx, None, jobs)
            assert rel_err(job.y, refs[0]) < TOL
            assert len(job.reads) == pieces and (rows_read(job) == 1).all()
            if lanes == 1:
                assert [r[0] for r in job.reads] == [0, 3855, 7710]
    finally:
        ctx.close()


def test_source_batch_reads_a_gguf_checkpoint(kb, oracle, cuda, tmp_path):
    """Packed rows read from a GGUF file by the library's own source
    (kb200_gguf_rows_source, on the read team's threads) give the oracle's
    outputs, first streamed, then from the bank."""
    from kadan_b200 import gguf_write as gw
    from kadan_b200 import synth
    from kadan_b200.gguf_file import GgufCheckpoint
    from kadan_b200.weight_bank import SourceJob, WeightBank, dense_gguf_source_batch

    # (name, encoding, ggml type, in, out): Q4_K in 2 chunks (7281 + 911
    # columns), Q8_0 in 2 chunks (3855 + 241).
    specs = [("blk.0.ffn_up.weight", kb.Q4_K, 12, 4096, 8192), ("blk.0.attn_q.weight", kb.Q8_0, 8, 4096, 4096)]
    weights = {name: synth.gguf(enc, out, in_, seed=60 + i) for i, (name, enc, _, in_, out) in enumerate(specs)}
    root = tmp_path / "ckpt"
    root.mkdir()
    gw.write_arrays(root / "model.gguf", [("general.architecture", gw.STRING, "llama")],
                    [(name, [in_, out], gtype, weights[name]) for name, _, gtype, in_, out in specs])
    ckpt = GgufCheckpoint(root)
    jobs, refs = [], []
    for i, (name, enc, _, in_, out) in enumerate(specs):
        x = synth.activations(in_, seed=70 + i, dtype="f32").reshape(1, in_)
        jobs.append(SourceJob(ckpt.identity(name), ckpt.rows(name), x, np.full((1, out), np.nan, np.float32), in_,
                              out, enc))
        refs.append(oracle.gemv_f64(enc, weights[name], x, in_, out))
    ctx = kb.Context(0)
    bank = WeightBank.cuda(0, 256 << 20)
    try:
        for _ in range(2):
            for j in jobs:
                j.y[:] = np.nan
            assert dense_gguf_source_batch(ctx, bank, jobs) == kb.RESULT_UNVALIDATED
            for j, ref in zip(jobs, refs):
                assert rel_err(j.y, ref) < TOL
        assert bank.entries() == 4
    finally:
        bank.close()
        ctx.close()
        ckpt.close()


def test_single_source_projection_with_bias(kb, oracle, cuda):
    """kb200_dense_gguf_source: bias added once per output, outputs certified
    finite; a non-finite bias and `precise` stop the call before any read."""
    from kadan_b200.weight_bank import WeightBank, dense_gguf_source

    jobs, refs = source_jobs(kb, oracle, [(kb.Q8_0, 2048, 300, 3)])
    job = jobs[0]
    bias = np.linspace(-1, 1, 300).astype(np.float32)
    ctx = kb.Context(0)
    bank = WeightBank.cuda(0, 64 << 20)
    try:
        assert dense_gguf_source(ctx, bank, job, bias=bias) == kb.RESULT_FINITE
        assert rel_err(job.y, refs[0] + bias) < TOL
        job.reads.clear()
        bad = bias.copy()
        bad[7] = np.nan
        with pytest.raises(kb.KadanError) as e:
            dense_gguf_source(ctx, bank, job, bias=bad)
        assert e.value.status == kb.NONFINITE_BIAS
        with pytest.raises(kb.Unsupported):
            dense_gguf_source(ctx, bank, job, bias=bias, precise=True)
        assert not job.reads
        # Served from the bank on the second call.
        assert dense_gguf_source(ctx, bank, job) == kb.RESULT_FINITE
        assert not job.reads and rel_err(job.y, refs[0]) < TOL
    finally:
        bank.close()
        ctx.close()


@pytest.mark.parametrize("enc,in_,out", [(1, 4096, 512), (3, 4096, 256), (2, 4096, 384)], ids=["q4_k", "q6_k", "q8_0"])
def test_prefill_through_dense_gguf_source(kb, oracle, cuda, enc, in_, out):
    """A T = 512 prefill through kb200_dense_gguf_source, the worker's own
    prefill call (IW/src/models/text/gguf_weights.cpp:570-582), runs on the
    tensor-core GEMM: one GEMM launch per chunk and no GEMV batch, when the
    rows stream from their source and again when they are bank hits; the
    outputs match the oracle (1e-3)."""
    from kadan_b200.weight_bank import WeightBank, dense_gguf_source

    jobs, refs = source_jobs(kb, oracle, [(enc, in_, out, 512)])
    job = jobs[0]
    ctx = kb.Context(0)
    bank = WeightBank.cuda(0, 64 << 20)
    try:
        before = ctx.counters()
        assert dense_gguf_source(ctx, bank, job) == kb.RESULT_FINITE
        after = ctx.counters()
        assert after["gemm_launches"] - before["gemm_launches"] == 1
        assert after["gemv_batches"] == before["gemv_batches"]
        assert rows_read(job).tolist() == [1] * out
        assert rel_err(job.y, refs[0]) <= TOL
        job.reads.clear()
        job.y[:] = np.nan
        assert dense_gguf_source(ctx, bank, job) == kb.RESULT_FINITE
        hits = ctx.counters()
        assert not job.reads
        assert hits["gemm_launches"] - after["gemm_launches"] == 1 and hits["gemm_fallbacks"] == 0
        assert rel_err(job.y, refs[0]) <= TOL
    finally:
        bank.close()
        ctx.close()


def test_dense_gguf_batch_switches_at_eight_rows(kb, oracle, cuda):
    """The resident batch path keeps jobs of up to 8 rows on the GEMV (one
    batch) and sends 9 rows and more to the GEMM, as the reference's
    project switches (h3_compute.cu:1863-1865); both within tolerance."""
    from kadan_b200 import synth

    ctx = kb.Context(0)
    in_, out = 2048, 320
    w = synth.gguf(kb.Q6_K, out, in_, seed=3)
    ptr = ctx.upload(w)
    try:
        for rows, gemm in ((8, 0), (9, 1), (200, 1)):
            x = synth.activations(rows * in_, seed=rows).reshape(rows, in_)
            y = np.full((rows, out), np.nan, dtype=np.float32)
            before = ctx.counters()
            assert ctx.dense_gguf_batch([kb.host_job(kb.Q6_K, ptr, x, y, in_=in_, out=out)]) == kb.RESULT_UNVALIDATED
            after = ctx.counters()
            assert after["gemm_launches"] - before["gemm_launches"] == gemm
            assert after["gemv_batches"] - before["gemv_batches"] == 1 - gemm
            assert rel_err(y, oracle.gemv_f64(kb.Q6_K, w, x, in_, out)) <= TOL
    finally:
        ctx.free(ptr)
        ctx.close()


def test_gemm_range_fallback_through_the_boundary(kb, oracle, cuda):
    """A Q8_0 block whose weights exceed fp16 (d = 1000): the boundary's GEMM
    reports it and the call recomputes that job on the GEMV path, so the
    outputs still match the oracle; the counters record one fallback."""
    from kadan_b200 import synth

    ctx = kb.Context(0)
    rows, in_, out = 64, 1024, 96
    w = synth.q8_0(out, in_, seed=8)
    w[11, 5 * 34:5 * 34 + 2] = [0xD0, 0x63]
    ptr = ctx.upload(w)
    try:
        x = synth.activations(rows * in_, seed=9).reshape(rows, in_)
        y = np.full((rows, out), np.nan, dtype=np.float32)
        assert ctx.dense_gguf_batch([kb.host_job(kb.Q8_0, ptr, x, y, in_=in_, out=out)]) == kb.RESULT_UNVALIDATED
        c = ctx.counters()
        assert c["gemm_launches"] == 1 and c["gemm_fallbacks"] == 1
        assert rel_err(y, oracle.gemv_f64(kb.Q8_0, w, x, in_, out)) <= TOL
    finally:
        ctx.free(ptr)
        ctx.close()
