"""GPU parity of the GGUF dequant and GEMV kernels against the pinned oracle.

Bars: dequant bit-exact (integer/byte work); GEMV outputs within the stated
tolerance 1e-3 of the double-precision oracle, measured as
max|y - ref| / max(max|ref|, 1) (the reference's GEMV check,
IW/tests/gguf_text.cpp:247-250).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def to_dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("name", ["q8_0", "q4_k", "q6_k", "q3_k", "iq4_nl", "iq4_xs", "bf16"])
def test_dequant_bit_exact_reference_blocks(kb, oracle, cuda, name):
    check_dequant(kb, oracle, cuda, name)


@pytest.fixture
def iq_grids(kb, oracle, ref):
    """The reference's IQ code grids, registered with the library (as the
    worker's adapter registers its own) and with the oracle."""
    grids = ref.iq_grids()
    kb.set_iq_grids(*grids)
    oracle.set_iq_grids(grids)
    return grids


@pytest.mark.parametrize("name", ["iq3_xxs", "iq2_s", "iq3_s"])
def test_dequant_grid_coded_bit_exact(kb, oracle, cuda, iq_grids, name):
    check_dequant(kb, oracle, cuda, name)


@pytest.mark.parametrize("enc_name", ["iq3_xxs", "iq2_s", "iq3_s"])
@pytest.mark.parametrize("rows", [1, 5])
def test_gemv_grid_coded_parity(kb, oracle, cuda, iq_grids, enc_name, rows):
    enc = getattr(kb, enc_name.upper())
    y, want = gemv_case(kb, oracle, cuda, enc, 512, 23, rows)
    assert rel_err(y, want) <= TOL


def check_dequant(kb, oracle, cuda, name):
    """The golden blocks of `name` decoded on the device: the reference's
    digest, the oracle's bits (NaN payloads aside) and the status word."""
    import torch

    from golden.make_golden import canonical_digest, reference_blocks

    spec = json.loads((GOLDEN / "gguf_blocks.json").read_text())["encodings"][name]
    blocks = reference_blocks(spec["encoding"], spec["trials"])
    n = blocks.shape[0] * kb.block_values(spec["encoding"])
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    kb.gguf_dequant(spec["encoding"], to_dev(blocks, cuda), n, out, status)
    got = out.cpu().numpy()
    assert canonical_digest(got) == spec["sha256_expected"]
    want = oracle.decode(spec["encoding"], blocks, n)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got.view(np.uint32)[~nan], want.view(np.uint32)[~nan])
    assert int(status.item()) == (1 if spec["nan_count"] or np.isinf(want).any() else 0)


def gemv_case(kb, oracle, cuda, enc, in_, out, rows, seed=0, x_dtype="f32"):
    import torch

    from kadan_b200 import synth

    if enc in (kb.Q8_0, kb.Q4_K, kb.Q6_K):
        w = synth.gguf(enc, out, in_, seed=seed)
    else:
        rng = np.random.default_rng(seed)
        w = rng.integers(0, 256, size=(out, in_ // kb.block_values(enc) * kb.block_bytes(enc)), dtype=np.uint8)
        if enc != kb.BF16:
            # keep the fp16 scales finite and modest
            bb, bv = kb.block_bytes(enc), kb.block_values(enc)
            off = {kb.Q3_K: 108}.get(enc, 0)
            blocks = w.reshape(-1, bb)
            blocks[:, off:off + 2] = (np.abs(rng.standard_normal(len(blocks))) * 0.02).astype(np.float16).view(
                np.uint8).reshape(-1, 2)
        else:
            w = (rng.standard_normal((out, in_)) * 0.05).astype(np.float32).view(np.uint32)
            w = ((w >> 16).astype(np.uint16)).view(np.uint8).reshape(out, -1)
    x = synth.activations(rows * in_, seed=seed + 1, dtype=x_dtype).reshape(rows, in_)
    want = oracle.gemv_f64(enc, w, x, in_, out)
    y = kb.gguf_gemv(enc, to_dev(w, cuda), to_dev(x, cuda), in_=in_, columns=out)
    torch.cuda.synchronize()
    return y.cpu().numpy(), want


@pytest.mark.parametrize("enc_name", ["q8_0", "q4_k", "q6_k"])
@pytest.mark.parametrize("in_,out", [(4096, 37), (4096, 1), (8192, 19), (14336, 64), (2048, 300), (256, 8)])
@pytest.mark.parametrize("rows", [1, 2, 3])
def test_gemv_staged_parity(kb, oracle, cuda, enc_name, in_, out, rows):
    enc = {"q8_0": kb.Q8_0, "q4_k": kb.Q4_K, "q6_k": kb.Q6_K}[enc_name]
    if enc == kb.Q6_K and (in_ // 256) % 8:
        pytest.skip("Q6_K rows of this width are not 16-byte multiples (generic path covers them)")
    y, want = gemv_case(kb, oracle, cuda, enc, in_, out, rows)
    assert rel_err(y, want) <= TOL


def test_q4k_uses_tensor_pipe_kernel(kb, cuda):
    import torch

    w = torch.zeros(64, 4352, dtype=torch.uint8, device=cuda)
    x = torch.zeros(1, 4096, device=cuda)
    y = torch.zeros(1, 64, device=cuda)
    assert kb.gemv_path(kb.gemv_job(kb.Q4_K, w, x, y, in_=4096, columns=64, rows=1, row_bytes_=4352)) == 2
    assert kb.gemv_path(kb.gemv_job(kb.Q8_0, w, x, y, in_=4096, columns=64, rows=1, row_bytes_=4352)) == 1


@pytest.mark.parametrize("rows", [4, 5, 8, 17])
def test_gemv_row_groups(kb, oracle, cuda, rows):
    y, want = gemv_case(kb, oracle, cuda, kb.Q4_K, 4096, 40, rows)
    assert rel_err(y, want) <= TOL


@pytest.mark.parametrize("enc_name,in_", [("q8_0", 160), ("q6_k", 256), ("q3_k", 512), ("iq4_nl", 96),
                                          ("iq4_xs", 512), ("bf16", 200), ("q4_k", 512)])
@pytest.mark.parametrize("rows", [1, 5])
def test_gemv_generic_parity(kb, oracle, cuda, enc_name, in_, rows):
    enc = getattr(kb, enc_name.upper())
    y, want = gemv_case(kb, oracle, cuda, enc, in_, 23, rows)
    assert rel_err(y, want) <= TOL


def test_gemv_golden_cpu_matvec_fixture(kb, cuda):
    import torch

    g = np.load(GOLDEN / "cpu_matvec.npz")
    x = to_dev(g["input"], cuda)
    for name, enc in (("q8_0", kb.Q8_0), ("q4_k", kb.Q4_K), ("q6_k", kb.Q6_K)):
        y = kb.gguf_gemv(enc, to_dev(g[f"{name}_packed"], cuda), x, in_=512, columns=37)
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), g[f"{name}_f64"]) <= TOL


def test_config1_golden(kb, cuda):
    import torch

    from kadan_b200 import synth

    g = np.load(GOLDEN / "config1_q8_0.npz")
    w = to_dev(synth.q8_0(4096, 4096, seed=0), cuda)
    y = kb.gguf_gemv(kb.Q8_0, w, to_dev(g["x"], cuda), in_=4096, columns=4096)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy()[0], g["y_f64"]) <= TOL


def test_batch_mixed_encodings_shared_input(kb, oracle, cuda):
    import torch

    from kadan_b200 import synth

    in_ = 4096
    x = synth.activations(2 * in_, seed=9).reshape(2, in_)
    xd = to_dev(x, cuda)
    cases = [(kb.Q4_K, 100), (kb.Q8_0, 33), (kb.Q6_K, 65), (kb.Q4_K, 8)]
    jobs, outs, wants = [], [], []
    for i, (enc, out) in enumerate(cases):
        w = synth.gguf(enc, out, in_, seed=20 + i)
        wd = to_dev(w, cuda)
        y = torch.full((2, out), float("nan"), device=cuda)
        outs.append((wd, y))
        jobs.append(kb.gemv_job(enc, wd, xd, y, in_=in_, columns=out, rows=2))
        wants.append(oracle.gemv_f64(enc, w, x, in_, out))
    kb.gguf_gemv_batch(jobs)
    torch.cuda.synchronize()
    for (_, y), want in zip(outs, wants):
        assert rel_err(y.cpu().numpy(), want) <= TOL


def test_strided_output_and_status(kb, oracle, cuda):
    import torch

    from kadan_b200 import synth

    in_, out = 4096, 24
    w = synth.q4_k(out, in_, seed=4)
    x = synth.activations(2 * in_, seed=5).reshape(2, in_)
    y = torch.full((2, 3 * out), -7.0, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    wd = to_dev(w, cuda)
    kb.gguf_gemv_batch([kb.gemv_job(kb.Q4_K, wd, to_dev(x, cuda), y[:, out:], in_=in_, columns=out, rows=2,
                                    stride=3 * out, status=status)])
    torch.cuda.synchronize()
    yy = y.cpu().numpy()
    assert rel_err(yy[:, out:2 * out], oracle.gemv_f64(kb.Q4_K, w, x, in_, out)) <= TOL
    assert np.all(yy[:, :out] == -7.0) and np.all(yy[:, 2 * out:] == -7.0)
    assert status.item() == 0
    # An infinite fp16 d in one block sets the job's status bit.
    bad = w.copy()
    bad[5, 144 * 3: 144 * 3 + 2] = [0x00, 0x7C]
    kb.gguf_gemv_batch([kb.gemv_job(kb.Q4_K, to_dev(bad, cuda), to_dev(x, cuda), y[:, :out], in_=in_,
                                    columns=out, rows=2, stride=3 * out, status=status)])
    torch.cuda.synchronize()
    assert status.item() == 1
    assert kb.take_device_error() == 0


def test_full_size_gate_projection_against_exact_dequant(kb, cuda):
    """Config 2 gate (14336 x 4096 Q4_K) at full size: the GEMV equals the
    float64 product of the bit-exact dequantised weights."""
    import torch

    from kadan_b200 import synth

    out, in_ = 14336, 4096
    wd = synth.device_gguf(kb.Q4_K, out, in_, seed=3, device=cuda)
    x = torch.randn(1, in_, device=cuda, generator=torch.Generator(device=cuda).manual_seed(1)).half().float()
    y = kb.gguf_gemv(kb.Q4_K, wd, x, in_=in_, columns=out)
    dec = torch.empty(out * in_, dtype=torch.float32, device=cuda)
    kb.gguf_dequant(kb.Q4_K, wd, out * in_, dec)
    want = (dec.view(out, in_).double() @ x.double().T).T
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), want.cpu().numpy()) <= TOL
    # Linearity in the input (size-independent property).
    x2 = torch.randn(1, in_, device=cuda, generator=torch.Generator(device=cuda).manual_seed(2))
    y2 = kb.gguf_gemv(kb.Q4_K, wd, x2, in_=in_, columns=out)
    y3 = kb.gguf_gemv(kb.Q4_K, wd, (2.0 * x - x2).contiguous(), in_=in_, columns=out)
    torch.cuda.synchronize()
    assert rel_err(y3.cpu().numpy(), (2.0 * y - y2).cpu().numpy()) <= TOL


def _dequant_product(kb, wd, x, in_, out):
    """float64 product of the bit-exact dequantised weights (device)."""
    import torch

    dec = torch.empty(out * in_, dtype=torch.float32, device=x.device)
    kb.gguf_dequant(kb.Q4_K, wd, out * in_, dec)
    return (dec.view(out, in_).double() @ x.double().T).T


@pytest.mark.parametrize("rows", [1, 3, 8])
def test_q4k_balanced_split_ragged_batch_deterministic(kb, cuda, rows):
    """One launch over Q4_K jobs of different widths and heights: the balanced
    split cuts tiles at CTA boundaries (K = 56 super-blocks, 40-column tails,
    a K = 4 job with fewer units than CTAs). Every output matches the exact
    product, and three launches agree bit for bit (the cut tiles are summed in
    a fixed order whatever piece finishes last; the counters re-arm)."""
    import torch

    from kadan_b200 import synth

    shapes = [(4096, 6144), (14336, 4096), (4096, 40), (1024, 999), (2048, 64)]
    gen = torch.Generator(device=cuda).manual_seed(7)
    mats, jobs, outs, xs = [], [], [], []
    for i, (in_, out) in enumerate(shapes):
        wd = synth.device_gguf(kb.Q4_K, out, in_, seed=40 + i, device=cuda)
        x = torch.randn(rows, in_, device=cuda, generator=gen).half().float()
        y = torch.full((rows, out), float("nan"), device=cuda)
        mats.append(wd), xs.append(x), outs.append(y)
        jobs.append(kb.gemv_job(kb.Q4_K, wd, x, y, in_=in_, columns=out, rows=rows))
    runs = []
    for _ in range(3):
        for y in outs:
            y.fill_(float("nan"))
        kb.gguf_gemv_batch(jobs)
        torch.cuda.synchronize()
        runs.append([y.cpu().numpy().copy() for y in outs])
    for (in_, out), wd, x, got in zip(shapes, mats, xs, runs[0]):
        want = _dequant_product(kb, wd, x, in_, out)
        assert rel_err(got, want.cpu().numpy()) <= TOL, (in_, out)
    for other in runs[1:]:
        for a, b in zip(runs[0], other):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert kb.take_device_error() == 0


def test_q4k_streams_share_nothing(kb, cuda):
    """Launches on two streams run concurrently, each with its own fixup
    buffer: both results match a single-stream run bit for bit."""
    import torch

    from kadan_b200 import synth

    in_, out = 14336, 4096
    wd = synth.device_gguf(kb.Q4_K, out, in_, seed=61, device=cuda)
    xa = torch.randn(1, in_, device=cuda, generator=torch.Generator(device=cuda).manual_seed(3))
    xb = torch.randn(1, in_, device=cuda, generator=torch.Generator(device=cuda).manual_seed(4))
    ref_a = kb.gguf_gemv(kb.Q4_K, wd, xa, in_=in_, columns=out)
    ref_b = kb.gguf_gemv(kb.Q4_K, wd, xb, in_=in_, columns=out)
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)
    ya, yb = torch.empty_like(ref_a), torch.empty_like(ref_b)
    ja = kb.gemv_job(kb.Q4_K, wd, xa, ya, in_=in_, columns=out, rows=1)
    jb = kb.gemv_job(kb.Q4_K, wd, xb, yb, in_=in_, columns=out, rows=1)
    for _ in range(4):
        kb.gguf_gemv_batch([ja], stream=s1)
        kb.gguf_gemv_batch([jb], stream=s2)
    torch.cuda.synchronize()
    assert torch.equal(ya, ref_a) and torch.equal(yb, ref_b)


@pytest.mark.parametrize("in_,out,rows", [(8192, 40, 1), (3584, 131, 1), (1024, 8192, 1), (256, 33, 3), (28672, 64, 2),
                                          (8192, 1280, 4), (14336, 17, 5), (2048, 4096, 8), (4096, 29, 7),
                                          (28672, 1024, 1), (2048, 333, 2), (8192, 2048, 2), (512, 7, 1)])
def test_q6k_tensor_pipe_parity(kb, oracle, cuda, in_, out, rows):
    """Q6_K on the integer tensor pipe: rows padded to a 16-byte pitch (as the
    tensor-parallel shards are), chunks of 8 blocks with ragged last chunks,
    the paired-sub-block kernel at 1-2 rows (activation windows shorter than
    K at 28672), up to 4 input rows per pass and row groups beyond, balanced
    and whole-tile launches."""
    import torch

    from kadan_b200 import synth
    from kadan_b200.tensor_parallel import pad_rows

    w = synth.q6_k(out, in_, seed=in_ + out + rows)
    pitch = (w.shape[1] + 15) // 16 * 16
    wd = to_dev(pad_rows(w, pitch), cuda)
    x = synth.activations(rows * in_, seed=rows + 3, dtype="bf16").reshape(rows, in_)
    y = torch.full((rows, out), float("nan"), device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    job = kb.gemv_job(kb.Q6_K, wd, to_dev(x, cuda), y, in_=in_, columns=out, rows=rows, row_bytes_=pitch,
                      status=status)
    assert kb.gemv_path(job) == 2
    kb.gguf_gemv_batch([job])
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.gemv_f64(kb.Q6_K, w, x, in_, out)) <= TOL
    assert status.item() == 0
    assert kb.take_device_error() == 0


# Batches whose activations are quantised once per launch: Q6_K at 1-2
# input rows (the pair kernel; q/k/v-like jobs sharing one input, a long-K
# job, mixed 1- and 2-row jobs with a ragged last chunk) and Q4_K at up to 8
# rows on 64-row tiles where each CTA's share of K is longer than its own
# activation segment (balanced splits; shared inputs, 3-, 4-, 6- and 8-row
# jobs, K of 19 super-blocks).
_STAGED_BATCHES = r"""
import numpy as np, torch
import kadan_b200 as kb
from kadan_b200 import synth
from kadan_b200.tensor_parallel import pad_rows

BATCHES = {
    "q6_k": (((8192, 1024, 1, 0), (8192, 256, 1, 0), (8192, 256, 1, 0), (28672, 512, 1, 1)),
             ((8192, 2048, 2, 2), (2304, 96, 1, 3)),
             ((256, 33, 2, 4),)),
    "q4_k": (((24576, 8192, 1, 0), (24576, 4096, 1, 0)),
             ((4096, 14336, 3, 1), (4096, 2048, 4, 2)),
             ((4864, 28672, 2, 3),),
             ((8192, 8192, 8, 5), (8192, 4096, 6, 6))),
}


def run_batches(name, dev, stream=None, capture=None):
    enc = getattr(kb, name.upper())
    make = synth.q6_k if name == "q6_k" else synth.q4_k
    outs = []
    for batch in BATCHES[name]:
        keep, jobs, ys, xs = [], [], [], {}
        for i, (in_, out, rows, xi) in enumerate(batch):
            w = make(out, in_, seed=10 * xi + i)
            pitch = (w.shape[1] + 15) // 16 * 16
            wd = torch.from_numpy(pad_rows(w, pitch)).to(dev)
            if xi not in xs:
                x = synth.activations(rows * in_, seed=100 + xi, dtype="bf16").reshape(rows, in_)
                xs[xi] = torch.from_numpy(x).to(dev)
            y = torch.full((rows, out), float("nan"), device=dev)
            keep.append(wd)
            ys.append(y)
            jobs.append(kb.gemv_job(enc, wd, xs[xi], y, in_=in_, columns=out, rows=rows, row_bytes_=pitch))
        if capture is None:
            kb.gguf_gemv_batch(jobs, stream=stream)
        else:
            capture(lambda: kb.gguf_gemv_batch(jobs, stream=stream))
        torch.cuda.synchronize()
        outs += [y.cpu().numpy() for y in ys]
    return outs
"""
_STAGED = {"q6_k": ("KB200_GEMV_Q6K_STAGED", "pair_quant_kernel", "gemv_q6k_pair_kernel"),
           "q4_k": ("KB200_GEMV_Q4K_STAGED", "q4k_quant_kernel", "gemv_q4k_mma_kernel")}


def _staged_namespace():
    ns = {}
    exec(_STAGED_BATCHES, ns)
    return ns


@pytest.mark.parametrize("name", ["q6_k", "q4_k"])
def test_staged_activations_match_per_cta_quantisation(kb, oracle, cuda, tmp_path, name):
    """Activations quantised once per launch (a quantisation kernel, its
    records copied into each weight stage) give the bit-identical outputs of
    the per-CTA activation segments (the staging switch off, another
    process), and both are within the tolerance of the oracle."""
    import os
    import subprocess
    import sys

    from conftest import ROOT
    from kadan_b200 import synth

    env_name, quant, gemv = _STAGED[name]
    ns = _staged_namespace()
    with kb.Phase() as ph:
        got = ns["run_batches"](name, cuda)
        calls = {k: v["calls"] for k, v in ph.snapshot()["kernels"].items()}
    ph.close()
    assert calls == {quant: len(ns["BATCHES"][name]), gemv: len(ns["BATCHES"][name])}
    out = tmp_path / "unstaged.npz"
    code = _STAGED_BATCHES + f"\nnp.savez({str(out)!r}, *run_batches({name!r}, torch.device('cuda:0')))\n"
    env = {**os.environ, env_name: "0", "KADAN_B200_NO_BUILD": "1", "PYTHONPATH": str(ROOT)}
    subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, check=True, timeout=600)
    with np.load(out) as z:
        want = [z[f"arr_{i}"] for i in range(len(z.files))]
    flat = [(i, job) for b in ns["BATCHES"][name] for i, job in enumerate(b)]
    assert len(want) == len(got) == len(flat)
    for a, b in zip(got, want):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    make = synth.q6_k if name == "q6_k" else synth.q4_k
    enc = getattr(kb, name.upper())
    for (i, (in_, cols, rows, xi)), y in zip(flat, got):
        w = make(cols, in_, seed=10 * xi + i)
        x = synth.activations(rows * in_, seed=100 + xi, dtype="bf16").reshape(rows, in_)
        assert rel_err(y, oracle.gemv_f64(enc, w, x, in_, cols)) <= TOL


@pytest.mark.parametrize("rows", [3, 4, 6, 8])
def test_q6k_multi_row_pairs_of_tokens(kb, oracle, cuda, rows):
    """Q6_K at 3-8 input rows: the pair kernel with two token pairs per pass
    (3-4 rows) or four (5-8 rows, eight consumer warps), activations staged
    once per launch; a
    batch of jobs sharing one input, one with a ragged last chunk, one with a
    long K; within the oracle's tolerance."""
    import torch

    from kadan_b200 import synth
    from kadan_b200.tensor_parallel import pad_rows

    shapes = [(8192, 1024), (8192, 256), (2304, 200), (28672, 160)]
    x = {in_: synth.activations(rows * in_, seed=rows + in_, dtype="bf16").reshape(rows, in_) for in_, _ in shapes}
    xd = {in_: to_dev(v, cuda) for in_, v in x.items()}
    keep, jobs, ys, ws = [], [], [], []
    for i, (in_, out) in enumerate(shapes):
        w = synth.q6_k(out, in_, seed=7 * i + rows)
        pitch = (w.shape[1] + 15) // 16 * 16
        wd = to_dev(pad_rows(w, pitch), cuda)
        y = torch.full((rows, out), float("nan"), device=cuda)
        keep.append(wd)
        ws.append(w)
        ys.append(y)
        jobs.append(kb.gemv_job(kb.Q6_K, wd, xd[in_], y, in_=in_, columns=out, rows=rows, row_bytes_=pitch))
    with kb.Phase() as ph:
        kb.gguf_gemv_batch(jobs)
        torch.cuda.synchronize()
        calls = {k: v["calls"] for k, v in ph.snapshot()["kernels"].items()}
    ph.close()
    assert calls == {"pair_quant_kernel": 1, "gemv_q6k_pair_kernel": 1}
    for (in_, out), w, y in zip(shapes, ws, ys):
        assert rel_err(y.cpu().numpy(), oracle.gemv_f64(kb.Q6_K, w, x[in_], in_, out)) <= TOL
    assert kb.take_device_error() == 0


@pytest.mark.parametrize("name", ["q6_k", "q4_k"])
def test_first_use_inside_capture_quantises_per_cta(kb, cuda, name):
    """A stream whose first launch is captured into a CUDA graph has no
    staging buffer (nor fixup buffer) yet: the captured launches quantise per
    CTA (no quantisation kernel is captured), and their replay matches the
    eager results of another stream within the oracle's tolerance."""
    import torch

    _, quant, gemv = _STAGED[name]
    ns = _staged_namespace()
    want = ns["run_batches"](name, cuda)
    stream = torch.cuda.Stream(cuda)
    graphs = []

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        graphs.append(g)
        g.replay()

    with kb.Phase() as ph:
        got = ns["run_batches"](name, cuda, stream=stream, capture=capture)
        calls = {k: v["calls"] for k, v in ph.snapshot()["kernels"].items()}
    ph.close()
    assert calls == {gemv: len(ns["BATCHES"][name])}
    for a, b in zip(got, want):
        assert rel_err(a, b) <= TOL
    del graphs


def test_q6k_tensor_pipe_nonfinite_scale_sets_status(kb, cuda):
    import torch

    from kadan_b200 import synth

    in_, out = 2048, 48
    w = synth.q6_k(out, in_, seed=1)
    w.reshape(-1, 210)[5 * (in_ // 256) + 3, 208:210] = np.array([0x7C00], dtype=np.uint16).view(np.uint8)  # +inf d
    x = synth.activations(in_, seed=2).reshape(1, in_)
    y = torch.zeros(1, out, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    job = kb.gemv_job(kb.Q6_K, to_dev(w, cuda), to_dev(x, cuda), y, in_=in_, columns=out, rows=1, status=status)
    assert kb.gemv_path(job) == 2
    kb.gguf_gemv_batch([job])
    torch.cuda.synchronize()
    assert status.item() == 1
