"""GPU parity of the Q4_K prefill GEMM (tensor cores) against the pinned oracle.

The reference's prefill path decodes the packed weights to fp32 and runs an
FP32 SGEMM (IW/src/cuda/h3_compute.cu:2201-2218, :2435-2468); its outputs are
checked here as the reference checks GEMV outputs, max|y - ref| /
max(max|ref|, 1) <= 1e-3 (IW/tests/gguf_text.cpp:247-250), against the
double-precision oracle on small shapes and against the float64 product of
the bit-exact device dequantisation at full size.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def to_dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def run_gemm(kb, cuda, w_dev, x_dev, rows, in_, out, stride=None, y=None, status=None):
    import torch

    if y is None:
        y = torch.full((rows, stride or out), float("nan"), device=cuda)
    ws = torch.empty(kb.gemm_workspace_bytes(rows, in_), dtype=torch.uint8, device=cuda)
    job = kb.gemv_job(kb.Q4_K, w_dev, x_dev, y, in_=in_, columns=out, rows=rows, stride=stride or out, status=status)
    kb.gguf_gemm(job, ws)
    return y


@pytest.mark.parametrize("rows,in_,out", [(9, 512, 37), (64, 1024, 200), (130, 512, 129), (257, 256, 64),
                                          (16, 2048, 300), (300, 512, 12840)])
def test_gemm_matches_oracle(kb, oracle, cuda, rows, in_, out):
    import torch

    from kadan_b200 import synth

    w = synth.q4_k(out, in_, seed=rows)
    x = synth.activations(rows * in_, seed=rows + 1).reshape(rows, in_)
    want = oracle.gemv_f64(kb.Q4_K, w, x, in_, out)
    y = run_gemm(kb, cuda, to_dev(w, cuda), to_dev(x, cuda), rows, in_, out)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), want) <= TOL


def _dequant_product(kb, wd, x, in_, out):
    import torch

    dec = torch.empty(out * in_, dtype=torch.float32, device=x.device)
    kb.gguf_dequant(kb.Q4_K, wd, out * in_, dec)
    return x.double() @ dec.view(out, in_).double().T


def test_gemm_full_size_prefill_layer(kb, cuda):
    """BASELINE config 2 prefill shape (T = 512, gate 14336 x 4096) against the
    float64 product of the bit-exact dequantised weights, plus linearity."""
    import torch

    from kadan_b200 import synth

    rows, in_, out = 512, 4096, 14336
    wd = synth.device_gguf(kb.Q4_K, out, in_, seed=5, device=cuda)
    gen = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(rows, in_, device=cuda, generator=gen)
    y = run_gemm(kb, cuda, wd, x, rows, in_, out)
    want = _dequant_product(kb, wd, x, in_, out)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), want.cpu().numpy()) <= TOL
    x2 = torch.randn(rows, in_, device=cuda, generator=gen)
    y2 = run_gemm(kb, cuda, wd, x2, rows, in_, out)
    y3 = run_gemm(kb, cuda, wd, (x + x2).contiguous(), rows, in_, out)
    torch.cuda.synchronize()
    assert rel_err(y3.cpu().numpy(), (y + y2).cpu().numpy()) <= TOL


def test_gemm_agrees_with_gemv_row_groups(kb, cuda):
    """The tensor-core GEMM and the packed GEMV (8 rows per pass) agree."""
    import torch

    from kadan_b200 import synth

    rows, in_, out = 40, 4096, 1024
    wd = synth.device_gguf(kb.Q4_K, out, in_, seed=8, device=cuda)
    x = torch.randn(rows, in_, device=cuda, generator=torch.Generator(device=cuda).manual_seed(9))
    y = run_gemm(kb, cuda, wd, x, rows, in_, out)
    y_gemv = kb.gguf_gemv(kb.Q4_K, wd, x, in_=in_, columns=out)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), y_gemv.cpu().numpy()) <= 2 * TOL


def test_gemm_power_of_two_scale_is_exact_and_deterministic(kb, cuda):
    """Each input row is normalised by a power of two before the fp16 cast, so
    scaling a row by 2^k scales its outputs by exactly 2^k; repeated launches
    agree bit for bit."""
    import torch

    from kadan_b200 import synth

    rows, in_, out = 200, 1024, 384
    wd = synth.device_gguf(kb.Q4_K, out, in_, seed=11, device=cuda)
    x = torch.randn(rows, in_, device=cuda, generator=torch.Generator(device=cuda).manual_seed(12))
    scale = torch.tensor([2.0 ** (20 if i % 3 == 0 else -20 if i % 3 == 1 else 0) for i in range(rows)],
                         device=cuda).unsqueeze(1)
    y = run_gemm(kb, cuda, wd, x, rows, in_, out)
    y_again = run_gemm(kb, cuda, wd, x, rows, in_, out)
    y_scaled = run_gemm(kb, cuda, wd, (x * scale).contiguous(), rows, in_, out)
    torch.cuda.synchronize()
    assert torch.equal(y, y_again)
    assert torch.equal(y_scaled, y * scale)


def test_gemm_strided_output_and_status(kb, oracle, cuda):
    import torch

    from kadan_b200 import synth

    rows, in_, out = 33, 512, 70
    w = synth.q4_k(out, in_, seed=21)
    x = synth.activations(rows * in_, seed=22).reshape(rows, in_)
    y = torch.full((rows, 3 * out), -7.0, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    run_gemm(kb, cuda, to_dev(w, cuda), to_dev(x, cuda), rows, in_, out, stride=3 * out, y=y[:, out:], status=status)
    torch.cuda.synchronize()
    yy = y.cpu().numpy()
    assert rel_err(yy[:, out:2 * out], oracle.gemv_f64(kb.Q4_K, w, x, in_, out)) <= TOL
    assert np.all(yy[:, :out] == -7.0) and np.all(yy[:, 2 * out:] == -7.0)
    assert status.item() == 0
    bad = w.copy()
    bad[17, 144:146] = [0x00, 0x7C]  # +inf fp16 d in super-block 1 of row 17
    run_gemm(kb, cuda, to_dev(bad, cuda), to_dev(x, cuda), rows, in_, out, stride=3 * out, y=y[:, out:],
             status=status)
    torch.cuda.synchronize()
    assert status.item() == 1
    assert kb.take_device_error() == 0


def test_gemm_rejects_other_encodings(kb, cuda):
    import torch

    w = torch.zeros(8, 1088, dtype=torch.uint8, device=cuda)
    x = torch.zeros(16, 1024, device=cuda)
    y = torch.zeros(16, 8, device=cuda)
    ws = torch.empty(kb.gemm_workspace_bytes(16, 1024), dtype=torch.uint8, device=cuda)
    job = kb.gemv_job(kb.Q8_0, w, x, y, in_=1024, columns=8, rows=16)
    with pytest.raises(kb.KadanError) as err:
        kb.gguf_gemm(job, ws)
    assert err.value.status == 1
