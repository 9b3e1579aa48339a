"""GPU parity of the prefill GEMM (tensor cores; Q4_K, Q6_K, Q8_0) against the pinned oracle.

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


def run_gemm(kb, cuda, w_dev, x_dev, rows, in_, out, stride=None, y=None, status=None, enc=None, row_bytes=None,
             ws=None):
    import torch

    if y is None:
        y = torch.full((rows, stride or out), float("nan"), device=cuda)
    if ws is None:
        ws = torch.empty(kb.gemm_workspace_bytes(rows, in_), dtype=torch.uint8, device=cuda)
    job = kb.gemv_job(kb.Q4_K if enc is None else enc, w_dev, x_dev, y, in_=in_, columns=out, rows=rows,
                      stride=stride or out, status=status, row_bytes_=row_bytes)
    kb.gguf_gemm(job, ws)
    return y


def padded(w):
    """Packed rows copied to a 16-byte pitch (the GEMM's row rule)."""
    pitch = (w.shape[1] + 15) // 16 * 16
    out = np.zeros((w.shape[0], pitch), dtype=np.uint8)
    out[:, :w.shape[1]] = w
    return out


@pytest.mark.parametrize("enc", [1, 3, 2], ids=["q4_k", "q6_k", "q8_0"])
@pytest.mark.parametrize("rows,in_,out", [(9, 512, 37), (64, 1024, 200), (130, 2048, 129), (257, 256, 64),
                                          (300, 768, 1284)])
def test_gemm_formats_match_oracle(kb, oracle, cuda, enc, rows, in_, out):
    """Every GEMM format at odd shapes (partial M and N tiles, K of one to
    eight 256-value steps, Q6_K's super-blocks at every offset within their
    16-byte words) against the double-precision oracle."""
    import torch

    from kadan_b200 import synth

    w = synth.gguf(enc, out, in_, seed=rows + 7 * enc)
    x = synth.activations(rows * in_, seed=rows + 1).reshape(rows, in_)
    want = oracle.gemv_f64(enc, w, x, in_, out)
    wp = padded(w)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    y = run_gemm(kb, cuda, to_dev(wp, cuda), to_dev(x, cuda), rows, in_, out, enc=enc, row_bytes=wp.shape[1],
                 status=status)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), want) <= TOL
    assert status.item() == 0


@pytest.mark.parametrize("enc,in_,out", [(3, 8192, 8192), (3, 28672, 2048), (2, 4096, 14336)],
                         ids=["q6_k-o", "q6_k-down", "q8_0"])
def test_gemm_full_size_other_formats(kb, cuda, enc, in_, out):
    """T = 512 prefill at BASELINE config-4 shapes (Q6_K o, a slice of down)
    and a Q8_0 matrix, against the float64 product of the bit-exact device
    dequantisation."""
    import torch

    from kadan_b200 import synth

    rows = 512
    wd = synth.device_gguf(enc, out, in_, seed=17, device=cuda)
    x = torch.randn(rows, in_, device=cuda, generator=torch.Generator(device=cuda).manual_seed(4))
    y = run_gemm(kb, cuda, wd, x, rows, in_, out, enc=enc)
    dec = torch.empty(out * in_, dtype=torch.float32, device=cuda)
    kb.gguf_dequant(enc, wd, out * in_, dec)
    want = x.double() @ dec.view(out, in_).double().T
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), want.cpu().numpy()) <= TOL


def test_gemm_flags_weights_beyond_fp16(kb, oracle, cuda):
    """A Q8_0 block with d = 1000 puts weights beyond fp16: the GEMM reports
    it (status bit 2 and the workspace's range word); a clean launch on the
    same workspace clears the word again."""
    import torch

    from kadan_b200 import synth

    rows, in_, out = 20, 1024, 64
    w = synth.q8_0(out, in_, seed=5)
    x = synth.activations(rows * in_, seed=6).reshape(rows, in_)
    bad = w.copy()
    bad[5, 3 * 34:3 * 34 + 2] = [0xD0, 0x63]  # fp16 1000.0
    ws = torch.empty(kb.gemm_workspace_bytes(rows, in_), dtype=torch.uint8, device=cuda)
    at = kb.gemm_range_offset(rows, in_)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    run_gemm(kb, cuda, to_dev(bad, cuda), to_dev(x, cuda), rows, in_, out, enc=kb.Q8_0, status=status, ws=ws)
    torch.cuda.synchronize()
    assert status.item() == 2
    assert int(ws[at:at + 4].view(torch.int32).item()) == 1
    y = run_gemm(kb, cuda, to_dev(w, cuda), to_dev(x, cuda), rows, in_, out, enc=kb.Q8_0, ws=ws)
    torch.cuda.synchronize()
    assert int(ws[at:at + 4].view(torch.int32).item()) == 0
    assert rel_err(y.cpu().numpy(), oracle.gemv_f64(kb.Q8_0, w, x, in_, out)) <= TOL


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

    w = torch.zeros(8, 544, dtype=torch.uint8, device=cuda)
    x = torch.zeros(16, 1024, device=cuda)
    y = torch.zeros(16, 8, device=cuda)
    ws = torch.empty(kb.gemm_workspace_bytes(16, 1024), dtype=torch.uint8, device=cuda)
    job = kb.gemv_job(kb.IQ4_NL, w, x, y, in_=1024, columns=8, rows=16)
    with pytest.raises(kb.KadanError) as err:
        kb.gguf_gemm(job, ws)
    assert err.value.status == 1
