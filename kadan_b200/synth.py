"""Seeded synthetic GGUF / MXFP4 tensors with the distributions BASELINE
configs name (there is no network and no checkpoint on the GPU machine).

Host generators use a counter-based splitmix64 stream and Box-Muller in numpy,
so the same seed always gives the same bytes. Device generators (for the
multi-GB bench stacks) use a seeded torch.Generator on the GPU.

Block layouts (GGUF, IW/third_party/ggml/src/ggml-common.h):
  Q8_0  34 B: fp16 d, 32 x int8
  Q4_K 144 B: fp16 d, fp16 dmin, 12 B packed 6-bit scales/mins, 128 B nibbles
  Q6_K 210 B: 128 B ql, 64 B qh, 16 x int8 scales, fp16 d
MXFP4 (safetensors expert layout, IW/src/weights/checkpoint.cpp:669-730):
  weights [rows, cols/2] low nibble first, scales [rows, cols/32] E8M0.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """n outputs of splitmix64 at counters stream*2^40 + [0, n) from `seed`."""
    with np.errstate(over="ignore"):
        i = np.arange(n, dtype=np.uint64) + np.uint64(stream << 40)
        z = np.uint64(seed) + (i + np.uint64(1)) * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform01(seed: int, n: int, stream: int = 0) -> np.ndarray:
    return (splitmix64(seed, n, stream) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))


def normal(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """Box-Muller N(0,1) doubles."""
    m = (n + 1) // 2
    u1 = uniform01(seed, m, 2 * stream)
    u2 = uniform01(seed, m, 2 * stream + 1)
    r = np.sqrt(-2.0 * np.log1p(-u1))
    z = np.empty(2 * m)
    z[0::2] = r * np.cos(2 * np.pi * u2)
    z[1::2] = r * np.sin(2 * np.pi * u2)
    return z[:n]


def random_bytes(seed: int, n: int, stream: int = 0) -> np.ndarray:
    words = splitmix64(seed, (n + 7) // 8, stream)
    return words.view(np.uint8)[:n].copy()


def _half_abs_normal(seed: int, n: int, stream: int, scale: float) -> np.ndarray:
    return (np.abs(normal(seed, n, stream)) * scale).astype(np.float16)


def q8_0(rows: int, cols: int, seed: int = 0) -> np.ndarray:
    """Q8_0 [rows, cols/32 blocks]: int8 uniform in [-127, 127], d = |N(0,1)|*0.01."""
    nb = rows * cols // 32
    blocks = np.empty((nb, 34), dtype=np.uint8)
    blocks[:, :2] = _half_abs_normal(seed, nb, 1, 0.01).view(np.uint8).reshape(nb, 2)
    codes = (splitmix64(seed, nb * 32, 2) % np.uint64(255)).astype(np.int16) - 127
    blocks[:, 2:] = codes.astype(np.int8).view(np.uint8).reshape(nb, 32)
    return blocks.reshape(rows, cols // 32 * 34)


def q4_k(rows: int, cols: int, seed: int = 0) -> np.ndarray:
    """Q4_K: every code/scale/min bit uniform, d and dmin = |N(0,1)|*0.02."""
    nb = rows * cols // 256
    blocks = random_bytes(seed, nb * 144, 3).reshape(nb, 144)
    blocks[:, 0:2] = _half_abs_normal(seed, nb, 4, 0.02).view(np.uint8).reshape(nb, 2)
    blocks[:, 2:4] = _half_abs_normal(seed, nb, 5, 0.02).view(np.uint8).reshape(nb, 2)
    return blocks.reshape(rows, cols // 256 * 144)


def q6_k(rows: int, cols: int, seed: int = 0) -> np.ndarray:
    """Q6_K: codes from uniform bytes, int8 scales uniform in [-32, 31], d = |N(0,1)|*0.02."""
    nb = rows * cols // 256
    blocks = random_bytes(seed, nb * 210, 6).reshape(nb, 210)
    scales = (splitmix64(seed, nb * 16, 7) % np.uint64(64)).astype(np.int16) - 32
    blocks[:, 192:208] = scales.astype(np.int8).view(np.uint8).reshape(nb, 16)
    blocks[:, 208:210] = _half_abs_normal(seed, nb, 8, 0.02).view(np.uint8).reshape(nb, 2)
    return blocks.reshape(rows, cols // 256 * 210)


def gguf(encoding: int, rows: int, cols: int, seed: int = 0) -> np.ndarray:
    from . import Q4_K, Q6_K, Q8_0

    return {Q8_0: q8_0, Q4_K: q4_k, Q6_K: q6_k}[encoding](rows, cols, seed)


def mxfp4(rows: int, cols: int, seed: int = 0, exp_lo: int = 118, exp_hi: int = 126):
    """MXFP4 checkpoint layout: codes uniform over 16, E8M0 uniform in [exp_lo, exp_hi]."""
    weights = random_bytes(seed, rows * cols // 2, 9).reshape(rows, cols // 2)
    span = np.uint64(exp_hi - exp_lo + 1)
    scales = (splitmix64(seed, rows * cols // 32, 10) % span).astype(np.uint8) + np.uint8(exp_lo)
    return weights, scales.reshape(rows, cols // 32)


def activations(n: int, seed: int = 0, dtype: str = "f16", stream: int = 11) -> np.ndarray:
    """N(0,1) activations rounded to `dtype` ("f16", "bf16" or "f32"), returned as float32."""
    v = normal(seed, n, stream).astype(np.float32)
    if dtype == "f16":
        return v.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        b = v.view(np.uint32).astype(np.uint64)
        b = (b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) & np.uint64(0xFFFF0000)
        return b.astype(np.uint32).view(np.float32)
    return v


# ---------------------------------------------------------------- device side
def device_gguf(encoding: int, rows: int, cols: int, seed: int, device):
    """Same distributions as the host generators, drawn on the GPU (torch)."""
    import torch

    from . import Q4_K, Q6_K, Q8_0, block_bytes, block_values

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nb = rows * cols // block_values(encoding)
    bb = block_bytes(encoding)
    blocks = torch.randint(0, 256, (nb, bb), dtype=torch.uint8, device=device, generator=g)

    def halves(scale):
        return (torch.randn(nb, device=device, generator=g).abs() * scale).half().view(torch.uint8).view(nb, 2)

    if encoding == Q8_0:
        blocks[:, 0:2] = halves(0.01)
        codes = torch.randint(-127, 128, (nb, 32), dtype=torch.int16, device=device, generator=g)
        blocks[:, 2:] = codes.to(torch.int8).view(torch.uint8)
    elif encoding == Q4_K:
        blocks[:, 0:2] = halves(0.02)
        blocks[:, 2:4] = halves(0.02)
    elif encoding == Q6_K:
        sc = torch.randint(-32, 32, (nb, 16), dtype=torch.int16, device=device, generator=g)
        blocks[:, 192:208] = sc.to(torch.int8).view(torch.uint8)
        blocks[:, 208:210] = halves(0.02)
    else:
        raise ValueError("unsupported encoding for the device generator")
    return blocks.view(rows, cols // block_values(encoding) * bb)
