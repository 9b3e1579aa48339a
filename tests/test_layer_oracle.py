"""The layer-math oracle (oracle/layer.c) pinned to the reference's own
known-answer tests of its host layer math, IW/tests/gguf_text.cpp: norms
(:46-58), rotation (:60-73), delta (:75-113), delta_passes (:115-154, bit for
bit) and attention (:263-302), with the test's tolerance
|a - e| <= 1e-5 max(1, |e|) (:23-27). IW = services/hikari/inference_worker."""
from __future__ import annotations

import math

import numpy as np
import pytest

F = np.float32


def near(actual, expected, tol=1e-5):
    actual, expected = float(actual), float(expected)
    assert abs(actual - expected) <= tol * max(1.0, abs(expected)), (actual, expected)


def test_norms(oracle):
    x = oracle.rms_norm([3, 4, 6, 8], [1, 2], width=2, eps=0.0)
    a, b = 1 / math.sqrt(12.5), 1 / math.sqrt(50.0)
    near(x[0], 3 * a)
    near(x[1], 8 * a)
    near(x[2], 6 * b)
    y = oracle.l2_norm([3, 4], width=2, eps=0.0)
    near(y[0], 0.6)
    near(y[1], 0.8)
    with pytest.raises(ValueError):
        oracle.rms_norm([np.inf, 1.0], [1.0, 1.0], width=2, eps=0.0)


def test_rotation(oracle):
    # Width 6 with four rotary values: pairs (0, 2) and (1, 3); 4 and 5 stay.
    x = oracle.rope([1, 2, 3, 4, 5, 6], rows=1, width=6, rotary=4, position=3, base=10000.0)
    t0, t1 = 3.0, 3.0 * 10000.0 ** -0.5
    near(x[0], 1 * math.cos(t0) - 3 * math.sin(t0))
    near(x[2], 1 * math.sin(t0) + 3 * math.cos(t0))
    near(x[1], 2 * math.cos(t1) - 4 * math.sin(t1))
    near(x[3], 2 * math.sin(t1) + 4 * math.cos(t1))
    assert x[4] == 5 and x[5] == 6
    origin = oracle.rope([1, 2, 3, 4], rows=1, width=4, rotary=4, position=0, base=10000.0)
    assert list(origin) == [1, 2, 3, 4]


def test_delta(oracle):
    dim = 3
    for per_key in (False, True):
        state = np.zeros(dim * dim, F)
        naive = np.zeros((dim, dim), np.float64)
        q = [F([.5, -.25, 1]), F([.1, .2, -.3])]
        k = [F([.3, .4, -.2]), F([-.6, .1, .5])]
        v = [F([1, -2, .5]), F([.25, .75, -1])]
        decay = F([.9, .8, .7]) if per_key else F([.95])
        beta = 0.6
        for t in range(2):
            out = oracle.delta_rule(state, q[t], k[t], v[t], decay, beta)
            g = decay if per_key else np.full(dim, decay[0])
            naive *= g[:, None]
            update = beta * (v[t] - naive.T @ k[t])
            naive += np.outer(k[t], update)
            expected = naive.T @ q[t]
            for j in range(dim):
                near(out[j], expected[j])
        for i in range(dim * dim):
            near(state[i], naive.reshape(-1)[i])


def test_delta_passes_bit_for_bit(oracle):
    """The fused two-pass recurrence equals the three-pass form bit for bit
    (the reference's LCG, seed 12345)."""
    dim = 128
    seed = [12345]

    def nxt():
        seed[0] = (seed[0] * 1664525 + 1013904223) & 0xFFFFFFFF
        return F((int(seed[0] >> 8) - (1 << 23)) / F(1 << 23))

    for per_key in (False, True):
        state = np.array([nxt() for _ in range(dim * dim)], F)
        ref = state.copy().reshape(dim, dim)
        for _ in range(4):
            q, k, v = (np.array([nxt() for _ in range(dim)], F) for _ in range(3))
            decay = np.array([F(0.5) + F(0.5) * F(abs(nxt())) for _ in range(dim if per_key else 1)], F)
            beta = F(F(0.5) + F(0.25) * nxt())
            out = oracle.delta_rule(state, q, k, v, decay, float(beta))
            g = decay if per_key else np.full(dim, decay[0], F)
            ref *= g[:, None]
            delta = v.copy()
            for i in range(dim):
                delta -= ref[i] * k[i]
            delta *= beta
            expected = np.zeros(dim, F)
            for i in range(dim):
                ref[i] += k[i] * delta
                expected += ref[i] * q[i]
            assert np.array_equal(out, expected)
            assert np.array_equal(state.reshape(dim, dim), ref)


def test_attention_causal(oracle):
    # Two query rows at positions 1 and 2, two heads sharing one KV head.
    heads, dim = 2, 2
    q = F([1, 0, 0, 1, .5, .5, -1, 2])
    k = F([1, 0, 0, 1, 1, 1])
    v = F([1, 2, 3, 4, 5, 6])
    scale = 0.7
    out = oracle.attend_cached(q, k, v, rows=2, position=1, heads=heads, kv_heads=1, dim=dim, scale=scale).reshape(-1)
    for row in range(2):
        for h in range(heads):
            visible = row + 2
            w = [math.exp((q[(row * heads + h) * dim] * k[t * dim] + q[(row * heads + h) * dim + 1] * k[t * dim + 1])
                          * scale) for t in range(visible)]
            total = sum(w)
            for d in range(dim):
                near(out[(row * heads + h) * dim + d], sum(w[t] / total * v[t * dim + d] for t in range(visible)))


def test_attention_selection_matches_gathered_keys(oracle):
    """A selected row attends exactly its listed positions (qwen_layers.cpp:
    300-330 gathers them and attends the gathered keys)."""
    rng = np.random.default_rng(3)
    heads, kv_heads, dim, pos = 4, 2, 8, 5
    k = rng.standard_normal((pos + 1) * kv_heads * dim).astype(F)
    v = rng.standard_normal(k.size).astype(F)
    q = rng.standard_normal(heads * dim).astype(F)
    sel = [0, 2, 5]
    got = oracle.attend_cached(q, k, v, rows=1, position=pos, heads=heads, kv_heads=kv_heads, dim=dim, scale=0.3,
                               selected=sel, offsets=[0, 3])
    kk = k.reshape(pos + 1, -1)[sel].reshape(-1)
    vv = v.reshape(pos + 1, -1)[sel].reshape(-1)
    want = oracle.attend_cached(q, kk, vv, rows=1, position=2, heads=heads, kv_heads=kv_heads, dim=dim, scale=0.3)
    assert np.array_equal(got, want)
