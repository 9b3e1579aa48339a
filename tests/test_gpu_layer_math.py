"""GPU parity of the layer math around the path (RMSNorm, L2 norm, RoPE,
cached attention, the gated delta-net step) against the oracle restatement of
the reference's host code (oracle/layer.c), on seeded inputs. Tolerances use
max|y - ref| / max(max|ref|, 1) (IW/tests/gguf_text.cpp:247-250); fp32
throughout, so 1e-5 for the elementwise ops and 1e-4 for attention and the
recurrent delta-net (different summation orders and CUDA's exp)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(cuda)


def test_rms_norm_and_l2_norm(kb, oracle, cuda):
    import torch

    rng = np.random.default_rng(1)
    rows, width = 7, 8192
    x = rng.standard_normal(rows * width).astype(np.float32) * 3
    w = rng.standard_normal(width).astype(np.float32)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    y = kb.rms_norm(dev(x, cuda), dev(w, cuda), width=width, eps=1e-6, status=status)
    assert rel_err(y.cpu().numpy().reshape(-1), oracle.rms_norm(x, w, width=width, eps=1e-6)) <= 1e-6
    assert int(status.item()) == 0
    # In place and unweighted.
    xd = dev(x, cuda)
    kb.rms_norm(xd, None, width=width, eps=1e-5, out=xd)
    assert rel_err(xd.cpu().numpy().reshape(-1), oracle.rms_norm(x, None, width=width, eps=1e-5)) <= 1e-6
    y2 = kb.l2_norm(dev(x, cuda), width=128, eps=1e-6)
    assert rel_err(y2.cpu().numpy().reshape(-1), oracle.l2_norm(x, width=128, eps=1e-6)) <= 1e-6
    # A non-finite output raises the status bit (gguf_text_norm_nonfinite).
    bad = x.copy()
    bad[5] = np.inf
    kb.rms_norm(dev(bad, cuda), dev(w, cuda), width=width, eps=1e-6, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1


@pytest.mark.parametrize("rotary", [128, 64])
def test_rope(kb, oracle, cuda, rotary):
    rng = np.random.default_rng(2)
    rows, heads, width, position = 3, 8, 128, 1000
    x = rng.standard_normal(rows * heads * width).astype(np.float32)
    y = kb.rope(dev(x, cuda), rows=rows, width=width, rotary=rotary, position=position, base=500000.0)
    want = oracle.rope(x, rows=rows, width=width, rotary=rotary, position=position, base=500000.0)
    assert rel_err(y.cpu().numpy().reshape(-1), want) <= 1e-5


ATTN = [
    # (rows, position, heads, kv_heads, dim): Llama-3-70B decode at 4k context,
    # a 4-row prefill chunk, and the other head sizes.
    (1, 4095, 64, 8, 128),
    (4, 1000, 64, 8, 128),
    (2, 300, 8, 2, 64),
    (3, 77, 16, 2, 256),
    (1, 0, 4, 4, 128),
]


@pytest.mark.parametrize("rows,position,heads,kv_heads,dim", ATTN)
def test_attend_cached(kb, oracle, cuda, rows, position, heads, kv_heads, dim):
    rng = np.random.default_rng(rows * 1000 + position)
    n = position + rows
    q = rng.standard_normal(rows * heads * dim).astype(np.float32)
    k = rng.standard_normal(n * kv_heads * dim).astype(np.float32)
    v = rng.standard_normal(n * kv_heads * dim).astype(np.float32)
    scale = 1.0 / np.sqrt(dim)
    got = kb.attend_cached(dev(q, cuda), dev(k, cuda), dev(v, cuda), rows=rows, position=position, heads=heads,
                           kv_heads=kv_heads, dim=dim, scale=scale)
    want = oracle.attend_cached(q, k, v, rows=rows, position=position, heads=heads, kv_heads=kv_heads, dim=dim,
                                scale=scale)
    assert rel_err(got.cpu().numpy(), want) <= 1e-4


def test_attend_cached_selected_positions(kb, oracle, cuda):
    import torch

    rng = np.random.default_rng(9)
    rows, position, heads, kv_heads, dim = 3, 600, 16, 4, 128
    n = position + rows
    q = rng.standard_normal(rows * heads * dim).astype(np.float32)
    k = rng.standard_normal(n * kv_heads * dim).astype(np.float32)
    v = rng.standard_normal(n * kv_heads * dim).astype(np.float32)
    sel, off = [], [0]
    for r in range(rows):
        own = position + r
        picks = sorted(rng.choice(own + 1, size=[5, 300, own + 1][r], replace=False).tolist())
        sel += picks
        off.append(len(sel))
    sel_d = torch.tensor(sel, dtype=torch.int32, device=cuda)
    off_d = torch.tensor(off, dtype=torch.int32, device=cuda)
    got = kb.attend_cached(dev(q, cuda), dev(k, cuda), dev(v, cuda), rows=rows, position=position, heads=heads,
                           kv_heads=kv_heads, dim=dim, scale=0.1, selected=sel_d, offsets=off_d)
    want = oracle.attend_cached(q, k, v, rows=rows, position=position, heads=heads, kv_heads=kv_heads, dim=dim,
                                scale=0.1, selected=sel, offsets=off)
    assert rel_err(got.cpu().numpy(), want) <= 1e-4


@pytest.mark.parametrize("key_heads,value_heads,dim,kernel,gate", [(16, 32, 128, 4, True), (2, 4, 256, 4, False),
                                                                   (4, 4, 64, 1, True)])
def test_delta_step_sequence(kb, oracle, cuda, key_heads, value_heads, dim, kernel, gate):
    """A 5-row step from zero state, then two 1-row steps on the carried state
    and history: outputs, state and history against the oracle after each."""
    import torch

    rng = np.random.default_rng(dim + kernel)
    channels = (2 * key_heads + value_heads) * dim
    inner = value_heads * dim
    conv = (rng.standard_normal(channels * kernel) * 0.5).astype(np.float32)
    dt = rng.standard_normal(value_heads).astype(np.float32)
    a = -np.abs(rng.standard_normal(value_heads)).astype(np.float32)
    norm = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    history = np.zeros(max(1, (kernel - 1) * channels), np.float32)
    state = np.zeros(value_heads * dim * dim, np.float32)
    hist_d = dev(history, cuda)
    state_d = dev(state, cuda)
    for rows in (5, 1, 1):
        qkv = rng.standard_normal(rows * channels).astype(np.float32)
        z = rng.standard_normal(rows * inner).astype(np.float32)
        alpha = rng.standard_normal(rows * value_heads).astype(np.float32)
        beta = rng.standard_normal(rows * value_heads).astype(np.float32)
        out_d = torch.empty(rows * inner, device=cuda)
        kb.delta_step(qkv=dev(qkv, cuda), z=dev(z, cuda), alpha=dev(alpha, cuda), beta=dev(beta, cuda),
                      conv=dev(conv, cuda), dt=dev(dt, cuda), a=dev(a, cuda), norm=dev(norm, cuda),
                      history=hist_d if kernel > 1 else None, state=state_d, output=out_d, rows=rows,
                      key_heads=key_heads, value_heads=value_heads, dim=dim, kernel=kernel, eps=1e-6,
                      sigmoid_gate=gate)
        want = oracle.delta_step(qkv, z, alpha, beta, conv, dt, a, norm, rows=rows, key_heads=key_heads,
                                 value_heads=value_heads, dim=dim, kernel=kernel, eps=1e-6, sigmoid_gate=gate,
                                 history=history, state=state)
        assert rel_err(out_d.cpu().numpy(), want) <= 1e-4
        assert rel_err(state_d.cpu().numpy(), state) <= 1e-4
        if kernel > 1:
            assert np.array_equal(hist_d.cpu().numpy(), history)


def test_attend_cached_host_mirrors_the_cache(kb, oracle, cuda):
    """attend_cached from host spans over the context's per-layer KV mirror:
    a 6-row prefill, then decode rows; positions mirrored earlier are reused
    (a change the caller makes to them below `position` is not seen), the
    call's own positions are uploaded again; two layers do not mix."""
    rng = np.random.default_rng(21)
    heads, kv_heads, dim, total = 16, 4, 128, 12
    k = rng.standard_normal((total, kv_heads * dim)).astype(np.float32)
    v = rng.standard_normal((total, kv_heads * dim)).astype(np.float32)
    ctx = kb.Context(0)
    scale = 0.088
    mirror_k, mirror_v = k.copy(), v.copy()
    for rows, position in ((6, 0), (1, 6), (2, 7), (1, 9)):
        q = rng.standard_normal(rows * heads * dim).astype(np.float32)
        if position:
            # Rewrite a position the context already mirrors: it keeps its copy.
            k[0] += 1.0
        got = kb.attend_cached_host(ctx, 7, q, k, v, rows=rows, position=position, heads=heads, kv_heads=kv_heads,
                                    dim=dim, scale=scale)
        mirror_k[position:position + rows] = k[position:position + rows]
        mirror_v[position:position + rows] = v[position:position + rows]
        want = oracle.attend_cached(q, mirror_k, mirror_v, rows=rows, position=position, heads=heads,
                                    kv_heads=kv_heads, dim=dim, scale=scale)
        assert rel_err(got, want) <= 1e-4
    # Another layer id starts its own mirror from the caller's current cache.
    q = rng.standard_normal(heads * dim).astype(np.float32)
    got = kb.attend_cached_host(ctx, 8, q, k, v, rows=1, position=9, heads=heads, kv_heads=kv_heads, dim=dim,
                                scale=scale)
    want = oracle.attend_cached(q, k, v, rows=1, position=9, heads=heads, kv_heads=kv_heads, dim=dim, scale=scale)
    assert rel_err(got, want) <= 1e-4
    with pytest.raises(kb.Unsupported):
        kb.attend_cached_host(ctx, 9, q, k, v, rows=1, position=9, heads=heads, kv_heads=kv_heads, dim=96,
                              scale=scale)
    kb.release_layers(ctx)
    ctx.close()


def test_delta_step_host_carries_state(kb, oracle, cuda):
    """delta_step from host spans: a fresh step, two later steps on the state
    the device carries, a snapshot equal to the oracle's state, a restore from
    that snapshot, and the lost-state rule after release."""
    rng = np.random.default_rng(5)
    key_heads, value_heads, dim, kernel = 4, 8, 128, 4
    channels = (2 * key_heads + value_heads) * dim
    conv = (rng.standard_normal(channels * kernel) * 0.5).astype(np.float32)
    dt = rng.standard_normal(value_heads).astype(np.float32)
    a = -np.abs(rng.standard_normal(value_heads)).astype(np.float32)
    norm = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    history = np.zeros((kernel - 1) * channels, np.float32)
    state = np.zeros(value_heads * dim * dim, np.float32)
    ctx = kb.Context(0)
    shape = dict(key_heads=key_heads, value_heads=value_heads, dim=dim, kernel=kernel, eps=1e-6, sigmoid_gate=True)

    def inputs(rows):
        return dict(qkv=rng.standard_normal(rows * channels), z=rng.standard_normal(rows * value_heads * dim),
                    alpha=rng.standard_normal(rows * value_heads), beta=rng.standard_normal(rows * value_heads))

    for i, rows in enumerate((3, 1, 1)):
        x = {n: t.astype(np.float32) for n, t in inputs(rows).items()}
        got = kb.delta_step_host(ctx, 3, fresh=i == 0, conv=conv, dt=dt, a=a, norm=norm, rows=rows, **x, **shape)
        want = oracle.delta_step(x["qkv"], x["z"], x["alpha"], x["beta"], conv, dt, a, norm, rows=rows,
                                 history=history, state=state, **shape)
        assert rel_err(got.reshape(-1), want) <= 1e-4
    snap_state, snap_hist = kb.recurrent_state_get(ctx, 3, state.size, history.size)
    assert rel_err(snap_state, state) <= 1e-4
    assert np.array_equal(snap_hist, history)
    # Restore the snapshot into a fresh layer and take the same next step on both.
    x = {n: t.astype(np.float32) for n, t in inputs(1).items()}
    a1 = kb.delta_step_host(ctx, 3, fresh=False, conv=conv, dt=dt, a=a, norm=norm, rows=1, **x, **shape)
    a2 = kb.delta_step_host(ctx, 4, fresh=True, conv=conv, dt=dt, a=a, norm=norm, rows=1, initial_state=snap_state,
                            initial_history=snap_hist, **x, **shape)
    assert np.array_equal(a1, a2)
    kb.release_layers(ctx)
    with pytest.raises(kb.KadanError, match="recurrent_state_lost"):
        kb.delta_step_host(ctx, 3, fresh=False, conv=conv, dt=dt, a=a, norm=norm, rows=1, **x, **shape)
    ctx.close()
