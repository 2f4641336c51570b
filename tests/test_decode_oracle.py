"""The oracle's support ops and decode-step composition, on CPU.

The C restatement of rust/src/backend_cpu.rs (rms_norm, rope, attention, the
fused compositions of rust/src/backend.rs:137-154) is checked against
independent numpy restatements written from the same Rust source, the masking
rules against brute force, and the decode step (rust/src/model.rs) for the
reference's own structural invariants (rust/tests/model.rs: finite logits,
deterministic re-run, KV sharing map).
"""
import numpy as np
import pytest

from gq import e2b, synth
from oracle import e2b_ref
from oracle import oracle as o


def rel(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def np_rms_norm(x, w, eps):
    x = x.astype(np.float64)
    inv = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    y = x * inv
    return y * w if w is not None else y


def np_rope(x, pos, theta, dh, heads, rot):
    y = x.astype(np.float64).copy()
    half = rot // 2
    j = np.arange(half)
    freq = np.float64(theta) ** (-(2.0 * j) / rot)
    for i, p in enumerate(pos):
        ang = p * freq
        a, b = y[i, :, :half].copy(), y[i, :, half:rot].copy()
        y[i, :, :half] = a * np.cos(ang) - b * np.sin(ang)
        y[i, :, half:rot] = b * np.cos(ang) + a * np.sin(ang)
    return y


def np_attention(q, k, v, qp, kp, scale, window, softcap=0.0):
    t, hq, dh = q.shape
    s, hkv, dv = v.shape
    g = hq // hkv
    out = np.zeros((t, hq, dv))
    for i in range(t):
        for h in range(hq):
            sc = np.array([np.dot(q[i, h].astype(np.float64), k[j, h // g]) * scale for j in range(s)])
            if softcap > 0:
                sc = softcap * np.tanh(sc / softcap)
            mask = np.array([(kp[j] <= qp[i]) and not (window > 0 and qp[i] - kp[j] >= window) for j in range(s)])
            if not mask.any():
                continue
            sc = np.where(mask, sc, -np.inf)
            p = np.exp(sc - sc.max())
            out[i, h] = (p[:, None] * v[:, h // g].astype(np.float64)).sum(0) / p.sum()
    return out.reshape(t, hq * dv)


@pytest.mark.parametrize("rows,d", [(5, 48), (3, 1536), (16, 256), (1, 7)])
def test_rms_norm_matches_float64(rows, d):
    x = synth.normal(10 + d, rows * d).reshape(rows, d)
    w = synth.uniform(11 + d, d, -0.1, 0.1)
    assert rel(o.rms_norm(x, w, 1e-6), np_rms_norm(x, w, 1e-6)) < 1e-6
    assert rel(o.rms_norm(x, None, 1e-6), np_rms_norm(x, None, 1e-6)) < 1e-6


def test_add_rms_norm_composition():
    x, r = synth.normal(20, 5 * 48).reshape(5, 48), synth.normal(21, 5 * 48).reshape(5, 48)
    w = synth.uniform(22, 48, -0.1, 0.1)
    s = np.array([1.37], np.float32)
    want = (r.astype(np.float64) + np_rms_norm(x, w, 1e-6)) * 1.37
    assert rel(o.add_rms_norm(r, x, w, 1e-6, s), want) < 1e-6
    # the exact composition of rust/src/backend.rs:137-144
    assert np.array_equal(o.add_rms_norm(r, x, w, 1e-6, s), o.scale(o.add(r, o.rms_norm(x, w, 1e-6)), 1.37))


@pytest.mark.parametrize("t,heads,dh,rot", [(4, 2, 16, 8), (2, 8, 256, 256), (2, 1, 512, 128), (3, 4, 16, 8)])
def test_rope_and_head_norm_rope(t, heads, dh, rot):
    x = synth.normal(30 + dh, t * heads * dh).reshape(t, heads, dh)
    pos = [0, 1, 5, 9][:t] if t <= 4 else list(range(t))
    assert rel(o.rope(x, pos, 1e4, dh, heads, rot), np_rope(x, pos, 1e4, dh, heads, rot)) < 1e-6
    w = synth.uniform(31 + dh, dh, -0.1, 0.1)
    hn = o.head_norm_rope(x, w, 1e-6, pos, 1e4, dh, heads, rot)
    want = np_rope(np_rms_norm(x.reshape(t * heads, dh), w, 1e-6).reshape(t, heads, dh), pos, 1e4, dh, heads, rot)
    assert rel(hn, want) < 1e-6
    # untouched tail past rotary_dim
    assert np.array_equal(o.rope(x, pos, 1e4, dh, heads, rot)[:, :, rot:], x[:, :, rot:])


@pytest.mark.parametrize("t,s,hq,hkv,dh,window", [(6, 6, 4, 1, 16, 3), (3, 300, 2, 1, 32, 0), (3, 300, 2, 1, 32, 150),
                                                  (1, 64, 8, 2, 32, 0), (5, 5, 8, 1, 16, 0)])
def test_attention_matches_brute_force(t, s, hq, hkv, dh, window):
    q = synth.normal(40 + s, t * hq * dh).reshape(t, hq, dh) * 0.5
    k = synth.normal(41 + s, s * hkv * dh).reshape(s, hkv, dh) * 0.5
    v = synth.normal(42 + s, s * hkv * dh).reshape(s, hkv, dh) * 0.5
    kp = np.arange(s)
    qp = np.arange(s - t, s)
    got = o.attention(q, k, v, qp, kp, 1.0 / np.sqrt(dh), window)
    assert rel(got, np_attention(q, k, v, qp, kp, 1.0 / np.sqrt(dh), window)) < 1e-5


def test_attention_masked_query_is_zero():
    q = np.ones((1, 2, 8), np.float32)
    k = np.ones((3, 1, 8), np.float32)
    v = np.ones((3, 1, 8), np.float32)
    # every key is in the future of the query
    assert not np.any(o.attention(q, k, v, [0], [5, 6, 7]))


def test_config_kv_sharing_map():
    """rust/tests/model.rs:14-27 on the tiny config, and the E2B map."""
    c = e2b.tiny_config(64)
    assert c.is_global(1) and not c.is_global(0)
    assert (c.dh(1), c.dh(0)) == (16, 8)
    assert all(c.kv_source(i) <= i for i in range(c.layers))
    assert c.kv_source(4) == 3 and c.kv_source(5) == 3
    e = e2b.e2b_config()
    assert e.global_layers == (4, 9, 14, 19, 24, 29, 34)
    assert [e.kv_source(i) for i in (15, 19, 34)] == [13, 14, 14]
    assert e.rope(4) == (1e6, 128) and e.rope(0) == (1e4, 256)


def test_decode_step_finite_and_deterministic():
    c = e2b.tiny_config(48)
    w = e2b.Weights(c, 42)
    a = e2b_ref.decode_step(c, w, [2, 10, 47], 4, e2b_ref.kv_from_weights(c, w, 3, 4, 8))
    b = e2b_ref.decode_step(c, w, [2, 10, 47], 4, e2b_ref.kv_from_weights(c, w, 3, 4, 8))
    assert a.shape == (3, 48) and np.isfinite(a).all()
    assert np.array_equal(a, b)


def test_decode_step_batch_rows_are_independent():
    """A batch of sequences gives each sequence the logits it gets alone."""
    c = e2b.small_config(512)
    w = e2b.Weights(c, 5)
    kv3 = e2b_ref.kv_from_weights(c, w, 3, 20, 24)
    got = e2b_ref.decode_step(c, w, [3, 200, 511], 20, kv3)
    kv1 = {i: (K[1:2].copy(), V[1:2].copy()) for i, (K, V) in e2b_ref.kv_from_weights(c, w, 3, 20, 24).items()}
    alone = e2b_ref.decode_step(c, w, [200], 20, kv1)
    assert np.array_equal(got[1], alone[0])
    # the step wrote slot 20 of every source layer
    assert all(np.any(K[:, 20]) and np.any(V[:, 20]) for K, V in kv3.values())
