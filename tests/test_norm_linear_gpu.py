"""gq_add_norm_linear: the decode step's residual add + RMSNorm fused into the
projection that reads it, one activation row (needs a B200).

The fused call must give exactly what its parts give: h_out equal to
gq_add_rms_norm / gq_add_rms_norm_norm bit for bit, and y equal to the CUDA-core
GEMV of that row (the register-x variant is switched off for the comparison,
GQ_GEMV_R1=0, so both sides run the same GEMV); y also against the oracle on the
row, at the GEMV bound. Shapes: the E2B projections that follow a norm in a
decode step (q|k|v with the layer scalar and the next input norm, gate|up GeGLU
after the post-attention norms, the PLE gate after the post-MLP norm).
"""
from ctypes import c_float, c_void_p

import numpy as np
import pytest

from oracle import oracle
from gq import CudaBackend, synth
from gq import _abi

pytestmark = pytest.mark.gpu

K = synth.HIDDEN
EPS = 1e-6


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.fixture(scope="module")
def g():
    be = CudaBackend(0)
    yield be
    be.close()


def ptr(t):
    return c_void_p(t.ptr()) if t is not None else None


def fused(g, mode, x, r, w1, s, w2, h, w, wu, b, b_off, y, k=K):
    return g.lib.gq_add_norm_linear(g.ctx, mode, ptr(x), ptr(r), k, ptr(w1), c_float(EPS), ptr(s), ptr(w2), ptr(h),
                                    c_void_p(w.qw), c_void_p(wu.qw) if wu is not None else None, ptr(b), b_off,
                                    ptr(y))


def composed(g, mode, x, r, w1, s, w2, w, wu, b, b_off, n, k=K):
    """The calls the fused one replaces: the norm(s), then the linear."""
    h = g.zeros((1, k))
    if w2 is not None:
        xn = g.zeros((1, k))
        g._check(g.lib.gq_add_rms_norm_norm(g.ctx, ptr(r), ptr(x), 1, k, ptr(w1), c_float(EPS), ptr(s), ptr(w2),
                                            ptr(h), ptr(xn)), "add_rms_norm_norm")
    else:
        g._check(g.lib.gq_add_rms_norm(g.ctx, ptr(r), ptr(x), 1, k, ptr(w1), c_float(EPS), ptr(s), ptr(h)),
                 "add_rms_norm")
        xn = h
    if mode == 1:
        y = g.linear_geglu(xn, w, wu)
    elif mode == 2:
        y = g.linear_gelu_mul_cols(xn, w, b, b_off)
    else:
        y = g.linear(xn, w)
    return h, xn, y


CASES = {  # mode, rows, bits, signed, layer scalar, second norm
    "qkv_after_ple_norm": (0, 2560, 8, True, True, True),
    "gate_up_after_post_attn": (1, synth.INTER, 4, False, False, True),
    "ple_gate_after_post_ffn": (2, synth.PLE_DIM, 8, True, False, False),
    "down_2bit_plain_norm": (0, 640, 2, False, False, False),
}


@pytest.mark.parametrize("case", list(CASES))
def test_equals_the_calls_it_fuses(g, monkeypatch, case):
    monkeypatch.setenv("GQ_GEMV_R1", "0")
    mode, n, bits, signed, with_s, with_w2 = CASES[case]
    seed = 8000 + n + bits
    x = g.tensor(synth.normal(seed, K).reshape(1, K), (1, K))
    r = g.tensor(synth.normal(seed + 1, K).reshape(1, K), (1, K))
    w1 = g.tensor(synth.uniform(seed + 2, K, 0.9, 1.1), (K,))
    w2 = g.tensor(synth.uniform(seed + 3, K, 0.9, 1.1), (K,)) if with_w2 else None
    s = g.tensor([1.07], (1,)) if with_s else None
    qw = synth.random_qweight(seed + 4, n, K, bits, signed)
    qu = synth.random_qweight(seed + 5, n, K, bits, signed) if mode == 1 else None
    w, wu = g.quant_tensor(qw), (g.quant_tensor(qu) if qu is not None else None)
    b = g.tensor(synth.normal(seed + 6, 9000).reshape(1, 9000), (1, 9000)) if mode == 2 else None
    b_off = 2048 if mode == 2 else 0
    h_ref, xn_ref, y_ref = composed(g, mode, x, r, w1, s, w2, w, wu, b, b_off, n)
    for _ in range(2):  # twice: nothing carried over between calls
        h = g.zeros((1, K))
        y = g.zeros((1, n))
        assert fused(g, mode, x, r, w1, s, w2, h, w, wu, b, b_off, y) == _abi.GQ_OK
        g.flush()
        assert np.array_equal(g.readback(h), g.readback(h_ref))
        assert np.array_equal(g.readback(y), g.readback(y_ref))
    xn = g.readback(xn_ref).reshape(1, K)
    if mode == 1:
        want = oracle.linear_geglu(xn, qw, qu)
    elif mode == 2:
        want = oracle.linear_gelu_mul_cols(xn, qw, g.readback(b).reshape(1, -1), b_off)
    else:
        want = oracle.linear(xn, qw)
    assert rel_l2(g.readback(y), want) <= 1e-5


def test_fallback_shapes_equal_the_calls(g):
    """Rows the fused GEMV does not take (k not a multiple of 4; grouped scales) run
    as the separate calls, with the same results."""
    for k, group in ((1534, None), (1536, 128)):
        x = g.tensor(synth.normal(8100 + k, k).reshape(1, k), (1, k))
        r = g.tensor(synth.normal(8101 + k, k).reshape(1, k), (1, k))
        w1 = g.tensor(synth.uniform(8102, k, 0.9, 1.1), (k,))
        w2 = g.tensor(synth.uniform(8103, k, 0.9, 1.1), (k,))
        qw = synth.random_qweight(8104 + k, 300, k, 8, True, group)
        w = g.quant_tensor(qw)
        h_ref, _, y_ref = composed(g, 0, x, r, w1, None, w2, w, None, None, 0, 300, k=k)
        h = g.zeros((1, k))
        y = g.zeros((1, 300))
        assert fused(g, 0, x, r, w1, None, w2, h, w, None, None, 0, y, k=k) == _abi.GQ_OK
        g.flush()
        assert np.array_equal(g.readback(h), g.readback(h_ref))
        assert np.array_equal(g.readback(y), g.readback(y_ref))


def test_rejections(g):
    x = g.tensor(synth.normal(8200, K).reshape(1, K), (1, K))
    r = g.tensor(synth.normal(8201, K).reshape(1, K), (1, K))
    w1 = g.tensor(synth.uniform(8202, K, 0.9, 1.1), (K,))
    w = g.quant_tensor(synth.random_qweight(8203, 64, K, 8, True))
    y = g.zeros((1, 64))
    h = g.zeros((1, K))
    bad = _abi.GQ_ERR_INVALID_ARGUMENT
    assert fused(g, 0, x, r, w1, None, None, r, w, None, None, 0, y) == bad  # h_out on the residual
    assert fused(g, 0, x, r, w1, None, None, h, w, None, None, 0, x) == bad  # y on x
    assert fused(g, 5, x, r, w1, None, None, h, w, None, None, 0, y) == bad  # mode
    assert fused(g, 1, x, r, w1, None, None, h, w, None, None, 0, y) == bad  # geglu without the up weight
    assert fused(g, 2, x, r, w1, None, None, h, w, None, None, 0, y) == bad  # gelu_mul_cols without b
    assert fused(g, 0, x, r, w1, None, None, h, w, None, None, 0, y, k=K - 4) == bad  # k != w.k
