"""Decode chains (gq_chain_*) against the CPU oracle, op by op (needs a B200).

A chain runs a list of one-row MATMUL_Q calls in one persistent launch, each op
reading what the ops before it wrote (rust/src/backend_wgpu.rs:768-835 issues the
same calls as one dispatch each). Every op is checked on the input it actually
read -- the GPU's outputs of the earlier ops, read back after the run -- against
the oracle at the GEMV bound (relative L2 <= 1e-5); replays of the same chain,
eager or from a captured graph, must give bit-identical outputs.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle
from gq import CudaBackend, GqError, synth
from gq import _abi

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5
# code standard deviation of the uniform codes per format: scales of ~1/(sqrt(K) * std)
# keep the activations of a long chain near unit size
QSTD = {2: 1.118, 4: 4.61, 8: 73.9}


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    nb = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (nb if nb > 0 else 1.0)


@pytest.fixture(scope="module")
def g():
    be = CudaBackend(0)
    yield be
    be.close()


def qw(seed, n, k, bits, signed=False, group=None):
    base = 1.0 / (np.sqrt(k) * QSTD[bits])
    return synth.random_qweight(seed, n, k, bits, signed, group, 0.7 * base, 1.3 * base)


def expect(op, x, b):
    """The oracle's output of one chain op given its input row x (and b)."""
    mode, w, w2, cap = op["mode"], op["w"], op.get("w2"), op.get("cap", 0.0)
    x = np.asarray(x, np.float32).reshape(1, -1)
    if mode == 1:
        return oracle.linear_geglu(x, w, w2)[0]
    if mode == 2:
        return oracle.linear_gelu_mul_cols(x, w, np.asarray(b, np.float32).reshape(1, -1), op["b_off"])[0]
    y = oracle.linear(x, w)[0]
    return oracle.softcap(y, cap) if (mode == 3 and cap > 0) else y


class Net:
    """Device buffers (name -> GqTensor) and chain ops that read/write them
    (x/y given as (buffer, element offset))."""

    def __init__(self, g):
        self.g, self.buf, self.ops = g, {}, []

    def add_buf(self, name, n, data=None):
        self.buf[name] = self.g.tensor(data, (n,)) if data is not None else self.g.zeros((n,))

    def add_op(self, mode, w, x, y, w2=None, b=None, b_off=0, cap=0.0):
        gw = self.g.quant_tensor(w)
        gw2 = self.g.quant_tensor(w2) if w2 is not None else None
        self.ops.append(dict(mode=mode, w=w, w2=w2, gw=gw, gw2=gw2, x=x, y=y, b=b, b_off=b_off, cap=cap))

    def ptr(self, ref):
        name, off = ref if isinstance(ref, tuple) else (ref, 0)
        return self.buf[name].ptr() + 4 * off

    def chain(self):
        return self.g.chain([(o["mode"], o["gw"], o["gw2"], self.ptr(o["x"]), self.ptr(o["y"]),
                              self.ptr(o["b"]) if o["b"] is not None else None, o["b_off"], o["cap"])
                             for o in self.ops])

    def snapshot(self):
        return {k: self.g.readback(v).copy() for k, v in self.buf.items()}

    def check(self, snap):
        for i, o in enumerate(self.ops):
            xn, xo = o["x"] if isinstance(o["x"], tuple) else (o["x"], 0)
            yn, yo = o["y"] if isinstance(o["y"], tuple) else (o["y"], 0)
            k, n = o["w"].shape[1], o["w"].shape[0]
            x = snap[xn][xo:xo + k]
            b = snap[o["b"]] if o["b"] is not None else None
            got = snap[yn][yo:yo + n]
            err = rel_l2(got, expect(o, x, b))
            assert err <= REL_L2, f"op {i} (mode {o['mode']}, {o['w'].bits}-bit {n}x{k}): rel L2 {err:.3g}"
            assert np.all(np.isfinite(got))


def e2b_layers(g, layers, seed=7000):
    """The six per-layer calls of a Gemma-4-E2B decode step, chained through their
    real data flow: h -> q|k|v -> o (reads the q part) -> gate+up GeGLU -> down ->
    PLE gate (gelu * this layer's 256 columns of the per-layer input) -> PLE
    projection -> the next layer's h."""
    net = Net(g)
    net.add_buf("h0", synth.HIDDEN, synth.normal(seed, synth.HIDDEN))
    net.add_buf("ple", synth.LAYERS * synth.PLE_DIM, synth.normal(seed + 1, synth.LAYERS * synth.PLE_DIM))
    s = seed + 10
    for i in range(layers):
        h, hn = f"h{i}", f"h{i + 1}"
        for name, n in (("qkv", 2560), ("a", synth.HIDDEN), ("inter", synth.INTER), ("d", synth.HIDDEN),
                        ("pg", synth.PLE_DIM), (hn, synth.HIDDEN)):
            net.add_buf(f"{name}{i}" if name != hn else hn, n)
        net.add_op(0, qw(s + 1, 2560, 1536, 8, True), h, f"qkv{i}")
        net.add_op(0, qw(s + 2, 1536, 2048, 8, True), (f"qkv{i}", 0), f"a{i}")
        net.add_op(1, qw(s + 3, 6144, 1536, 4), f"a{i}", f"inter{i}", w2=qw(s + 4, 6144, 1536, 4))
        net.add_op(0, qw(s + 5, 1536, 6144, 2), f"inter{i}", f"d{i}")
        net.add_op(2, qw(s + 6, 256, 1536, 8, True), f"d{i}", f"pg{i}", b="ple", b_off=i * synth.PLE_DIM)
        net.add_op(0, qw(s + 7, 1536, 256, 8, True), f"pg{i}", hn)
        s += 10
    return net


@pytest.mark.parametrize("layers", [1, 3])
def test_e2b_layers_chain_matches_oracle(g, layers):
    net = e2b_layers(g, layers)
    ch = net.chain()
    try:
        ch.run()
        g.flush()
        snap = net.snapshot()
        net.check(snap)
        # a second run (counters cleared by the first) gives the same bits
        ch.run()
        g.flush()
        again = net.snapshot()
        for k in snap:
            assert np.array_equal(snap[k], again[k]), k
    finally:
        ch.close()


def test_every_format_and_mode(g):
    """U8 / 4-bit / 2-bit / I8 weights in every mode, odd row counts (fewer rows
    than SMs, several ring slots per CTA), and an op reading an older op's output."""
    net = Net(g)
    net.add_buf("x0", 512, synth.normal(7101, 512))
    net.add_buf("b", 6000, synth.normal(7102, 6000))
    for name, n in (("y0", 640), ("y1", 384), ("y2", 320), ("y3", 448), ("y4", 77), ("y5", 1024),
                    ("y6", 4992), ("y7", 3)):
        net.add_buf(name, n)
    net.add_op(3, qw(7110, 640, 512, 8, False), "x0", "y0", cap=5.0)
    net.add_op(0, qw(7111, 384, 640, 4), "y0", "y1")
    net.add_op(1, qw(7112, 320, 384, 2), "y1", "y2", w2=qw(7113, 320, 384, 2))
    net.add_op(2, qw(7114, 448, 320, 8, True), "y2", "y3", b="b", b_off=100)
    net.add_op(1, qw(7115, 77, 448, 8, False), "y3", "y4", w2=qw(7116, 77, 448, 8, False))
    net.add_op(3, qw(7117, 1024, 448, 2), "y3", "y5", cap=0.0)
    net.add_op(2, qw(7118, 4992, 1024, 4), "y5", "y6", b="b", b_off=1000)
    net.add_op(0, qw(7119, 3, 4992, 8, True), "y6", "y7")
    ch = net.chain()
    try:
        ch.run()
        g.flush()
        net.check(net.snapshot())
    finally:
        ch.close()


@pytest.fixture(scope="module")
def gs():
    be = CudaBackend(0, own_stream=True)  # graphs are recorded from the backend's own stream
    yield be
    be.close()


def test_graph_replay_is_bit_identical(gs):
    g = gs
    net = e2b_layers(g, 2, seed=7300)
    ch = net.chain()
    try:
        ch.run()
        g.flush()
        ref = net.snapshot()
        graph = g.record(lambda: [ch.run() for _ in range(3)])
        try:
            for _ in range(2):
                g.replay(graph)
            g.flush()
            got = net.snapshot()
        finally:
            g.destroy_graph(graph)
        for k in ref:
            assert np.array_equal(ref[k], got[k]), k
    finally:
        ch.close()


def test_chain_equals_single_calls(g):
    """The chain against the same calls made one by one through gq_linear & co."""
    net = e2b_layers(g, 1, seed=7400)
    ch = net.chain()
    try:
        ch.run()
        g.flush()
        snap = net.snapshot()
    finally:
        ch.close()
    for o in net.ops:
        xn, xo = o["x"] if isinstance(o["x"], tuple) else (o["x"], 0)
        k = o["w"].shape[1]
        x = g.tensor(snap[xn][xo:xo + k].reshape(1, k), (1, k))
        if o["mode"] == 1:
            y = g.linear_geglu(x, o["gw"], o["gw2"])
        elif o["mode"] == 2:
            y = g.linear_gelu_mul_cols(x, o["gw"], g.tensor(snap[o["b"]].reshape(1, -1), (1, snap[o["b"]].size)),
                                       o["b_off"])
        else:
            y = g.linear(x, o["gw"])
        yn = o["y"] if not isinstance(o["y"], tuple) else o["y"][0]
        assert rel_l2(snap[yn], g.readback(y)) <= 2 * REL_L2


def test_rejections(g):
    lib = g.lib
    x = g.zeros((1024,))
    y = g.zeros((1024,))
    w = g.quant_tensor(qw(7500, 256, 512, 8, True))
    wg = g.quant_tensor(qw(7501, 256, 512, 8, True, group=128))

    def status(ops):
        arr = (_abi.ChainOp * len(ops))(*[_abi.ChainOp(*o) for o in ops])
        out = ctypes.c_void_p()
        rc = lib.gq_chain_create(g.ctx, arr, len(ops), ctypes.byref(out))
        if out.value:
            lib.gq_chain_destroy(out)
        return rc

    ok = (0, w.qw, None, x.ptr(), y.ptr(), None, 0, 0.0)
    assert status([ok]) == _abi.GQ_OK
    assert status([(0, wg.qw, None, x.ptr(), y.ptr(), None, 0, 0.0)]) == _abi.GQ_ERR_UNSUPPORTED  # grouped
    assert status([(0, w.qw, None, x.ptr() + 4, y.ptr(), None, 0, 0.0)]) == _abi.GQ_ERR_UNSUPPORTED  # x align
    assert status([(0, w.qw, None, x.ptr(), x.ptr() + 64, None, 0, 0.0)]) == _abi.GQ_ERR_INVALID_ARGUMENT  # y on x
    assert status([(7, w.qw, None, x.ptr(), y.ptr(), None, 0, 0.0)]) == _abi.GQ_ERR_INVALID_ARGUMENT  # mode
    assert status([(1, w.qw, None, x.ptr(), y.ptr(), None, 0, 0.0)]) == _abi.GQ_ERR_INVALID_ARGUMENT  # no up
    assert status([(2, w.qw, None, x.ptr(), y.ptr(), None, 0, 0.0)]) == _abi.GQ_ERR_INVALID_ARGUMENT  # no b
    assert status([ok, (0, None, None, x.ptr(), y.ptr(), None, 0, 0.0)]) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_chain_create(g.ctx, None, 0, ctypes.byref(ctypes.c_void_p())) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_chain_run(None) == _abi.GQ_ERR_INVALID_ARGUMENT
    with pytest.raises(GqError):
        g.chain([(0, wg, None, x.ptr(), y.ptr(), None, 0, 0.0)])
