"""The tcgen05 prefill GEMM (M >= 128) against the CPU oracle (needs a B200).

The kernel rounds each activation row to f16 after scaling it by a power of two
(2^e with |x| * 2^e < 2^14, undone exactly in the epilogue). Two bars per case:
  * against the f32 oracle: relative L2 <= 1e-2 (the tensor-core path's bound);
  * against the oracle run on the same row-scaled, f16-rounded activations:
    relative L2 <= 1e-5 — products of f16 activations and integer codes are
    exact, so only the accumulation order differs. This pins the widening, the
    permuted K order, the swizzled operand layout and the epilogue, not just the
    rounding budget.
"""
import numpy as np
import pytest

from oracle import oracle
from gq import CudaBackend, GqError, QuantWeight
from gq import synth
from numerics import f16_round, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    be = CudaBackend(0)
    yield be
    be.close()


CASES = [  # (m, n, k, bits, signed)
    (512, 6144, 1536, 4, False),   # config 3 gate/up shape
    (512, 1536, 6144, 2, False),   # config 3 down shape
    (128, 256, 64, 8, True),
    (130, 300, 128, 4, False),     # M and N tails
    (200, 520, 192, 2, False),
    (256, 2048, 1536, 8, True),    # I8 q_proj at prefill
    (384, 96, 256, 8, False),      # U8 8-bit, N < one tile
]


@pytest.mark.parametrize("m,n,k,bits,signed", CASES)
def test_prefill_linear(g, m, n, k, bits, signed):
    w = synth.make_qweight(100 + n + k, n, k, bits, signed)
    x = synth.normal(200 + m, m * k).reshape(m, k)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w))).reshape(m, n)
    assert rel_l2(got, oracle.linear(x, w)) <= 1e-2
    assert rel_l2(got, oracle.linear(f16_round(x), w)) <= 1e-5


@pytest.mark.parametrize("m,n,k,bits", [(512, 6144, 1536, 4), (160, 200, 128, 2)])
def test_prefill_geglu(g, m, n, k, bits):
    wg = synth.make_qweight(300 + n, n, k, bits)
    wu = synth.make_qweight(301 + n, n, k, bits)
    x = synth.normal(302, m * k).reshape(m, k)
    got = g.readback(g.linear_geglu(g.tensor(x, x.shape), g.quant_tensor(wg), g.quant_tensor(wu))).reshape(m, n)
    assert rel_l2(got, oracle.linear_geglu(x, wg, wu)) <= 1e-2
    assert rel_l2(got, oracle.linear_geglu(f16_round(x), wg, wu)) <= 1e-5


def test_prefill_gelu_mul_cols_and_softcap(g):
    m, n, k = 192, 256, 1536
    w = synth.make_qweight(401, n, k, 8, True)
    x = synth.normal(402, m * k).reshape(m, k)
    ple = synth.normal(403, m * 8960).reshape(m, 8960)
    got = g.readback(g.linear_gelu_mul_cols(g.tensor(x, x.shape), g.quant_tensor(w), g.tensor(ple, ple.shape),
                                            7 * 256)).reshape(m, n)
    assert rel_l2(got, oracle.linear_gelu_mul_cols(f16_round(x), w, ple, 7 * 256)) <= 1e-5
    wl = synth.make_qweight(404, 4096, k, 8, True)
    xs = (4.0 * synth.normal(405, m * k)).reshape(m, k)
    full = g.zeros((m, 3 * 4096))
    g.linear_softcap(g.tensor(xs, xs.shape), g.quant_tensor(wl), 30.0, out=full, col0=4096)
    got = g.readback(full).reshape(m, 3 * 4096)
    ref = oracle.softcap(oracle.linear(f16_round(xs), wl), 30.0)
    assert rel_l2(got[:, 4096:8192], ref) <= 1e-5
    assert not got[:, :4096].any() and not got[:, 8192:].any()


def test_prefill_reference_tile_sizes(g):
    """The reference's tiled-path cases (rust/tests/gpu.rs:335-349 shapes scaled to
    K % 64 == 0): partial 128-row tiles and N not a multiple of the tile."""
    for bits in (2, 4, 8):
        w = synth.make_qweight(500 + bits, 70, 128, bits, bits == 8)
        for m in (128, 129, 255):
            x = synth.normal(600 + m, m * 128).reshape(m, 128)
            got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w))).reshape(m, 70)
            assert rel_l2(got, oracle.linear(f16_round(x), w)) <= 1e-5, (bits, m)


@pytest.mark.parametrize("m,n,k,bits,mode", [(512, 1536, 6144, 2, 0), (256, 1024, 2048, 4, 1), (129, 640, 4096, 8, 0),
                                             (300, 96, 2048, 4, 3)])
def test_prefill_split_k_over_a_cluster(g, m, n, k, bits, mode):
    """Grids with fewer output tiles than SMs split K over a cluster of up to 8 CTAs
    (partials added over distributed shared memory): the config-3 down projection (24
    tiles, 4 splits), GeGLU pairs, a ragged token tile and the soft-capped epilogue,
    at the same bars as the unsplit kernel."""
    w = synth.make_qweight(900 + n + k, n, k, bits, bits == 8)
    x = synth.normal(901 + m, m * k).reshape(m, k)
    gx = g.tensor(x, x.shape)
    if mode == 1:
        wu = synth.make_qweight(902 + n, n, k, bits)
        got = g.readback(g.linear_geglu(gx, g.quant_tensor(w), g.quant_tensor(wu))).reshape(m, n)
        ref = oracle.linear_geglu(f16_round(x), w, wu)
    elif mode == 3:
        full = g.zeros((m, n + 32))
        g.linear_softcap(gx, g.quant_tensor(w), 30.0, out=full, col0=16)
        got = g.readback(full).reshape(m, n + 32)[:, 16:16 + n]
        ref = oracle.softcap(oracle.linear(f16_round(x), w), 30.0)
    else:
        got = g.readback(g.linear(gx, g.quant_tensor(w))).reshape(m, n)
        ref = oracle.linear(f16_round(x), w)
        assert rel_l2(got, oracle.linear(x, w)) <= 1e-2
    assert rel_l2(got, ref) <= 1e-5


@pytest.mark.parametrize("nt", [64, 192])
@pytest.mark.parametrize("m,n,k,bits,mode", [(512, 1536, 6144, 2, 0), (512, 768, 1536, 4, 1), (200, 300, 2048, 8, 2)])
def test_prefill_token_tiles(g, monkeypatch, nt, m, n, k, bits, mode):
    """Token tiles of 64 and 192 (GQ_PREFILL_NT; the default is 256, or 128 for
    short prefills): ragged last tiles, K split over clusters where the grid is
    small, GeGLU pairs and the column-slice epilogue, at the unsplit bars."""
    monkeypatch.setenv("GQ_PREFILL_NT", str(nt))
    w = synth.make_qweight(950 + n + k, n, k, bits, bits == 8)
    x = synth.normal(951 + m, m * k).reshape(m, k)
    gx = g.tensor(x, x.shape)
    if mode == 1:
        wu = synth.make_qweight(952 + n, n, k, bits)
        got = g.readback(g.linear_geglu(gx, g.quant_tensor(w), g.quant_tensor(wu))).reshape(m, n)
        ref = oracle.linear_geglu(f16_round(x), w, wu)
    elif mode == 2:
        b = synth.normal(953, m * (n + 40)).reshape(m, n + 40)
        got = g.readback(g.linear_gelu_mul_cols(gx, g.quant_tensor(w), g.tensor(b, b.shape), 40)).reshape(m, n)
        ref = oracle.linear_gelu_mul_cols(f16_round(x), w, b, 40)
    else:
        got = g.readback(g.linear(gx, g.quant_tensor(w))).reshape(m, n)
        ref = oracle.linear(f16_round(x), w)
    assert rel_l2(got, ref) <= 1e-5
