"""Both decode GEMVs against the CPU oracle (needs a B200).

Decode rows (M <= 64) have two CUDA implementations: the CUDA-core GEMV and the
tensor-core ones (exact integer dot products on tcgen05.mma.kind::i8; x staged
in the CTA for M <= 2, streamed as a limb matrix for 3 <= M <= 64: one M=64 MMA
up to 16 rows, one or two M=128 MMAs up to 32 / 64 rows; weights taller than one
tile per SM run as row slices, e.g. the 40000-row case below). The
library picks one per shape; GQ_DECODE_TC forces the choice (0 = CUDA cores,
2 = tensor cores wherever they apply), so every shape family here runs through
both, at the FFMA-path bound (relative L2 <= 1e-5 against the oracle).
"""
import numpy as np
import pytest

from oracle import oracle
from gq import CudaBackend
from gq import synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5


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


PATHS = ["0", "2"]

# (rows, K, bits, signed): E2B projections and odd sizes
SHAPES = [(2048, 1536, 8, True), (256, 1536, 8, True), (1536, 2048, 8, True), (6144, 1536, 4, False),
          (1536, 6144, 2, False), (300, 640, 8, False), (77, 256, 4, False), (5000, 512, 2, False),
          (40000, 1536, 8, True)]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("n,k,bits,signed", SHAPES)
@pytest.mark.parametrize("m", [1, 2, 3, 8, 16, 24, 40, 64])
def test_linear_both_paths(g, monkeypatch, path, n, k, bits, signed, m):
    monkeypatch.setenv("GQ_DECODE_TC", path)
    w = synth.random_qweight(3000 + n + k + bits, n, k, bits, signed)
    x = synth.normal(3001 + m, m * k).reshape(m, k)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m", [1, 2, 8, 33, 64])
def test_geglu_both_paths(g, monkeypatch, path, m):
    monkeypatch.setenv("GQ_DECODE_TC", path)
    n, k = 6144, 1536
    wg = synth.random_qweight(3101, n, k, 4, False)
    wu = synth.random_qweight(3102, n, k, 4, False)
    x = synth.normal(3103, m * k).reshape(m, k)
    got = g.readback(g.linear_geglu(g.tensor(x, x.shape), g.quant_tensor(wg), g.quant_tensor(wu)))
    assert rel_l2(got, oracle.linear_geglu(x, wg, wu)) <= REL_L2


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m", [2, 5, 40])
def test_gelu_mul_cols_both_paths(g, monkeypatch, path, m):
    monkeypatch.setenv("GQ_DECODE_TC", path)
    n, k, off = 256, 1536, 512
    w = synth.random_qweight(3201, n, k, 8, True)
    x = synth.normal(3202, m * k).reshape(m, k)
    b = synth.normal(3203, m * 8960).reshape(m, 8960)
    got = g.readback(g.linear_gelu_mul_cols(g.tensor(x, x.shape), g.quant_tensor(w), g.tensor(b, b.shape), off))
    assert rel_l2(got, oracle.linear_gelu_mul_cols(x, w, b, off)) <= REL_L2


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m,n", [(4, 32768), (48, 32768), (6, 65536)])
def test_softcap_slice_both_paths(g, monkeypatch, path, m, n):
    """A vocab shard written into its column range of a wider logits row."""
    monkeypatch.setenv("GQ_DECODE_TC", path)
    k, cap = 1536, 30.0
    w = synth.random_qweight(3301, n, k, 8, True)
    x = synth.normal(3302, m * k).reshape(m, k) * 4.0
    out = g.zeros((m, 3 * n))
    g.linear_softcap(g.tensor(x, x.shape), g.quant_tensor(w), cap, out=out, col0=n)
    got = g.readback(out).reshape(m, 3 * n)
    ref = oracle.softcap(oracle.linear(x, w), cap)
    assert rel_l2(got[:, n:2 * n], ref) <= REL_L2
    assert not np.any(got[:, :n]) and not np.any(got[:, 2 * n:])


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m", [6, 36])
def test_extreme_activations_both_paths(g, monkeypatch, path, m):
    """Fixed-point scaling across the f32 range: tiny, huge, large mean, outlier."""
    monkeypatch.setenv("GQ_DECODE_TC", path)
    n, k = 1024, 1536
    w = synth.make_qweight(3401, n, k, 4)
    base = synth.normal(3402, m * k).reshape(m, k)
    for label, x in [("tiny", base * 1e-30), ("huge", base * 1e25), ("mean", base + 5.0)]:
        x = x.astype(np.float32)
        got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
        assert rel_l2(got, oracle.linear(x, w)) <= REL_L2, label
    x = base.copy()
    x[:, 7] = 300.0
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2, "outlier"


@pytest.mark.parametrize("wa", ["0", "1"])
@pytest.mark.parametrize("n,k,bits,signed", [(2048, 1536, 8, True), (6144, 1536, 4, False), (1536, 6144, 2, False),
                                             (300, 640, 8, False), (40000, 1536, 8, True)])
@pytest.mark.parametrize("m", [5, 16, 24, 64])
def test_short_m_tensor_core_layouts(g, monkeypatch, wa, n, k, bits, signed, m):
    """Both operand layouts of the short-M tensor-core GEMV (limb rows as A with
    weight tiles as N, or weight tiles as A with limb rows as N) at every size."""
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    monkeypatch.setenv("GQ_TCX_WA", wa)
    w = synth.random_qweight(3500 + n + k + bits, n, k, bits, signed)
    x = synth.normal(3501 + m, m * k).reshape(m, k)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2


@pytest.mark.parametrize("wa", ["0", "1"])
@pytest.mark.parametrize("m", [7, 40])
def test_short_m_tensor_core_layouts_fused(g, monkeypatch, wa, m):
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    monkeypatch.setenv("GQ_TCX_WA", wa)
    n, k = 6144, 1536
    wg = synth.random_qweight(3601, n, k, 4, False)
    wu = synth.random_qweight(3602, n, k, 4, False)
    x = synth.normal(3603, m * k).reshape(m, k)
    got = g.readback(g.linear_geglu(g.tensor(x, x.shape), g.quant_tensor(wg), g.quant_tensor(wu)))
    assert rel_l2(got, oracle.linear_geglu(x, wg, wu)) <= REL_L2
    w = synth.random_qweight(3604, 256, k, 8, True)
    b = synth.normal(3605, m * 8960).reshape(m, 8960)
    got = g.readback(g.linear_gelu_mul_cols(g.tensor(x, x.shape), g.quant_tensor(w), g.tensor(b, b.shape), 768))
    assert rel_l2(got, oracle.linear_gelu_mul_cols(x, w, b, 768)) <= REL_L2


# (rows, K, bits, signed, M, "splits:tile"): split-K plans that fit (one CTA
# cluster of `splits` CTAs per weight tile, at most one CTA per SM)
SPLITS = [(1536, 6144, 2, False, 64, "8:128"), (1536, 6144, 2, False, 8, "8:128"), (1536, 6144, 2, False, 24, "4:64"),
          (2048, 1536, 8, True, 64, "8:128"), (2048, 1536, 8, True, 5, "4:128"), (6144, 1536, 4, False, 40, "2:128"),
          (300, 640, 8, False, 16, "2:64"), (1536, 2048, 8, True, 33, "8:128"), (77, 256, 4, False, 7, "2:16")]


@pytest.mark.parametrize("n,k,bits,signed,m,split", SPLITS)
def test_short_m_split_k_is_exact(g, monkeypatch, n, k, bits, signed, m, split):
    """Split-K over a CTA cluster: every split's exact int64 partial sums are
    added over distributed shared memory before the one conversion, so the
    output is bit-identical to the unsplit kernel's (and within the FFMA bound
    of the oracle)."""
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    monkeypatch.setenv("GQ_TCX_WA", "0")
    w = synth.random_qweight(3700 + n + k + bits, n, k, bits, signed)
    x = synth.normal(3701 + m, m * k).reshape(m, k)
    gw, gx = g.quant_tensor(w), g.tensor(x, x.shape)
    monkeypatch.setenv("GQ_TCX_SPLIT", "1")  # one CTA per tile, all K-blocks
    base = g.readback(g.linear(gx, gw))
    monkeypatch.setenv("GQ_TCX_SPLIT", split)
    got = g.readback(g.linear(gx, gw))
    again = g.readback(g.linear(gx, gw))
    assert np.array_equal(got, base) and np.array_equal(again, base)
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2


# (rows, K, bits, signed, M, splits) with the weights as the A operand (128-row
# tiles): every plan below fits, so each runs split (grid = tiles x splits <= SMs)
SPLITS_WA = [(1536, 6144, 2, False, 64, "8"), (1536, 6144, 2, False, 8, "8"), (2048, 1536, 8, True, 64, "6"),
             (2048, 1536, 8, True, 5, "4"), (6144, 1536, 4, False, 40, "3"), (300, 640, 8, False, 16, "5"),
             (1536, 2048, 8, True, 33, "8"), (77, 256, 4, False, 7, "2"), (2560, 1536, 8, True, 64, "6")]


@pytest.mark.parametrize("n,k,bits,signed,m,split", SPLITS_WA)
def test_short_m_split_k_weights_as_a_is_exact(g, monkeypatch, n, k, bits, signed, m, split):
    """The same cluster split-K with weight rows as the MMA's A operand: each
    thread's int64 limb sums for its weight row go to the shared partials, and
    the cluster's finalisation gives the unsplit kernel's output bit for bit."""
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    monkeypatch.setenv("GQ_TCX_WA", "1")
    w = synth.random_qweight(3750 + n + k + bits, n, k, bits, signed)
    x = synth.normal(3751 + m, m * k).reshape(m, k)
    gw, gx = g.quant_tensor(w), g.tensor(x, x.shape)
    monkeypatch.setenv("GQ_TCX_SPLIT", "1")
    base = g.readback(g.linear(gx, gw))
    for sp in (split, ""):  # the forced split, then the default (automatic) one
        monkeypatch.setenv("GQ_TCX_SPLIT", sp)
        got = g.readback(g.linear(gx, gw))
        assert np.array_equal(got, base), sp
    assert rel_l2(base, oracle.linear(x, w)) <= REL_L2


# (rows, K, bits, signed, M, weights-as-A, splits): plans whose CTAs convert x into
# their own limb tiles (no pre-pass launch), split and unsplit, both layouts
XIN = [(2048, 1536, 8, True, 8, "0", ""), (6144, 1536, 4, False, 8, "0", ""), (1536, 6144, 2, False, 8, "0", ""),
       (1536, 2048, 8, True, 16, "0", ""), (256, 1536, 8, True, 5, "0", ""), (1536, 256, 8, True, 64, "0", ""),
       (2048, 1536, 8, True, 8, "1", ""), (1536, 6144, 2, False, 33, "1", ""), (300, 640, 8, False, 16, "1", ""),
       (2048, 1536, 8, True, 64, "1", "6"), (77, 256, 4, False, 7, "0", ""), (40000, 1536, 8, True, 6, "0", "")]


@pytest.mark.parametrize("n,k,bits,signed,m,wa,split", XIN)
def test_short_m_in_kernel_limbs_equal_the_pre_pass(g, monkeypatch, n, k, bits, signed, m, wa, split):
    """Limb tiles made inside the GEMV (row maxima exchanged over the K-split
    cluster, zero points removed per split) give the pre-pass kernel's output bit
    for bit: same exponent, same digits, same integer sums. Rows with an outlier,
    tiny values and a non-finite entry included."""
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    monkeypatch.setenv("GQ_TCX_WA", wa)
    monkeypatch.setenv("GQ_TCX_SPLIT", split)
    w = synth.random_qweight(3900 + n + k + bits + m, n, k, bits, signed)
    x = synth.normal(3901 + m, m * k).reshape(m, k)
    x[0, 5] = 300.0
    x[m - 1] *= 1e-30
    if m > 2:
        x[1, k - 1] = np.inf
    gw, gx = g.quant_tensor(w), g.tensor(x, x.shape)
    monkeypatch.setenv("GQ_TCX_XIN", "0")
    base = g.readback(g.linear(gx, gw))
    monkeypatch.setenv("GQ_TCX_XIN", "1")
    got = g.readback(g.linear(gx, gw))
    assert np.array_equal(got, base, equal_nan=True)
    ok = np.ones(m, bool)
    if m > 2:
        ok[1] = False
        assert np.isnan(got.reshape(m, n)[1]).all()
    assert rel_l2(got.reshape(m, n)[ok], oracle.linear(x[ok], w)) <= REL_L2


def test_short_m_in_kernel_limbs_fused_modes(g, monkeypatch):
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    k, m = 1536, 8
    x = synth.normal(3951, m * k).reshape(m, k)
    gx = g.tensor(x, x.shape)
    wg = g.quant_tensor(synth.random_qweight(3952, 6144, k, 4, False))
    wu = g.quant_tensor(synth.random_qweight(3953, 6144, k, 4, False))
    gwp = g.quant_tensor(synth.random_qweight(3954, 256, k, 8, True))
    b = synth.normal(3955, m * 8960).reshape(m, 8960)
    gb = g.tensor(b, b.shape)
    gwl = g.quant_tensor(synth.random_qweight(3956, 2000, k, 8, True))
    outs = []
    for wa in ("0", "1"):
        monkeypatch.setenv("GQ_TCX_WA", wa)
        for xin in ("0", "1"):
            monkeypatch.setenv("GQ_TCX_XIN", xin)
            outs.append((g.readback(g.linear_geglu(gx, wg, wu)),
                         g.readback(g.linear_gelu_mul_cols(gx, gwp, gb, 768)),
                         g.readback(g.linear_softcap(gx, gwl, 30.0))))
    for o in outs[1:]:
        for a, b0 in zip(o, outs[0]):
            assert np.array_equal(a, b0)


def test_short_m_in_kernel_limbs_launch_one_kernel(g, monkeypatch):
    """With the in-kernel limbs an M = 8 projection is one launch (no limb pre-pass)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    k, m = 1536, 8
    x = synth.normal(3961, m * k).reshape(m, k)
    gx = g.tensor(x, x.shape)
    gw = g.quant_tensor(synth.random_qweight(3962, 2048, k, 8, True))
    g.linear(gx, gw)
    g.flush()
    names = {}
    for xin in ("1", "0"):
        monkeypatch.setenv("GQ_TCX_XIN", xin)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            g.linear(gx, gw)
            g.flush()
            torch.cuda.synchronize()
        names[xin] = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert any("gemv_tcx_kernel" in nm for nm in names["1"]) and not any("xlimbs" in nm for nm in names["1"])
    assert any("xlimbs" in nm for nm in names["0"])


@pytest.mark.parametrize("wa", ["0", "1"])
def test_short_m_split_k_fused_modes(g, monkeypatch, wa):
    monkeypatch.setenv("GQ_DECODE_TC", "2")
    monkeypatch.setenv("GQ_TCX_WA", wa)
    k = 1536
    x = synth.normal(3801, 40 * k).reshape(40, k)
    gx = g.tensor(x, x.shape)
    wg = g.quant_tensor(synth.random_qweight(3802, 6144, k, 4, False))
    wu = g.quant_tensor(synth.random_qweight(3803, 6144, k, 4, False))
    wp = synth.random_qweight(3804, 256, k, 8, True)
    gwp = g.quant_tensor(wp)
    b = synth.normal(3805, 40 * 8960).reshape(40, 8960)
    gb = g.tensor(b, b.shape)
    wl = synth.random_qweight(3806, 2000, k, 8, True)
    gwl = g.quant_tensor(wl)
    outs = []
    for split in ("1", "", "2:128", "4:32", "8:128", "3"):
        monkeypatch.setenv("GQ_TCX_SPLIT", split)
        outs.append((g.readback(g.linear_geglu(gx, wg, wu)),
                     g.readback(g.linear_gelu_mul_cols(gx, gwp, gb, 768)),
                     g.readback(g.linear_softcap(gx, gwl, 30.0))))
    for o in outs[1:]:
        for a, b0 in zip(o, outs[0]):
            assert np.array_equal(a, b0)
    assert rel_l2(outs[0][2], oracle.softcap(oracle.linear(x, wl), 30.0)) <= REL_L2


# M = 1 has two CUDA-core kernels: the register-x GEMV (gemv_r1.cu, for rows of a
# multiple of 128 bytes whose slice fits in shared memory) and the shared-memory GEMV
# (gemv_q.cu); GQ_GEMV_R1 selects (1) or deselects (0) the former.
R1_SHAPES = SHAPES + [(4608, 1536, 8, True), (1536, 4096, 8, True), (2560, 1536, 8, True), (96, 4096, 2, False),
                      (130, 1024, 4, False)]


@pytest.mark.parametrize("r1", ["0", "1"])
@pytest.mark.parametrize("n,k,bits,signed", R1_SHAPES)
def test_m1_kernels_linear(g, monkeypatch, r1, n, k, bits, signed):
    monkeypatch.setenv("GQ_DECODE_TC", "0")
    monkeypatch.setenv("GQ_GEMV_R1", r1)
    w = synth.random_qweight(3300 + n + k + bits, n, k, bits, signed)
    for seed, shift in ((3301, 0.0), (3302, 3.0)):  # zero-mean and shifted activations
        x = (synth.normal(seed, k) + shift).reshape(1, k)
        got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
        assert rel_l2(got, oracle.linear(x, w)) <= REL_L2


@pytest.mark.parametrize("r1", ["0", "1"])
def test_m1_kernels_fused_modes(g, monkeypatch, r1):
    """GeGLU (two weights), gelu * PLE slice and the soft-capped lm_head slice at M = 1."""
    monkeypatch.setenv("GQ_DECODE_TC", "0")
    monkeypatch.setenv("GQ_GEMV_R1", r1)
    k = 1536
    x = synth.normal(3401, k).reshape(1, k)
    gx = g.tensor(x, x.shape)
    wg = synth.random_qweight(3402, 6144, k, 4, False)
    wu = synth.random_qweight(3403, 6144, k, 4, False)
    got = g.readback(g.linear_geglu(gx, g.quant_tensor(wg), g.quant_tensor(wu)))
    assert rel_l2(got, oracle.linear_geglu(x, wg, wu)) <= REL_L2
    w = synth.random_qweight(3404, 256, k, 8, True)
    b = synth.normal(3405, 8960).reshape(1, 8960)
    for off in (0, 17 * 256, 34 * 256):
        got = g.readback(g.linear_gelu_mul_cols(gx, g.quant_tensor(w), g.tensor(b, b.shape), off))
        assert rel_l2(got, oracle.linear_gelu_mul_cols(x, w, b, off)) <= REL_L2
    wl = synth.random_qweight(3406, 4096, k, 8, True)
    xs = (4.0 * synth.normal(3407, k)).reshape(1, k)
    full = g.zeros((1, 3 * 4096))
    g.linear_softcap(g.tensor(xs, xs.shape), g.quant_tensor(wl), 30.0, out=full, col0=4096)
    got = g.readback(full).reshape(1, 3 * 4096)
    assert rel_l2(got[:, 4096:8192], oracle.softcap(oracle.linear(xs, wl), 30.0)) <= REL_L2
    assert not got[:, :4096].any() and not got[:, 8192:].any()


@pytest.mark.parametrize("m", [65, 96, 127])
@pytest.mark.parametrize("n,k,bits,signed", [(2048, 1536, 8, True), (1536, 6144, 2, False), (6144, 1536, 4, False),
                                             (300, 640, 8, False)])
def test_rows_65_to_127_blocked_tensor_core_gemv(g, monkeypatch, m, n, k, bits, signed):
    """Between the short-M GEMV (<= 64 rows) and the prefill GEMM (>= 128 rows): the
    short-M tensor-core GEMV in equal row blocks of at most 64, exact integer dot
    products, so the FFMA-path bound holds (the reference switches to its tiled
    kernel here, rust/src/backend_wgpu.rs:663-673)."""
    monkeypatch.delenv("GQ_DECODE_TC", raising=False)
    w = synth.random_qweight(3500 + n + k + bits, n, k, bits, signed)
    x = synth.normal(3501 + m, m * k).reshape(m, k)
    gw = g.quant_tensor(w)
    got = g.readback(g.linear(g.tensor(x, x.shape), gw))
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2
    if n == 6144:
        wu = synth.random_qweight(3502, n, k, bits, signed)
        got = g.readback(g.linear_geglu(g.tensor(x, x.shape), gw, g.quant_tensor(wu)))
        assert rel_l2(got, oracle.linear_geglu(x, w, wu)) <= REL_L2
    if n == 2048:
        full = g.zeros((m, n + 64))
        g.linear_softcap(g.tensor(x, x.shape), gw, 30.0, out=full, col0=64)
        got = g.readback(full).reshape(m, n + 64)
        assert rel_l2(got[:, 64:], oracle.softcap(oracle.linear(x, w), 30.0)) <= REL_L2
        b = synth.normal(3503, m * 4096).reshape(m, 4096)
        got = g.readback(g.linear_gelu_mul_cols(g.tensor(x, x.shape), gw, g.tensor(b, b.shape), 1024))
        assert rel_l2(got, oracle.linear_gelu_mul_cols(x, w, b, 1024)) <= REL_L2
