"""CUDA path vs the CPU oracle through the C ABI (needs a B200).

The first two tests rebuild the quantized cases of the reference's GPU suite
value for value (same LCG, same draw order, same shapes):
  quantized_kernel_parity  rust/tests/gpu.rs:145-188
  fused_op_parity          rust/tests/gpu.rs:298-383 (quantized parts)
and hold them to the reference's max-abs tolerance (2e-3 / 4e-3,
rust/tests/gpu.rs:30-35) AND to the north-star bound for the FFMA path:
relative L2 <= 1e-5. The generic (MATMUL_Q_SCALAR) path and EMBED_Q are
checked bit for bit. The rest covers the E2B shapes and the edge cases.
"""
import numpy as np
import pytest

from oracle import oracle
from gq import CudaBackend, GqError, QuantWeight
from gq import synth

pytestmark = pytest.mark.gpu

REL_L2_FFMA = 1e-5


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


def close(label, got, ref, tol, rel=REL_L2_FFMA):
    got = np.asarray(got).reshape(np.asarray(ref).shape)
    d = float(np.max(np.abs(got - ref))) if np.size(ref) else 0.0
    r = rel_l2(got, ref)
    assert d < tol, f"{label}: max diff {d:.3e} >= {tol:.1e}"
    assert r <= rel, f"{label}: rel L2 {r:.3e} > {rel:.1e}"


def qw_u(r, n, k, bits, base=0.01, width=0.05):
    vals = r.randu(n * k, bits)
    return QuantWeight(qbytes=synth.pack_unsigned(vals, bits), scales=r.scales(n, base, width), shape=(n, k),
                       bits=bits, signed_i8=False, group_size=k)


def qw_i8(r, n, k, base=0.01, width=0.05):
    qbytes = np.array([int(np.floor(r.next() * np.float32(256.0))) & 0xFF for _ in range(n * k)], np.uint8)
    return QuantWeight(qbytes=qbytes, scales=r.scales(n, base, width), shape=(n, k), bits=8, signed_i8=True,
                       group_size=k)


def run_linear(g, x, q, m, k):
    return g.readback(g.linear(g.tensor(x, (m, k)), g.quant_tensor(q)))


def test_quantized_kernel_parity(g):
    """rust/tests/gpu.rs:145-188."""
    r = synth.Lcg(9)
    for bits in (4, 2):
        n, k = 40, 64
        q = qw_u(r, n, k, bits)
        for m in (5, 1):
            x = r.rand(m * k, 1.0)
            close(f"linear q{bits} M={m}", run_linear(g, x, q, m, k), oracle.linear(x.reshape(m, k), q), 2e-3)
    # odd K -> generic path: same operation order as the CPU, so bit-exact
    n, k, m = 21, 52, 3
    q = qw_u(r, n, k, 4)
    x = r.rand(m * k, 1.0)
    got = run_linear(g, x, q, m, k)
    ref = oracle.linear(x.reshape(m, k), q)
    assert np.array_equal(got.reshape(ref.shape), ref), "generic path must be bit-exact"
    # signed int8
    n, k, m = 30, 48, 4
    q = qw_i8(r, n, k, 0.01, 0.03)
    x = r.rand(m * k, 1.0)
    close("linear i8", run_linear(g, x, q, m, k), oracle.linear(x.reshape(m, k), q), 2e-3)
    # quantized embedding with grouped scales (2 groups per row): bit-exact
    v, d, bits, group = 50, 32, 4, 16
    vals = r.randu(v * d, bits)
    q = QuantWeight(qbytes=synth.pack_unsigned(vals, bits), scales=r.scales(v * (d // group), 0.02, 0.04),
                    shape=(v, d), bits=bits, signed_i8=False, group_size=group)
    ids = [3, 7, 49, 0, 21]
    got = g.readback(g.embed_rows(g.quant_tensor(q), ids, float(np.sqrt(np.float32(d)))))
    ref = oracle.embed_rows(q, ids, float(np.sqrt(np.float32(d))))
    assert np.array_equal(got.reshape(ref.shape), ref)


def test_fused_op_parity(g):
    """rust/tests/gpu.rs:298-383, the quantized cases (the norm/rope draws are
    consumed so every later value matches the reference's)."""
    r = synth.Lcg(33)
    r.rand(5 * 48, 1.0), r.rand(5 * 48, 1.0), r.rand(48, 0.1)  # add_rms_norm block
    for (t, heads, dh, _rot) in [(3, 4, 16, 8), (2, 8, 256, 256), (2, 1, 512, 128)]:
        r.rand(t * heads * dh, 1.0), r.rand(dh, 0.1)  # head_norm_rope block
    for bits in (2, 4, 8):
        n, k = 70, 96
        q = qw_i8(r, n, k) if bits == 8 else qw_u(r, n, k, bits)
        for m in (8, 9, 64, 70):
            x = r.rand(m * k, 1.0)
            close(f"linear q{bits} M={m}", run_linear(g, x, q, m, k), oracle.linear(x.reshape(m, k), q), 4e-3)
    for bits in (2, 4):
        n, k = 40, 64
        wg, wu = qw_u(r, n, k, bits), qw_u(r, n, k, bits)
        gwg, gwu = g.quant_tensor(wg), g.quant_tensor(wu)
        for m in (1, 4, 9, 40):
            x = r.rand(m * k, 1.0)
            got = g.readback(g.linear_geglu(g.tensor(x, (m, k)), gwg, gwu))
            close(f"linear_geglu q{bits} M={m}", got, oracle.linear_geglu(x.reshape(m, k), wg, wu), 2e-3)
    n, k, stride, off = 24, 32, 96, 48
    w = qw_i8(r, n, k)
    gw = g.quant_tensor(w)
    for m in (1, 6, 33):
        x = r.rand(m * k, 1.0)
        b = r.rand(m * stride, 1.0)
        got = g.readback(g.linear_gelu_mul_cols(g.tensor(x, (m, k)), gw, g.tensor(b, (m, stride)), off))
        ref = oracle.linear_gelu_mul_cols(x.reshape(m, k), w, b.reshape(m, stride), off)
        close(f"linear_gelu_mul_cols i8 M={m}", got, ref, 2e-3)


E2B = [  # (name, n, k, bits, signed)
    ("gate 4b 6144x1536 (config 1)", 6144, 1536, 4, False),
    ("q_local i8 2048x1536", 2048, 1536, 8, True),
    ("q_global i8 4096x1536", 4096, 1536, 8, True),
    ("k_local i8 256x1536", 256, 1536, 8, True),
    ("v_global i8 512x1536", 512, 1536, 8, True),
    ("o_local i8 1536x2048", 1536, 2048, 8, True),
    ("down 2b 1536x6144", 1536, 6144, 2, False),
    ("ple_proj i8 1536x256", 1536, 256, 8, True),
    ("q 4b 2048x1536 (checkpoint width)", 2048, 1536, 4, False),
]


@pytest.mark.parametrize("name,n,k,bits,signed", E2B, ids=[e[0] for e in E2B])
@pytest.mark.parametrize("m", [1, 2, 3, 8])
def test_e2b_shapes(g, name, n, k, bits, signed, m):
    q = synth.make_qweight(1000 + n + k + bits, n, k, bits, signed)
    x = synth.normal(77 + m, m * k).reshape(m, k)
    got = g.readback(g.linear(g.tensor(x, (m, k)), g.quant_tensor(q)))
    ref = oracle.linear(x, q)
    assert rel_l2(got, ref) <= REL_L2_FFMA, name


@pytest.mark.parametrize("m", [1, 8])
def test_e2b_gate_up_geglu(g, m):
    wg = synth.make_qweight(11, 6144, 1536, 4)
    wu = synth.make_qweight(12, 6144, 1536, 4)
    x = synth.normal(13, m * 1536).reshape(m, 1536)
    got = g.readback(g.linear_geglu(g.tensor(x, x.shape), g.quant_tensor(wg), g.quant_tensor(wu)))
    ref = oracle.linear_geglu(x, wg, wu)
    assert rel_l2(got, ref) <= REL_L2_FFMA


@pytest.mark.parametrize("m", [1, 3])
def test_e2b_ple_gate(g, m):
    w = synth.make_qweight(21, 256, 1536, 8, True)
    x = synth.normal(22, m * 1536).reshape(m, 1536)
    ple = synth.normal(23, m * 8960).reshape(m, 8960)
    for layer in (0, 17, 34):
        got = g.readback(g.linear_gelu_mul_cols(g.tensor(x, x.shape), g.quant_tensor(w), g.tensor(ple, ple.shape),
                                                layer * 256))
        ref = oracle.linear_gelu_mul_cols(x, w, ple, layer * 256)
        assert rel_l2(got, ref) <= REL_L2_FFMA


@pytest.mark.parametrize("m", [1, 2])
def test_lm_head_softcap_and_shard_slice(g, m):
    """lm_head rows with the soft-cap fused, written into a column slice of a
    wider logits buffer (what one vocab shard does)."""
    n, k, cap = 8192, 1536, 30.0
    w = synth.make_qweight(31, n, k, 8, True)
    x = (3.0 * synth.normal(32, m * k)).reshape(m, k)
    ref = oracle.softcap(oracle.linear(x, w), cap)
    full = g.zeros((m, 3 * n))
    g.linear_softcap(g.tensor(x, x.shape), g.quant_tensor(w), cap, out=full, col0=n)
    got = g.readback(full).reshape(m, 3 * n)
    assert rel_l2(got[:, n:2 * n], ref) <= REL_L2_FFMA
    assert not got[:, :n].any() and not got[:, 2 * n:].any()


@pytest.mark.parametrize("n,k,bits,signed", [(65536, 1536, 8, True), (32768, 1536, 8, True),
                                              (40000, 1536, 4, False), (20000, 6144, 2, False)])
def test_lm_head_scale_shapes(g, n, k, bits, signed):
    """Row counts of a full or sharded vocab projection (thousands of rows per
    CTA, deep pipelines, large stage sizes)."""
    w = synth.random_qweight(900 + n, n, k, bits, signed)
    x = synth.normal(901, k).reshape(1, k)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2_FFMA


@pytest.mark.parametrize("kind", ["mean", "outlier", "tiny", "huge"])
def test_precision_robustness(g, kind):
    """Activations with a large mean, an outlier channel, or extreme scale."""
    n, k = 1024, 1536
    w = synth.make_qweight(41, n, k, 4)
    x = synth.normal(42, 2 * k).reshape(2, k)
    if kind == "mean":
        x = x + 5.0
    elif kind == "outlier":
        x[:, 7] = 300.0
    elif kind == "tiny":
        x = x * 1e-30
    else:
        x = x * 1e25
    x = x.astype(np.float32)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    ref = oracle.linear(x, w)
    assert rel_l2(got, ref) <= REL_L2_FFMA, kind


@pytest.mark.parametrize("n", [1, 3, 149, 297, 5000])
def test_odd_row_counts(g, n):
    w = synth.make_qweight(50 + n, n, 512, 2)
    x = synth.normal(51, 4 * 512).reshape(4, 512)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2_FFMA


def test_unsigned_8bit_and_grouped_scales(g):
    """U8 8-bit (offset binary, zp 128) and grouped scales (generic path, exact)."""
    w = synth.make_qweight(61, 96, 256, 8, signed_i8=False)
    x = synth.normal(62, 2 * 256).reshape(2, 256)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    assert rel_l2(got, oracle.linear(x, w)) <= REL_L2_FFMA
    wg = synth.make_qweight(63, 40, 128, 4, group_size=32)
    got = g.readback(g.linear(g.tensor(x[:, :128].copy(), (2, 128)), g.quant_tensor(wg)))
    ref = oracle.linear(x[:, :128], wg)
    assert np.array_equal(got.reshape(ref.shape), ref)


def test_embed_config4_shapes_bit_exact(g):
    """EMBED_Q at the config-4 row widths (fewer ids/rows to keep the CPU check fast)."""
    v = 4096
    tok = synth.make_qweight(71, v, 1536, 4)
    ple = synth.make_qweight(72, v, 35 * 256, 8, True, group_size=256)
    ids = synth.int_codes(73, 512, 0, v - 1).astype(np.uint32)
    for table, emb in ((tok, float(np.sqrt(np.float32(1536)))), (ple, 16.0)):
        got = g.readback(g.embed_rows(g.quant_tensor(table), ids, emb))
        ref = oracle.embed_rows(table, ids, emb)
        assert np.array_equal(got.reshape(ref.shape), ref)


def test_embed_config4_full_size_bit_exact(g):
    """BASELINE config 4 at its own size: the 262,144-row 4-bit token table and the
    I8 per-layer table [262,144, 35 x 256 = 8960] with one scale per 256-column
    block, 4096 ids including row 0, the last row (262,143, whose byte offset in the
    I8 table passes 2^31) and duplicates; bit-exact against the oracle
    (rust/src/backend_cpu.rs:127-137)."""
    v = 262144
    tok = synth.random_qweight(7401, v, 1536, 4)
    ple = synth.random_qweight(7402, v, 35 * 256, 8, True, group_size=256)
    ids = synth.int_codes(7403, 4096, 0, v - 1).astype(np.uint32)
    ids[:4] = [0, v - 1, v - 1, 0]
    ids[100:110] = ids[200:210]
    ids[-1] = v - 1
    assert int(v - 1) * 8960 > 2 ** 31
    for table, emb in ((tok, float(np.sqrt(np.float32(1536)))), (ple, 16.0)):
        qt = g.quant_tensor(table)
        got = g.readback(g.embed_rows(qt, ids, emb))
        g.free_quant(qt)
        ref = oracle.embed_rows(table, ids, emb)
        assert np.array_equal(got.reshape(ref.shape), ref)


def test_embed_odd_width_and_duplicates(g):
    t = synth.make_qweight(81, 20, 18, 4)  # D % 4 != 0 -> per-element kernel
    ids = [0, 19, 19, 5, 0]
    got = g.readback(g.embed_rows(g.quant_tensor(t), ids, 0.5))
    assert np.array_equal(got.reshape(5, 18), oracle.embed_rows(t, ids, 0.5))
    # K not a multiple of the values per byte cannot be packed (row_bytes = K / per_byte
    # truncates in rust/src/backend.rs:33-36): rejected at upload
    with pytest.raises(GqError):
        g.quant_tensor(QuantWeight(np.zeros(40, np.uint8), np.ones(20, np.float32), (20, 18), 2, False, 18))


def test_embed_bad_id_raises(g):
    t = synth.make_qweight(82, 10, 32, 4)
    out = g.embed_rows(g.quant_tensor(t), [1, 10], 1.0)
    with pytest.raises(GqError):
        g.readback(out)
    # the context stays usable and the error was cleared
    ok = g.readback(g.embed_rows(g.quant_tensor(t), [1, 9], 1.0))
    assert np.array_equal(ok.reshape(2, 32), oracle.embed_rows(t, [1, 9], 1.0))


def test_empty_and_invalid(g):
    w = g.quant_tensor(synth.make_qweight(91, 16, 64, 4))
    y = g.linear(g.zeros((0, 64)), w)
    assert y.shape == (0, 16)
    e = g.embed_rows(w, [], 1.0)
    assert e.shape == (0, 64)
    with pytest.raises(GqError):
        g.linear(g.zeros((2, 32)), w)  # K mismatch
    with pytest.raises(GqError):
        g.linear_gelu_mul_cols(g.zeros((1, 64)), w, g.zeros((1, 20)), 8)  # offset + N > stride
    with pytest.raises(GqError):
        g.quant_tensor(QuantWeight(np.zeros(8, np.uint8), np.ones(2, np.float32), (2, 8), 3, False, 8))


def test_softcap_and_geglu_elementwise(g):
    x = synth.normal(95, 4096) * 40
    got = g.readback(g.softcap(g.tensor(x, (4096,)), 30.0))
    assert rel_l2(got, oracle.softcap(x, 30.0)) <= 1e-6
    u = synth.normal(96, 4096)
    got = g.readback(g.geglu(g.tensor(x, (4096,)), g.tensor(u, (4096,))))
    assert rel_l2(got, oracle.geglu(x, u)) <= 1e-6
