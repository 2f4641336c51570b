"""Checkpoint loading (gq_st_* in libgq) on the committed tiny checkpoint in the real
on-disk layout (tests/golden/tiny_real_format.safetensors, written by
tests/golden/make_checkpoint.py as the analogue of rust/tests/common/mod.rs:160-235).

CPU: header parse and names, dtypes/shapes/payload slices against the writer's
manifest, the float decodes (BF16 of the fixture; F16 with subnormals, infinities and
NaN against numpy), name resolution (rust/src/weights.rs:37-48), the bit-width table
(rust/src/config.rs:161-169) and malformed headers.
GPU: every quantized tensor uploaded as ModelWeights::load builds it
(rust/src/weights.rs:86-110) — shape, bits, signedness and group size (the 4-bit
per-layer table with one scale per layer block, group = K / L) — and the uploaded
weights used by EMBED_Q (bit-exact) and MATMUL_Q (FFMA bound) against the oracle on
QuantWeights built from the same bytes in Python.
"""
import json
import os
import struct

import numpy as np
import pytest

from gq import QuantWeight, _abi, loader, synth
from oracle import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
CKPT = os.path.join(HERE, "golden", "tiny_real_format.safetensors")
MANIFEST = json.load(open(os.path.join(HERE, "golden", "tiny_real_format.json")))
RULES = [tuple(r) for r in MANIFEST["quant_rules"]]
KAT = json.load(open(os.path.join(HERE, "golden", "kat.json")))


@pytest.fixture(scope="module")
def f():
    st = loader.SafetensorsFile(CKPT)
    yield st
    st.close()


def quant_logicals():
    """Logical names of the quantized tensors, as the model asks for them."""
    out = []
    for name, dtype, _ in MANIFEST["tensors"]:
        if dtype not in ("U8", "I8"):
            continue
        if name.endswith(".embedding_quantized"):
            out.append(name[len("model."): -len(".embedding_quantized")] + ".weight")
        elif name == "lm_head.weight":
            out.append("lm_head.weight")
        else:
            out.append(name[len("model."):])
    return out


def expected_quant(logical):
    """QuantWeight fields as rust/src/weights.rs:86-110 derives them, from the manifest."""
    weight, scale, _ = loader.resolve(logical)
    meta = {n: (d, s) for n, d, s in MANIFEST["tensors"]}
    dtype, (n, cols) = meta[weight]
    base = logical[: -len(".weight")] if logical.endswith(".weight") else logical
    signed = dtype == "I8"
    bits = 8 if signed else loader.bits_for(base, RULES)
    k = cols * (1 if signed else 8 // bits)
    scale_cols = meta[scale][1][1]
    return n, k, bits, signed, k // scale_cols


def host_quant(f, logical):
    weight, scale, _ = loader.resolve(logical)
    n, k, bits, signed, group = expected_quant(logical)
    _, _, payload = f.info(weight)
    return QuantWeight(qbytes=np.frombuffer(payload, dtype=np.uint8).copy(), scales=f.read_f32(scale).ravel(),
                       shape=(n, k), bits=bits, signed_i8=signed, group_size=group)


def test_header_names_and_payloads_match_the_writer(f):
    names = f.names()
    assert names == sorted(n for n, _, _ in MANIFEST["tensors"])  # __metadata__ skipped
    blob = open(CKPT, "rb").read()
    hlen = struct.unpack("<Q", blob[:8])[0]
    hdr = json.loads(blob[8: 8 + hlen])
    for name, dtype, shape in MANIFEST["tensors"]:
        d, s, payload = f.info(name)
        assert d == dtype and list(s) == shape
        a, b = hdr[name]["data_offsets"]
        assert payload == blob[8 + hlen + a: 8 + hlen + b]


def test_float_decodes(f):
    w = f.read_f32("model.language_model.norm.weight")
    _, _, payload = f.info("model.language_model.norm.weight")
    want = (np.frombuffer(payload, dtype="<u2").astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(w, want)
    # F16 (safetensors.rs:75-86): normals, subnormals, signed zeros, infinities, NaN
    h = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0xC000, 0x7BFF, 0x7C00, 0xFC00, 0x7E00, 0x3555],
                 dtype="<u2")
    f32 = np.array([1.5, -2.25], dtype=np.float32)
    from golden.make_checkpoint import build_safetensors as build
    st = loader.SafetensorsFile(blob=build([("h", "F16", [len(h)], h.tobytes()), ("f", "F32", [2], f32.tobytes())]))
    got = st.read_f32("h")
    want = h.view(np.float16).astype(np.float32)
    assert np.array_equal(got[~np.isnan(want)], want[~np.isnan(want)]) and np.isnan(got[10])
    assert np.array_equal(np.signbit(got), np.signbit(want))
    assert np.array_equal(st.read_f32("f"), f32)
    st.close()


def test_name_resolution():
    """rust/src/weights.rs:37-48."""
    assert loader.resolve("lm_head.weight") == ("lm_head.weight", "lm_head.weight_scale", "")
    assert loader.resolve("language_model.embed_tokens.weight") == (
        "model.language_model.embed_tokens.embedding_quantized", "model.language_model.embed_tokens.embedding_scale", "")
    assert loader.resolve("language_model.embed_tokens_per_layer.weight")[0] == \
        "model.language_model.embed_tokens_per_layer.embedding_quantized"
    assert loader.resolve("language_model.layers.2.self_attn.q_proj.weight") == (
        "model.language_model.layers.2.self_attn.q_proj.weight",
        "model.language_model.layers.2.self_attn.q_proj.weight_scale",
        "model.language_model.layers.2.self_attn.q_proj")
    assert loader.resolve("language_model.layers.0.layer_scalar")[2] == "model.language_model.layers.0.layer_scalar"


def test_bits_for_matches_the_reference_table():
    """rust/tests/weights.rs:64-71 through the table of rust/assets/config.json:57-89
    (first match wins, 16 when nothing matches)."""
    rules = [tuple(r) for r in KAT["quant_rules"]]
    for name, bits in KAT["bits_for"].items():
        assert loader.bits_for(name, rules) == bits, name
    assert loader.bits_for("language_model.layers.3.mlp.gate_proj", RULES) == 4
    assert loader.bits_for("model.audio_tower.layers.2.lconv1d.linear_start.w", rules) == 4
    assert loader.bits_for("model.audio_tower.layers.2.ffw.w", rules) == 2
    with pytest.raises(_abi.GqError):
        loader.bits_for("x", [("([", 4)])


def test_malformed_files_are_errors_not_crashes(tmp_path):
    from golden.make_checkpoint import build_safetensors as build

    good = build([("a", "F32", [1], b"\0\0\0\0")])
    bad = [b"", b"\x05\0\0\0\0\0\0\0{}", good[:8] + b"[]" + good[10:],
           struct.pack("<Q", 2**40) + b"{}"]
    for blob in bad:
        with pytest.raises(_abi.GqError):
            loader.SafetensorsFile(blob=blob if blob else b"\0")
    # offsets past the end of the file: the header parses, the slice is refused
    js = json.dumps({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode()
    st = loader.SafetensorsFile(blob=struct.pack("<Q", len(js)) + js + b"\0" * 8)
    with pytest.raises(_abi.GqError):
        st.info("a")
    with pytest.raises(_abi.GqError):
        st.info("missing")
    st.close()
    p = tmp_path / "x.safetensors"
    p.write_bytes(good)
    st = loader.SafetensorsFile(str(p))
    assert st.names() == ["a"]
    st.close()
    with pytest.raises(_abi.GqError):
        loader.SafetensorsFile(str(tmp_path / "none.safetensors"))


@pytest.mark.gpu
def test_upload_every_quantized_tensor_and_use_it(f):
    import ctypes
    from ctypes import c_int32, c_int64

    from gq import CudaBackend

    g = CudaBackend(0)
    try:
        logicals = quant_logicals()
        assert len(logicals) == 2 + 1 + 9 * MANIFEST["config"]["layers"]
        for logical in logicals:
            t = loader.load_quant(g, f, logical, RULES)
            n, k, bits, signed, group = expected_quant(logical)
            vals = [c_int64(), c_int64(), c_int32(), c_int32(), c_int64()]
            g.lib.gq_qweight_info(ctypes.c_void_p(t.qw), *[ctypes.byref(v) for v in vals])
            assert [v.value for v in vals] == [n, k, bits, int(signed), group], logical
            q = host_quant(f, logical)
            if logical.startswith("language_model.embed_tokens"):
                ids = [0, q.shape[0] - 1, 7, 7, 3]
                emb = float(np.sqrt(np.float32(q.shape[1])))
                got = g.readback(g.embed_rows(t, ids, emb)).reshape(len(ids), q.shape[1])
                assert np.array_equal(got, oracle.embed_rows(q, ids, emb)), logical
            else:
                x = synth.normal(len(logical), 3 * q.shape[1]).reshape(3, q.shape[1])
                got = g.readback(g.linear(g.tensor(x, x.shape), t)).reshape(3, q.shape[0])
                ref = oracle.linear(x, q)
                assert np.linalg.norm(got - ref) <= 1e-5 * np.linalg.norm(ref), logical
        # the per-layer table: 4-bit, one scale per layer block of 12 columns
        assert expected_quant("language_model.embed_tokens_per_layer.weight")[2:] == (4, False, 12)
        with pytest.raises(_abi.GqError):
            loader.load_quant(g, f, "language_model.norm.weight", RULES)  # BF16: not quantized
        with pytest.raises(_abi.GqError):
            loader.load_quant(g, f, "language_model.layers.99.mlp.up_proj.weight", RULES)
    finally:
        g.close()
