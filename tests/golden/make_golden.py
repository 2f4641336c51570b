"""Writes tests/golden/kat.json: the known-answer vectors of the reference's own
CPU tests for the quantized path, restated as data.

Sources (Dhruba531/gemma-4-webgpu-kernels):
  rust/tests/weights.rs:32-42  int_pack_unpack_roundtrip — 33 values per width
                               spanning [-2^(b-1), 2^(b-1)-1], exact round trip
  rust/tests/weights.rs:44-52  dequantize_per_row — q=[1,-2,3,0,2,2,-1,4],
                               scales=[0.5,2.0], group 4 -> [0.5,-1,1.5,0,4,4,-2,8]
  rust/tests/weights.rs:64-71  per-tensor bit widths of the E2B quantization table
  rust/assets/config.json:57-89 the regex table those widths come from
  rust/tests/model.rs:77-101   sampler: greedy, top-k = 1, the once-per-token
                               repetition penalty, top-p head, seed determinism

The packed byte images are derived from the documented format (offset binary,
LSB-first; I8 two's complement: rust/src/dequant.rs:1-12) by the independent
packer below, so the oracle's pack_int is checked byte for byte, not only by
round trip. Run: python tests/golden/make_golden.py
"""
import json
import os


def pack(vals, bits):
    if bits == 8:
        return [v & 0xFF for v in vals]
    pb = 8 // bits
    out = [0] * (-(-len(vals) // pb))
    for i, v in enumerate(vals):
        raw = (v + (1 << (bits - 1))) & ((1 << bits) - 1)
        out[i // pb] |= raw << ((i % pb) * bits)
    return out


def main():
    kat = {"roundtrip": [], "dequantize_per_row": {}, "bits_for": {}, "quant_rules": []}
    for bits in (2, 4, 8):
        lo, hi = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
        vals = [lo + (i % (hi - lo + 1)) for i in range(33)]
        kat["roundtrip"].append({"bits": bits, "values": vals, "packed": pack(vals, bits)})
    q = [1, -2, 3, 0, 2, 2, -1, 4]
    kat["dequantize_per_row"] = {
        "q": q, "scales": [0.5, 2.0], "rows": 2, "cols": 4, "group_size": 4,
        "expected": [0.5, -1.0, 1.5, 0.0, 4.0, 4.0, -2.0, 8.0], "packed_4bit": pack(q, 4),
    }
    # rust/assets/config.json:57-89, in match order (first match wins)
    kat["quant_rules"] = [
        ["^lm_head$", 2],
        ["audio_tower(?!.*lconv1d\\.linear_start)", 2],
        ["audio_tower\\.layers\\.\\d+\\.lconv1d\\.linear_start\\.", 4],
        ["language_model\\.embed_tokens$", 2],
        ["language_model\\.embed_tokens_per_layer$", 4],
        ["language_model\\.layers\\.(\\d|1[0-4])\\.mlp\\.", 4],
        ["language_model\\.layers\\.\\d+\\.mlp\\.", 2],
        ["language_model\\.layers\\.\\d+\\.per_layer_input_gate$", 8],
        ["language_model\\.layers\\.\\d+\\.per_layer_projection$", 8],
        ["language_model\\.layers\\.\\d+\\.self_attn\\.", 4],
        ["vision_tower", 8],
    ]
    kat["bits_for"] = {
        "lm_head": 2,
        "language_model.layers.3.mlp.gate_proj": 4,
        "language_model.layers.15.mlp.gate_proj": 2,
        "language_model.layers.15.per_layer_input_gate": 8,
        "language_model.layers.0.self_attn.q_proj": 4,
        "language_model.norm": 16,
    }
    # rust/tests/model.rs:77-101 (fn sampler): logits, options, the draw its closure
    # returns, and the asserted token; "determinism" has no asserted token (the test
    # checks two equal runs from Rng::new(1) and the range)
    kat["sampler"] = [
        {"logits": [0.1, 5.0, 0.2, -1.0], "temperature": 0.0, "top_k": 0, "top_p": 1.0, "penalty": 1.0,
         "recent": [], "u": 0.99, "token": 1},
        {"logits": [0.0, 10.0, 9.0, -5.0], "temperature": 1.0, "top_k": 1, "top_p": 1.0, "penalty": 1.0,
         "recent": [], "u": 0.99, "token": 1},
        {"logits": [10.0, 4.0], "temperature": 0.0, "top_k": 0, "top_p": 1.0, "penalty": 2.0,
         "recent": [0, 0], "u": 0.99, "token": 0},
        {"logits": [0.0, 10.0, 9.9, -5.0], "temperature": 1.0, "top_k": 0, "top_p": 0.5, "penalty": 1.0,
         "recent": [], "u": 0.0, "token": 1},
    ]
    kat["sampler_determinism"] = {"n": 100, "step": 0.37, "seed": 1, "temperature": 1.0, "top_k": 64, "top_p": 0.95}
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat.json")
    with open(path, "w") as f:
        json.dump(kat, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
