"""Writes tests/golden/tiny_real_format.safetensors and tiny_real_format.json: a tiny
checkpoint in the reference's REAL on-disk format, the analogue of the reference's own
fixture (rust/tests/common/mod.rs:160-235, real_format_config_json +
real_format_tensors with seed 5 and vocab 40, the configuration of
rust/tests/gpu.rs:235-244):
  * U8 sub-byte packed / I8 weights with F32 scale tensors `<name>_scale`;
  * BF16 norms and per_layer_model_projection (truncated f32 -> bf16, as f32_to_bf16);
  * `model.language_model.*` names, `lm_head.weight` without the prefix, and the
    embeddings as `.embedding_quantized` / `.embedding_scale`;
  * the 4-bit per-layer embedding table with one scale per layer block
    (scale_cols = L, group = K / L), and a vision tensor the text model ignores.
Values come from the reference's test Lcg (rust/tests/common/mod.rs:29-42) in the
same draw order, so the tensors hold the same numbers as the reference's fixture.
The JSON holds the tiny config's shapes and the checkpoint's quantization rules in
match order. Run: python tests/golden/make_checkpoint.py
"""
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "gemma-4-webgpu-kernels_b200"))
from gq import synth  # noqa: E402

# rust/tests/common/mod.rs:44-55 (vocab 40) and :162-175 (the quantization rules)
CFG = {"vocab": 40, "hidden": 32, "inter": 64, "layers": 6, "heads_q": 4, "heads_kv": 1, "head_dim": 8,
       "global_head_dim": 16, "ple_dim": 12, "global_layers": [1]}
RULES = [
    ["^lm_head$", 2],
    ["language_model\\.embed_tokens$", 2],
    ["language_model\\.embed_tokens_per_layer$", 4],
    ["language_model\\.layers\\.(\\d|1[0-4])\\.mlp\\.", 4],
    ["language_model\\.layers\\.\\d+\\.mlp\\.", 2],
    ["language_model\\.layers\\.\\d+\\.per_layer_input_gate$", 8],
    ["language_model\\.layers\\.\\d+\\.per_layer_projection$", 8],
    ["language_model\\.layers\\.\\d+\\.self_attn\\.", 4],
]


def tensors(seed: int = 5):
    r = synth.Lcg(seed)
    out = []
    f32 = np.float32

    def nxt():
        return r.next()

    def scales(count):
        return np.array([f32(0.02) + nxt() * f32(0.05) for _ in range(count)], dtype=np.float32).tobytes()

    def add_q(real, n, k, bits, signed, scale_cols):
        if signed:
            vals = [(int(np.floor(nxt() * f32(256.0))) - 128) & 0xFF for _ in range(n * k)]
            payload = bytes(vals)
        else:
            span = f32(1 << bits)
            vals = [int(np.floor(nxt() * span)) % (1 << bits) for _ in range(n * k)]
            payload = synth.pack_unsigned(np.array(vals, dtype=np.uint32), bits).tobytes()
        cols = k if signed else k // (8 // bits)
        out.append((real, "I8" if signed else "U8", [n, cols], payload))
        out.append((real + "_scale", "F32", [n, scale_cols], scales(n * scale_cols)))

    def add_bf(real, shape):
        n = int(np.prod(shape))
        vals = np.array([(nxt() * f32(2.0) - f32(1.0)) * f32(0.05) for _ in range(n)], dtype=np.float32)
        out.append((real, "BF16", list(shape), (vals.view(np.uint32) >> 16).astype("<u2").tobytes()))

    def add_embed(base, n, k, bits, scale_cols):
        span = f32(1 << bits)
        vals = [int(np.floor(nxt() * span)) % (1 << bits) for _ in range(n * k)]
        out.append((base + ".embedding_quantized", "U8", [n, k // (8 // bits)],
                    synth.pack_unsigned(np.array(vals, dtype=np.uint32), bits).tobytes()))
        out.append((base + ".embedding_scale", "F32", [n, scale_cols], scales(n * scale_cols)))

    c = CFG
    h, i_, v, dple, L, hq, hkv = c["hidden"], c["inter"], c["vocab"], c["ple_dim"], c["layers"], c["heads_q"], c["heads_kv"]
    add_embed("model.language_model.embed_tokens", v, h, 2, 1)
    add_embed("model.language_model.embed_tokens_per_layer", v, L * dple, 4, L)
    add_bf("model.language_model.per_layer_model_projection.weight", [L * dple, h])
    add_bf("model.language_model.per_layer_projection_norm.weight", [dple])
    add_bf("model.language_model.norm.weight", [h])
    add_q("lm_head.weight", v, h, 2, False, 1)
    for i in range(L):
        p = f"model.language_model.layers.{i}"
        dh = c["global_head_dim"] if i in c["global_layers"] else c["head_dim"]
        for nm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                   "post_feedforward_layernorm", "post_per_layer_input_norm"):
            add_bf(f"{p}.{nm}.weight", [h])
        add_bf(f"{p}.layer_scalar", [1])
        add_bf(f"{p}.self_attn.q_norm.weight", [dh])
        add_bf(f"{p}.self_attn.k_norm.weight", [dh])
        add_q(f"{p}.self_attn.q_proj.weight", hq * dh, h, 4, False, 1)
        add_q(f"{p}.self_attn.k_proj.weight", hkv * dh, h, 4, False, 1)
        add_q(f"{p}.self_attn.v_proj.weight", hkv * dh, h, 4, False, 1)
        add_q(f"{p}.self_attn.o_proj.weight", h, hq * dh, 4, False, 1)
        add_q(f"{p}.mlp.gate_proj.weight", i_, h, 4, False, 1)
        add_q(f"{p}.mlp.up_proj.weight", i_, h, 4, False, 1)
        add_q(f"{p}.mlp.down_proj.weight", h, i_, 4, False, 1)
        add_q(f"{p}.per_layer_input_gate.weight", dple, h, 8, True, 1)
        add_q(f"{p}.per_layer_projection.weight", h, dple, 8, True, 1)
    out.append(("model.vision_tower.patch.weight", "F32", [4], bytes(16)))
    return out


def build_safetensors(entries, metadata=None) -> bytes:
    """build_safetensors (rust/src/safetensors.rs:186-205): payloads in the given order."""
    header = {}
    if metadata:
        header["__metadata__"] = metadata
    off = 0
    for name, dtype, shape, payload in entries:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(payload)]}
        off += len(payload)
    js = json.dumps(header, separators=(",", ":")).encode()
    return struct.pack("<Q", len(js)) + js + b"".join(e[3] for e in entries)


def main():
    entries = tensors(5)
    blob = build_safetensors(entries, {"format": "pt"})
    with open(os.path.join(HERE, "tiny_real_format.safetensors"), "wb") as f:
        f.write(blob)
    with open(os.path.join(HERE, "tiny_real_format.json"), "w") as f:
        json.dump({"config": CFG, "quant_rules": RULES, "seed": 5,
                   "tensors": [[n, d, s] for n, d, s, _ in entries]}, f, indent=1)
    print("wrote", len(blob), "bytes")


if __name__ == "__main__":
    main()
