"""CPU restatement of the Gemma-4 forward graph for one decode step.

TEST INFRASTRUCTURE ONLY: the checker of the CUDA decode step (tests/ and the
cpu_baseline leg of bench.py). The product never imports it.

Follows rust/src/model.rs:142-300 op for op — forward (:142-205),
decoder_layer (:207-252), attention (:254-300) — over the oracle's CPU ops
(oracle.py, the restatement of rust/src/backend_cpu.rs), for `batch`
independent sequences that each decode one token at the same position. Rows of
a batch go through linear / norms / rope together: the CPU backend computes
every row with the same arithmetic whatever the row count, so batching changes
no result; attention runs per sequence over that sequence's cache. The
lm_head output is soft-capped (the reference model itself
leaves it off, rust/src/model.rs:193-195).

`cfg` and `weights` are duck-typed: the fields of gq.e2b.Config and the
``q`` (QuantWeight) / ``f`` (f32 arrays) dictionaries of gq.e2b.Weights.
"""
from __future__ import annotations

import numpy as np

from . import oracle as o

FRAC_1_SQRT_2 = np.float32(0.70710677)  # std::f32::consts::FRAC_1_SQRT_2


def _sqrt32(v: int) -> float:
    return float(np.sqrt(np.float32(v)))


def decode_step(cfg, weights, ids, position: int, kv: dict, threads: int = 0) -> np.ndarray:
    """Logits [batch, vocab] of one step. kv maps each KV source layer to (K, V)
    arrays [batch, capacity, heads_kv*dh]; slot `position` is written (the step's
    key/value rows) and slots [0, position] are attended."""
    c, W, F = cfg, weights.q, weights.f
    ids = np.asarray(ids, dtype=np.uint32)
    B, H, L, P = ids.size, c.hidden, c.layers, c.ple_dim
    pos = np.full(B, position, dtype=np.uint32)
    kpos = np.arange(position + 1, dtype=np.uint32)

    # embeddings + per-layer inputs (rust/src/model.rs:152-177)
    h = o.embed_rows(W["embed"], ids, _sqrt32(H))
    emb = o.embed_rows(W["embed_ple"], ids, _sqrt32(P))
    proj = o.linear_f32(h, F["ple_model_proj"], threads)
    proj = o.rms_norm(proj.reshape(B * L, P), F["ple_proj_norm"], c.eps).reshape(B, L * P)
    ple = o.scale(o.add(proj, emb), FRAC_1_SQRT_2)

    for i in range(L):
        p = f"l{i}."
        dh = c.dh(i)
        theta, rot = c.rope(i)
        src = c.kv_source(i)
        # attention block
        residual = h
        x = o.rms_norm(residual, F[p + "input_ln"], c.eps)
        q = o.linear(x, W[p + "q_proj"], threads).reshape(B, c.heads_q, dh)
        q = o.head_norm_rope(q, F[p + "q_norm"], c.eps, pos, theta, dh, c.heads_q, rot)
        K, V = kv[src]
        if src == i:
            k = o.linear(x, W[p + "k_proj"], threads).reshape(B, c.heads_kv, dh)
            v = o.linear(x, W[p + "v_proj"], threads).reshape(B, c.heads_kv, dh)
            k = o.head_norm_rope(k, F[p + "k_norm"], c.eps, pos, theta, dh, c.heads_kv, rot)
            v = o.rms_norm(v.reshape(B * c.heads_kv, dh), None, c.eps)  # unweighted (rust/src/model.rs:272-273)
            K[:, position] = k.reshape(B, -1)
            V[:, position] = v.reshape(B, -1)
        outs = []
        for b in range(B):
            kb = K[b, : position + 1].reshape(position + 1, c.heads_kv, dh)
            vb = V[b, : position + 1].reshape(position + 1, c.heads_kv, dh)
            outs.append(o.attention(q[b: b + 1], kb, vb, pos[b: b + 1], kpos, 1.0, c.window_of(i), 0.0, threads))
        attn = o.linear(np.concatenate(outs, axis=0), W[p + "o_proj"], threads)
        h = o.add_rms_norm(residual, attn, F[p + "post_attn_ln"], c.eps)
        # GeGLU MLP
        residual = h
        x = o.rms_norm(residual, F[p + "pre_ffn_ln"], c.eps)
        ff = o.linear_geglu(x, W[p + "gate"], W[p + "up"], threads)
        ff = o.linear(ff, W[p + "down"], threads)
        h = o.add_rms_norm(residual, ff, F[p + "post_ffn_ln"], c.eps)
        # per-layer input injection, then the layer scalar
        inj = o.linear_gelu_mul_cols(h, W[p + "ple_gate"], ple, i * P, threads)
        inj = o.linear(inj, W[p + "ple_proj"], threads)
        h = o.add_rms_norm(h, inj, F[p + "ple_norm"], c.eps, F[p + "layer_scalar"])

    h = o.rms_norm(h, F["final_norm"], c.eps)
    return o.softcap(o.linear(h, W["lm_head"], threads), c.lm_softcap)


def kv_from_weights(cfg, weights, batch: int, cache_len: int, capacity: int) -> dict:
    """The seeded cache prefix of every KV source layer, in host arrays of the
    decoder's layout [batch, capacity, heads_kv*dh]."""
    kv = {}
    for i in range(cfg.layers):
        if cfg.kv_source(i) != i:
            continue
        d = cfg.heads_kv * cfg.dh(i)
        K = np.zeros((batch, capacity, d), dtype=np.float32)
        V = np.zeros((batch, capacity, d), dtype=np.float32)
        if cache_len:
            kk, vv = weights.kv_prefix(i, batch, cache_len)
            K[:, :cache_len] = kk
            V[:, :cache_len] = vv
        kv[i] = (K, V)
    return kv
