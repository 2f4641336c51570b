"""A Gemma-4 (E2B-shaped) decode step on the B200 backend: BASELINE config 5.

The forward graph of rust/src/model.rs:142-300 (token and per-layer embeddings,
35 decoder layers with MQA attention over a KV cache, GeGLU MLP, per-layer
input injection, final norm, lm_head) written against the C ABI of libgq for
`batch` independent sequences that each decode one token per step. It is the
caller of the quantized hot path, kept here so the whole step can be measured
and checked against the CPU oracle; nothing in it computes on the host.

* ``Config``   — the text config fields the graph reads (rust/src/config.rs:28-52),
  with the layer-type, head_dim, RoPE and KV-sharing rules of :118-158.
* ``Weights``  — seeded synthetic weights at the config's shapes: quantized
  projections and embeddings with the BASELINE bit widths, f32 norms near 1
  (the reference's test weights, rust/tests/common/mod.rs:100-118), the
  per-layer model projection as bf16 values, and a seeded KV-cache prefix.
* ``Decoder``  — device buffers, KV caches and the pre-bound C-ABI calls of one
  step; ``run()`` enqueues them, ``record()`` captures them into a graph.

Layout: KV cache of source layer i is K/V [batch, capacity, head_dim] f32; a
step at position p writes the new key/value rows into slot p directly from the
norm kernels and attends over slots [0, p]. Shared layers (the last
``kv_shared``) read their source layer's cache (rust/src/config.rs:148-158).
"""
from __future__ import annotations

import math
import os
import zlib
from ctypes import c_float, c_void_p
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import QuantWeight, synth
from ._abi import GQ_ATTN_KPOS_IDENTITY, GqError


@dataclass
class Config:
    vocab: int = 262144
    hidden: int = 1536
    inter: int = 6144
    layers: int = 35
    heads_q: int = 8
    heads_kv: int = 1
    head_dim: int = 256
    global_head_dim: int = 512
    ple_dim: int = 256
    kv_shared: int = 20
    window: int = 512
    eps: float = 1e-6
    theta_local: float = 1e4
    partial_local: float = 1.0
    theta_global: float = 1e6
    partial_global: float = 0.25
    global_layers: Tuple[int, ...] = ()
    lm_softcap: float = 30.0
    # bit widths (attention I8, MLP 4/4/2, PLE I8, lm_head I8)
    attn_bits: int = 8
    mlp_bits: int = 4
    down_bits: int = 2
    ple_bits: int = 8
    lm_bits: int = 8
    embed_bits: int = 4
    ple_table_bits: int = 8

    def __post_init__(self):
        if not self.global_layers:
            # every 5th layer is full attention (rust/src/config.rs:81-88 fallback)
            self.global_layers = tuple(i for i in range(self.layers) if (i + 1) % 5 == 0)

    def is_global(self, i: int) -> bool:
        return i in self.global_layers

    def dh(self, i: int) -> int:
        """rust/src/config.rs:130-132"""
        return self.global_head_dim if self.is_global(i) else self.head_dim

    def rope(self, i: int) -> Tuple[float, int]:
        """(theta, rotary_dim) of layer i (rust/src/config.rs:134-136, rust/src/model.rs:246)."""
        theta, part = (self.theta_global, self.partial_global) if self.is_global(i) else (self.theta_local,
                                                                                           self.partial_local)
        return theta, int(round(self.dh(i) * part))

    def kv_source(self, i: int) -> int:
        """rust/src/config.rs:148-158"""
        first_shared = max(0, self.layers - self.kv_shared)
        if i < first_shared:
            return i
        for j in range(first_shared - 1, -1, -1):
            if self.is_global(j) == self.is_global(i):
                return j
        return i

    def window_of(self, i: int) -> int:
        return 0 if self.is_global(i) else self.window


def e2b_config() -> Config:
    """Gemma-4 E2B text shapes."""
    return Config()


def tiny_config(vocab: int = 48) -> Config:
    """The reference's tiny test model (rust/tests/common/mod.rs:44-55): layer 1 is
    global, the last 2 layers share KV, window 3."""
    return Config(vocab=vocab, hidden=32, inter=64, layers=6, heads_q=4, heads_kv=1, head_dim=8, global_head_dim=16,
                  ple_dim=12, kv_shared=2, window=3, global_layers=(1,))


def small_config(vocab: int = 4096) -> Config:
    """A mid-sized config with the E2B structure (MQA 8/1, both head_dims, KV sharing,
    sliding window) for batched parity tests."""
    return Config(vocab=vocab, hidden=256, inter=512, layers=7, heads_q=8, heads_kv=1, head_dim=64,
                  global_head_dim=128, ple_dim=32, kv_shared=3, window=16, global_layers=(1, 4))


def _bf16_round(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


@dataclass
class Weights:
    """Seeded synthetic weights of a Config (host arrays; uploaded by Decoder)."""

    cfg: Config
    seed: int = 123
    q: Dict[str, QuantWeight] = field(default_factory=dict)
    f: Dict[str, np.ndarray] = field(default_factory=dict)

    def __post_init__(self):
        c, s = self.cfg, self.seed * 100003
        k = [0]

        def nxt() -> int:
            k[0] += 1
            return s + 7919 * k[0]

        def qw(name, n, kk, bits, group=None):
            self.q[name] = synth.random_qweight(nxt(), n, kk, bits, signed_i8=(bits == 8), group_size=group)

        def norm(name, n, base=1.0, width=0.05):
            self.f[name] = (base + synth.uniform(nxt(), n, -width, width)).astype(np.float32)

        L, P = c.layers, c.ple_dim
        qw("embed", c.vocab, c.hidden, c.embed_bits)
        qw("embed_ple", c.vocab, L * P, c.ple_table_bits, group=P)
        self.f["ple_model_proj"] = _bf16_round(synth.uniform(nxt(), L * P * c.hidden, -0.04, 0.04)).reshape(
            L * P, c.hidden)
        norm("ple_proj_norm", P)
        norm("final_norm", c.hidden)
        qw("lm_head", c.vocab, c.hidden, c.lm_bits)
        for i in range(L):
            dh = c.dh(i)
            p = f"l{i}."
            for nm in ("input_ln", "post_attn_ln", "pre_ffn_ln", "post_ffn_ln", "ple_norm"):
                norm(p + nm, c.hidden)
            norm(p + "q_norm", dh)
            norm(p + "layer_scalar", 1)
            qw(p + "q_proj", c.heads_q * dh, c.hidden, c.attn_bits)
            if c.kv_source(i) == i:
                qw(p + "k_proj", c.heads_kv * dh, c.hidden, c.attn_bits)
                qw(p + "v_proj", c.heads_kv * dh, c.hidden, c.attn_bits)
                norm(p + "k_norm", dh)
            qw(p + "o_proj", c.hidden, c.heads_q * dh, c.attn_bits)
            qw(p + "gate", c.inter, c.hidden, c.mlp_bits)
            qw(p + "up", c.inter, c.hidden, c.mlp_bits)
            qw(p + "down", c.hidden, c.inter, c.down_bits)
            qw(p + "ple_gate", P, c.hidden, c.ple_bits)
            qw(p + "ple_proj", c.hidden, P, c.ple_bits)

    def kv_prefix(self, layer: int, batch: int, length: int) -> Tuple[np.ndarray, np.ndarray]:
        """Seeded cache contents [batch, length, heads_kv * dh] for source layer `layer`
        (keys and values ~N(0,1), the scale of normalised rows)."""
        d = self.cfg.heads_kv * self.cfg.dh(layer)
        base = self.seed * 1_000_003 + 1009 * layer
        kk = synth.normal(base + 1, batch * length * d).reshape(batch, length, d)
        vv = synth.normal(base + 2, batch * length * d).reshape(batch, length, d)
        return kk, vv


class Decoder:
    """One decode step of `batch` sequences through the C ABI, with device-resident
    weights, KV caches and activations (all buffers fixed, so a step records into a
    graph). The cache holds `cache_len` seeded tokens (positions 0..cache_len-1);
    ``set_position(p)`` selects the slot a step writes and attends up to.

    lm_shard=(rank, world, group): the lm_head is split by vocab rows over `world`
    ranks (one process per GPU, torch.distributed initialised). This rank holds
    rows [r0, r1) and runs the fused sharded lm_head (gq.parallel.PeerLmHead,
    device barrier): its GEMV stores its logits into every rank's buffer over
    NVLink, so every rank ends the step with the full logits. The trunk is
    replicated. Steps alternate between two logits buffers, so ``record`` then
    captures two steps (one per buffer) and a replay runs both.

    kv_device_seed: draw the cache prefix ~N(0,1) on the device from this seed even
    when host weights are given (large batches: the host draw of a 64-sequence,
    2047-token cache takes minutes); a checker reads it back from ``kcache`` /
    ``vcache``."""

    def __init__(self, g, cfg: Config, weights: Optional[Weights], batch: int, cache_len: int,
                 capacity: Optional[int] = None, device_init_seed: Optional[int] = None, lm_shard=None,
                 kv_device_seed: Optional[int] = None, fuse_norms: Optional[bool] = None):
        import torch

        self.g, self.cfg, self.batch = g, cfg, batch
        self.torch = torch
        lib, ctx = g.lib, g.ctx
        dev = g.torch_device
        self.capacity = capacity or (cache_len + 1)
        if cache_len >= self.capacity:
            raise GqError(1, "Decoder: cache_len must be < capacity")
        self.cache_len = cache_len
        c = cfg
        f32 = torch.float32
        self._keep: List[object] = []
        gen = None
        if weights is None:
            gen = torch.Generator(device=dev)
            gen.manual_seed(device_init_seed or 1)
        kv_gen = gen
        if kv_device_seed is not None:  # cache prefix drawn on the device even with host weights
            kv_gen = torch.Generator(device=dev)
            kv_gen.manual_seed(kv_device_seed)

        # ---- weights -------------------------------------------------------------
        self.meta: Dict[str, Tuple[int, int, int, int]] = {}  # name -> (n, k, bits, group)

        def qt(name, n, k, bits, group=None):
            self.meta[name] = (n, k, bits, group or k)
            if weights is not None:
                return g.quant_tensor(weights.q[name])
            rb = k if bits == 8 else k * bits // 8
            payload = torch.randint(0, 256, (n * rb,), generator=gen, device=dev, dtype=torch.uint8)
            ss = -(-k // (group or k))
            sc = synth.uniform(zlib.crc32(name.encode()), n * ss, 0.005, 0.02)
            torch.cuda.synchronize(dev)
            t = g.quant_tensor_from_device(payload, sc, (n, k), bits, bits == 8, group or k)
            del payload
            return t

        def qt_stack(pre, parts, k, bits):
            """One device weight holding the rows of several projections of the same
            input, stacked in order (packed rows are independent, so one GEMV over
            the stack gives each projection's outputs side by side)."""
            for nm, rows in parts:
                self.meta[pre + nm] = (rows, k, bits, k)
            n = sum(rows for _, rows in parts)
            if weights is not None:
                qs = [weights.q[pre + nm] for nm, _ in parts]
                from . import QuantWeight
                return g.quant_tensor(QuantWeight(
                    qbytes=np.concatenate([np.asarray(q.qbytes, dtype=np.uint8) for q in qs]),
                    scales=np.concatenate([np.asarray(q.scales, dtype=np.float32) for q in qs]),
                    shape=(n, k), bits=qs[0].bits, signed_i8=qs[0].signed_i8, group_size=qs[0].group_size))
            rb = k if bits == 8 else k * bits // 8
            payload = torch.cat([torch.randint(0, 256, (rows * rb,), generator=gen, device=dev, dtype=torch.uint8)
                                 for _, rows in parts])
            sc = np.concatenate([synth.uniform(zlib.crc32((pre + nm).encode()), rows, 0.005, 0.02)
                                 for nm, rows in parts])
            torch.cuda.synchronize(dev)
            t = g.quant_tensor_from_device(payload, sc, (n, k), bits, bits == 8, k)
            del payload
            return t

        def ft(name, n):
            if weights is not None:
                a = weights.f[name].reshape(-1)
            else:
                a = (1.0 + synth.uniform(zlib.crc32(name.encode()) + 1, n, -0.05, 0.05)).astype(np.float32)
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)

        L, P, H = c.layers, c.ple_dim, c.hidden
        self.w = {}
        self.w["embed"] = qt("embed", c.vocab, H, c.embed_bits)
        self.w["embed_ple"] = qt("embed_ple", c.vocab, L * P, c.ple_table_bits, group=P)
        if weights is not None:
            self.w["ple_model_proj"] = g.tensor_bf16(weights.f["ple_model_proj"], (L * P, H))
        else:
            v = (torch.rand(L * P, H, generator=gen, device=dev) * 0.08 - 0.04).to(torch.bfloat16)
            from . import GqTensor
            self.w["ple_model_proj"] = GqTensor(shape=(L * P, H), data=v.view(torch.int16), bf16=True)
        self.w["ple_proj_norm"] = ft("ple_proj_norm", P)
        self.w["final_norm"] = ft("final_norm", H)
        self.peer = None
        if lm_shard is None:
            self.w["lm_head"] = qt("lm_head", c.vocab, H, c.lm_bits)
        else:
            from .parallel import PeerLmHead, shard_rows, slice_rows
            rank, world, group = lm_shard
            r0, r1 = shard_rows(c.vocab, world, rank)
            self.meta["lm_head"] = (c.vocab, H, c.lm_bits, H)
            if weights is not None:
                shard = g.quant_tensor(slice_rows(weights.q["lm_head"], r0, r1))
            else:  # the same random stream as the full table, then this rank's rows
                rb = H if c.lm_bits == 8 else H * c.lm_bits // 8
                payload = torch.randint(0, 256, (c.vocab * rb,), generator=gen, device=dev, dtype=torch.uint8)
                sc = synth.uniform(zlib.crc32(b"lm_head"), c.vocab, 0.005, 0.02)
                torch.cuda.synchronize(dev)
                shard = g.quant_tensor_from_device(payload[r0 * rb: r1 * rb].contiguous(), sc[r0:r1], (r1 - r0, H),
                                                   c.lm_bits, c.lm_bits == 8, H)
                del payload
            self.w["lm_head"] = shard
            self.peer = PeerLmHead(g, shard, c.vocab, rank, world, max_m=batch, cap=c.lm_softcap, group=group,
                                   barrier="fused")
        for i in range(L):
            dh = c.dh(i)
            p = f"l{i}."
            for nm in ("input_ln", "post_attn_ln", "pre_ffn_ln", "post_ffn_ln", "ple_norm"):
                self.w[p + nm] = ft(p + nm, H)
            self.w[p + "q_norm"] = ft(p + "q_norm", dh)
            self.w[p + "layer_scalar"] = ft(p + "layer_scalar", 1)
            if c.kv_source(i) == i:
                # q, k and v read the same normed input: one stacked weight, one GEMV
                self.w[p + "qkv_proj"] = qt_stack(p, [("q_proj", c.heads_q * dh), ("k_proj", c.heads_kv * dh),
                                                      ("v_proj", c.heads_kv * dh)], H, c.attn_bits)
                self.w[p + "k_norm"] = ft(p + "k_norm", dh)
            else:
                self.w[p + "q_proj"] = qt(p + "q_proj", c.heads_q * dh, H, c.attn_bits)
            self.w[p + "o_proj"] = qt(p + "o_proj", H, c.heads_q * dh, c.attn_bits)
            self.w[p + "gate"] = qt(p + "gate", c.inter, H, c.mlp_bits)
            self.w[p + "up"] = qt(p + "up", c.inter, H, c.mlp_bits)
            self.w[p + "down"] = qt(p + "down", H, c.inter, c.down_bits)
            self.w[p + "ple_gate"] = qt(p + "ple_gate", P, H, c.ple_bits)
            self.w[p + "ple_proj"] = qt(p + "ple_proj", H, P, c.ple_bits)

        # ---- KV caches of the source layers ----------------------------------------
        self.kcache, self.vcache = {}, {}
        for i in range(L):
            if c.kv_source(i) != i:
                continue
            d = c.heads_kv * c.dh(i)
            kc = torch.zeros(batch, self.capacity, d, dtype=f32, device=dev)
            vc = torch.zeros(batch, self.capacity, d, dtype=f32, device=dev)
            if cache_len:
                if weights is not None and kv_device_seed is None:
                    kk, vv = weights.kv_prefix(i, batch, cache_len)
                    kc[:, :cache_len] = torch.from_numpy(kk).to(dev)
                    vc[:, :cache_len] = torch.from_numpy(vv).to(dev)
                else:
                    kc[:, :cache_len].normal_(generator=kv_gen)
                    vc[:, :cache_len].normal_(generator=kv_gen)
            self.kcache[i], self.vcache[i] = kc, vc

        # ---- activations and step inputs ------------------------------------------
        B = batch
        dq = c.heads_q * c.global_head_dim
        z = lambda *s: torch.zeros(*s, dtype=f32, device=dev)  # noqa: E731
        self.ids = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.kpos = torch.arange(self.capacity, dtype=torch.int32, device=dev)
        self.rsqrt2 = torch.tensor([np.float32(1.0 / math.sqrt(2.0))], dtype=f32, device=dev)
        self.h, self.x = z(B, H), z(B, H)
        # fuse_norms (one sequence): the residual add + RMSNorm before gate|up, the PLE
        # gate and the next layer's q(|k|v) run inside those projections
        # (gq_add_norm_linear); the residual then alternates between h and h2 (the
        # fused op must not write the row it reads). Off by default: with the
        # launches chained under programmatic dependent launch the separate norm
        # kernels cost less than the prologue adds to each projection (E2B batch 1:
        # 1.700-1.708 ms separate, 1.727 ms fused). GQ_E2B_FUSE=1 turns it on.
        if fuse_norms is None:
            fuse_norms = batch == 1 and os.environ.get("GQ_E2B_FUSE", "0") == "1"
        self.fuse_norms = bool(fuse_norms) and batch == 1
        self.h2 = z(B, H)
        self.emb, self.proj, self.ple = z(B, L * P), z(B, L * P), z(B, L * P)
        self.q, self.qr, self.attn = z(B, dq), z(B, dq), z(B, dq)
        self.qkv = z(B, (c.heads_q + 2 * c.heads_kv) * c.global_head_dim)
        self.o, self.ff, self.inj = z(B, H), z(B, c.inter), z(B, P)
        self.logits = z(B, c.vocab)
        self._par = 0
        self.position = -1
        self.set_position(cache_len)

    # ---- the step --------------------------------------------------------------------
    def set_position(self, p: int) -> None:
        """Steps write cache slot p (all sequences) and attend over slots [0, p]."""
        if not 0 <= p < self.capacity:
            raise GqError(1, f"position {p} outside the cache capacity {self.capacity}")
        self.position = p
        self.pos.fill_(p)
        self._calls = self._build_calls(p)

    def set_ids(self, ids) -> None:
        t = self.torch.as_tensor(np.asarray(ids, dtype=np.int32).reshape(self.batch))
        self.ids.copy_(t.to(self.ids.device), non_blocking=False)

    def _build_calls(self, p: int):
        g, c, lib, ctx = self.g, self.cfg, self.g.lib, self.g.ctx
        B, H, L, P = self.batch, c.hidden, c.layers, c.ple_dim
        V = lambda t: c_void_p(t.data_ptr())  # noqa: E731
        Q = lambda name: c_void_p(self.w[name].qw)  # noqa: E731
        F = lambda name: c_void_p(self.w[name].data.data_ptr())  # noqa: E731
        eps = c_float(c.eps)
        calls = []
        add = lambda label, fn, *args: calls.append((label, fn, args))  # noqa: E731

        # embeddings and per-layer inputs (rust/src/model.rs:152-177)
        add("embed", lib.gq_embed_rows, ctx, Q("embed"), V(self.ids), B, c_float(math.sqrt(H)), V(self.h))
        add("embed_ple", lib.gq_embed_rows, ctx, Q("embed_ple"), V(self.ids), B, c_float(math.sqrt(P)), V(self.emb))
        add("ple_model_proj", lib.gq_linear_bf16, ctx, V(self.h), B, H, F("ple_model_proj"), L * P, V(self.proj))
        add("ple_combine", lib.gq_add_rms_norm, ctx, V(self.emb), V(self.proj), B * L, P, F("ple_proj_norm"), eps,
            V(self.rsqrt2), V(self.ple))
        S = p + 1
        # input norm of layer 0; later layers get theirs fused into the previous layer's last norm
        add("l0.input_norm", lib.gq_rms_norm, ctx, V(self.h), B, H, F("l0.input_ln"), eps, V(self.x), H)
        fuse = self.fuse_norms
        hc, halt = self.h, self.h2  # residual: current row, the other buffer

        def fused(label, mode, w_norm, scale, w_norm2, w, w_up, b, b_off, y):
            nonlocal hc, halt
            add(label, lib.gq_add_norm_linear, ctx, mode, V(self.o), V(hc), H, F(w_norm), eps,
                F(scale) if scale else None, F(w_norm2) if w_norm2 else None, V(halt), Q(w),
                Q(w_up) if w_up else None, V(b) if b is not None else None, b_off, V(y))
            hc, halt = halt, hc

        for i in range(L):
            pre = f"l{i}."
            dh = c.dh(i)
            theta, rot = c.rope(i)
            src = c.kv_source(i)
            kc, vc = self.kcache[src], self.vcache[src]
            kvd = c.heads_kv * dh
            cstride = self.capacity * kvd
            # attention block (rust/src/model.rs:214-219, 233-300)
            # the previous layer's closing norm (residual + PLE norm, layer scalar,
            # this layer's input norm), fused into this layer's first projection
            prev = f"l{i - 1}."
            pro = fuse and i > 0
            if src == i:
                # q|k|v in one GEMV, then the q and k norms + RoPE and the unweighted
                # value norm (rust/src/model.rs:258-273) in one launch, k and v written
                # straight into slot p of every sequence's cache
                if pro:
                    fused(pre + "qkv_proj", 0, prev + "ple_norm", prev + "layer_scalar", pre + "input_ln",
                          pre + "qkv_proj", None, None, 0, self.qkv)
                else:
                    add(pre + "qkv_proj", lib.gq_linear, ctx, V(self.x), B, H, Q(pre + "qkv_proj"), V(self.qkv))
                add(pre + "qkv_norm_rope", lib.gq_qkv_norm_rope, ctx, V(self.qkv), B, (c.heads_q + 2 * c.heads_kv) * dh,
                    c.heads_q, c.heads_kv, dh, F(pre + "q_norm"), F(pre + "k_norm"), eps, V(self.pos),
                    c_float(theta), rot, V(self.qr), c.heads_q * dh, c_void_p(kc.data_ptr() + 4 * p * kvd), cstride,
                    c_void_p(vc.data_ptr() + 4 * p * kvd), cstride)
            else:
                if pro:
                    fused(pre + "q_proj", 0, prev + "ple_norm", prev + "layer_scalar", pre + "input_ln",
                          pre + "q_proj", None, None, 0, self.q)
                else:
                    add(pre + "q_proj", lib.gq_linear, ctx, V(self.x), B, H, Q(pre + "q_proj"), V(self.q))
                add(pre + "q_norm_rope", lib.gq_head_norm_rope, ctx, V(self.q), B, c.heads_q, dh, F(pre + "q_norm"),
                    eps, V(self.pos), c_float(theta), rot, V(self.qr), c.heads_q * dh)
            add(pre + "attention", lib.gq_attention, ctx, V(self.qr), B, 1, c.heads_q, dh, V(kc), V(vc), S,
                c.heads_kv, cstride, V(self.pos), None, 0, c_float(1.0), c.window_of(i), c_float(0.0),
                GQ_ATTN_KPOS_IDENTITY, V(self.attn))
            add(pre + "o_proj", lib.gq_linear, ctx, V(self.attn), B, c.heads_q * dh, Q(pre + "o_proj"), V(self.o))
            # h = h + post_attn_norm(o), then x = pre_ffn_norm(h): one pass (rust/src/model.rs:219, 223)
            # GeGLU MLP (rust/src/model.rs:221-227)
            if fuse:
                fused(pre + "gate_up", 1, pre + "post_attn_ln", None, pre + "pre_ffn_ln", pre + "gate", pre + "up",
                      None, 0, self.ff)
            else:
                add(pre + "post_attn", lib.gq_add_rms_norm_norm, ctx, V(self.h), V(self.o), B, H,
                    F(pre + "post_attn_ln"), eps, None, F(pre + "pre_ffn_ln"), V(self.h), V(self.x))
                add(pre + "gate_up", lib.gq_linear_geglu, ctx, V(self.x), B, H, Q(pre + "gate"), Q(pre + "up"),
                    V(self.ff))
            add(pre + "down", lib.gq_linear, ctx, V(self.ff), B, c.inter, Q(pre + "down"), V(self.o))
            # h = h + post_ffn_norm(o); per-layer input injection + layer scalar (rust/src/model.rs:229-242)
            if fuse:
                fused(pre + "ple_gate", 2, pre + "post_ffn_ln", None, None, pre + "ple_gate", None, self.ple, i * P,
                      self.inj)
            else:
                add(pre + "post_ffn", lib.gq_add_rms_norm, ctx, V(self.h), V(self.o), B, H, F(pre + "post_ffn_ln"),
                    eps, None, V(self.h))
                add(pre + "ple_gate", lib.gq_linear_gelu_mul_cols, ctx, V(self.h), B, H, Q(pre + "ple_gate"),
                    V(self.ple), L * P, i * P, V(self.inj))
            add(pre + "ple_proj", lib.gq_linear, ctx, V(self.inj), B, P, Q(pre + "ple_proj"), V(self.o))
            # h = (h + ple_norm(inj)) * layer_scalar, then the next layer's input norm (or the
            # final norm, rust/src/model.rs:183) of h: one pass (fused into the next layer's
            # first projection when the norms are fused; the last one always here, into h)
            if not fuse or i + 1 == L:
                nxt = f"l{i + 1}.input_ln" if i + 1 < L else "final_norm"
                add(pre + "ple_norm", lib.gq_add_rms_norm_norm, ctx, V(hc), V(self.o), B, H, F(pre + "ple_norm"),
                    eps, F(pre + "layer_scalar"), F(nxt), V(self.h), V(self.x))
                hc, halt = self.h, self.h2
        # lm_head with the soft-cap on the final-normed h (rust/src/model.rs:183-192)
        if self.peer is None:
            add("lm_head", lib.gq_linear_softcap, ctx, V(self.x), B, H, Q("lm_head"), c_float(c.lm_softcap),
                V(self.logits), c.vocab, 0)
        else:  # this rank's vocab rows, stored into every rank's logits buffer `par` (set per step)
            self._lm_calls = [self.peer.device_calls(self.x.data_ptr(), B, H, par) for par in (0, 1)]
        return calls

    def run(self) -> None:
        """Enqueue one step (no host synchronisation)."""
        calls = self._calls
        if self.peer is not None:
            calls = calls + self._lm_calls[self._par]
            self.logits = self.peer.logits[self._par][: self.batch]
            self._par ^= 1
        for label, fn, args in calls:
            rc = fn(*args)
            if rc != 0:
                self.g._check(rc, label)

    def read(self, t) -> np.ndarray:
        """Blocking copy of one of the decoder's device tensors (after the queued work)."""
        out = np.empty(tuple(t.shape), dtype=np.float32)
        self.g._check(self.g.lib.gq_readback(self.g.ctx, c_void_p(out.ctypes.data), c_void_p(t.data_ptr()), out.size),
                      "readback")
        return out

    def record(self):
        """Capture one step into a graph (the backend must own its stream; run once
        first). With a sharded lm_head the graph holds two steps, one per logits
        buffer, and ``logits`` is the second one's."""
        if self.peer is None:
            return self.g.record(self.run)
        self._par = 0

        def two():
            self.run()
            self.run()
        return self.g.record(two)

    @property
    def steps_per_graph(self) -> int:
        return 1 if self.peer is None else 2

    def close(self) -> None:
        """Free the decoder's quantized weights (device memory of the rest is torch's)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None
        for t in self.w.values():
            if getattr(t, "qw", None) is not None:
                self.g.free_quant(t)
        self.w.clear()
        self.kcache.clear()
        self.vcache.clear()

    @property
    def launches(self) -> int:
        return len(self._calls) + (len(self._lm_calls[0]) if self.peer is not None else 0)

    def labels(self) -> List[str]:
        return [c[0] for c in self._calls]

    def weight_bytes(self) -> int:
        """Packed weight + scale bytes the step reads once (lm_head included, the two
        embedding tables excluded: they are gathered, see ``gather_bytes``)."""
        c = self.cfg
        tot = 0
        for name, (n, k, bits, group) in self.meta.items():
            if name in ("embed", "embed_ple"):
                continue
            rb = k if bits == 8 else k * bits // 8
            tot += n * rb + 4 * n * (-(-k // group))
        tot += 2 * c.layers * c.ple_dim * c.hidden  # bf16 per-layer model projection
        return tot

    def gather_bytes(self) -> int:
        """Embedding rows gathered per step (packed bytes + scales of both tables)."""
        c = self.cfg
        row = c.hidden * c.embed_bits // 8 + 4 + c.layers * c.ple_dim * c.ple_table_bits // 8 + 4 * c.layers
        return self.batch * row

    def kv_bytes(self) -> int:
        """K and V bytes the step's attention reads (per sequence, summed over layers)."""
        c, S = self.cfg, self.position + 1
        tot = 0
        for i in range(c.layers):
            keys = S if c.window_of(i) == 0 else min(S, c.window_of(i))
            tot += 2 * keys * c.heads_kv * c.dh(i) * 4
        return tot * self.batch
