"""Seeded synthetic inputs at the E2B shapes, and the packing rules of the
reference's on-disk format.

* ``pack_codes`` follows pack_int (rust/src/dequant.rs:37-50): sub-byte values
  are stored offset binary (raw = code + 2^(bits-1)), LSB-first; 8-bit as two's
  complement.
* The generator is splitmix64 (one independent stream per tensor seed),
  uniform doubles from the top 53 bits, normals by Box–Muller.
* ``Lcg`` restates the LCG of the reference's GPU tests
  (rust/tests/common/mod.rs:29-42) with its f32 arithmetic, so the parity cases
  of rust/tests/gpu.rs can be rebuilt value for value.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import QuantWeight

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int) -> np.ndarray:
    """n outputs of the splitmix64 stream started at `seed` (vectorised)."""
    with np.errstate(over="ignore"):
        s = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + _GOLDEN * (np.arange(1, n + 1, dtype=np.uint64))
        z = s
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, n: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    u = (splitmix64(seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
    return (lo + (hi - lo) * u).astype(np.float32)


def normal(seed: int, n: int) -> np.ndarray:
    m = (n + 1) // 2
    z = splitmix64(seed, 2 * m)
    u1 = ((z[:m] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / (1 << 53))  # (0, 1]
    u2 = (z[m:] >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(2 * np.pi * u2)
    out[1::2] = r * np.sin(2 * np.pi * u2)
    return out[:n].astype(np.float32)


def int_codes(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """Uniform integers in [lo, hi]."""
    span = np.uint64(hi - lo + 1)
    return (lo + (splitmix64(seed, n) % span).astype(np.int64)).astype(np.int32)


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """pack_int of rust/src/dequant.rs:37-50 (row-major, LSB-first)."""
    codes = np.asarray(codes, dtype=np.int32).ravel()
    if bits == 8:
        return codes.astype(np.int8).view(np.uint8).copy()
    pb = 8 // bits
    raw = ((codes + (1 << (bits - 1))) & ((1 << bits) - 1)).astype(np.uint8)
    pad = (-raw.size) % pb
    if pad:
        raw = np.concatenate([raw, np.zeros(pad, np.uint8)])
    raw = raw.reshape(-1, pb)
    out = np.zeros(raw.shape[0], dtype=np.uint8)
    for j in range(pb):
        out |= (raw[:, j] << (j * bits)).astype(np.uint8)
    return out


def pack_unsigned(vals: np.ndarray, bits: int) -> np.ndarray:
    """pack_unsigned of rust/src/dequant.rs:53-62."""
    vals = np.asarray(vals, dtype=np.uint32).ravel() & ((1 << bits) - 1)
    pb = 8 // bits
    pad = (-vals.size) % pb
    if pad:
        vals = np.concatenate([vals, np.zeros(pad, np.uint32)])
    vals = vals.reshape(-1, pb)
    out = np.zeros(vals.shape[0], dtype=np.uint8)
    for j in range(pb):
        out |= (vals[:, j] << (j * bits)).astype(np.uint8)
    return out


def make_qweight(seed: int, n: int, k: int, bits: int, signed_i8: bool = False, group_size: int | None = None,
                 scale_lo: float = 0.005, scale_hi: float = 0.02) -> QuantWeight:
    """Random codes uniform over the signed range, scales ~U(scale_lo, scale_hi)."""
    lo, hi = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    codes = int_codes(seed, n * k, lo, hi)
    g = group_size or k
    ss = -(-k // g)
    return QuantWeight(qbytes=pack_codes(codes, bits), scales=uniform(seed + 7, n * ss, scale_lo, scale_hi),
                       shape=(n, k), bits=bits, signed_i8=bool(signed_i8 and bits == 8), group_size=g)


def random_bytes(seed: int, nbytes: int) -> np.ndarray:
    """nbytes uniform bytes (8 per splitmix64 output)."""
    return splitmix64(seed, -(-nbytes // 8)).view(np.uint8)[:nbytes].copy()


def random_qweight(seed: int, n: int, k: int, bits: int, signed_i8: bool = False, group_size: int | None = None,
                   scale_lo: float = 0.005, scale_hi: float = 0.02) -> QuantWeight:
    """Same distribution as make_qweight (codes uniform over the whole signed
    range) built from uniform payload bytes: every packed field of a uniform
    byte is uniform. Fast enough for GB-sized tables."""
    pb = 1 if (bits == 8) else 8 // bits
    g = group_size or k
    ss = -(-k // g)
    return QuantWeight(qbytes=random_bytes(seed, n * (k // pb)), scales=uniform(seed + 7, n * ss, scale_lo, scale_hi),
                       shape=(n, k), bits=bits, signed_i8=bool(signed_i8 and bits == 8), group_size=g)


class Lcg:
    """rust/tests/common/mod.rs:29-42, with its f32 arithmetic."""

    def __init__(self, seed: int):
        self.s = seed & 0xFFFFFFFF

    def next(self) -> np.float32:
        self.s = (self.s * 1103515245 + 12345) & 0x7FFFFFFF
        return np.float32(self.s) / np.float32(0x7FFFFFFF)

    def rand(self, n: int, s: float) -> np.ndarray:
        s = np.float32(s)
        return np.array([(self.next() * np.float32(2.0) - np.float32(1.0)) * s for _ in range(n)], dtype=np.float32)

    def randu(self, n: int, bits: int) -> np.ndarray:
        f = np.float32(1 << bits)
        return np.array([int(np.floor(self.next() * f)) % (1 << bits) for _ in range(n)], dtype=np.uint32)

    def scales(self, n: int, base: float, width: float) -> np.ndarray:
        return np.array([np.float32(base) + self.next() * np.float32(width) for _ in range(n)], dtype=np.float32)


# ---- E2B shapes (rust/assets/config.json text_config) -------

HIDDEN = 1536
INTER = 6144
LAYERS = 35
HEADS_Q = 8
HEAD_DIM_LOCAL = 256
HEAD_DIM_GLOBAL = 512
PLE_DIM = 256
VOCAB = 262144
KV_LAYERS = 15  # layers 15..34 reuse an earlier layer's KV (num_kv_shared_layers = 20)


def is_global(i: int) -> bool:
    """Every 5th layer is full attention (layer_types in the E2B config)."""
    return i % 5 == 4


@dataclass
class Proj:
    name: str
    n: int
    k: int
    bits: int
    signed: bool
    mode: int = 0  # 0 linear, 1 geglu (gate+up pair), 2 gelu * PLE slice


def layer_projections(i: int, stack_qkv: bool = False) -> list:
    """The quantized projections of decoder layer i at the BASELINE config-2 bit
    widths: I8 attention and PLE, 4-bit gate/up (fused GeGLU), 2-bit down.
    stack_qkv: the q, k and v projections of a KV layer as one stacked weight
    (they read the same input; the decode step runs them as one GEMV)."""
    dh = HEAD_DIM_GLOBAL if is_global(i) else HEAD_DIM_LOCAL
    if stack_qkv and i < KV_LAYERS:
        out = [Proj(f"l{i}.qkv_proj", (HEADS_Q + 2) * dh, HIDDEN, 8, True)]
    else:
        out = [Proj(f"l{i}.q_proj", HEADS_Q * dh, HIDDEN, 8, True)]
    if i < KV_LAYERS and not stack_qkv:
        out += [Proj(f"l{i}.k_proj", dh, HIDDEN, 8, True), Proj(f"l{i}.v_proj", dh, HIDDEN, 8, True)]
    out += [
        Proj(f"l{i}.o_proj", HIDDEN, HEADS_Q * dh, 8, True),
        Proj(f"l{i}.gate_up", INTER, HIDDEN, 4, False, mode=1),
        Proj(f"l{i}.down_proj", HIDDEN, INTER, 2, False),
        Proj(f"l{i}.ple_gate", PLE_DIM, HIDDEN, 8, True, mode=2),
        Proj(f"l{i}.ple_proj", HIDDEN, PLE_DIM, 8, True),
    ]
    return out


def proj_bytes(p: Proj, m: int) -> int:
    """Algorithmic HBM bytes of one call: packed weights + f32 scales (x2 for the
    GeGLU pair) + f32 activations in + f32 outputs (+ the PLE slice read)."""
    row_bytes = p.k if p.signed else p.k * p.bits // 8
    nw = 2 if p.mode == 1 else 1
    b = nw * (p.n * row_bytes + 4 * p.n) + 4 * m * p.k + 4 * m * p.n
    if p.mode == 2:
        b += 4 * m * p.n
    return b
