"""ctypes wrapper of the CPU oracle (libgq_oracle.so, built from gq_oracle.c).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py as the checker and the timed
CPU baseline. The product library never imports this module.

Weights are any object with the QuantWeight fields of rust/src/backend.rs:16-24
(qbytes, scales, shape, bits, signed_i8, group_size).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, Structure, c_float, c_int32, c_int64, c_size_t, c_uint8, c_uint32, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgq_oracle.so")


class _QW(Structure):
    _fields_ = [("qbytes", c_void_p), ("scales", c_void_p), ("n", c_int64), ("k", c_int64),
                ("bits", c_int32), ("signed_i8", c_int32), ("group_size", c_int64)]


_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    P = POINTER(_QW)
    sig = {
        "gqo_per_byte": (c_int64, [P]), "gqo_row_bytes": (c_int64, [P]), "gqo_scale_stride": (c_int64, [P]),
        "gqo_code": (c_int32, [P, c_int64, c_int64]), "gqo_deq": (c_float, [P, c_int64, c_int64]),
        "gqo_unpack_int": (None, [c_void_p, c_int32, c_size_t, c_void_p]),
        "gqo_pack_int": (c_size_t, [c_void_p, c_size_t, c_int32, c_void_p]),
        "gqo_pack_unsigned": (c_size_t, [c_void_p, c_size_t, c_int32, c_void_p]),
        "gqo_dequantize": (None, [c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p]),
        "gqo_default_threads": (c_int32, []),
        "gqo_linear": (c_int32, [c_void_p, c_int64, c_int64, P, c_void_p, c_int32]),
        "gqo_linear_f32": (c_int32, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int32]),
        "gqo_embed_rows": (c_int32, [P, c_void_p, c_int64, c_float, c_void_p]),
        "gqo_gelu_tanh": (c_float, [c_float]),
        "gqo_geglu": (None, [c_void_p, c_void_p, c_size_t, c_void_p]),
        "gqo_softcap": (None, [c_void_p, c_size_t, c_float, c_void_p]),
        "gqo_slice_cols": (None, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p]),
        "gqo_linear_geglu": (c_int32, [c_void_p, c_int64, c_int64, P, P, c_void_p, c_int32]),
        "gqo_linear_gelu_mul_cols": (c_int32, [c_void_p, c_int64, c_int64, P, c_void_p, c_int64, c_int64,
                                               c_void_p, c_int32]),
        "gqo_rms_norm": (None, [c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p]),
        "gqo_add": (None, [c_void_p, c_void_p, c_size_t, c_void_p]),
        "gqo_mul": (None, [c_void_p, c_void_p, c_size_t, c_void_p]),
        "gqo_scale": (None, [c_void_p, c_size_t, c_float, c_void_p]),
        "gqo_add_rms_norm": (None, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p, c_void_p]),
        "gqo_rope": (None, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_float, c_int64, c_void_p]),
        "gqo_head_norm_rope": (None, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p, c_float,
                                      c_int64, c_void_p]),
        "gqo_attention": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                                    c_int64, c_void_p, c_void_p, c_float, c_uint32, c_float, c_void_p, c_int32]),
        "gqo_rng_next_u64": (ctypes.c_uint64, [c_void_p]),
        "gqo_rng_next_f64": (ctypes.c_double, [c_void_p]),
        "gqo_sample": (c_int32, [c_void_p, c_int64, c_float, c_int64, c_float, c_float, c_void_p, c_int64,
                                 ctypes.c_double]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _p(a: np.ndarray) -> c_void_p:
    return c_void_p(a.ctypes.data)


class _Held:
    """A QuantWeight as the C struct plus the arrays it points into."""

    def __init__(self, q):
        self.qb = np.ascontiguousarray(np.asarray(q.qbytes, dtype=np.uint8))
        self.sc = np.ascontiguousarray(np.asarray(q.scales, dtype=np.float32))
        n, k = q.shape
        self.s = _QW(self.qb.ctypes.data, self.sc.ctypes.data, n, k, q.bits, int(bool(q.signed_i8)),
                     q.group_size)
        self.ref = ctypes.byref(self.s)


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def default_threads() -> int:
    return int(load().gqo_default_threads())


def code(q, n: int, k: int) -> int:
    return int(load().gqo_code(_Held(q).ref, n, k))


def deq(q, n: int, k: int) -> float:
    return float(load().gqo_deq(_Held(q).ref, n, k))


def unpack_int(b: np.ndarray, bits: int, count: int) -> np.ndarray:
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint8))
    out = np.empty(count, dtype=np.int32)
    load().gqo_unpack_int(_p(b), bits, count, _p(out))
    return out


def pack_int(v, bits: int) -> np.ndarray:
    v = np.ascontiguousarray(np.asarray(v, dtype=np.int32))
    pb = 1 if bits == 8 else 8 // bits
    out = np.zeros(max(1, -(-v.size // pb)), dtype=np.uint8)
    nb = load().gqo_pack_int(_p(v), v.size, bits, _p(out))
    return out[:nb]


def pack_unsigned(v, bits: int) -> np.ndarray:
    v = np.ascontiguousarray(np.asarray(v, dtype=np.uint32))
    pb = 8 // bits
    out = np.zeros(max(1, -(-v.size // pb)), dtype=np.uint8)
    nb = load().gqo_pack_unsigned(_p(v), v.size, bits, _p(out))
    return out[:nb]


def dequantize(q, scales, rows: int, cols: int, group_size: int) -> np.ndarray:
    q = np.ascontiguousarray(np.asarray(q, dtype=np.int32))
    s = _f32(scales)
    out = np.empty(rows * cols, dtype=np.float32)
    load().gqo_dequantize(_p(q), _p(s), rows, cols, group_size, _p(out))
    return out


def linear(x, q, threads: int = 0) -> np.ndarray:
    x = _f32(x)
    k = q.shape[1]
    t = x.size // k if k else 0
    y = np.empty((t, q.shape[0]), dtype=np.float32)
    h = _Held(q)
    rc = load().gqo_linear(_p(x), t, k, h.ref, _p(y), threads)
    if rc != 0:
        raise ValueError("oracle linear: bad shape")
    return y


def linear_f32(x, w, threads: int = 0) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    n, k = w.shape
    t = x.size // k
    y = np.empty((t, n), dtype=np.float32)
    load().gqo_linear_f32(_p(x), t, k, _p(w), n, _p(y), threads)
    return y


def linear_geglu(x, wg, wu, threads: int = 0) -> np.ndarray:
    x = _f32(x)
    k = wg.shape[1]
    t = x.size // k
    y = np.empty((t, wg.shape[0]), dtype=np.float32)
    hg, hu = _Held(wg), _Held(wu)
    if load().gqo_linear_geglu(_p(x), t, k, hg.ref, hu.ref, _p(y), threads) != 0:
        raise ValueError("oracle linear_geglu: bad shape")
    return y


def linear_gelu_mul_cols(x, w, b, offset: int, threads: int = 0) -> np.ndarray:
    x, b = _f32(x), _f32(b)
    k = w.shape[1]
    t = x.size // k
    stride = b.shape[-1]
    y = np.empty((t, w.shape[0]), dtype=np.float32)
    h = _Held(w)
    if load().gqo_linear_gelu_mul_cols(_p(x), t, k, h.ref, _p(b), stride, offset, _p(y), threads) != 0:
        raise ValueError("oracle linear_gelu_mul_cols: bad offset")
    return y


def embed_rows(table, ids, scale: float) -> np.ndarray:
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
    out = np.empty((ids.size, table.shape[1]), dtype=np.float32)
    h = _Held(table)
    if load().gqo_embed_rows(h.ref, _p(ids), ids.size, scale, _p(out)) != 0:
        raise IndexError("oracle embed_rows: id out of range")
    return out


def gelu_tanh(v: float) -> float:
    return float(load().gqo_gelu_tanh(v))


def geglu(g, u) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    load().gqo_geglu(_p(g), _p(u), g.size, _p(out))
    return out


def softcap(x, cap: float) -> np.ndarray:
    x = _f32(x)
    out = np.empty_like(x)
    load().gqo_softcap(_p(x), x.size, cap, _p(out))
    return out


# ---- support ops of the decode step (rust/src/backend_cpu.rs, rust/src/backend.rs) ----

def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def rms_norm(x, w, eps: float) -> np.ndarray:
    """rust/src/backend_cpu.rs:149-172, per row of the last axis (w None: unweighted)."""
    x = _f32(x)
    d = x.shape[-1]
    out = np.empty_like(x)
    wp = None if w is None else _f32(w)
    load().gqo_rms_norm(_p(x), x.size // d, d, None if wp is None else _p(wp), eps, _p(out))
    return out


def add(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    load().gqo_add(_p(a), _p(b), a.size, _p(out))
    return out


def mul(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    load().gqo_mul(_p(a), _p(b), a.size, _p(out))
    return out


def scale(a, s: float) -> np.ndarray:
    a = _f32(a)
    out = np.empty_like(a)
    load().gqo_scale(_p(a), a.size, s, _p(out))
    return out


def add_rms_norm(residual, x, w, eps: float, scale_by=None) -> np.ndarray:
    """rust/src/backend.rs:137-144: (residual + rms_norm(x, w)) * scale_by[0]."""
    r, x, w = _f32(residual), _f32(x), _f32(w)
    d = x.shape[-1]
    out = np.empty_like(x)
    sb = None if scale_by is None else _f32(np.atleast_1d(scale_by))
    load().gqo_add_rms_norm(_p(r), _p(x), x.size // d, d, _p(w), eps, None if sb is None else _p(sb), _p(out))
    return out


def rope(x, positions, theta: float, head_dim: int, heads: int, rotary_dim: int) -> np.ndarray:
    """rust/src/backend_cpu.rs:248-268 on [t, heads, head_dim]."""
    x, pos = _f32(x), _u32(positions)
    out = np.empty_like(x)
    load().gqo_rope(_p(x), pos.size, heads, head_dim, _p(pos), theta, rotary_dim, _p(out))
    return out


def head_norm_rope(x, w, eps: float, positions, theta: float, head_dim: int, heads: int,
                   rotary_dim: int) -> np.ndarray:
    """rust/src/backend.rs:148-154."""
    x, w, pos = _f32(x), _f32(w), _u32(positions)
    out = np.empty_like(x)
    load().gqo_head_norm_rope(_p(x), pos.size, heads, head_dim, _p(w), eps, _p(pos), theta, rotary_dim, _p(out))
    return out


def attention(q, k, v, q_pos, k_pos, scale: float = 1.0, sliding_window: int = 0, attn_softcap: float = 0.0,
              threads: int = 0) -> np.ndarray:
    """rust/src/backend_cpu.rs:270-336: q [t, hq, dh], k [s, hkv, dh], v [s, hkv, dv] -> [t, hq*dv]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    qp, kp = _u32(q_pos), _u32(k_pos)
    t, hq, dh = q.shape
    s, hkv, dv = v.shape
    out = np.empty((t, hq * dv), dtype=np.float32)
    rc = load().gqo_attention(_p(q), t, hq, dh, _p(k), _p(v), s, hkv, dv, _p(qp), _p(kp), scale,
                              int(sliding_window), attn_softcap, _p(out), threads)
    if rc != 0:
        raise ValueError("oracle attention: bad shape")
    return out


def rng_next_f64(state: int):
    """Rng::next_f64 (rust/src/sampler.rs:23-26): (u in [0, 1), the advanced state)."""
    st = ctypes.c_uint64(state & 0xFFFFFFFFFFFFFFFF)
    u = load().gqo_rng_next_f64(ctypes.byref(st))
    return float(u), int(st.value)


def sample(logits, temperature: float, top_k: int, top_p: float, repetition_penalty: float = 1.0,
           recent=None, u: float = 0.0) -> int:
    """sample (rust/src/sampler.rs:116-190) of one logits row with the draw u."""
    lg = _f32(logits).ravel()
    rc = _u32(recent if recent is not None else []).ravel()
    tok = load().gqo_sample(_p(lg), lg.size, temperature, int(top_k), top_p, repetition_penalty,
                            _p(rc) if rc.size else None, rc.size, float(u))
    if tok < 0:
        raise ValueError("oracle sample: bad argument")
    return int(tok)
