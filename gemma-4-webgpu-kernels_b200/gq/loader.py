"""Checkpoint loading through libgq (the C ABI's gq_st_* entry points): the
reference's SafetensorsFile (rust/src/safetensors.rs) and ModelWeights
(rust/src/weights.rs:37-118) for the quantized weights of the real QAT layout.

    f = SafetensorsFile(path)            # memory-mapped, header parsed in libgq
    rules = [("^lm_head$", 2), ...]      # config.quantization_config, match order
    w = load_quant(backend, f, "language_model.layers.3.mlp.gate_proj.weight", rules)

`load_quant` returns a device weight (a gq_qweight) exactly as the reference's
`ModelWeights::get` builds its QuantWeight: bits from the rules (8 for I8), K = stored
columns x values per byte, group_size = K / scale columns.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char, c_char_p, c_int32, c_int64, c_size_t, c_void_p
from typing import List, Sequence, Tuple

import numpy as np

from . import _abi


class SafetensorsFile:
    """A safetensors file parsed (and memory-mapped) by libgq."""

    def __init__(self, path: str = None, blob: bytes = None):
        self.lib = _abi.load()
        self.h = c_void_p()
        self._blob = None
        if blob is not None:
            self._blob = ctypes.create_string_buffer(bytes(blob), len(blob))
            rc = self.lib.gq_st_open_memory(ctypes.cast(self._blob, c_void_p), len(blob), ctypes.byref(self.h))
        else:
            rc = self.lib.gq_st_open(path.encode(), ctypes.byref(self.h))
        if rc != _abi.GQ_OK:
            raise _abi.GqError(rc, f"gq_st_open: {self.lib.gq_status_string(rc).decode()}")

    def close(self) -> None:
        if self.h:
            self.lib.gq_st_close(self.h)
            self.h = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> List[str]:
        return [self.lib.gq_st_name(self.h, i).decode() for i in range(self.lib.gq_st_count(self.h))]

    def info(self, name: str) -> Tuple[str, Tuple[int, ...], bytes]:
        """(dtype, shape, payload bytes) of a tensor."""
        dtype = (c_char * 16)()
        shape = (c_int64 * 8)()
        ndim = c_int32()
        data = c_void_p()
        nbytes = c_size_t()
        rc = self.lib.gq_st_info(self.h, name.encode(), dtype, shape, ctypes.byref(ndim), ctypes.byref(data),
                                 ctypes.byref(nbytes))
        if rc != _abi.GQ_OK:
            raise _abi.GqError(rc, f"gq_st_info({name})")
        payload = ctypes.string_at(data.value, nbytes.value) if nbytes.value else b""
        return dtype.value.decode(), tuple(shape[i] for i in range(ndim.value)), payload

    def read_f32(self, name: str) -> np.ndarray:
        """decode_to_f32 of an F32 / F16 / BF16 tensor, in its shape."""
        _, shape, _ = self.info(name)
        out = np.empty(shape, dtype=np.float32)
        rc = self.lib.gq_st_read_f32(self.h, name.encode(), out.ctypes.data_as(c_void_p), out.size)
        if rc != _abi.GQ_OK:
            raise _abi.GqError(rc, f"gq_st_read_f32({name})")
        return out


def bits_for(name: str, rules: Sequence[Tuple[str, int]]) -> int:
    """Gemma4Config::bits_for (rust/src/config.rs:161-169), evaluated by libgq."""
    lib = _abi.load()
    pats = (c_char_p * max(1, len(rules)))(*[p.encode() for p, _ in rules])
    bits = (c_int32 * max(1, len(rules)))(*[int(b) for _, b in rules])
    v = lib.gq_bits_for(name.encode(), pats, bits, len(rules))
    if v < 0:
        raise _abi.GqError(_abi.GQ_ERR_INVALID_ARGUMENT, f"bits_for({name}): bad pattern")
    return int(v)


def resolve(logical: str) -> Tuple[str, str, str]:
    """resolve_tensor_names (rust/src/weights.rs:37-48): (weight, scale, bare)."""
    lib = _abi.load()
    bufs = [ctypes.create_string_buffer(256) for _ in range(3)]
    rc = lib.gq_st_resolve(logical.encode(), *bufs)
    if rc != _abi.GQ_OK:
        raise _abi.GqError(rc, f"resolve({logical})")
    return tuple(b.value.decode() for b in bufs)


def load_quant(g, f: SafetensorsFile, logical: str, rules: Sequence[Tuple[str, int]]):
    """ModelWeights::load for a quantized weight (rust/src/weights.rs:86-110), onto
    backend g's device."""
    from . import GqTensor

    base = logical[: -len(".weight")] if logical.endswith(".weight") else logical
    out = c_void_p()
    rc = g.lib.gq_st_upload_quant(g.ctx, f.h, logical.encode(), bits_for(base, rules), ctypes.byref(out))
    g._check(rc, f"load_quant({logical})")
    g._qweights.append(out.value)
    n, k = c_int64(), c_int64()
    g.lib.gq_qweight_info(out, ctypes.byref(n), ctypes.byref(k), None, None, None)
    return GqTensor(shape=(n.value, k.value), qw=out.value, quant=None)
