"""ctypes binding of libgq.so (the C ABI declared in include/gq.h).

The library is loaded from this package directory. If it is missing the import
fails loudly: there is no CPU fallback behind this API.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint8, c_uint32, c_uint64, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgq.so")

GQ_OK = 0
GQ_ERR_INVALID_ARGUMENT = 1
GQ_ERR_UNSUPPORTED = 2
GQ_ERR_CUDA = 3
GQ_ERR_OUT_OF_MEMORY = 4
GQ_ERR_DEVICE = 5

GQ_DEVERR_BAD_ID = 0x1
GQ_DEVERR_WAIT_TIMEOUT = 0x2
GQ_DEVERR_SAMPLE_CAP = 0x4


class SampleOpts(ctypes.Structure):
    """gq_sample_opts (include/gq.h): the reference's SampleOpts (rust/src/sampler.rs:29-39)."""
    _fields_ = [("temperature", c_float), ("top_k", c_int32), ("top_p", c_float), ("repetition_penalty", c_float)]


class ChainOp(ctypes.Structure):
    """gq_chain_op (include/gq.h): one one-row MATMUL_Q call of a decode chain."""
    _fields_ = [("mode", c_int32), ("w", c_void_p), ("w2", c_void_p), ("x", c_void_p), ("y", c_void_p),
                ("b", c_void_p), ("b_offset", c_int64), ("cap", c_float)]


class GqError(RuntimeError):
    """A non-zero status from libgq (the Rust trait would panic here)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


# name -> (restype, argtypes). Every symbol include/gq.h declares.
SIGNATURES = {
    "gq_abi_version": (c_int, []),
    "gq_status_string": (c_char_p, [c_int]),
    "gq_ctx_create": (c_int, [c_int, POINTER(c_void_p)]),
    "gq_ctx_destroy": (c_int, [c_void_p]),
    "gq_ctx_set_stream": (c_int, [c_void_p, c_void_p]),
    "gq_ctx_get_stream": (c_void_p, [c_void_p]),
    "gq_ctx_num_sms": (c_int, [c_void_p]),
    "gq_last_error": (c_char_p, [c_void_p]),
    "gq_sync": (c_int, [c_void_p]),
    "gq_alloc": (c_int, [c_void_p, c_size_t, POINTER(c_void_p)]),
    "gq_free": (c_int, [c_void_p, c_void_p]),
    "gq_memcpy_h2d": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t]),
    "gq_memcpy_d2h": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t]),
    "gq_memset": (c_int, [c_void_p, c_void_p, c_int, c_size_t]),
    "gq_readback": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t]),
    "gq_qweight_upload": (
        c_int,
        [c_void_p, POINTER(c_uint8), c_size_t, POINTER(c_float), c_size_t, c_int64, c_int64, c_int32,
         c_int32, c_int64, POINTER(c_void_p)],
    ),
    "gq_qweight_upload_device": (
        c_int,
        [c_void_p, c_void_p, c_size_t, POINTER(c_float), c_size_t, c_int64, c_int64, c_int32,
         c_int32, c_int64, POINTER(c_void_p)],
    ),
    "gq_qweight_free": (c_int, [c_void_p]),
    "gq_qweight_info": (
        c_int,
        [c_void_p, POINTER(c_int64), POINTER(c_int64), POINTER(c_int32), POINTER(c_int32), POINTER(c_int64)],
    ),
    "gq_graph_begin": (c_int, [c_void_p]),
    "gq_graph_end": (c_int, [c_void_p, POINTER(c_void_p)]),
    "gq_graph_launch": (c_int, [c_void_p, c_void_p]),
    "gq_graph_destroy": (c_int, [c_void_p]),
    "gq_linear": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "gq_linear_geglu": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "gq_linear_gelu_mul_cols": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "gq_linear_softcap": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p, c_int64, c_int64]),
    "gq_linear_softcap_peers": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p, c_int64, c_int64, c_void_p,
                c_int32]),
    "gq_linear_softcap_peers_signal": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p, c_int64, c_int64, c_void_p,
                c_int32, c_void_p, c_void_p, c_int32]),
    "gq_linear_softcap_peers_sync": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p, c_int64, c_int64, c_void_p,
                c_int32, c_void_p, c_void_p, c_int32]),
    "gq_peer_wait": (c_int, [c_void_p, c_void_p, c_int32, c_void_p]),
    "gq_ctx_set_wait_limit": (c_int, [c_void_p, c_uint64]),
    "gq_chain_create": (c_int, [c_void_p, c_void_p, c_int32, POINTER(c_void_p)]),
    "gq_chain_run": (c_int, [c_void_p]),
    "gq_chain_reset": (c_int, [c_void_p]),
    "gq_chain_destroy": (c_int, [c_void_p]),
    "gq_argmax_rows": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "gq_sample_rows": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                               c_void_p, c_void_p]),
    "gq_topk_rows": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int32, c_float, c_void_p,
                             c_int64, c_int64, c_void_p, c_void_p]),
    "gq_sample_candidates": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                                     c_void_p]),
    "gq_ipc_get_handle": (c_int, [c_void_p, c_void_p, c_void_p]),
    "gq_ipc_open": (c_int, [c_void_p, c_void_p, POINTER(c_void_p)]),
    "gq_ipc_close": (c_int, [c_void_p, c_void_p]),
    "gq_embed_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_float, c_void_p]),
    "gq_st_open": (c_int, [c_char_p, POINTER(c_void_p)]),
    "gq_st_open_memory": (c_int, [c_void_p, c_size_t, POINTER(c_void_p)]),
    "gq_st_close": (c_int, [c_void_p]),
    "gq_st_count": (c_int64, [c_void_p]),
    "gq_st_name": (c_char_p, [c_void_p, c_int64]),
    "gq_st_info": (c_int, [c_void_p, c_char_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "gq_st_read_f32": (c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
    "gq_bits_for": (c_int32, [c_char_p, c_void_p, c_void_p, c_int32]),
    "gq_st_resolve": (c_int, [c_char_p, c_void_p, c_void_p, c_void_p]),
    "gq_st_upload_quant": (c_int, [c_void_p, c_void_p, c_char_p, c_int32, POINTER(c_void_p)]),
    "gq_linear_prefill_static": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "gq_linear_prefill_static_status": (c_int, [c_void_p, POINTER(c_uint32)]),
    "gq_softcap": (c_int, [c_void_p, c_void_p, c_int64, c_float, c_void_p]),
    "gq_geglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "gq_rms_norm": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p, c_int64]),
    "gq_add_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p,
                                c_void_p]),
    "gq_add_rms_norm_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_float, c_void_p,
                                     c_void_p, c_void_p, c_void_p]),
    "gq_add_norm_linear": (c_int, [c_void_p, c_int32, c_void_p, c_void_p, c_int64, c_void_p, c_float, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "gq_head_norm_rope": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p,
                                  c_float, c_int64, c_void_p, c_int64]),
    "gq_qkv_norm_rope": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_float, c_void_p,
                c_float, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64]),
    "gq_rope": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_float, c_int64, c_void_p,
                        c_int64]),
    "gq_attention": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64,
                             c_int64, c_int64, c_void_p, c_void_p, c_int64, c_float, c_uint32, c_float, c_uint32,
                             c_void_p]),
    "gq_linear_bf16": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p]),
    "gq_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "gq_mul": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "gq_scale": (c_int, [c_void_p, c_void_p, c_int64, c_float, c_void_p]),
    "gq_scale_by_tensor": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "gq_copy_rows": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64]),
}

GQ_ATTN_KPOS_ASCENDING = 0x1
GQ_ATTN_KPOS_IDENTITY = 0x2

_lib = None


def load() -> ctypes.CDLL:
    """Load libgq.so once and attach the signatures. Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libgq.so not found at {LIB_PATH}: build it with "
            "`make -C gemma-4-webgpu-kernels_b200` (there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, ctx=None, what: str = "") -> None:
    if status == GQ_OK:
        return
    lib = load()
    msg = lib.gq_last_error(ctx).decode() if ctx else lib.gq_status_string(status).decode()
    raise GqError(status, f"{what}: {msg}" if what else msg)
