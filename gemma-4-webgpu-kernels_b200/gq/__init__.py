"""gq — B200 backend for the quantized-weight hot path of the Gemma-4 engine.

Host-side mirror of the reference's `Backend` trait (rust/src/backend.rs:88-180)
for the quantized ops, on top of the C ABI in include/gq.h (libgq.so). Method
names, argument meaning and error behaviour follow the trait:

* ``quant_tensor(QuantWeight)``                        rust/src/backend.rs:95
* ``linear(x, w)``                                     rust/src/backend.rs:105-106
* ``linear_geglu(x, w_gate, w_up)``                    rust/src/backend.rs:155-160
* ``linear_gelu_mul_cols(x, w, b, offset)``            rust/src/backend.rs:161-167
* ``embed_rows(table, ids, scale)``                    rust/src/backend.rs:101-102
* ``softcap(a, cap)`` / ``geglu(gate, up)``            rust/src/backend.rs:113-116
* ``tensor`` / ``zeros`` / ``reshape`` / ``readback`` / ``flush`` /
  ``begin_frame`` / ``end_frame`` / ``free_tensor``    rust/src/backend.rs:94-98, 169-179
* support ops of a decode step: ``rms_norm``, ``add``, ``mul``, ``scale``,
  ``scale_by_tensor``, ``rope``, ``attention``, ``slice_rows``, ``slice_cols``,
  ``concat_rows``, ``kv_append`` (rust/src/backend.rs:103-130), ``add_rms_norm``,
  ``head_norm_rope`` (:137-154), and ``linear`` with a bf16-stored plain weight

Ops enqueue on the backend's stream (torch's current stream of the device) and
return immediately; ``readback`` blocks, like the reference. Failures raise
``GqError`` where the Rust trait panics. Device memory for f32 tensors comes from
torch's caching allocator; the quantized weights are owned by libgq.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int32, c_int64, c_uint8, c_void_p
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _abi
from ._abi import GqError

__all__ = ["QuantWeight", "GqTensor", "CudaBackend", "GqError", "AttnOpts", "KvAppend"]


@dataclass
class QuantWeight:
    """A weight kept in its packed, quantized form (rust/src/backend.rs:16-24).

    ``qbytes``: raw payload (U8 sub-byte packed LSB-first offset-binary, or
    native I8); ``scales``: one f32 per (row, group); ``shape``: logical [N, K].
    """

    qbytes: np.ndarray
    scales: np.ndarray
    shape: tuple
    bits: int
    signed_i8: bool
    group_size: int

    def per_byte(self) -> int:  # rust/src/backend.rs:28-30
        return 1 if self.signed_i8 else 8 // self.bits

    def row_bytes(self) -> int:  # rust/src/backend.rs:33-36
        k = self.shape[1]
        return k if self.signed_i8 else k // self.per_byte()

    def scale_stride(self) -> int:  # rust/src/backend.rs:39-41
        return -(-self.shape[1] // self.group_size)

    def codes(self) -> np.ndarray:
        """All integer codes [N, K] (the integer part of deq, backend.rs:46-54)."""
        n, k = self.shape
        b = np.asarray(self.qbytes, dtype=np.uint8)[: n * self.row_bytes()].reshape(n, self.row_bytes())
        if self.signed_i8:
            return b.view(np.int8).astype(np.int32)
        pb = self.per_byte()
        shifts = (np.arange(pb, dtype=np.uint32) * self.bits)[None, None, :]
        raw = (b.astype(np.uint32)[:, :, None] >> shifts) & ((1 << self.bits) - 1)
        return raw.reshape(n, k).astype(np.int32) - (1 << (self.bits - 1))


@dataclass
class GqTensor:
    """A backend tensor: dense row-major f32 on the device, a quantized weight, or a
    plain weight stored as bf16 (``bf16=True``: ``data`` is a cuda int16 tensor of
    the bf16 bit patterns)."""

    shape: tuple
    data: object = None          # torch.Tensor (cuda, float32, contiguous) for f32 tensors
    qw: Optional[int] = None     # gq_qweight* for quantized tensors
    quant: Optional[QuantWeight] = field(default=None, repr=False)
    bf16: bool = False

    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def ptr(self) -> int:
        return self.data.data_ptr()


@dataclass
class AttnOpts:
    """rust/src/backend.rs:59-69: query / key positions, score scale, sliding
    window (0 = none) and attention soft-cap (0 = none)."""

    q_pos: Sequence[int]
    k_pos: Sequence[int]
    scale: float = 1.0
    sliding_window: int = 0
    attn_softcap: float = 0.0


@dataclass
class KvAppend:
    """rust/src/backend.rs:71-77: the grown tensor and the one it superseded."""

    tensor: GqTensor
    dead: Optional[GqTensor] = None


class Chain:
    """A created decode chain (gq_chain): run() enqueues it on the backend's
    stream (recordable into a graph), reset() clears its counters after a
    timed-out run, close() frees it."""

    def __init__(self, backend: "CudaBackend", handle: c_void_p):
        self.backend = backend
        self.handle = handle

    def run(self) -> None:
        self.backend._check(self.backend.lib.gq_chain_run(self.handle), "chain_run")

    def reset(self) -> None:
        self.backend._check(self.backend.lib.gq_chain_reset(self.handle), "chain_reset")

    def close(self) -> None:
        if self.handle is not None and self.handle.value:
            self.backend.lib.gq_chain_destroy(self.handle)
        self.handle = None


class CudaBackend:
    """The Backend-trait surface of the quantized hot path, on one CUDA device."""

    def __init__(self, device: int = 0, own_stream: bool = False):
        """own_stream=False runs on torch's current stream of the device;
        True keeps the context's own non-blocking stream (needed to record graphs)."""
        import torch  # device memory + streams (plumbing only)

        self._torch = torch
        self.lib = _abi.load()
        self.device = int(device)
        self.torch_device = torch.device("cuda", self.device)
        ctx = c_void_p()
        rc = self.lib.gq_ctx_create(self.device, ctypes.byref(ctx))
        if rc != _abi.GQ_OK:
            raise GqError(rc, f"gq_ctx_create(device={device}) failed: {self.lib.gq_status_string(rc).decode()}")
        self.ctx = ctx
        self._frame: list = []
        self._qweights: list = []
        self.own_stream = own_stream
        if not own_stream:
            self._bind_stream()

    # ---- plumbing ---------------------------------------------------------
    def _bind_stream(self) -> None:
        s = self._torch.cuda.current_stream(self.torch_device).cuda_stream
        # torch's default stream is the legacy NULL stream (handle 0); pass it as
        # cudaStreamLegacy (0x1), since NULL means "the context's own stream" here
        if not s:
            s = 1
        _abi.check(self.lib.gq_ctx_set_stream(self.ctx, c_void_p(s)), self.ctx, "set_stream")

    def _check(self, rc: int, what: str) -> None:
        _abi.check(rc, self.ctx, what)

    def _alloc(self, shape) -> GqTensor:
        t = self._torch.empty(tuple(shape), dtype=self._torch.float32, device=self.torch_device)
        g = GqTensor(shape=tuple(shape), data=t)
        self._frame.append(g)
        return g

    def close(self) -> None:
        if getattr(self, "ctx", None):
            for q in self._qweights:
                self.lib.gq_qweight_free(q)
            self._qweights.clear()
            self.lib.gq_ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def name(self) -> str:
        return "cuda-b200"

    def num_sms(self) -> int:
        return self.lib.gq_ctx_num_sms(self.ctx)

    def stream_ptr(self) -> int:
        return int(self.lib.gq_ctx_get_stream(self.ctx) or 0)

    # ---- record / replay (include/gq.h gq_graph_*) ------------------------------
    def record(self, fn):
        """Record the ops `fn()` issues into a replayable graph (own_stream only)."""
        self._check(self.lib.gq_graph_begin(self.ctx), "graph_begin")
        try:
            fn()
        except BaseException:
            tmp = c_void_p()
            self.lib.gq_graph_end(self.ctx, ctypes.byref(tmp))
            if tmp.value:
                self.lib.gq_graph_destroy(tmp)
            raise
        out = c_void_p()
        self._check(self.lib.gq_graph_end(self.ctx, ctypes.byref(out)), "graph_end")
        return out

    def replay(self, graph) -> None:
        self._check(self.lib.gq_graph_launch(self.ctx, graph), "graph_launch")

    def destroy_graph(self, graph) -> None:
        self.lib.gq_graph_destroy(graph)

    # ---- decode chains (include/gq.h gq_chain_*) ------------------------------------
    def chain(self, ops) -> "Chain":
        """A decode chain over `ops`: tuples (mode, w, w2, x, y, b, b_offset, cap)
        with w/w2 quantized GqTensors (w2 None unless mode 1), x/y/b device
        pointers (int) or f32 GqTensors (b None unless mode 2). One activation row
        per op; `Chain.run()` issues them all as one launch."""
        arr = (_abi.ChainOp * len(ops))()
        for i, (mode, w, w2, x, y, b, b_off, cap) in enumerate(ops):
            ptr = lambda t: None if t is None else (t if isinstance(t, int) else t.ptr())
            arr[i] = _abi.ChainOp(int(mode), c_void_p(w.qw), c_void_p(w2.qw if w2 is not None else None),
                                  c_void_p(ptr(x)), c_void_p(ptr(y)), c_void_p(ptr(b)), int(b_off), float(cap))
        out = c_void_p()
        self._check(self.lib.gq_chain_create(self.ctx, arr, len(ops), ctypes.byref(out)), "chain_create")
        return Chain(self, out)

    # ---- construction (rust/src/backend.rs:94-98) ----------------------------
    def tensor(self, data, shape: Sequence[int]) -> GqTensor:
        arr = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(tuple(shape)))
        t = self._torch.from_numpy(arr).to(self.torch_device)
        return GqTensor(shape=tuple(shape), data=t)

    def from_torch(self, t) -> GqTensor:
        """Wrap an existing cuda float32 contiguous tensor (no copy)."""
        assert t.is_cuda and t.dtype == self._torch.float32 and t.is_contiguous()
        return GqTensor(shape=tuple(t.shape), data=t)

    def quant_tensor(self, q: QuantWeight) -> GqTensor:
        qb = np.ascontiguousarray(np.asarray(q.qbytes, dtype=np.uint8))
        sc = np.ascontiguousarray(np.asarray(q.scales, dtype=np.float32))
        out = c_void_p()
        n, k = q.shape
        rc = self.lib.gq_qweight_upload(
            self.ctx, qb.ctypes.data_as(ctypes.POINTER(c_uint8)), qb.size,
            sc.ctypes.data_as(ctypes.POINTER(c_float)), sc.size, n, k, q.bits, int(bool(q.signed_i8)),
            q.group_size, ctypes.byref(out))
        self._check(rc, "quant_tensor")
        self._qweights.append(out.value)
        return GqTensor(shape=(n, k), qw=out.value, quant=q)

    def quant_tensor_from_device(self, qbytes_dev, scales, shape, bits: int, signed_i8: bool,
                                 group_size: int) -> GqTensor:
        """WgpuBackend::quant_tensor_from_gpu (rust/src/backend_wgpu.rs:447-456):
        the packed payload is a cuda uint8 tensor already on this device."""
        sc = np.ascontiguousarray(np.asarray(scales, dtype=np.float32))
        out = c_void_p()
        n, k = shape
        rc = self.lib.gq_qweight_upload_device(
            self.ctx, c_void_p(qbytes_dev.data_ptr()), qbytes_dev.numel(), sc.ctypes.data_as(ctypes.POINTER(c_float)),
            sc.size, n, k, bits, int(bool(signed_i8)), group_size, ctypes.byref(out))
        self._check(rc, "quant_tensor_from_device")
        self._qweights.append(out.value)
        return GqTensor(shape=(n, k), qw=out.value, quant=None)

    def free_quant(self, t: GqTensor) -> None:
        if t.qw in self._qweights:
            self._qweights.remove(t.qw)
            self.lib.gq_qweight_free(t.qw)
            t.qw = None

    def zeros(self, shape: Sequence[int]) -> GqTensor:
        t = self._torch.zeros(tuple(shape), dtype=self._torch.float32, device=self.torch_device)
        return GqTensor(shape=tuple(shape), data=t)

    def reshape(self, x: GqTensor, shape: Sequence[int]) -> GqTensor:
        if x.qw is not None:
            return GqTensor(shape=tuple(shape), qw=x.qw, quant=x.quant)
        return GqTensor(shape=tuple(shape), data=x.data.view(tuple(shape)))

    # ---- ops ------------------------------------------------------------------
    def _xm(self, x: GqTensor):
        k = x.shape[-1]
        m = x.size() // k if k else 0
        return m, k

    def linear(self, x: GqTensor, w: GqTensor) -> GqTensor:
        """y = x · Wᵀ; x [M, K], W [N, K] quantized (rust/src/backend.rs:105-106)."""
        self._require_quant(w, "linear")
        m, k = self._xm(x)
        y = self._alloc((m, w.shape[0]))
        self._check(self.lib.gq_linear(self.ctx, c_void_p(x.ptr()), m, k, c_void_p(w.qw), c_void_p(y.ptr())),
                    "linear")
        return y

    def linear_geglu(self, x: GqTensor, w_gate: GqTensor, w_up: GqTensor) -> GqTensor:
        """gelu(x · Wgᵀ) * (x · Wuᵀ) (rust/src/backend.rs:155-160)."""
        self._require_quant(w_gate, "linear_geglu")
        self._require_quant(w_up, "linear_geglu")
        m, k = self._xm(x)
        y = self._alloc((m, w_gate.shape[0]))
        self._check(self.lib.gq_linear_geglu(self.ctx, c_void_p(x.ptr()), m, k, c_void_p(w_gate.qw),
                                             c_void_p(w_up.qw), c_void_p(y.ptr())), "linear_geglu")
        return y

    def linear_gelu_mul_cols(self, x: GqTensor, w: GqTensor, b: GqTensor, offset: int) -> GqTensor:
        """gelu(x · Wᵀ) * b[:, offset:offset+N], b [M, stride] (rust/src/backend.rs:161-167)."""
        self._require_quant(w, "linear_gelu_mul_cols")
        m, k = self._xm(x)
        if len(b.shape) != 2 or b.shape[0] != m:
            raise GqError(_abi.GQ_ERR_INVALID_ARGUMENT, "linear_gelu_mul_cols: b must be [M, stride]")
        y = self._alloc((m, w.shape[0]))
        self._check(self.lib.gq_linear_gelu_mul_cols(self.ctx, c_void_p(x.ptr()), m, k, c_void_p(w.qw),
                                                     c_void_p(b.ptr()), b.shape[1], offset, c_void_p(y.ptr())),
                    "linear_gelu_mul_cols")
        return y

    def linear_softcap(self, x: GqTensor, w: GqTensor, cap: float, out: Optional[GqTensor] = None,
                       col0: int = 0) -> GqTensor:
        """softcap(linear(x, w), cap) in one pass — the lm_head of rust/src/model.rs:192
        followed by Backend::softcap. ``out``/``col0`` write a vocab shard into its
        column slice of a wider logits tensor."""
        self._require_quant(w, "linear_softcap")
        m, k = self._xm(x)
        y = out if out is not None else self._alloc((m, w.shape[0]))
        ldy = y.shape[-1]
        self._check(self.lib.gq_linear_softcap(self.ctx, c_void_p(x.ptr()), m, k, c_void_p(w.qw), float(cap),
                                               c_void_p(y.ptr()), ldy, col0), "linear_softcap")
        return y

    def embed_rows(self, table: GqTensor, ids: Sequence[int], scale: float) -> GqTensor:
        """out[i, :] = deq(table)[ids[i], :] * scale (rust/src/backend.rs:101-102)."""
        self._require_quant(table, "embed_rows")
        if isinstance(ids, self._torch.Tensor) and ids.is_cuda:
            dids = ids.to(self._torch.int32).contiguous()
        else:
            arr = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
            dids = self._torch.from_numpy(arr.view(np.int32)).to(self.torch_device)
        t = int(dids.numel())
        out = self._alloc((t, table.shape[1]))
        self._check(self.lib.gq_embed_rows(self.ctx, c_void_p(table.qw), c_void_p(dids.data_ptr()), t,
                                           float(scale), c_void_p(out.ptr())), "embed_rows")
        self._frame.append(GqTensor(shape=(t,), data=dids))  # keep ids alive until the frame ends
        return out

    def softcap(self, a: GqTensor, cap: float) -> GqTensor:
        y = self._alloc(a.shape)
        self._check(self.lib.gq_softcap(self.ctx, c_void_p(a.ptr()), a.size(), float(cap), c_void_p(y.ptr())),
                    "softcap")
        return y

    def geglu(self, gate: GqTensor, up: GqTensor) -> GqTensor:
        y = self._alloc(gate.shape)
        self._check(self.lib.gq_geglu(self.ctx, c_void_p(gate.ptr()), c_void_p(up.ptr()), gate.size(),
                                      c_void_p(y.ptr())), "geglu")
        return y

    # ---- support ops of a decode step (rust/src/backend.rs:103-154) ------------
    def _u32_dev(self, vals):
        if isinstance(vals, self._torch.Tensor) and vals.is_cuda:
            t = vals.to(self._torch.int32).contiguous()
        else:
            arr = np.ascontiguousarray(np.asarray(vals, dtype=np.uint32))
            t = self._torch.from_numpy(arr.view(np.int32)).to(self.torch_device)
        self._frame.append(GqTensor(shape=(t.numel(),), data=t))  # alive until the frame ends
        return t

    def tensor_bf16(self, data, shape: Sequence[int]) -> GqTensor:
        """A plain weight stored as bf16 (round to nearest even; exact for values that
        are bf16 on disk, like the reference's BF16 checkpoint tensors)."""
        arr = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(tuple(shape)))
        u = arr.view(np.uint32)
        rounded = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
        t = self._torch.from_numpy(rounded.view(np.int16)).to(self.torch_device)
        return GqTensor(shape=tuple(shape), data=t, bf16=True)

    def rms_norm(self, x: GqTensor, w: Optional[GqTensor], eps: float) -> GqTensor:
        """y = x / sqrt(mean(x²) + eps) * w per row (rust/src/backend.rs:103-104)."""
        d = x.shape[-1]
        y = self._alloc(x.shape)
        self._check(self.lib.gq_rms_norm(self.ctx, c_void_p(x.ptr()), x.size() // d, d,
                                         c_void_p(w.ptr()) if w is not None else None, float(eps),
                                         c_void_p(y.ptr()), d), "rms_norm")
        return y

    def add_rms_norm(self, residual: GqTensor, x: GqTensor, w: GqTensor, eps: float,
                     scale_by: Optional[GqTensor] = None) -> GqTensor:
        """(residual + rms_norm(x, w)) * scale_by[0] (rust/src/backend.rs:137-144)."""
        d = x.shape[-1]
        y = self._alloc(x.shape)
        self._check(self.lib.gq_add_rms_norm(self.ctx, c_void_p(residual.ptr()), c_void_p(x.ptr()), x.size() // d,
                                             d, c_void_p(w.ptr()), float(eps),
                                             c_void_p(scale_by.ptr()) if scale_by is not None else None,
                                             c_void_p(y.ptr())), "add_rms_norm")
        return y

    def head_norm_rope(self, x: GqTensor, w: GqTensor, eps: float, positions, theta: float, head_dim: int,
                       heads: int, rotary_dim: int) -> GqTensor:
        """Per-head weighted RMSNorm then partial RoPE (rust/src/backend.rs:148-154)."""
        pos = self._u32_dev(positions)
        t = x.size() // (heads * head_dim)
        y = self._alloc(x.shape)
        self._check(self.lib.gq_head_norm_rope(self.ctx, c_void_p(x.ptr()), t, heads, head_dim, c_void_p(w.ptr()),
                                               float(eps), c_void_p(pos.data_ptr()), float(theta), rotary_dim,
                                               c_void_p(y.ptr()), 0), "head_norm_rope")
        return y

    def rope(self, x: GqTensor, positions, theta: float, head_dim: int, heads: int, rotary_dim: int) -> GqTensor:
        """Half-split partial RoPE on [T, heads, head_dim] (rust/src/backend.rs:118-119)."""
        pos = self._u32_dev(positions)
        t = x.size() // (heads * head_dim)
        y = self._alloc(x.shape)
        self._check(self.lib.gq_rope(self.ctx, c_void_p(x.ptr()), t, heads, head_dim, c_void_p(pos.data_ptr()),
                                     float(theta), rotary_dim, c_void_p(y.ptr()), 0), "rope")
        return y

    def attention(self, q: GqTensor, k: GqTensor, v: GqTensor, opts: AttnOpts) -> GqTensor:
        """q [T, Hq, Dh], k/v [S, Hkv, Dh] -> [T, Hq*Dh] (rust/src/backend.rs:120-121)."""
        t, hq, dh = q.shape
        s, hkv = k.shape[0], k.shape[1]
        if v.shape[-1] != dh or k.shape[-1] != dh:
            raise GqError(_abi.GQ_ERR_UNSUPPORTED, "attention: value head_dim must equal key head_dim")
        qp, kp = self._u32_dev(opts.q_pos), self._u32_dev(opts.k_pos)
        kpos = np.asarray(opts.k_pos, dtype=np.int64)
        flags = _abi.GQ_ATTN_KPOS_ASCENDING if (kpos.size < 2 or bool(np.all(np.diff(kpos) > 0))) else 0
        y = self._alloc((t, hq * dh))
        self._check(self.lib.gq_attention(self.ctx, c_void_p(q.ptr()), 1, t, hq, dh, c_void_p(k.ptr()),
                                          c_void_p(v.ptr()), s, hkv, 0, c_void_p(qp.data_ptr()),
                                          c_void_p(kp.data_ptr()), 0, float(opts.scale), int(opts.sliding_window),
                                          float(opts.attn_softcap), flags, c_void_p(y.ptr())), "attention")
        return y

    def linear_plain(self, x: GqTensor, w: GqTensor) -> GqTensor:
        """linear with a plain (bf16-stored) weight [N, K] (rust/src/backend_cpu.rs:174-222)."""
        if not w.bf16:
            raise GqError(_abi.GQ_ERR_INVALID_ARGUMENT, "linear_plain: weight must come from tensor_bf16")
        m, k = self._xm(x)
        n = w.shape[0]
        y = self._alloc((m, n))
        self._check(self.lib.gq_linear_bf16(self.ctx, c_void_p(x.ptr()), m, k, c_void_p(w.ptr()), n,
                                            c_void_p(y.ptr())), "linear_bf16")
        return y

    def _ew(self, fn, *args, shape, what):
        y = self._alloc(shape)
        self._check(fn(self.ctx, *args, c_void_p(y.ptr())), what)
        return y

    def add(self, a: GqTensor, b: GqTensor) -> GqTensor:
        return self._ew(self.lib.gq_add, c_void_p(a.ptr()), c_void_p(b.ptr()), a.size(), shape=a.shape, what="add")

    def mul(self, a: GqTensor, b: GqTensor) -> GqTensor:
        return self._ew(self.lib.gq_mul, c_void_p(a.ptr()), c_void_p(b.ptr()), a.size(), shape=a.shape, what="mul")

    def scale(self, a: GqTensor, s: float) -> GqTensor:
        return self._ew(self.lib.gq_scale, c_void_p(a.ptr()), a.size(), float(s), shape=a.shape, what="scale")

    def scale_by_tensor(self, a: GqTensor, s: GqTensor) -> GqTensor:
        return self._ew(self.lib.gq_scale_by_tensor, c_void_p(a.ptr()), a.size(), c_void_p(s.ptr()), shape=a.shape,
                        what="scale_by_tensor")

    def _copy_rows(self, src: GqTensor, rows: int, cols: int, src_stride: int, src_off: int, dst: GqTensor,
                   dst_stride: int, dst_off: int) -> None:
        self._check(self.lib.gq_copy_rows(self.ctx, c_void_p(src.ptr() + 4 * src_off), rows, cols, src_stride,
                                          c_void_p(dst.ptr() + 4 * dst_off), dst_stride), "copy_rows")

    def slice_rows(self, x: GqTensor, start: int, count: int) -> GqTensor:
        """Rows [start, start+count) of [rows, dim] (rust/src/backend.rs:122-123)."""
        dim = x.shape[1]
        y = self._alloc((count, dim))
        self._copy_rows(x, count, dim, dim, start * dim, y, dim, 0)
        return y

    def slice_cols(self, x: GqTensor, offset: int, width: int) -> GqTensor:
        """[:, offset:offset+width] of [rows, stride] (rust/src/backend.rs:124-125)."""
        rows, stride = x.shape
        y = self._alloc((rows, width))
        self._copy_rows(x, rows, width, stride, offset, y, width, 0)
        return y

    def concat_rows(self, a: Optional[GqTensor], b: GqTensor) -> GqTensor:
        """Concatenate along dim 0 (rust/src/backend.rs:126-127)."""
        if a is None:
            y = self._alloc(b.shape)
            self._copy_rows(b, 1, b.size(), b.size(), 0, y, b.size(), 0)
            return y
        shape = (a.shape[0] + b.shape[0],) + tuple(a.shape[1:])
        y = self._alloc(shape)
        self._copy_rows(a, 1, a.size(), a.size(), 0, y, a.size(), 0)
        self._copy_rows(b, 1, b.size(), b.size(), 0, y, b.size(), a.size())
        return y

    def kv_append(self, existing: Optional[GqTensor], add: GqTensor) -> KvAppend:
        """Append rows (rust/src/backend.rs:128-130): a new tensor holding old ++ new;
        the old one is reported dead, as on the CPU backend."""
        return KvAppend(tensor=self.concat_rows(existing, add), dead=existing)

    # ---- sync / lifecycle (rust/src/backend.rs:169-179) ------------------------
    def readback(self, t: GqTensor) -> np.ndarray:
        """Blocking read of a tensor's f32 contents; raises on a device-reported error."""
        out = np.empty(t.size(), dtype=np.float32)
        self._check(self.lib.gq_readback(self.ctx, out.ctypes.data_as(c_void_p), c_void_p(t.ptr()), out.size),
                    "readback")
        return out

    def flush(self) -> None:
        self._check(self.lib.gq_sync(self.ctx), "flush")

    def begin_frame(self) -> None:
        self._frame = []

    def end_frame(self, keep: Sequence[GqTensor] = (), also_free: Sequence[GqTensor] = ()) -> None:
        keep_ids = {id(k.data) for k in keep if k.data is not None}
        self._frame = [t for t in self._frame if id(t.data) in keep_ids]
        for t in also_free:
            self.free_tensor(t)

    def free_tensor(self, t: GqTensor) -> None:
        if t.qw is not None:
            self.free_quant(t)
        t.data = None

    @staticmethod
    def _require_quant(w: GqTensor, op: str) -> None:
        if w.qw is None:
            raise GqError(_abi.GQ_ERR_INVALID_ARGUMENT, f"{op}: weight is not a quantized tensor")
