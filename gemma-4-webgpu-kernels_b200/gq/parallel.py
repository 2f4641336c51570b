"""Vocab-row sharding of the lm_head across the GPUs of one box.

The lm_head [V, K] is the only part of the quantized path that shards: rank r
owns rows [r*V/G, (r+1)*V/G) (its packed bytes and scales), computes the
soft-capped logits of its rows with the streaming GEMV, and the shards are
gathered over NVLink with NCCL. Every rank runs the (small) trunk itself, so no
broadcast of the hidden state is needed. The reference engine is single-device
(rust/src/model.rs:192 computes the whole lm_head in one linear); the gathered
logits equal that single-device result row for row.

The host logic here (row split, slicing a packed weight, reassembling the
gathered [G, M, V/G] blocks into [M, V]) is backend-agnostic so it is tested on
CPU with gloo ranks and the oracle as the per-shard compute.

Two exchanges: ShardedLmHead gathers the shards with NCCL's all-gather;
PeerLmHead fuses the exchange into the shard GEMV (its epilogue stores every
logit into all ranks' buffers over NVLink through CUDA IPC mappings).
"""
from __future__ import annotations

from typing import Tuple

import numpy as np

from . import QuantWeight


def shard_rows(vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [r0, r1) of rank `rank`; every shard has ceil(V/G) rows except a
    shorter (or empty) tail."""
    per = -(-vocab // world)
    r0 = min(vocab, rank * per)
    return r0, min(vocab, r0 + per)


def slice_rows(q: QuantWeight, r0: int, r1: int) -> QuantWeight:
    """Rows [r0, r1) of a packed weight: rows are contiguous in the packed layout
    (rust/src/backend.rs:26-41), so this is a byte range and a scale range."""
    rb, ss = q.row_bytes(), q.scale_stride()
    qb = np.asarray(q.qbytes, dtype=np.uint8)[r0 * rb: r1 * rb]
    sc = np.asarray(q.scales, dtype=np.float32)[r0 * ss: r1 * ss]
    return QuantWeight(qbytes=qb, scales=sc, shape=(r1 - r0, q.shape[1]), bits=q.bits, signed_i8=q.signed_i8,
                       group_size=q.group_size)


def assemble(gathered, m: int, world: int, per: int, vocab: int):
    """[G * M * per] (rank-major, as all_gather_into_tensor lays it out) -> [M, V].
    Works on numpy arrays and torch tensors."""
    g = gathered.reshape(world, m, per)
    if m == 1:
        return g.reshape(1, world * per)[:, :vocab]
    if hasattr(g, "permute"):
        return g.permute(1, 0, 2).reshape(m, world * per)[:, :vocab]
    return g.transpose(1, 0, 2).reshape(m, world * per)[:, :vocab]


class ShardedLmHead:
    """One rank's share of the lm_head on a CudaBackend, gathered with NCCL.

    forward(x) returns the full soft-capped logits [M, V] on every rank."""

    def __init__(self, backend, shard, vocab: int, rank: int, world: int, cap: float = 30.0, group=None):
        """shard: this rank's rows as a QuantWeight (uploaded here) or an already
        uploaded GqTensor."""
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.g = backend
        self.rank, self.world, self.vocab, self.cap, self.group = rank, world, vocab, cap, group
        self.r0, self.r1 = shard_rows(vocab, world, rank)
        self.per = -(-vocab // world)
        assert shard.shape[0] == self.r1 - self.r0
        if getattr(shard, "qw", None) is not None:
            self.w = shard
        else:
            self.w = backend.quant_tensor(shard) if shard.shape[0] else None
        self._bufs = {}

    def _buffers(self, m: int):
        if m not in self._bufs:
            t = self.torch
            local = t.zeros((m, self.per), dtype=t.float32, device=self.g.torch_device)
            gathered = t.empty((self.world * m * self.per,), dtype=t.float32, device=self.g.torch_device)
            self._bufs[m] = (local, gathered)
        return self._bufs[m]

    def forward(self, x):
        """x: GqTensor [M, K] on this rank's device -> torch tensor [M, V]."""
        m = x.shape[0]
        local, gathered = self._buffers(m)
        if self.w is not None:
            self.g.linear_softcap(x, self.w, self.cap, out=self.g.from_torch(local), col0=0)
        self.dist.all_gather_into_tensor(gathered, local, group=self.group)
        return assemble(gathered, m, self.world, self.per, self.vocab)


class _DeviceArray:
    """A raw device float32 buffer exposed to torch (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape), "typestr": "<f4",
                                         "version": 3}


class PeerLmHead:
    """One rank's share of the lm_head with the all-gather fused into the GEMV.

    Every rank owns two logits buffers [max_m, V] (one gq_alloc, an allocation
    base CUDA IPC can export) and maps every peer's into its own device
    (gq_ipc_open). forward(x) runs the shard GEMV whose epilogue stores each logit
    of this rank's vocab columns into its own buffer and, over NVLink, into every
    peer's buffer at the same offset. Calls alternate between the two buffers, so
    a rank that runs ahead writes the buffer its peers finished reading a call
    earlier (a rank can be at most one call ahead: each call waits for all ranks).
    The buffer is chosen on the host, so a CUDA graph should capture calls in
    pairs.

    Completion barrier, `barrier=`:
      "device" (default): gq_linear_softcap_peers_signal — the GEMV's last CTA
        increments a device-resident epoch and stores it into a flag slot of
        every rank (release, system scope) — then gq_peer_wait on this rank's
        flags. No NCCL call per step, and the pair replays inside a graph.
      "fused": gq_linear_softcap_peers_sync — the same, with the wait done by the
        GEMV's last CTA itself (one launch instead of two).
      "nccl": gq_linear_softcap_peers then a 1-element NCCL all-reduce on the same
        stream: when it finishes on a rank, every rank's GEMV (and its
        system-fenced peer stores) finished before it.
    The data never goes through NCCL. forward returns a torch view [M, V] of this
    rank's buffer, valid until the call after the next one."""

    def __init__(self, backend, shard, vocab: int, rank: int, world: int, max_m: int, cap: float = 30.0, group=None,
                 barrier: str = "device"):
        import ctypes
        from ctypes import c_uint8, c_void_p

        import torch
        import torch.distributed as dist

        from . import _abi

        if barrier not in ("device", "fused", "nccl"):
            raise ValueError(f"barrier must be 'device', 'fused' or 'nccl', not {barrier!r}")
        self.torch, self.dist, self.g, self.barrier = torch, dist, backend, barrier
        self.rank, self.world, self.vocab, self.cap, self.group, self.max_m = rank, world, vocab, cap, group, max_m
        self.r0, self.r1 = shard_rows(vocab, world, rank)
        assert shard.shape[0] == self.r1 - self.r0
        self.w = shard if getattr(shard, "qw", None) is not None else backend.quant_tensor(shard)
        lib, ctx = backend.lib, backend.ctx
        self.buf_floats = max_m * vocab
        # [2 logits buffers][flags: world u32, padded to 256 B]; the {CTA counter, epoch} pair is local
        self.flag_off = 2 * self.buf_floats * 4
        nbytes = self.flag_off + 256
        ptr, sync = c_void_p(), c_void_p()
        _abi.check(lib.gq_alloc(ctx, nbytes, ctypes.byref(ptr)), ctx, "alloc logits")
        self.buf = ptr.value
        _abi.check(lib.gq_alloc(ctx, 256, ctypes.byref(sync)), ctx, "alloc sync words")
        self.sync = sync.value
        _abi.check(lib.gq_memset(ctx, c_void_p(self.buf + self.flag_off), 0, 256), ctx, "zero flags")
        _abi.check(lib.gq_memset(ctx, c_void_p(self.sync), 0, 256), ctx, "zero sync words")
        _abi.check(lib.gq_sync(ctx), ctx, "sync")
        handle = (c_uint8 * 64)()
        _abi.check(lib.gq_ipc_get_handle(ctx, c_void_p(self.buf), handle), ctx, "ipc handle")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peers = []
        for r, h in enumerate(handles):
            if r == rank:
                continue
            p = c_void_p()
            _abi.check(lib.gq_ipc_open(ctx, (c_uint8 * 64).from_buffer_copy(h), ctypes.byref(p)), ctx, "ipc open")
            self.peers.append(p.value)
        n = max(1, len(self.peers))
        self.peer_arr = [(c_void_p * n)(*[p + k * self.buf_floats * 4 for p in self.peers]) for k in (0, 1)]
        self.flag_arr = (c_void_p * (1 + len(self.peers)))(
            *[b + self.flag_off for b in [self.buf] + self.peers])
        self.logits = [torch.as_tensor(_DeviceArray(self.buf + k * self.buf_floats * 4, (max_m, vocab)),
                                       device=backend.torch_device) for k in (0, 1)]
        self.calls = 0
        self.flag = torch.zeros(1, device=backend.torch_device)
        self.stream = torch.cuda.ExternalStream(backend.stream_ptr(), device=backend.torch_device) \
            if backend.own_stream else torch.cuda.current_stream(backend.torch_device)
        dist.barrier(group=group)  # every rank's flags are zero before any rank signals

    def forward(self, x):
        """x: GqTensor [M, K] (M <= max_m) -> torch view [M, V], complete on this rank's stream."""
        from ctypes import c_float, c_void_p

        from . import _abi

        m, k = x.shape
        assert m <= self.max_m
        lib, ctx = self.g.lib, self.g.ctx
        self.calls += 1
        par = self.calls & 1
        y = self.buf + par * self.buf_floats * 4
        if self.barrier in ("device", "fused"):
            for label, fn, args in self.device_calls(x.ptr(), m, k, par):
                _abi.check(fn(*args), ctx, label)
        else:
            _abi.check(lib.gq_linear_softcap_peers(ctx, c_void_p(x.ptr()), m, k, c_void_p(self.w.qw),
                                                   c_float(self.cap), c_void_p(y), self.vocab, self.r0,
                                                   self.peer_arr[par], len(self.peers)), ctx, "linear_softcap_peers")
            with self.torch.cuda.stream(self.stream):
                self.dist.all_reduce(self.flag, group=self.group)
        return self.logits[par][:m]

    def device_calls(self, x_ptr: int, m: int, k: int, par: int):
        """The two C-ABI calls of one device-barrier forward into buffer `par` (0 or 1),
        with their arguments bound, as (label, fn, args) for a caller's launch list
        (a captured graph replays them with fresh epochs); the logits are then
        ``self.logits[par][:m]``."""
        from ctypes import c_float, c_void_p

        lib, ctx = self.g.lib, self.g.ctx
        y = self.buf + par * self.buf_floats * 4
        args = (ctx, c_void_p(x_ptr), m, k, c_void_p(self.w.qw), c_float(self.cap), c_void_p(y), self.vocab,
                self.r0, self.peer_arr[par], len(self.peers), self.flag_arr, c_void_p(self.sync), self.rank)
        if self.barrier == "fused":  # one launch: the GEMV's last CTA also waits for every rank
            return [("lm_head_shard", lib.gq_linear_softcap_peers_sync, args)]
        return [("lm_head_shard", lib.gq_linear_softcap_peers_signal, args),
                ("lm_head_wait", lib.gq_peer_wait,
                 (ctx, c_void_p(self.buf + self.flag_off), self.world, c_void_p(self.sync)))]

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank stopped writing)."""
        from ctypes import c_void_p

        self.torch.cuda.synchronize(self.g.torch_device)
        self.g.lib.gq_sync(self.g.ctx)
        self.dist.barrier(group=self.group)
        for p in self.peers:
            self.g.lib.gq_ipc_close(self.g.ctx, c_void_p(p))
        self.peers = []
        self.dist.barrier(group=self.group)
        for attr in ("buf", "sync"):
            if getattr(self, attr):
                self.g.lib.gq_free(self.g.ctx, c_void_p(getattr(self, attr)))
                setattr(self, attr, 0)


def argmax_key(val, idx):
    """Order of (value, index) candidates for a row argmax: larger value first, NaN
    above every number, -0 equal to +0, and among equal values the smaller index
    (numpy.argmax semantics). Returns uint64 keys (numpy)."""
    v = np.asarray(val, dtype=np.float32)
    v = np.where(v == 0.0, np.float32(0.0), v)
    u = v.view(np.uint32).astype(np.uint64)
    order = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    order = np.where(np.isnan(v), np.uint64(0xFFFFFFFF), order)
    return (order << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(idx, dtype=np.uint64))


def merge_argmax(vals, idxs):
    """Per row, the best of G shards' (value, global index) candidates: vals, idxs
    [G, M] -> (val [M], idx [M]); equals numpy.argmax over the concatenated shards
    when each shard's candidate is its own first maximum."""
    vals = np.asarray(vals, dtype=np.float32)
    idxs = np.asarray(idxs, dtype=np.int64)
    best = np.argmax(argmax_key(vals, idxs), axis=0)
    cols = np.arange(vals.shape[1])
    return vals[best, cols], idxs[best, cols]


class ShardedGreedy:
    """Greedy decoding over a vocab-sharded lm_head: each rank computes its
    shard's soft-capped logits, reduces every row to (max, first index) on the GPU
    (gq_argmax_rows) and all-gathers those pairs (M * 12 bytes per rank instead
    of its M * V/G logits). forward(x) returns the token ids [M] (and values) of
    the full vocabulary's argmax on every rank."""

    def __init__(self, backend, shard, vocab: int, rank: int, world: int, max_m: int, cap: float = 30.0,
                 group=None):
        import torch
        import torch.distributed as dist

        self.torch, self.dist, self.g = torch, dist, backend
        self.rank, self.world, self.vocab, self.cap, self.group = rank, world, vocab, cap, group
        self.r0, self.r1 = shard_rows(vocab, world, rank)
        self.per = self.r1 - self.r0
        assert shard.shape[0] == self.per
        self.w = shard if getattr(shard, "qw", None) is not None else backend.quant_tensor(shard)
        dev = backend.torch_device
        self.logits = torch.empty(max_m, max(1, self.per), device=dev)
        self.val = torch.empty(max_m, device=dev)
        self.idx = torch.empty(max_m, dtype=torch.int64, device=dev)
        self.max_m = max_m

    def forward(self, x):
        from ctypes import c_float, c_void_p

        from . import _abi

        m, k = x.shape
        assert m <= self.max_m
        lib, ctx = self.g.lib, self.g.ctx
        torch, dist = self.torch, self.dist
        if self.per > 0:
            _abi.check(lib.gq_linear_softcap(ctx, c_void_p(x.ptr()), m, k, c_void_p(self.w.qw), c_float(self.cap),
                                             c_void_p(self.logits.data_ptr()), self.per, 0), ctx, "shard logits")
            _abi.check(lib.gq_argmax_rows(ctx, c_void_p(self.logits.data_ptr()), m, self.per, self.per, self.r0,
                                          c_void_p(self.val.data_ptr()), c_void_p(self.idx.data_ptr())), ctx,
                       "argmax_rows")
        else:  # an empty shard offers no candidate
            self.val[:m].fill_(float("-inf"))
            self.idx[:m].fill_(self.vocab)
        self.g.flush()
        vals = torch.empty(self.world * m, device=self.val.device)
        idxs = torch.empty(self.world * m, dtype=torch.int64, device=self.idx.device)
        dist.all_gather_into_tensor(vals, self.val[:m].contiguous(), group=self.group)
        dist.all_gather_into_tensor(idxs, self.idx[:m].contiguous(), group=self.group)
        return merge_argmax(vals.cpu().numpy().reshape(self.world, m), idxs.cpu().numpy().reshape(self.world, m))


class ShardedSampler:
    """Sampling over a vocab-sharded lm_head with the per-shard top-k exchange: each
    rank computes its shard's soft-capped logits, keeps every row's k best (value,
    id) pairs after the repetition penalty (gq_topk_rows, ids offset by the shard's
    first row), all-gathers the G*k pairs per row (G*k*12 bytes instead of its M*V/G
    logits), and samples them on the device (gq_sample_candidates) with a splitmix64
    state per row that every rank advances identically, so every rank draws the same
    token. Greedy (temperature <= 0) and top-k (+ top-p) options, as the reference's
    sample() (rust/src/sampler.rs:116-190); the union of the shards' top k holds the
    vocabulary's top k, so the result equals sampling the whole row."""

    def __init__(self, backend, shard, vocab: int, rank: int, world: int, max_m: int, opts, seeds, cap: float = 30.0,
                 group=None):
        import torch
        import torch.distributed as dist

        from . import _abi

        if opts.temperature > 0 and opts.top_k == 0:
            raise ValueError("ShardedSampler: top_k > 0 (or greedy) is needed for the per-shard exchange")
        self.torch, self.dist, self.g, self.opts = torch, dist, backend, opts
        self.rank, self.world, self.vocab, self.cap, self.group = rank, world, vocab, cap, group
        self.r0, self.r1 = shard_rows(vocab, world, rank)
        self.per = self.r1 - self.r0
        assert shard.shape[0] == self.per
        self.w = shard if getattr(shard, "qw", None) is not None else backend.quant_tensor(shard)
        self.k = max(1, int(opts.top_k)) if opts.temperature > 0 else 1
        dev = backend.torch_device
        self.max_m = max_m
        self.logits = torch.empty(max_m, max(1, self.per), device=dev)
        self.val = torch.empty(max_m, self.k, device=dev)
        self.idx = torch.empty(max_m, self.k, dtype=torch.int64, device=dev)
        seeds = np.asarray(seeds, dtype=np.uint64).reshape(-1)
        assert seeds.size >= max_m
        self.state = torch.from_numpy(seeds[:max_m].view(np.int64).copy()).to(dev)
        self.tokens = torch.empty(max_m, dtype=torch.int32, device=dev)
        self._abi = _abi

    def forward(self, x, recent=None):
        """x: GqTensor [M, K]; recent: optional device int32 [M, R] history (ids of the
        whole vocabulary). Returns the token ids [M] (numpy), the same on every rank."""
        import ctypes
        from ctypes import c_float, c_void_p

        _abi = self._abi
        m, k = x.shape
        assert m <= self.max_m
        lib, ctx = self.g.lib, self.g.ctx
        torch, dist = self.torch, self.dist
        n_rec = 0 if recent is None else int(recent.shape[1])
        rec_p = None if recent is None else c_void_p(recent.data_ptr())
        if self.per > 0:
            _abi.check(lib.gq_linear_softcap(ctx, c_void_p(x.ptr()), m, k, c_void_p(self.w.qw), c_float(self.cap),
                                             c_void_p(self.logits.data_ptr()), self.per, 0), ctx, "shard logits")
            _abi.check(lib.gq_topk_rows(ctx, c_void_p(self.logits.data_ptr()), m, self.per, self.per, self.r0, self.k,
                                        c_float(self.opts.repetition_penalty), rec_p, n_rec, n_rec,
                                        c_void_p(self.val.data_ptr()), c_void_p(self.idx.data_ptr())), ctx, "topk_rows")
        else:  # an empty shard offers no candidate
            self.val[:m].fill_(float("-inf"))
            self.idx[:m].fill_(-1)
        self.g.flush()
        vals = torch.empty(self.world, m, self.k, device=self.val.device)
        idxs = torch.empty(self.world, m, self.k, dtype=torch.int64, device=self.idx.device)
        dist.all_gather_into_tensor(vals, self.val[:m].contiguous(), group=self.group)
        dist.all_gather_into_tensor(idxs, self.idx[:m].contiguous(), group=self.group)
        cv = vals.permute(1, 0, 2).reshape(m, self.world * self.k).contiguous()  # [M][rank][k]
        ci = idxs.permute(1, 0, 2).reshape(m, self.world * self.k).contiguous()
        _abi.check(lib.gq_sample_candidates(ctx, c_void_p(cv.data_ptr()), c_void_p(ci.data_ptr()), m,
                                            self.world * self.k, ctypes.byref(self.opts),
                                            c_void_p(self.state.data_ptr()), c_void_p(self.tokens.data_ptr())),
                   ctx, "sample_candidates")
        self.g.flush()
        return self.tokens[:m].cpu().numpy().copy()
