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
