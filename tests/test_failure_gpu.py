"""Failure detection on one GPU without faulting it (needs a B200).

The cross-GPU completion wait of the vocab-sharded lm_head (gq_peer_wait) is the
failure detector of a multi-GPU step: when a peer rank dies or stalls, its flags
never reach the epoch, and the wait must end with an error status instead of
holding the GPU. Here the peer is simulated by a flag array that nothing ever
sets: the wait runs out after the context's wait limit (set to 50 ms), the next
gq_sync returns GQ_ERR_DEVICE naming the timeout, and the context stays usable
(the error word is cleared; a linear call afterwards matches the oracle). No
kernel traps, asserts or spins without a bound.
"""
import ctypes
import time
from ctypes import c_void_p

import numpy as np
import pytest

from gq import CudaBackend, _abi, synth
from numerics import rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    be = CudaBackend(0)
    yield be
    be.close()


def test_peer_wait_times_out_and_context_survives(g):
    torch = g._torch
    lib, ctx = g.lib, g.ctx
    assert lib.gq_ctx_set_wait_limit(ctx, 50_000_000) == _abi.GQ_OK
    world = 2
    flags = torch.zeros(world, dtype=torch.int32, device=g.torch_device)  # no rank ever signals
    sync = torch.tensor([0, 5], dtype=torch.int32, device=g.torch_device)  # {CTA counter, epoch 5}
    g.flush()
    t0 = time.perf_counter()
    assert lib.gq_peer_wait(ctx, c_void_p(flags.data_ptr()), world, c_void_p(sync.data_ptr())) == _abi.GQ_OK
    rc = lib.gq_sync(ctx)
    elapsed = time.perf_counter() - t0
    assert rc == _abi.GQ_ERR_DEVICE
    assert b"wait timed out" in lib.gq_last_error(ctx)
    assert 0.045 <= elapsed < 5.0, elapsed
    # the error word was cleared and the context still runs work
    assert lib.gq_sync(ctx) == _abi.GQ_OK
    w = synth.make_qweight(9101, 512, 1536, 4)
    x = synth.normal(9102, 1536).reshape(1, 1536)
    got = g.readback(g.linear(g.tensor(x, x.shape), g.quant_tensor(w)))
    assert rel_l2(got, oracle.linear(x, w)) <= 1e-5
    # a wait whose flags have reached the epoch passes without an error
    flags.fill_(5)
    g.flush()
    t0 = time.perf_counter()
    assert lib.gq_peer_wait(ctx, c_void_p(flags.data_ptr()), world, c_void_p(sync.data_ptr())) == _abi.GQ_OK
    assert lib.gq_sync(ctx) == _abi.GQ_OK
    assert time.perf_counter() - t0 < 0.045
    assert lib.gq_ctx_set_wait_limit(ctx, 2_000_000_000) == _abi.GQ_OK


def test_wait_limit_range_is_checked(g):
    lib, ctx = g.lib, g.ctx
    assert lib.gq_ctx_set_wait_limit(ctx, 0) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_ctx_set_wait_limit(ctx, 61_000_000_000) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_ctx_set_wait_limit(None, 50_000_000) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_ctx_set_wait_limit(ctx, 2_000_000_000) == _abi.GQ_OK
