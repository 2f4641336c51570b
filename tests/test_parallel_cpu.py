"""Host logic of the vocab-sharded lm_head on CPU: 2 gloo ranks, the oracle as
the per-shard compute, gathered and reassembled logits equal to the
single-device lm_head (bit for bit: the split is by output row, so each row's
arithmetic is unchanged). Also: a rank that never joins makes the collective
fail with a timeout error instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gq import parallel, synth


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, vocab, m, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "gemma-4-webgpu-kernels_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle import oracle
    from gq import parallel as par, synth as syn

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = syn.make_qweight(5, vocab, 64, 8, True)
        x = syn.normal(6, m * 64).reshape(m, 64)
        r0, r1 = par.shard_rows(vocab, world, rank)
        per = -(-vocab // world)
        local = np.zeros((m, per), np.float32)
        if r1 > r0:
            local[:, : r1 - r0] = oracle.softcap(oracle.linear(x, par.slice_rows(full, r0, r1)), 30.0)
        out = torch.empty(world * m * per)
        dist.all_gather_into_tensor(out, torch.from_numpy(local.ravel().copy()))
        logits = par.assemble(out, m, world, per, vocab).numpy()
        ref = oracle.softcap(oracle.linear(x, full), 30.0)
        q.put((rank, bool(np.array_equal(logits, ref))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("vocab,m", [(1000, 1), (1003, 3)])
def test_sharded_lm_head_gloo(vocab, m):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, vocab, m, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert res == {0: True, 1: True}


def test_shard_rows_cover_vocab():
    for vocab, world in [(262144, 8), (262144, 3), (10, 4), (3, 8)]:
        spans = [parallel.shard_rows(vocab, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == vocab
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_slice_rows_matches_codes():
    q = synth.make_qweight(9, 40, 64, 4)
    s = parallel.slice_rows(q, 10, 25)
    assert np.array_equal(s.codes(), q.codes()[10:25])
    assert np.array_equal(s.scales, q.scales[10:25])


def _lonely(port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=timedelta(seconds=3))
        q.put("joined")
    except Exception as e:  # the peer never joins: rendezvous times out
        q.put(type(e).__name__)


def test_missing_rank_times_out():
    """Failure detection on the host: the second rank never joins; the first gets
    an error from the short process-group timeout instead of waiting forever."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), q))
    p.start()
    p.join(timeout=60)
    assert p.exitcode == 0
    assert q.get(timeout=5) != "joined"
