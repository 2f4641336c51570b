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


def _greedy_worker(rank, world, port, vocab, m, q):
    """Each rank's shard candidate = its own first maximum (the semantics of
    gq_argmax_rows, computed here by numpy on the oracle's logits), gathered
    over gloo and merged."""
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
        full = syn.make_qweight(15, vocab, 64, 8, True)
        x = syn.normal(16, m * 64).reshape(m, 64)
        r0, r1 = par.shard_rows(vocab, world, rank)
        logits = oracle.softcap(oracle.linear(x, par.slice_rows(full, r0, r1)), 30.0).reshape(m, r1 - r0)
        a = np.argmax(logits, axis=1)
        vals = torch.empty(world * m)
        idxs = torch.empty(world * m, dtype=torch.int64)
        dist.all_gather_into_tensor(vals, torch.from_numpy(logits[np.arange(m), a].astype(np.float32)))
        dist.all_gather_into_tensor(idxs, torch.from_numpy((a + r0).astype(np.int64)))
        _, idx = par.merge_argmax(vals.numpy().reshape(world, m), idxs.numpy().reshape(world, m))
        ref = np.argmax(oracle.softcap(oracle.linear(x, full), 30.0).reshape(m, vocab), axis=1)
        q.put((rank, bool(np.array_equal(idx, ref))))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("vocab,m", [(1000, 1), (1003, 4)])
def test_sharded_greedy_gloo(vocab, m):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_greedy_worker, args=(r, world, port, vocab, m, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert all(v is True for v in res.values()), res


def test_merge_argmax_is_numpy_argmax():
    """Shard candidates merged in rank order give numpy.argmax of the whole row,
    with ties across shards, NaN and signed zeros."""
    rng = np.random.default_rng(1)
    for trial in range(300):
        g, per, m = int(rng.integers(1, 5)), int(rng.integers(1, 7)), 3
        full = rng.integers(-3, 4, (m, g * per)).astype(np.float32)
        if trial % 7 == 0:
            full[0, rng.integers(0, g * per)] = np.nan
        if trial % 5 == 0:
            full[1, :] = -0.0
            full[1, rng.integers(0, g * per)] = 0.0
        vals, idxs = [], []
        for gi in range(g):
            sh = full[:, gi * per:(gi + 1) * per]
            a = np.argmax(sh, axis=1)
            vals.append(sh[np.arange(m), a])
            idxs.append(a + gi * per)
        _, idx = parallel.merge_argmax(vals, idxs)
        assert np.array_equal(idx, np.argmax(full, axis=1)), trial
