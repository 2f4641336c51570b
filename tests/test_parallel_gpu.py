"""The vocab-sharded lm_head on 2 GPUs (needs two B200s; skipped with fewer).

Both exchanges against the single-device oracle and against each other: the
NCCL all-gather (ShardedLmHead) and the fused GEMV + peer stores over NVLink
(PeerLmHead, gq_linear_softcap_peers), the latter with either completion barrier
(NCCL all-reduce, or the GEMV's own epoch flags and gq_peer_wait). Each rank computes the same kernels on the
same shard bytes, so the two full logits tensors must be identical; against the
oracle the FFMA bound applies (relative L2 <= 1e-5)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V, K, CAP = 20000, 1536, 30.0


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from gq import CudaBackend, synth
        from gq.parallel import PeerLmHead, ShardedLmHead, shard_rows, slice_rows
        from oracle import oracle

        full = synth.random_qweight(4100, V, K, 8, True)
        r0, r1 = shard_rows(V, world, rank)
        shard = slice_rows(full, r0, r1)
        g = CudaBackend(rank)
        res = {}
        for m in (1, 5, 40):
            x = synth.normal(4101 + m, m * K).reshape(m, K).astype(np.float32)
            gx = g.tensor(x, x.shape)
            nccl = ShardedLmHead(g, shard, V, rank, world, CAP).forward(gx).cpu().numpy()
            ref = oracle.softcap(oracle.linear(x, full), CAP)
            for barrier in ("nccl", "device", "fused"):
                peer = PeerLmHead(g, shard, V, rank, world, max_m=m, cap=CAP, barrier=barrier)
                got = peer.forward(gx).cpu().numpy().copy()
                # later calls alternate buffers and epochs
                again = [peer.forward(gx).cpu().numpy().copy() for _ in range(3)]
                g.flush()
                peer.close()
                rel = float(np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref))
                res[(m, barrier)] = (rel, bool(np.array_equal(got, nccl)),
                                     all(np.array_equal(got, a) for a in again))
        # the device barriers replayed from a CUDA graph (device-resident epochs)
        gg = CudaBackend(rank, own_stream=True)
        x = synth.normal(4199, 3 * K).reshape(3, K).astype(np.float32)
        gx = gg.tensor(x, x.shape)
        ref = oracle.softcap(oracle.linear(x, full), CAP)
        for barrier in ("device", "fused"):
            peer = PeerLmHead(gg, shard, V, rank, world, max_m=3, cap=CAP, barrier=barrier)
            outs = []
            graph = gg.record(lambda: outs.extend([peer.forward(gx), peer.forward(gx)]))
            reps = []
            for _ in range(3):
                gg.replay(graph)
                gg.flush()
                reps.append([o.cpu().numpy().copy() for o in outs])
            gg.destroy_graph(graph)
            peer.close()
            rel = float(np.linalg.norm(reps[0][0].astype(np.float64) - ref) / np.linalg.norm(ref))
            res[("graph", barrier)] = (rel, True, all(np.array_equal(reps[0][0], o) for r in reps for o in r))
        gg.close()
        g.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_sharded_lm_head_two_gpus_both_exchanges():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    for rank, res in out.items():
        assert isinstance(res, dict), f"rank {rank}: {res}"
        for m, (rel, same_as_nccl, repeatable) in res.items():
            assert rel <= 1e-5, (rank, m, rel)
            assert same_as_nccl and repeatable, (rank, m)


def _decoder_worker(rank, world, port, q):
    """The decode step with its lm_head sharded over the ranks (fused exchange,
    device barrier) against the same step with the whole lm_head on one GPU."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from gq import CudaBackend, e2b

        c = e2b.small_config(2000)
        w = e2b.Weights(c, 21)
        ids = [5, 1999, 777]
        g = CudaBackend(rank, own_stream=True)
        full = e2b.Decoder(g, c, w, batch=3, cache_len=20, capacity=24)
        full.set_ids(ids)
        full.run()
        g.flush()
        want = full.read(full.logits)
        full.close()
        dec = e2b.Decoder(g, c, w, batch=3, cache_len=20, capacity=24, lm_shard=(rank, world, None))
        dec.set_ids(ids)
        g.flush()
        dist.barrier()  # the step's exchange waits are bounded: start the ranks together
        dec.run()
        g.flush()
        eager = dec.read(dec.logits)
        graph = dec.record()  # two steps, one per logits buffer
        outs = []
        for _ in range(2):
            g.replay(graph)
            g.flush()
            outs.append(dec.read(dec.logits))
        g.destroy_graph(graph)
        spg = dec.steps_per_graph
        dec.close()
        g.close()
        rel = float(np.linalg.norm(eager.astype(np.float64) - want) / np.linalg.norm(want))
        same = all(np.array_equal(o, eager) for o in outs)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, (rel, same, spg)))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_decode_step_with_sharded_lm_head_two_gpus():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_decoder_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    for rank, res in out.items():
        assert isinstance(res, tuple), f"rank {rank}: {res}"
        rel, same, spg = res
        assert rel <= 1e-5, (rank, rel)
        assert same and spg == 2, rank


def _greedy_worker(rank, world, port, q):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from gq import CudaBackend, synth
        from gq.parallel import ShardedGreedy, shard_rows, slice_rows
        from oracle import oracle

        full = synth.random_qweight(4200, V, K, 8, True)
        r0, r1 = shard_rows(V, world, rank)
        g = CudaBackend(rank)
        sg = ShardedGreedy(g, slice_rows(full, r0, r1), V, rank, world, max_m=5, cap=CAP)
        x = synth.normal(4201, 5 * K).reshape(5, K).astype(np.float32)
        _, idx = sg.forward(g.tensor(x, x.shape))
        ref = oracle.softcap(oracle.linear(x, full), CAP).reshape(5, V)
        g.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, (idx.tolist(), np.argmax(ref, axis=1).tolist())))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_sharded_greedy_two_gpus():
    """Greedy decoding with the vocab split over 2 GPUs: each shard's (max, first
    index) on the GPU, pairs all-gathered, merged: the token ids of the oracle's
    argmax over the full logits (the GEMV is within 1e-5 of the oracle, so this
    holds unless a row's two largest logits lie within that rounding)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_greedy_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    for rank, res in out.items():
        assert isinstance(res, tuple), f"rank {rank}: {res}"
        assert res[0] == res[1], rank


def _sampler_worker(rank, world, port, q):
    from ctypes import byref, c_float, c_void_p
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from gq import CudaBackend, _abi, synth
        from gq.parallel import ShardedSampler, shard_rows, slice_rows

        full = synth.random_qweight(4300, V, K, 8, True)
        r0, r1 = shard_rows(V, world, rank)
        g = CudaBackend(rank)
        m = 4
        x = (3.0 * synth.normal(4301, m * K)).reshape(m, K).astype(np.float32)
        gx = g.tensor(x, x.shape)
        seeds = [int(s) for s in synth.splitmix64(4302, m)]
        recent = torch.from_numpy(np.array([[1, 2, 2, V + 9]] * m, dtype=np.int32)).to(g.torch_device)
        res = {}
        for name, o in (("greedy", _abi.SampleOpts(0.0, 0, 1.0, 1.3)),
                        ("top_k64_top_p", _abi.SampleOpts(1.0, 64, 0.95, 1.3)),
                        ("top_k8", _abi.SampleOpts(0.7, 8, 1.0, 1.0))):
            ss = ShardedSampler(g, slice_rows(full, r0, r1), V, rank, world, max_m=m, opts=o, seeds=seeds, cap=CAP)
            got = ss.forward(gx, recent=recent)
            # the same draws on the whole row, on this GPU
            wq = g.quant_tensor(full)
            logits = torch.empty(m, V, device=g.torch_device)
            g._check(g.lib.gq_linear_softcap(g.ctx, c_void_p(gx.ptr()), m, K, c_void_p(wq.qw), c_float(CAP),
                                             c_void_p(logits.data_ptr()), V, 0), "full logits")
            st = torch.from_numpy(np.array(seeds, dtype=np.uint64).view(np.int64)).to(g.torch_device)
            tok = torch.empty(m, dtype=torch.int32, device=g.torch_device)
            g._check(g.lib.gq_sample_rows(g.ctx, c_void_p(logits.data_ptr()), m, V, 0, byref(o),
                                          c_void_p(recent.data_ptr()), recent.shape[1], recent.shape[1],
                                          c_void_p(st.data_ptr()), c_void_p(tok.data_ptr())), "sample_rows")
            g.flush()
            res[name] = (got.tolist(), tok.cpu().numpy().tolist(), ss.state.cpu().numpy().tolist(),
                         st.cpu().numpy().tolist())
            g.free_quant(wq)
        g.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_sharded_sampler_two_gpus():
    """Sampling with the vocab split over 2 GPUs through the per-shard top-k exchange
    (gq_topk_rows with the penalty, all-gather of the pairs, gq_sample_candidates):
    every rank draws the token gq_sample_rows draws on the whole row with the same
    seeds, and advances the states the same way, for greedy and top-k (+ top-p)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_sampler_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    for rank, res in out.items():
        assert isinstance(res, dict), f"rank {rank}: {res}"
        for name, (got, want, st, want_st) in res.items():
            assert got == want and st == want_st, (rank, name)
    assert out[0] == out[1]
