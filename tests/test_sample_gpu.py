"""On-device sampling (gq_sample_rows, gq_topk_rows, gq_sample_candidates) against the
CPU restatement of the reference's sampler (rust/src/sampler.rs:116-190), needs a B200.

Draws: both sides use the reference's Rng (splitmix64, sampler.rs:5-27) from the same
seed; the device advances one state per row and the test checks the advanced state.
Token ids must match exactly, except for a draw that lands within rounding of a
boundary between two tokens (the oracle picks different tokens for u - d and u + d):
the device sums a whole row in chunks and its expf may differ from libm's in the last
place, so such draws are not decided by the arithmetic contract and are skipped (and
counted, and kept rare).
"""
import ctypes
from ctypes import c_void_p

import numpy as np
import pytest

from gq import CudaBackend, _abi, synth
from oracle import oracle

pytestmark = pytest.mark.gpu

V = 262144


@pytest.fixture(scope="module")
def g():
    be = CudaBackend(0)
    yield be
    be.close()


def opts(temperature=1.0, top_k=0, top_p=1.0, penalty=1.0):
    return _abi.SampleOpts(temperature, top_k, top_p, penalty)


def dev(g, a, dtype):
    return g._torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).to(g.torch_device)


def sample_rows(g, logits, o, seeds, recent=None, vocab=None):
    """logits [m, ld]; the first `vocab` columns of each row are the row (ld = the
    array's width)."""
    torch = g._torch
    m, ld = logits.shape
    vocab = vocab or ld
    lg = dev(g, logits, np.float32)
    st = dev(g, np.array(seeds, dtype=np.uint64).view(np.int64), np.int64)
    tok = torch.full((m,), -7, dtype=torch.int32, device=g.torch_device)
    rec = None
    n_rec = 0
    if recent is not None:
        rec = dev(g, np.asarray(recent, dtype=np.uint32).view(np.int32), np.int32)
        n_rec = recent.shape[1]
    rc = g.lib.gq_sample_rows(g.ctx, c_void_p(lg.data_ptr()), m, vocab, ld, ctypes.byref(o),
                              c_void_p(rec.data_ptr()) if rec is not None else None, n_rec, n_rec,
                              c_void_p(st.data_ptr()), c_void_p(tok.data_ptr()))
    assert rc == _abi.GQ_OK, g.lib.gq_last_error(g.ctx)
    sync = g.lib.gq_sync(g.ctx)
    return tok.cpu().numpy(), st.cpu().numpy().view(np.uint64), sync


def penalized(row, penalty, recent):
    """The repetition penalty of rust/src/sampler.rs:120-133 on a copy (f32)."""
    l = np.array(row, dtype=np.float32).copy()
    if penalty != 1.0 and recent is not None:
        seen = set()
        for t in np.asarray(recent).ravel():
            t = int(t)
            if t < l.size and t not in seen:
                seen.add(t)
                l[t] = l[t] / np.float32(penalty) if l[t] > 0 else l[t] * np.float32(penalty)
    return l


def check_sample_all(row, o, seed, tok, state, recent=None, eps=2e-5):
    """sample_all (rust/src/sampler.rs:58-69) sums the whole row: the device's chunked
    sums round differently from the reference's sequential f32 sum, so the check is
    that the draw falls inside the token's interval of the float64 CDF (index order),
    widened by eps; and the state advanced by one draw."""
    u, st = oracle.rng_next_f64(seed)
    assert state == st
    l = penalized(row, o.repetition_penalty, recent).astype(np.float64)
    w = np.exp((l - l.max()) / np.float64(o.temperature))
    cdf = np.cumsum(w) / w.sum()
    lo = cdf[tok - 1] if tok > 0 else 0.0
    assert lo - eps <= u <= cdf[tok] + eps, (tok, u, lo, cdf[tok])
    return 1


def check_row(row, o, seed, tok, state, recent=None, delta=1e-6):
    """1 when the token is decided by the draw (and must match), 0 when skipped."""
    if o.temperature <= 0:
        want = oracle.sample(row, o.temperature, o.top_k, o.top_p, o.repetition_penalty, recent, 0.0)
        assert tok == want
        assert state == seed  # greedy rows draw nothing
        return 1
    if o.top_k == 0 and o.top_p >= 1.0:
        return check_sample_all(row, o, seed, tok, state, recent)
    u, st = oracle.rng_next_f64(seed)
    assert state == st
    want = oracle.sample(row, o.temperature, o.top_k, o.top_p, o.repetition_penalty, recent, u)
    lo = oracle.sample(row, o.temperature, o.top_k, o.top_p, o.repetition_penalty, recent, max(0.0, u - delta))
    hi = oracle.sample(row, o.temperature, o.top_k, o.top_p, o.repetition_penalty, recent, min(1 - 1e-12, u + delta))
    if lo != hi:
        return 0
    assert tok == want, (tok, want, u)
    return 1


def test_reference_sampler_cases(g):
    """rust/tests/model.rs:77-101, through the device sampler."""
    tok, _, _ = sample_rows(g, np.array([[0.1, 5.0, 0.2, -1.0]]), opts(temperature=0.0), [9])
    assert tok[0] == 1  # greedy picks argmax
    tok, _, _ = sample_rows(g, np.array([[0.0, 10.0, 9.0, -5.0]]), opts(top_k=1), [9])
    assert tok[0] == 1  # top-k = 1 is the argmax
    tok, _, _ = sample_rows(g, np.array([[10.0, 4.0]]), opts(temperature=0.0, penalty=2.0), [9],
                            recent=np.array([[0, 0]]))
    assert tok[0] == 0  # the penalty applies once per distinct token
    tok, _, _ = sample_rows(g, np.array([[0.0, 10.0, 9.9, -5.0]]), opts(top_p=0.5), [9])
    assert tok[0] == 1  # top-p keeps only the head
    row = np.array([np.float32(np.sin(np.float32(i) * np.float32(0.37))) for i in range(100)], dtype=np.float32)
    d = opts(temperature=1.0, top_k=64, top_p=0.95)  # SampleOpts::default of the engine (rust/src/engine.rs:47)
    t1, s1, _ = sample_rows(g, row[None, :], d, [1])
    t2, s2, _ = sample_rows(g, row[None, :], d, [1])
    assert t1[0] == t2[0] and s1[0] == s2[0] and 0 <= t1[0] < 100
    assert check_row(row, d, 1, int(t1[0]), int(s1[0])) == 1


MODES = {
    "greedy": opts(temperature=0.0),
    "engine_default": opts(temperature=1.0, top_k=64, top_p=0.95),
    "top_k_40": opts(temperature=0.8, top_k=40),
    "top_k_256_top_p": opts(temperature=1.3, top_k=256, top_p=0.6),
    "sample_all": opts(temperature=1.0),
    "sample_all_cold": opts(temperature=0.5),
}


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("penalty", [1.0, 1.3])
def test_sample_rows_against_oracle(g, mode, penalty):
    o = MODES[mode]
    o = opts(o.temperature, o.top_k, o.top_p, penalty)
    m = 6
    rng = np.random.default_rng(11 + int(penalty * 10))
    logits = (rng.standard_normal((m, V)) * 2.5).astype(np.float32)
    logits[:, rng.integers(0, V, 40)] += 9.0  # a head of likely tokens
    recent = rng.integers(0, V, (m, 24)).astype(np.uint32)
    recent[:, 1] = recent[:, 0]                    # a repeat: penalised once
    recent[:, 2] = V + 5                           # an id past the vocabulary: ignored
    recent[:, 3] = np.argmax(logits, axis=1)       # the leader is penalised
    seeds = [int(s) for s in synth.splitmix64(404 + len(mode), m)]
    tok, st, sync = sample_rows(g, logits, o, seeds, recent=recent if penalty != 1.0 else None)
    assert sync == _abi.GQ_OK
    decided = 0
    for r in range(m):
        decided += check_row(logits[r], o, seeds[r], int(tok[r]), int(st[r]),
                             recent=recent[r] if penalty != 1.0 else None,
                             delta=1e-4 if o.top_k == 0 else 1e-6)
    assert decided >= m - 1


def test_top_p_only_nucleus_and_its_cap(g):
    """top_k = 0 with top_p < 1: a peaked row whose nucleus fits the device's 256
    candidates matches the oracle (which sorts the whole row); a flat row's nucleus
    does not, and is reported (-1 and GQ_DEVERR_SAMPLE_CAP at the sync)."""
    rng = np.random.default_rng(5)
    peaked = (rng.standard_normal((2, V))).astype(np.float32)
    peaked[:, :30] += 14.0
    o = opts(temperature=1.0, top_p=0.9)
    seeds = [77, 78]
    tok, st, sync = sample_rows(g, peaked, o, seeds)
    assert sync == _abi.GQ_OK
    for r in range(2):
        assert check_row(peaked[r], o, seeds[r], int(tok[r]), int(st[r]), delta=1e-4) in (0, 1)
    flat = (rng.standard_normal((1, V)) * 0.1).astype(np.float32)
    tok, st, sync = sample_rows(g, flat, o, [79])
    assert tok[0] == -1 and sync == _abi.GQ_ERR_DEVICE
    assert b"nucleus" in g.lib.gq_last_error(g.ctx)
    assert g.lib.gq_sync(g.ctx) == _abi.GQ_OK


def test_small_vocab_strided_rows_and_ties(g):
    """A vocabulary smaller than top_k and a row stride wider than the vocabulary
    (the padding columns are never read); greedy over exact ties and a NaN (the first
    of the tied maxima, NaN never wins: the reference's strict `x > best`)."""
    n, ld = 10, 16
    rows = np.full((3, ld), 123.0, dtype=np.float32)
    rows[:, :n] = [[1, 3, 3, 0, -2, np.nan, 3, -1, 0.5, 2]] * 3
    tok, _, _ = sample_rows(g, rows, opts(temperature=0.0), [1, 2, 3], vocab=n)
    assert list(tok) == [1, 1, 1]
    rng = np.random.default_rng(3)
    rows[:, :n] = rng.standard_normal((3, n)).astype(np.float32)
    o = opts(temperature=1.0, top_k=64)
    seeds = [5, 6, 7]
    tok, st, _ = sample_rows(g, rows, o, seeds, vocab=n)
    for r in range(3):
        assert 0 <= tok[r] < n
        assert check_row(rows[r, :n], o, seeds[r], int(tok[r]), int(st[r])) in (0, 1)


@pytest.mark.parametrize("top_k", [1, 7, 64, 256])
def test_top_k_over_heavy_ties(g, top_k):
    """Logits on a few levels, so thousands of columns tie across chunks. The merged
    candidate list (radix select of the chunks' candidates, then a sort of the
    selected) holds the same candidates as the reference (among equal values, the
    first columns: its size-k heap admits only larger values once full) in column
    order; the reference lists equal candidates in its heap's internal order, so a
    draw may land on a different one of several EQUAL-probability candidates. The
    check: the state advanced as the oracle's, the token is one of the oracle's
    candidates and carries the value the oracle's token has; and the sorted top-k
    pairs of gq_topk_rows match numpy's stable order exactly."""
    rng = np.random.default_rng(44)
    m = 3
    logits = (rng.integers(0, 6, (m, V)) * 0.5).astype(np.float32)
    logits[1, 100000:100300] = 3.0  # a block of tied maxima inside one chunk
    o = opts(temperature=0.8, top_k=top_k, top_p=0.9)
    seeds = [11, 12, 13]
    tok, st, _ = sample_rows(g, logits, o, seeds)
    for r in range(m):
        u, want_st = oracle.rng_next_f64(seeds[r])
        assert int(st[r]) == want_st
        want = oracle.sample(logits[r], o.temperature, o.top_k, o.top_p, 1.0, None, u)
        cands = np.argsort(-logits[r], kind="stable")[:top_k]
        assert int(tok[r]) in set(cands.tolist())
        assert logits[r][int(tok[r])] == logits[r][want]
    torch = g._torch
    lg = dev(g, logits, np.float32)
    val = torch.empty(m, top_k, dtype=torch.float32, device=g.torch_device)
    idx = torch.empty(m, top_k, dtype=torch.int64, device=g.torch_device)
    rc = g.lib.gq_topk_rows(g.ctx, c_void_p(lg.data_ptr()), m, V, V, 0, top_k, 1.0, None, 0, 0,
                            c_void_p(val.data_ptr()), c_void_p(idx.data_ptr()))
    assert rc == _abi.GQ_OK
    g.flush()
    for r in range(m):
        want = np.argsort(-logits[r], kind="stable")[:top_k]
        assert np.array_equal(idx[r].cpu().numpy(), want)
        assert np.array_equal(val[r].cpu().numpy(), logits[r][want])


@pytest.mark.parametrize("mode", ["greedy", "engine_default", "top_k_40"])
def test_sharded_candidates_equal_whole_row(g, mode):
    """A vocab-sharded lm_head: each of 4 shards' top k (gq_topk_rows with the shard's
    first id and the penalty) gathered, then gq_sample_candidates, gives the token of
    gq_sample_rows on the whole row, and advances the states the same way."""
    torch = g._torch
    o = MODES[mode]
    o = opts(o.temperature, o.top_k, o.top_p, 1.2)
    m, G = 3, 4
    k = max(1, o.top_k)
    rng = np.random.default_rng(21)
    logits = (rng.standard_normal((m, V)) * 2.0).astype(np.float32)
    recent = rng.integers(0, V, (m, 16)).astype(np.uint32)
    recent[:, 0] = np.argmax(logits, axis=1)
    seeds = [int(s) for s in synth.splitmix64(999, m)]
    want, want_st, _ = sample_rows(g, logits, o, seeds, recent=recent)
    lg = dev(g, logits, np.float32)
    rec = dev(g, recent.view(np.int32), np.int32)
    val = torch.empty(G, m, k, dtype=torch.float32, device=g.torch_device)
    idx = torch.empty(G, m, k, dtype=torch.int64, device=g.torch_device)
    w = V // G
    for s in range(G):
        rc = g.lib.gq_topk_rows(g.ctx, c_void_p(lg.data_ptr() + 4 * s * w), m, w, V, s * w, k, o.repetition_penalty,
                                c_void_p(rec.data_ptr()), recent.shape[1], recent.shape[1],
                                c_void_p(val[s].data_ptr()), c_void_p(idx[s].data_ptr()))
        assert rc == _abi.GQ_OK
    cv = val.permute(1, 0, 2).reshape(m, G * k).contiguous()  # the all-gather's re-layout
    ci = idx.permute(1, 0, 2).reshape(m, G * k).contiguous()
    st = dev(g, np.array(seeds, dtype=np.uint64).view(np.int64), np.int64)
    tok = torch.full((m,), -7, dtype=torch.int32, device=g.torch_device)
    rc = g.lib.gq_sample_candidates(g.ctx, c_void_p(cv.data_ptr()), c_void_p(ci.data_ptr()), m, G * k,
                                    ctypes.byref(o), c_void_p(st.data_ptr()), c_void_p(tok.data_ptr()))
    assert rc == _abi.GQ_OK
    g.flush()
    assert np.array_equal(tok.cpu().numpy(), want)
    assert np.array_equal(st.cpu().numpy().view(np.uint64), want_st)


def test_sample_argument_checks(g):
    st = g._torch.zeros(1, dtype=g._torch.int64, device=g.torch_device)
    tok = g._torch.zeros(1, dtype=g._torch.int32, device=g.torch_device)
    lg = g._torch.zeros(1, 8, device=g.torch_device)
    bad_k = opts(top_k=257)
    assert g.lib.gq_sample_rows(g.ctx, c_void_p(lg.data_ptr()), 1, 8, 0, ctypes.byref(bad_k), None, 0, 0,
                                c_void_p(st.data_ptr()), c_void_p(tok.data_ptr())) == _abi.GQ_ERR_UNSUPPORTED
    assert g.lib.gq_sample_rows(g.ctx, c_void_p(lg.data_ptr()), 0, 8, 0, ctypes.byref(opts()), None, 0, 0,
                                c_void_p(st.data_ptr()), c_void_p(tok.data_ptr())) == _abi.GQ_OK
    nocand = opts(temperature=1.0, top_k=0)
    assert g.lib.gq_sample_candidates(g.ctx, c_void_p(lg.data_ptr()), c_void_p(st.data_ptr()), 1, 1,
                                      ctypes.byref(nocand), c_void_p(st.data_ptr()),
                                      c_void_p(tok.data_ptr())) == _abi.GQ_ERR_UNSUPPORTED
