"""The allocation-free prefill entry point (gq_linear_prefill_static), through the
C ABI (needs a B200).

gq_linear_prefill_static serves callers that cannot allocate device memory at
call time (a serving process that reserved its HBM at start-up, an embedder
whose buffers all come from its own arena): its scratch, the f16 copy of the
activations, is a fixed 8 MiB device array inside the library instead of a
context workspace. The checks:
  * against the regular entry point (gq_linear) on the same inputs, called twice
    in a row (the second call reuses the array the first one left behind), at
    the relative-L2 bound the prefill tests use;
  * against the CPU oracle at the tensor-core path's bounds: 1e-2 against the
    f32 oracle, 1e-5 against the oracle fed the same row-scaled f16-rounded
    activations, including row counts below one 128-row tile (m = 1, 15, 17, 64,
    127), which the regular entry point never sends to this kernel;
  * sizes beyond the scratch are rejected, and the status word reads clean.
The file is named so that pytest collects it last; it also passes run alone.
"""
import ctypes

import numpy as np
import pytest

from gq import CudaBackend, _abi
from gq import synth
from numerics import f16_round, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5


@pytest.fixture(scope="module")
def g():
    be = CudaBackend(0)
    yield be
    be.close()


def _stream(g):
    return g._torch.cuda.current_stream(g.torch_device).cuda_stream


def _static_linear(g, x_dev, m, k, qb_dev, sc_dev, n, bits, signed, y_dev):
    return g.lib.gq_linear_prefill_static(ctypes.c_void_p(_stream(g)), ctypes.c_void_p(x_dev.data_ptr()), m, k,
                                          ctypes.c_void_p(qb_dev.data_ptr()), ctypes.c_void_p(sc_dev.data_ptr()), n,
                                          bits, int(signed), ctypes.c_void_p(y_dev.data_ptr()))


def _status(g):
    bits = ctypes.c_uint32(0xFFFFFFFF)
    rc = g.lib.gq_linear_prefill_static_status(ctypes.c_void_p(_stream(g)), ctypes.byref(bits))
    return rc, bits.value


def _device_weight(g, w):
    torch = g._torch
    qb = torch.from_numpy(np.ascontiguousarray(w.qbytes)).to(g.torch_device)
    sc = torch.from_numpy(np.ascontiguousarray(w.scales)).to(g.torch_device)
    return qb, sc


@pytest.mark.parametrize("m,n,k,bits,signed", [(256, 2048, 1536, 4, False), (130, 300, 640, 8, True),
                                               (512, 1536, 6144, 2, False)])
def test_static_matches_regular_twice(g, m, n, k, bits, signed):
    torch = g._torch
    w = synth.make_qweight(7000 + n + k, n, k, bits, signed)
    gw = g.quant_tensor(w)  # the regular entry point's own upload
    qb, sc = _device_weight(g, w)
    for call in range(2):
        x = synth.normal(7100 + 10 * call + m, m * k).reshape(m, k) * (1.0 + call)
        gx = g.tensor(x, x.shape)
        ref = g.readback(g.linear(gx, gw))
        y = torch.empty(m, n, dtype=torch.float32, device=g.torch_device)
        rc = _static_linear(g, gx.data, m, k, qb, sc, n, bits, signed, y)
        assert rc == _abi.GQ_OK, f"call {call}: status {rc}"
        got = g.readback(g.from_torch(y))
        assert rel_l2(got, ref) <= REL_L2, f"call {call}"
    assert _status(g) == (_abi.GQ_OK, 0)


@pytest.mark.parametrize("m", [1, 15, 17, 64, 127, 129])
@pytest.mark.parametrize("bits,signed", [(2, False), (4, False), (8, True)])
def test_static_against_oracle(g, m, bits, signed):
    """Against the CPU oracle (rust/src/backend_cpu.rs:174-222) for row counts inside
    and just past one 128-row tile, each bit width; two calls in a row with
    different activations."""
    torch = g._torch
    n, k = 300, 640
    w = synth.make_qweight(7300 + bits, n, k, bits, signed)
    qb, sc = _device_weight(g, w)
    for call in range(2):
        x = (synth.normal(7400 + 13 * m + call, m * k) * (0.5 + call)).reshape(m, k)
        gx = g.tensor(x, x.shape)
        y = torch.empty(m, n, dtype=torch.float32, device=g.torch_device)
        assert _static_linear(g, gx.data, m, k, qb, sc, n, bits, signed, y) == _abi.GQ_OK
        got = g.readback(g.from_torch(y)).reshape(m, n)
        assert rel_l2(got, oracle.linear(x, w)) <= 1e-2, (m, bits, call)
        assert rel_l2(got, oracle.linear(f16_round(x), w)) <= REL_L2, (m, bits, call)
    assert _status(g) == (_abi.GQ_OK, 0)


def test_static_rejects_sizes_beyond_its_scratch(g):
    torch = g._torch
    m, k, n = 4097, 1024, 64  # m*k > 4,194,304
    x = torch.zeros(m, k, dtype=torch.float32, device=g.torch_device)
    qb = torch.zeros(n * k // 2, dtype=torch.uint8, device=g.torch_device)
    sc = torch.ones(n, dtype=torch.float32, device=g.torch_device)
    y = torch.empty(m, n, dtype=torch.float32, device=g.torch_device)
    assert _static_linear(g, x, m, k, qb, sc, n, 4, False, y) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert _static_linear(g, x[:, :1000].contiguous(), 4, 1000, qb, sc, n, 4, False, y) == _abi.GQ_ERR_UNSUPPORTED
    # more weight rows than 65,535 tiles of 128: refused before anything is enqueued
    assert _static_linear(g, x[:1], 1, 1024, qb, sc, 65535 * 128 + 1, 4, False, y) == _abi.GQ_ERR_UNSUPPORTED
    assert _status(g) == (_abi.GQ_OK, 0)
