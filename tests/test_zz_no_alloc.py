"""The allocation-free prefill entry point (gq_linear_prefill_static) against the
regular one (gq_linear), through the C ABI (needs a B200).

gq_linear_prefill_static serves callers that cannot allocate device memory at
call time (a serving process that reserved its HBM at start-up, an embedder
whose buffers all come from its own arena): its scratch, the f16 copy of the
activations, is a fixed 8 MiB device array inside the library instead of a
context workspace. These checks call it twice in a row (the second call reuses
the array the first one left behind) and compare each result with gq_linear on
the same inputs, at the relative-L2 bound the prefill tests use. The file is
named so that pytest collects it last; it also passes run alone.
"""
import ctypes

import numpy as np
import pytest

from gq import CudaBackend, _abi
from gq import synth

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.fixture(scope="module")
def g():
    be = CudaBackend(0)
    yield be
    be.close()


def _static_linear(g, x_dev, m, k, qb_dev, sc_dev, n, bits, signed, y_dev):
    torch = g._torch
    stream = torch.cuda.current_stream(g.torch_device).cuda_stream
    return g.lib.gq_linear_prefill_static(ctypes.c_void_p(stream), ctypes.c_void_p(x_dev.data_ptr()), m, k,
                                          ctypes.c_void_p(qb_dev.data_ptr()), ctypes.c_void_p(sc_dev.data_ptr()), n,
                                          bits, int(signed), ctypes.c_void_p(y_dev.data_ptr()))


@pytest.mark.parametrize("m,n,k,bits,signed", [(256, 2048, 1536, 4, False), (130, 300, 640, 8, True),
                                               (512, 1536, 6144, 2, False)])
def test_static_matches_regular_twice(g, m, n, k, bits, signed):
    torch = g._torch
    w = synth.make_qweight(7000 + n + k, n, k, bits, signed)
    gw = g.quant_tensor(w)  # the regular entry point's own upload
    qb = torch.from_numpy(np.ascontiguousarray(w.qbytes)).to(g.torch_device)
    sc = torch.from_numpy(np.ascontiguousarray(w.scales)).to(g.torch_device)
    for call in range(2):
        x = synth.normal(7100 + 10 * call + m, m * k).reshape(m, k) * (1.0 + call)
        gx = g.tensor(x, x.shape)
        ref = g.readback(g.linear(gx, gw))
        y = torch.empty(m, n, dtype=torch.float32, device=g.torch_device)
        rc = _static_linear(g, gx.data, m, k, qb, sc, n, bits, signed, y)
        assert rc == _abi.GQ_OK, f"call {call}: status {rc}"
        got = g.readback(g.from_torch(y))
        assert rel_l2(got, ref) <= REL_L2, f"call {call}"


def test_static_rejects_sizes_beyond_its_scratch(g):
    torch = g._torch
    m, k, n = 4097, 1024, 64  # m*k > 4,194,304
    x = torch.zeros(m, k, dtype=torch.float32, device=g.torch_device)
    qb = torch.zeros(n * k // 2, dtype=torch.uint8, device=g.torch_device)
    sc = torch.ones(n, dtype=torch.float32, device=g.torch_device)
    y = torch.empty(m, n, dtype=torch.float32, device=g.torch_device)
    assert _static_linear(g, x, m, k, qb, sc, n, 4, False, y) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert _static_linear(g, x[:, :1000].contiguous(), 4, 1000, qb, sc, n, 4, False, y) == _abi.GQ_ERR_UNSUPPORTED
