"""The latency floor of a chain of dependent phases on the B200 (needs a GPU).

tests/native/chain_latency.cu times 210 dependent phases (the per-layer GEMV count of
an E2B decode step) that do no MAC work: as launches in a CUDA graph with and without
programmatic dependent launch, and as one persistent kernel with a grid barrier
between phases. Those times bound what the decode-step GEMV chain can reach at batch
1: at ~2 us per dependent phase, 210 phases take ~0.44 ms however fast each GEMV
streams its weights. The test builds the harness with nvcc, runs it, checks that it
reports sane figures (and no barrier timeout), and prints them.
"""
import os
import re
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "native", "chain_latency.cu")


def test_chain_latency_floor(tmp_path, capsys):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = str(tmp_path / "chain_latency")
    subprocess.run([nvcc, "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-o", exe, SRC], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=120).stdout
    with capsys.disabled():
        print("\n" + out)
    pdl = [float(v) for v in re.findall(r"pdl=1: ([0-9.]+) us", out)]
    nopdl = [float(v) for v in re.findall(r"pdl=0: ([0-9.]+) us", out)]
    persist = [float(v) for v in re.findall(r"persistent chain: ([0-9.]+) us per phase \(err=0", out)]
    assert len(pdl) == 1 and len(nopdl) == 1 and len(persist) == 3, out
    assert 0.3 < pdl[0] < 20 and 0.3 < nopdl[0] < 20 and 0.3 < min(persist) < 20
