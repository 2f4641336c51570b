"""The short-M tensor-core GEMV's planner on the CPU: its translation unit is
compiled for the host (no kernel runs) and its plans for the E2B projections,
odd shapes and every decode row count are checked against the invariants the
kernel relies on: a split-K plan has every split non-empty, one CTA per SM at
most and one row slice; the int64 partials fit below the scales in shared
memory; TMEM columns are a power of two within 512; the limb ring is a power of
two per issuer, or, with the limbs made inside the GEMV, every K-block of a CTA
has a resident limb tile; the weights-as-A layout has one issuer; and the
default choice follows the measured rule (4 splits with 64-row tiles for
K >= 3072, 2 splits with 32-row tiles for K >= 2048, 4 splits with 32-row tiles
for short weights with K >= 1024)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "gemma-4-webgpu-kernels_b200", "_build")
SRC = os.path.join(ROOT, "tests", "native", "tcx_plan_dump.cu")
NUM_SMS, BUDGET = 148, 232448 - 1024


@pytest.fixture(scope="module")
def plans(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    objs = [os.path.join(BUILD, f) for f in sorted(os.listdir(BUILD))] if os.path.isdir(BUILD) else []
    objs = [o for o in objs if o.endswith(".o") and not o.endswith("gemv_tcx.o")]
    if not os.path.exists(nvcc) or not objs:
        pytest.skip("needs nvcc and the built objects (run the build first)")
    exe = str(tmp_path_factory.mktemp("plan") / "tcx_plan_dump")
    subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a",
                    "--expt-relaxed-constexpr", "-o", exe, SRC, *objs, "-lcuda"], check=True, capture_output=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    # the same plans with the in-kernel limbs enabled (GQ_TCX_XIN=1), tagged "+xin"
    env = dict(os.environ, GQ_TCX_XIN="1")
    out_xin = subprocess.run([exe], check=True, capture_output=True, text=True, env=env).stdout
    out += "".join(line.split(" ", 1)[0] + "+xin " + line.split(" ", 1)[1] + "\n" for line in out_xin.splitlines())
    rows = []
    for line in out.splitlines():
        f = line.split()
        name, vals = f[0], [int(v) for v in f[1:]]
        keys = ("m nw tile ks tile_rows gx kb_per kblocks slice_rows issuers xi xa_stages tmem_cols smem part "
                "sc_off ok xin wa raw_stages mma_stages").split()
        rows.append(dict(name=name, **dict(zip(keys, vals))))
    return rows


SHAPE_N = {n + t: v for n, v in {"qkv_l": 2560, "q_g": 4096, "o_l": 1536, "o_g": 1536, "gate_up": 6144,
                                 "down": 1536, "ple_gate": 256, "ple_proj": 1536, "lm_head": 262144, "odd": 300,
                                 "tiny": 77}.items() for t in ("", "+xin")}


def test_every_plan_meets_the_kernel_invariants(plans):
    ok = [p for p in plans if p["ok"]]
    assert len(ok) > 100
    for p in ok:
        ks = p["ks"] if p["ks"] > 0 else None
        assert p["smem"] <= BUDGET, p
        assert 32 <= p["tmem_cols"] <= 512 and p["tmem_cols"] & (p["tmem_cols"] - 1) == 0, p
        if p["xin"]:  # limbs made in the GEMV: one resident tile per K-block of the CTA, x held in registers
            assert p["xa_stages"] >= p["kb_per"], p
            gk = p["kb_per"] * 8
            gp = 8 if gk <= 8 else 16 if gk <= 16 else -(-gk // 32) * 32  # a row's lane slots
            assert p["m"] * gp <= 256 * 4, p
        else:
            assert p["xi"] >= 2 and p["xi"] & (p["xi"] - 1) == 0 and p["xa_stages"] == p["issuers"] * p["xi"], p
        if p["wa"]:
            assert p["issuers"] == 1 and p["tile_rows"] == 128, p
        assert p["raw_stages"] >= 1, p
        assert p["tile_rows"] % 16 == 0 and p["slice_rows"] <= NUM_SMS * p["tile_rows"], p
        splits = -(-p["kblocks"] // p["kb_per"])
        if splits > 1 or (ks or 1) > 1:
            assert p["slice_rows"] == SHAPE_N[p["name"]], p  # one slice
            assert p["gx"] * splits <= NUM_SMS, p          # one CTA per SM at most
            assert (splits - 1) * p["kb_per"] < p["kblocks"], p  # every split owns K-blocks
            assert p["part"] <= p["sc_off"], p              # partials below the scales


def test_default_choice_follows_the_measured_rule(plans):
    chosen = {(p["name"], p["m"]): p for p in plans if p["ks"] == 0 and p["ok"] and not p["wa"]}
    assert not any(p["xin"] for p in plans if "+xin" not in p["name"])  # the pre-pass is the default
    for m in (5, 8, 16, 24, 33, 64):
        d = chosen[("down", m)]        # K = 6144
        assert (d["tile_rows"], -(-d["kblocks"] // d["kb_per"])) == (64, 4), d
        og = chosen[("o_g", m)]        # K = 4096
        assert (og["tile_rows"], -(-og["kblocks"] // og["kb_per"])) == (64, 4), og
        ol = chosen[("o_l", m)]        # K = 2048
        assert (ol["tile_rows"], -(-ol["kblocks"] // ol["kb_per"])) == (32, 2), ol
        pg = chosen[("ple_gate", m)]   # N = 256, K = 1536
        assert (pg["tile_rows"], -(-pg["kblocks"] // pg["kb_per"])) == (32, 4), pg
        for name in ("qkv_l", "q_g", "gate_up", "ple_proj", "lm_head"):  # no split
            assert chosen[(name, m)]["kb_per"] == chosen[(name, m)]["kblocks"], (name, m)


def test_in_kernel_limbs_cover_the_small_decode_batches(plans):
    """With GQ_TCX_XIN=1, every E2B projection at M = 8 runs without the limb pre-pass."""
    chosen = {(p["name"], p["m"]): p for p in plans if p["ks"] == 0 and p["ok"] and not p["wa"]}
    for name in ("qkv_l", "q_g", "o_l", "o_g", "gate_up", "down", "ple_gate", "ple_proj"):
        assert chosen[(name + "+xin", 8)]["xin"] == 1, (name, chosen[(name + "+xin", 8)])
