"""The C-ABI library loads and exports every symbol its header declares (no GPU
compute here), and the oracle library does the same for its header."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gq.h")
LIB = os.path.join(ROOT, "gemma-4-webgpu-kernels_b200", "gq", "libgq.so")
ORACLE_H = os.path.join(ROOT, "oracle", "gq_oracle.h")
ORACLE_LIB = os.path.join(ROOT, "oracle", "libgq_oracle.so")


def declared(header: str, prefix: str):
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(%s\w+)\s*\(" % prefix, text)))


def exported(lib: str):
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_header_declares_the_trait_surface():
    names = declared(HEADER, "gq_")
    for required in ["gq_linear", "gq_linear_geglu", "gq_linear_gelu_mul_cols", "gq_embed_rows",
                     "gq_qweight_upload", "gq_softcap", "gq_readback", "gq_sync", "gq_last_error"]:
        assert required in names


def test_libgq_exports_every_declared_symbol():
    assert os.path.exists(LIB), "libgq.so not built (make -C gemma-4-webgpu-kernels_b200)"
    missing = set(declared(HEADER, "gq_")) - exported(LIB)
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_python_binding_covers_header():
    from gq import _abi

    assert set(declared(HEADER, "gq_")) == set(_abi.SIGNATURES)
    lib = _abi.load()
    assert lib.gq_abi_version() == 1
    assert lib.gq_status_string(0) == b"ok"


def test_oracle_exports_every_declared_symbol():
    missing = set(declared(ORACLE_H, "gqo_")) - exported(ORACLE_LIB)
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_null_arguments_are_errors_not_crashes():
    """Every entry point returns a status; nothing aborts (no device needed)."""
    from gq import _abi

    lib = _abi.load()
    assert lib.gq_ctx_create(0, None) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_linear(None, None, 1, 1, None, None) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_embed_rows(None, None, None, 1, 1.0, None) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_sync(None) == _abi.GQ_ERR_INVALID_ARGUMENT
    assert lib.gq_qweight_free(None) == _abi.GQ_OK
    assert lib.gq_ctx_destroy(None) == _abi.GQ_OK


def test_no_gpu_context_create_fails_cleanly():
    """Without a device, context creation reports an error status."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from gq import _abi

    lib = _abi.load()
    ctx = ctypes.c_void_p()
    assert lib.gq_ctx_create(0, ctypes.byref(ctx)) != _abi.GQ_OK
    assert not ctx.value


RUST = os.path.join(ROOT, "gemma-4-webgpu-kernels_b200", "rust")


def header_params(header: str, prefix: str = "gq_"):
    """name -> number of parameters of every function the header declares."""
    text = re.sub(r"/\*.*?\*/", "", open(header).read(), flags=re.S)
    out = {}
    for name, args in re.findall(r"\b(%s\w+)\s*\(([^)]*)\)\s*;" % prefix, text):
        args = " ".join(args.split())
        out[name] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def rust_params(path: str):
    """name -> number of parameters of every `pub fn gq_*` in a Rust extern block."""
    text = re.sub(r"//[^\n]*", "", open(path).read())
    out = {}
    for name, args in re.findall(r"pub fn (gq_\w+)\(([^)]*)\)", text):
        parts = [a for a in (x.strip() for x in args.split(",")) if a]
        out[name] = len(parts)
    return out


def test_rust_binding_declares_every_entry_point():
    """The Rust extern block a maintainer drops into the engine
    (rust/src/backend_cuda/ffi.rs) declares every entry point of the header with
    the same number of parameters."""
    want = header_params(HEADER)
    assert set(want) == set(declared(HEADER, "gq_"))
    got = rust_params(os.path.join(RUST, "src", "backend_cuda", "ffi.rs"))
    assert set(want) <= set(got), sorted(set(want) - set(got))
    wrong = {n: (want[n], got[n]) for n in want if want[n] != got[n]}
    assert not wrong, wrong


def test_rust_backend_implements_the_trait_surface():
    """rust/src/backend_cuda.rs implements every method of the reference's `trait
    Backend` (rust/src/backend.rs:88-180, listed here) and calls only symbols
    that ffi.rs declares; build.rs builds and links libgq."""
    src = open(os.path.join(RUST, "src", "backend_cuda.rs")).read()
    trait = ["name", "tensor", "quant_tensor", "zeros", "reshape", "embed_rows", "rms_norm", "linear", "add", "mul",
             "scale", "scale_by_tensor", "gelu_tanh", "geglu", "softcap", "rope", "attention", "slice_rows",
             "slice_cols", "concat_rows", "kv_append", "add_rms_norm", "head_norm_rope", "linear_geglu",
             "linear_gelu_mul_cols", "readback", "flush", "end_frame", "free_tensor"]
    impl = src[src.index("impl Backend for CudaBackend"):]
    have = set(re.findall(r"\bfn (\w+)\(", impl))
    assert set(trait) <= have, sorted(set(trait) - have)
    called = set(re.findall(r"ffi::(gq_\w+)", src))
    assert called <= set(rust_params(os.path.join(RUST, "src", "backend_cuda", "ffi.rs"))), called
    build = open(os.path.join(RUST, "build.rs")).read()
    assert "rustc-link-lib=dylib=gq" in build and '"make"' in build
