"""Numeric helpers shared by the GPU test files (no GPU needed to import)."""
import numpy as np


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def f16_round(x):
    """The activations the tensor-core prefill kernel multiplies: per row, x * 2^e
    rounded to f16 (nearest even) with e = 14 - (exponent of max|x| as frexp gives
    it), then scaled back by 2^-e; returned as f32."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, np.shape(x)[-1])
    out = np.empty_like(x)
    for i, row in enumerate(x):
        mx = float(np.max(np.abs(row))) if row.size else 0.0
        e = int(np.frexp(mx)[1]) if (mx > 0 and np.isfinite(mx)) else 0
        s = 14 - e
        scaled = (row.astype(np.float64) * 2.0 ** s).astype(np.float32)
        out[i] = (scaled.astype(np.float16).astype(np.float64) * 2.0 ** -s).astype(np.float32)
    return out
