"""Shared tolerances and comparisons for the parity tests.

The gate (north star): max |out - ref| / max |ref| <= 2e-3 on the attention output, fp32
accumulation.  The reference CPU graph rounds q, P and the attention output to f16 before each
mul_mat (ggml-cpu.c:1330-1375), so kernel and oracle sit in the same rounding class; the measured
gap is ~1e-4.
"""
import numpy as np

ATTN_TOL = 2e-3      # attention output and the W_UV output (the north-star gate)
QABS_TOL = 1e-5      # absorption gemv: same f16 operands, f32 vs double accumulation only


def rel_to_max(x, ref) -> float:
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    if den == 0.0:
        return float(np.abs(x).max())
    return float(np.abs(x - ref).max() / den)


def elementwise_ok(x, ref, rtol=2e-3, atol_frac=1e-5) -> bool:
    """|x - ref| <= rtol*|ref| + atol_frac*max|ref| everywhere (the survey's secondary check)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return bool(np.all(np.abs(x - ref) <= rtol * np.abs(ref) + atol_frac * np.abs(ref).max()))
