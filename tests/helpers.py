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
    """|x - ref| <= rtol*|ref| + atol_frac*max|ref| everywhere (an elementwise check beside the
    rel-to-max one)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return bool(np.all(np.abs(x - ref) <= rtol * np.abs(ref) + atol_frac * np.abs(ref).max()))


def fp64_layer(q, w_uk, kc, w_uv, mask=None, nope=128):
    """The layer step in float64 on the host, as the arbiter between the kernels and the reference
    CPU graph: q_nope and Qcur rounded to f16 (the tensor-core operands, and the CPU mul_mat's f16
    conversion of src1), the attention output rounded to f16 before W_UV; every sum in float64.
    Shapes: q (H, nope + rope) f32, w_uk (H, R, nope) f16, kc (N, R + rope) f16, w_uv (H, V, R)
    f16, mask (N,) or None.  Returns (attn (H, R), out (H, V))."""
    R = w_uk.shape[1]
    qn = q[:, :nope].astype(np.float16).astype(np.float64)
    qabs = np.einsum("hrk,hk->hr", w_uk.astype(np.float64), qn)
    qcur = np.concatenate([qabs, q[:, nope:].astype(np.float64)], 1)
    qcur = qcur.astype(np.float16).astype(np.float64)
    K = kc.astype(np.float64)
    s = (K @ qcur.T) / np.sqrt(q.shape[1])            # (N, H)
    if mask is not None:
        s = s + np.asarray(mask, np.float64)[:, None]
    s = s - s.max(0, keepdims=True)
    p = np.exp(s)
    p /= p.sum(0, keepdims=True)
    attn = p.T @ K[:, :R]
    out = np.einsum("hvr,hr->hv", w_uv.astype(np.float64),
                    attn.astype(np.float16).astype(np.float64))
    return attn, out
