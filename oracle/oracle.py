"""TEST INFRASTRUCTURE ONLY: ctypes front end of the MLA decode-attention oracle.

Two implementations of the reference's *unfused CPU ggml graph* live behind this module:

* ``liboracle.so`` -- ``oracle/mla_oracle.c``, our plain-C restatement of the graph's arithmetic
  (the rounding points of vendor/llama.cpp/ggml/src/ggml-cpu/ggml-cpu.c:1330-1375 and
  ops.cpp:5813-5910; the op sequence of engine/m1_layer.cpp:437-502).
* ``_ref/libggml_ref_v{3,4}.so`` -- the reference's own ggml + ggml-cpu sources, compiled by
  ``oracle/ref.mk`` with our graph-building harness ``oracle/ref_harness.c``.  Present wherever
  ``__graft_entry__.build()`` ran with the reference tree mounted; the built files travel.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use this module,
always as the checker / the baseline, never as the product path.

Array conventions: numpy row-major views of the ggml tensors (ggml ne[] reversed), f16 arrays as
``np.float16``; see the header of ``mla_oracle.c``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_C_SRC = os.path.join(HERE, "mla_oracle.c")
_C_LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def build_restatement(force: bool = False) -> str:
    """Compile ``mla_oracle.c`` into ``liboracle.so`` (gcc; seconds)."""
    if force or not os.path.exists(_C_LIB) or os.path.getmtime(_C_LIB) < os.path.getmtime(_C_SRC):
        subprocess.check_call(["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared",
                               "-o", _C_LIB, _C_SRC, "-lm"])
    return _C_LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build_restatement())
        i64, c_int, c_float = ctypes.c_int64, ctypes.c_int, ctypes.c_float
        _lib.orc_wkb_f16.argtypes = [_u16p, _f32p, i64, c_int, c_int, c_int, _f32p, i64]
        _lib.orc_kqkv.argtypes = [_u16p, i64, c_int, c_int, _f32p, i64, c_int, _f32p, c_float, _f32p]
        _lib.orc_kqkv_exact.argtypes = _lib.orc_kqkv.argtypes
        _lib.orc_wvb_f16.argtypes = [_u16p, _f32p, i64, c_int, c_int, c_int, _f32p]
        _lib.orc_kqkv_partial.argtypes = [_u16p, i64, i64, c_int, c_int, _f32p, i64, c_int, _f32p,
                                          c_float, _f32p]
        _lib.orc_combine.argtypes = [_f32p, c_int, c_int, c_int, _f32p]
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_f32p)


def _f16(a):
    a = np.asarray(a)
    if a.dtype == np.uint16:  # raw f16 bit patterns
        a = a.view(np.float16)
    a = np.ascontiguousarray(a, dtype=np.float16)
    return a, a.ctypes.data_as(_u16p)


def wkb(w_uk: np.ndarray, q: np.ndarray, nope: int) -> np.ndarray:
    """q_abs[h] = W_UK[h] . f16(q[h, :nope]).  w_uk f16 (H, R, nope); q f32 (H, q_stride)."""
    H, R, K = w_uk.shape
    assert K == nope and q.shape[0] == H
    w, wp = _f16(w_uk)
    qq, qp = _f32(q)
    out = np.empty((H, R), np.float32)
    lib().orc_wkb_f16(wp, qp, qq.shape[1], H, R, K, out.ctypes.data_as(_f32p), R)
    return out


def kqkv(kc: np.ndarray, qcur: np.ndarray, mask: np.ndarray | None, scale: float, R: int,
         exact: bool = False) -> np.ndarray:
    """Unfused K.Q -> soft_max_ext -> V^T.P.  kc f16 (N, D); qcur f32 (H, >=D); mask f32 (N,)."""
    N, D = kc.shape
    H = qcur.shape[0]
    k, kp = _f16(kc)
    qq, qp = _f32(qcur)
    if mask is not None:
        mm, mp = _f32(mask)
        assert mm.shape[0] == N
    else:
        mm, mp = None, None
    out = np.empty((H, R), np.float32)
    fn = lib().orc_kqkv_exact if exact else lib().orc_kqkv
    fn(kp, N, D, R, qp, qq.shape[1], H, mp, float(scale), out.ctypes.data_as(_f32p))
    return out


def wvb(w_uv: np.ndarray, x: np.ndarray) -> np.ndarray:
    """out[h] = W_UV[h] . f16(x[h]).  w_uv f16 (H, V, R); x f32 (H, >=R)."""
    H, V, R = w_uv.shape
    w, wp = _f16(w_uv)
    xx, xp = _f32(x)
    out = np.empty((H, V), np.float32)
    lib().orc_wvb_f16(wp, xp, xx.shape[1], H, V, R, out.ctypes.data_as(_f32p))
    return out


def kqkv_partial(kc, k0, k1, qcur, mask, scale, R) -> np.ndarray:
    """Exact split-K partial over keys [k0, k1): (H, R + 4) = {o[R], m (log2 units), l, 0, 0}."""
    N, D = kc.shape
    H = qcur.shape[0]
    k, kp = _f16(kc)
    qq, qp = _f32(qcur)
    mm, mp = _f32(mask) if mask is not None else (None, None)
    part = np.empty((H, R + 4), np.float32)
    lib().orc_kqkv_partial(kp, k0, k1, D, R, qp, qq.shape[1], H, mp, float(scale),
                           part.ctypes.data_as(_f32p))
    return part


def combine(part: np.ndarray) -> np.ndarray:
    """Merge (S, H, R + 4) partial records with the online-softmax rule -> (H, R)."""
    S, H, W = part.shape
    pp, ptr = _f32(part)
    out = np.empty((H, W - 4), np.float32)
    lib().orc_combine(ptr, S, H, W - 4, out.ctypes.data_as(_f32p))
    return out


def mla_step(w_uk, q, kc, mask, w_uv, scale, nope):
    """The whole unfused layer step: (q_abs, qcur, attn, out) with the restatement."""
    q_abs = wkb(w_uk, q, nope)
    qcur = np.concatenate([q_abs, q[:, nope:]], axis=1)
    attn = kqkv(kc, qcur, mask, scale, w_uk.shape[1])
    out = wvb(w_uv, attn)
    return q_abs, qcur, attn, out


# ---------------------------------------------------------------------------------------------
# The reference's own ggml-cpu (oracle/_ref)
# ---------------------------------------------------------------------------------------------

def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
    except OSError:
        return False
    return all(x in flags for x in ("avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"))


def ref_library_path() -> str | None:
    """Path of the widest oracle/_ref variant this host can run, or None when not built."""
    order = ["v4", "v3"] if _cpu_has_avx512() else ["v3"]
    for v in order:
        p = os.path.join(REF_DIR, f"libggml_ref_{v}.so")
        if os.path.exists(p):
            return p
    return None


_ref = None


def ref_lib():
    global _ref
    if _ref is None:
        path = ref_library_path()
        if path is None:
            raise FileNotFoundError("oracle/_ref not built (run __graft_entry__.build() where the "
                                    "reference tree is mounted)")
        _ref = ctypes.CDLL(path)
        vp = ctypes.c_void_p
        _ref.ref_mla_create.restype = vp
        _ref.ref_mla_create.argtypes = [ctypes.c_int] * 5 + [ctypes.c_int64, ctypes.c_float,
                                                             ctypes.c_int]
        _ref.ref_mla_destroy.argtypes = [vp]
        _ref.ref_mla_set_inputs.argtypes = [vp, _f32p, _u16p, _u16p, _f32p, _u16p]
        _ref.ref_mla_compute.argtypes = [vp]
        _ref.ref_mla_compute.restype = ctypes.c_int
        _ref.ref_mla_get_outputs.argtypes = [vp, _f32p, _f32p, _f32p, _f32p]
        _ref.ref_mla_n_nodes.argtypes = [vp]
        _ref.ref_mla_n_nodes.restype = ctypes.c_int
    return _ref


class RefMLA:
    """The reference's unfused MLA decode graph on its own ggml-cpu backend (built once)."""

    def __init__(self, H, nope, rope, R, V, N, scale, n_threads=None):
        self.H, self.nope, self.rope, self.R, self.V, self.N = H, nope, rope, R, V, N
        self.n_threads = n_threads or os.cpu_count() or 1
        self._h = ref_lib().ref_mla_create(H, nope, rope, R, V, N, float(scale), self.n_threads)
        if not self._h:
            raise RuntimeError("ref_mla_create failed")
        self._keep = []

    def set_inputs(self, q=None, w_uk=None, kc=None, mask=None, w_uv=None):
        args, keep = [], []
        for a, conv in ((q, _f32), (w_uk, _f16), (kc, _f16), (mask, _f32), (w_uv, _f16)):
            if a is None:
                args.append(None)
            else:
                arr, ptr = conv(a)
                keep.append(arr)
                args.append(ptr)
        ref_lib().ref_mla_set_inputs(self._h, *args)

    def compute(self):
        rc = ref_lib().ref_mla_compute(self._h)
        if rc != 0:
            raise RuntimeError(f"ggml_graph_compute returned {rc}")

    def outputs(self):
        H, R, V, D = self.H, self.R, self.V, self.R + self.rope
        q_abs = np.empty((H, R), np.float32)
        qcur = np.empty((H, D), np.float32)
        attn = np.empty((H, R), np.float32)
        out = np.empty((H, V), np.float32)
        ref_lib().ref_mla_get_outputs(self._h, q_abs.ctypes.data_as(_f32p),
                                      qcur.ctypes.data_as(_f32p), attn.ctypes.data_as(_f32p),
                                      out.ctypes.data_as(_f32p))
        return q_abs, qcur, attn, out

    def n_nodes(self) -> int:
        return ref_lib().ref_mla_n_nodes(self._h)

    def close(self):
        if self._h:
            ref_lib().ref_mla_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
