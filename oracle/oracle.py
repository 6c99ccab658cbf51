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
        u8p = ctypes.POINTER(ctypes.c_uint8)
        _lib.orc_q8_0_quantize.argtypes = [_f32p, i64, c_int, u8p]
        _lib.orc_wkb_q8.argtypes = [u8p, _f32p, i64, c_int, c_int, c_int, _f32p, i64, c_int]
        _lib.orc_wvb_q8.argtypes = [u8p, _f32p, i64, c_int, c_int, c_int, _f32p, c_int]
        _lib.orc_rope_corr_dims.argtypes = [c_int, c_int, c_float, c_float, c_float, _f32p]
        _lib.orc_kvwrite.argtypes = [_f32p, c_int, u8p, _f32p, c_int, c_int, _u16p, i64, c_int,
                                     c_float, c_float, c_float, c_float, c_float, c_float,
                                     c_float, c_int, c_int, _f32p]
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


# ---------------------------------------------------------------------------------------------
# Q8_0 weights (the Mistral-Small-4 geometry).  numerics: CPU = the unfused CPU graph (the
# oracle), FUSED = the reference's fused kernels (MMVQ's Q8_1 activation form).
# ---------------------------------------------------------------------------------------------
CPU, FUSED = 0, 1
_u8p = ctypes.POINTER(ctypes.c_uint8)


def _u8(a):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a, a.ctypes.data_as(_u8p)


def q8_0_quantize(w: np.ndarray) -> np.ndarray:
    """Float rows (..., K) -> Q8_0 bytes (..., K // 32 * 34), ggml's reference quantizer."""
    w32, wp = _f32(w)
    K = w32.shape[-1]
    rows = w32.size // K
    out = np.empty(w32.shape[:-1] + (K // 32 * 34,), np.uint8)
    lib().orc_q8_0_quantize(wp, rows, K, out.ctypes.data_as(_u8p))
    return out


def q8_0_dequantize(wq: np.ndarray, K: int) -> np.ndarray:
    """Q8_0 bytes (..., K // 32 * 34) -> float32 (..., K)."""
    b = np.ascontiguousarray(wq).reshape(-1, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (d * q).reshape(wq.shape[:-1] + (K,))


def wkb_q8(w_uk_q8: np.ndarray, q: np.ndarray, nope: int, R: int, numerics: int = CPU) -> np.ndarray:
    """q_abs[h] = W_UK[h] . Q8(q[h, :nope]).  w_uk_q8 Q8_0 bytes (H, R, nope/32*34)."""
    H = q.shape[0]
    w, wp = _u8(w_uk_q8)
    qq, qp = _f32(q)
    out = np.empty((H, R), np.float32)
    lib().orc_wkb_q8(wp, qp, qq.shape[1], H, R, nope, out.ctypes.data_as(_f32p), R, numerics)
    return out


def wvb_q8(w_uv_q8: np.ndarray, x: np.ndarray, V: int, numerics: int = CPU) -> np.ndarray:
    """out[h] = W_UV[h] . Q8(x[h]).  w_uv_q8 Q8_0 bytes (H, V, R/32*34); x f32 (H, R)."""
    H, R = x.shape
    w, wp = _u8(w_uv_q8)
    xx, xp = _f32(x)
    out = np.empty((H, V), np.float32)
    lib().orc_wvb_q8(wp, xp, xx.shape[1], H, V, R, out.ctypes.data_as(_f32p), numerics)
    return out


def rope_corr_dims(n_dims, n_ctx_orig, freq_base, beta_fast, beta_slow):
    d = np.zeros(2, np.float32)
    lib().orc_rope_corr_dims(n_dims, n_ctx_orig, freq_base, beta_fast, beta_slow,
                             d.ctypes.data_as(_f32p))
    return d


def kvwrite(cur, w_q8, norm_w, kcache, kidx, pos, rp, numerics: int = CPU):
    """Selector-0 KV-write for one token.  cur f32 (n_in,); w_q8 Q8_0 bytes (D, n_in/32*34);
    norm_w f32 (R,); kcache f16 (N, D), updated in place at row kidx (None: no cache);
    rp: dict eps, freq_base, freq_scale, ext_factor, attn_factor, beta_fast, beta_slow, n_dims,
    n_ctx_orig.  Returns Kcur f32 (D,)."""
    cc, cp = _f32(cur)
    w, wp = _u8(w_q8)
    nw, np_ = _f32(norm_w)
    R = nw.shape[0]
    D = w.shape[0]
    kcur = np.empty(D, np.float32)
    kc_ptr = None
    if kcache is not None:
        assert kcache.dtype == np.float16 and kcache.flags.c_contiguous
        kc_ptr = kcache.ctypes.data_as(_u16p)
    lib().orc_kvwrite(cp, cc.shape[0], wp, np_, R, D - R, kc_ptr, int(kidx), int(pos),
                      rp["eps"], rp["freq_base"], rp["freq_scale"], rp["ext_factor"],
                      rp["attn_factor"], rp["beta_fast"], rp["beta_slow"], int(rp["n_ctx_orig"]),
                      numerics, kcur.ctypes.data_as(_f32p))
    return kcur


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
        _ref.ref_mla_create_typed.restype = vp
        _ref.ref_mla_create_typed.argtypes = _ref.ref_mla_create.argtypes + [ctypes.c_int]
        _ref.ref_mla_set_inputs.argtypes = [vp, _f32p, vp, _u16p, _f32p, vp]
        cf, ci = ctypes.c_float, ctypes.c_int
        _ref.ref_kvw_create.restype = vp
        _ref.ref_kvw_create.argtypes = [ci, ci, ci, ctypes.c_int64] + [cf] * 7 + [ci, ci]
        _ref.ref_kvw_set_inputs.argtypes = [vp, _f32p, vp, _f32p, _u16p, ctypes.c_int64,
                                            ctypes.c_int32]
        _ref.ref_kvw_compute.argtypes = [vp]
        _ref.ref_kvw_compute.restype = ctypes.c_int
        _ref.ref_kvw_get_outputs.argtypes = [vp, _f32p, _u16p]
        _ref.ref_kvw_destroy.argtypes = [vp]
        _ref.ref_mla_compute.argtypes = [vp]
        _ref.ref_mla_compute.restype = ctypes.c_int
        _ref.ref_mla_get_outputs.argtypes = [vp, _f32p, _f32p, _f32p, _f32p]
        _ref.ref_mla_n_nodes.argtypes = [vp]
        _ref.ref_mla_n_nodes.restype = ctypes.c_int
    return _ref


class RefMLA:
    """The reference's unfused MLA decode graph on its own ggml-cpu backend (built once)."""

    GGML_F16, GGML_Q8_0 = 1, 8

    def __init__(self, H, nope, rope, R, V, N, scale, n_threads=None, weights="f16"):
        """weights: "f16" (BASELINE) or "q8_0" (the Mistral-Small-4 geometry; w_uk / w_uv are
        then passed as Q8_0 bytes)."""
        self.H, self.nope, self.rope, self.R, self.V, self.N = H, nope, rope, R, V, N
        self.n_threads = n_threads or os.cpu_count() or 1
        self.q8 = weights == "q8_0"
        wt = self.GGML_Q8_0 if self.q8 else self.GGML_F16
        self._h = ref_lib().ref_mla_create_typed(H, nope, rope, R, V, N, float(scale),
                                                 self.n_threads, wt)
        if not self._h:
            raise RuntimeError("ref_mla_create failed")
        self._keep = []

    def set_inputs(self, q=None, w_uk=None, kc=None, mask=None, w_uv=None):
        wconv = _u8 if self.q8 else _f16
        keep, args = [], []
        for a, conv in ((q, _f32), (w_uk, wconv), (kc, _f16), (mask, _f32), (w_uv, wconv)):
            if a is None:
                args.append(None)
            else:
                arr, ptr = conv(a)
                keep.append(arr)        # alive until the copy below has run
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


class RefKVWrite:
    """The reference's unfused KV-write sequence (m1_layer.cpp:422-460) on its own ggml-cpu."""

    def __init__(self, n_in, R, rope, N, rp, n_threads=None):
        self.n_in, self.R, self.rope, self.N = n_in, R, rope, N
        self.D = R + rope
        self._h = ref_lib().ref_kvw_create(n_in, R, rope, N, rp["eps"], rp["freq_base"],
                                           rp["freq_scale"], rp["ext_factor"], rp["attn_factor"],
                                           rp["beta_fast"], rp["beta_slow"], int(rp["n_ctx_orig"]),
                                           n_threads or os.cpu_count() or 1)
        if not self._h:
            raise RuntimeError("ref_kvw_create failed")

    def run(self, cur, w_q8, norm_w, kcache, kidx, pos):
        """Returns (Kcur f32 (D,), the cache f16 (N, D) after the write)."""
        c, cp = _f32(cur)
        w, wp = _u8(w_q8)
        nw, nwp = _f32(norm_w)
        kc, kcp = _f16(kcache)
        ref_lib().ref_kvw_set_inputs(self._h, cp, ctypes.cast(wp, ctypes.c_void_p), nwp, kcp,
                                     int(kidx), int(pos))
        rc = ref_lib().ref_kvw_compute(self._h)
        if rc != 0:
            raise RuntimeError(f"ggml_graph_compute returned {rc}")
        kcur = np.empty(self.D, np.float32)
        out = np.empty((self.N, self.D), np.float16)
        ref_lib().ref_kvw_get_outputs(self._h, kcur.ctypes.data_as(_f32p),
                                      out.ctypes.data_as(_u16p))
        return kcur, out

    def close(self):
        if self._h:
            ref_lib().ref_kvw_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
