"""Host-side mirror of aubier's M4 op API, over the C ABI of ``libm4b.so`` (include/m4b.h).

The reference exposes the path as ggml ops built by ``ggml_m4_wkb``, ``ggml_m4_kqkv``,
``ggml_m4_phase_kvwrite`` and ``ggml_m4_phase_wvb`` (vendor/llama.cpp/ggml/src/ggml.c:3398-3540)
and run by ggml-cuda's ``ggml_cuda_m4_*`` launchers.  This module keeps those names, argument
meanings and error behaviour for torch-allocated device tensors:

* shapes are the ggml shapes read right to left (ggml ne[] = reversed torch shape): W_UK is
  (32, 512, 128) = ggml [128, 512, 32]; the KV cache is (N, 576) = ggml [576, N]; the attention
  output is (32, 512) = ggml [512, 1, 32];
* a contract violation raises ``M4Error`` (the reference's GGML_ASSERT); a host tensor raises
  ``M4Error`` as well -- the ops have no CPU handler (ggml-cpu.c:2064-2082 aborts);
* every call is a plain launch on the current torch CUDA stream: no synchronisation, no
  allocation inside the library (outputs / scratch are allocated here, by torch, when the caller
  does not pass them), so it can be captured in a CUDA graph.

There is no fallback: if ``libm4b.so`` is missing, importing this module fails.
"""
from __future__ import annotations

import ctypes
import math
import os
from ctypes import c_float, c_int, c_int32, c_int64, c_uint32, c_uint64, c_void_p

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libm4b.so")

# geometry of the measured shape (BASELINE); engine/m1_layer.h:47-55 has the Mistral constants
HEADS, NOPE, ROPE, LATENT, VHEAD = 32, 128, 64, 512, 128
M_NOPE, M_LATENT = 64, 256   # the Mistral-Small-4 geometry (Q8_0 weights, KV row 320)
Q8_BLOCK = 34                # ggml block_q8_0: f16 scale + 32 int8
KROW = LATENT + ROPE
PART_STRIDE = LATENT + 4   # o[512], m (log2 units), l, 2 pad
TILE_KEYS = 128            # keys per KQKV tile: splits are balanced over ceil(N / 128) tiles

F32, F16, Q8_0, I32, I64 = 0, 1, 8, 26, 27
FLAG_PDL, FLAG_KV_STATIC, FLAG_QCAT, FLAG_EARLY_RELEASE = 1, 2, 4, 8
OK, EINVAL, ESCRATCH, ECUDA, EDEVICE, ENOTSUP, ETIMEOUT = range(7)

OP_WKB, OP_KQKV, OP_PHASE = 0, 1, 2
PHASE_KVWRITE, PHASE_WVB, PHASE_COMBINE_WVB, PHASE_MERGE = 0, 1, 2, 3


class Tensor(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("type", c_int32), ("_pad", c_int32),
                ("ne", c_int64 * 4), ("nb", c_uint64 * 4)]


class WkbArgs(ctypes.Structure):
    _fields_ = [("src0", Tensor), ("src1", Tensor), ("dst", Tensor), ("flags", c_uint32)]


class KqkvArgs(ctypes.Structure):
    _fields_ = [("src0", Tensor), ("src1", Tensor), ("src2", Tensor), ("dst", Tensor),
                ("kq_scale", c_float), ("flags", c_uint32), ("scratch", c_void_p),
                ("scratch_bytes", c_uint64)]


class PhaseArgs(ctypes.Structure):
    _fields_ = [("src", Tensor * 6), ("dst", Tensor), ("op_params", c_int32 * 16),
                ("flags", c_uint32), ("scratch", c_void_p), ("scratch_bytes", c_uint64)]


class RaggedArgs(ctypes.Structure):
    _fields_ = [("kcache", Tensor), ("q", Tensor), ("seq_base", Tensor), ("seq_len", Tensor),
                ("dst", Tensor), ("kq_scale", c_float), ("flags", c_uint32),
                ("scratch", c_void_p), ("scratch_bytes", c_uint64)]


class M4Error(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {strerror(code)} (code {code})")


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run aubier_b200.build.build_library() "
                          "(the M4 ops have no CPU or Python fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name in ("m4b_wkb",):
        getattr(lib, name).argtypes = [ctypes.POINTER(WkbArgs), c_void_p]
    for name in ("m4b_kqkv", "m4b_kqkv_partials"):
        getattr(lib, name).argtypes = [ctypes.POINTER(KqkvArgs), c_void_p]
    lib.m4b_phase.argtypes = [ctypes.POINTER(PhaseArgs), c_void_p]
    lib.m4b_phase_kvwrite_slab.argtypes = [ctypes.POINTER(PhaseArgs), c_int64, c_void_p]
    lib.m4b_kqkv_ragged.argtypes = [ctypes.POINTER(RaggedArgs), c_void_p]
    lib.m4b_kqkv_ragged_scratch_bytes.argtypes = [c_int64]
    lib.m4b_kqkv_ragged_scratch_bytes.restype = c_uint64
    lib.m4b_kqkv_scratch_bytes.argtypes = [c_int, c_int64]
    lib.m4b_kqkv_scratch_bytes.restype = c_uint64
    lib.m4b_phase_scratch_bytes.argtypes = [c_int]
    lib.m4b_phase_scratch_bytes.restype = c_uint64
    lib.m4b_kqkv_default_splits.argtypes = [c_int64]
    lib.m4b_supports_op.argtypes = [c_int, ctypes.POINTER(Tensor), c_int, ctypes.POINTER(Tensor),
                                    ctypes.POINTER(c_int32)]
    lib.m4b_resolve_flag.argtypes = [c_int, c_int, c_int, c_int, ctypes.POINTER(c_int)]
    lib.m4b_device_status.argtypes = [c_void_p]
    lib.m4b_set_wait_limit_cycles.argtypes = [c_int64]
    lib.m4b_last_cuda_error.argtypes = [ctypes.POINTER(ctypes.c_char_p)]
    lib.m4b_strerror.argtypes = [c_int]
    lib.m4b_strerror.restype = ctypes.c_char_p
    return lib


_lib = _load()


def lib():
    return _lib


def strerror(code: int) -> str:
    return _lib.m4b_strerror(code).decode()


def abi_version() -> int:
    return _lib.m4b_abi_version()


# ---------------------------------------------------------------------------------------------
# descriptors
# ---------------------------------------------------------------------------------------------
_DT = {torch.float32: F32, torch.float16: F16, torch.int32: I32, torch.int64: I64,
       torch.uint8: Q8_0}


def gtensor(t: torch.Tensor | None, ne, nb=None, type_id=None) -> Tensor:
    """An m4b_tensor for a view of ``t`` with ggml ``ne`` (innermost first) and byte strides
    ``nb`` (default: the torch strides of the reversed shape, trailing dims packed)."""
    g = Tensor()
    if t is None:
        return g
    g.data = t.data_ptr()
    g.type = _DT[t.dtype] if type_id is None else type_id
    ne = list(ne) + [1] * (4 - len(ne))
    if nb is None:
        es = t.element_size()
        st = [s * es for s in reversed(t.stride())]
        nb = st + [0] * (4 - len(st))
        for i in range(len(st), 4):
            nb[i] = nb[i - 1] * ne[i - 1]
    for i in range(4):
        g.ne[i] = int(ne[i])
        g.nb[i] = int(nb[i])
    return g


def _rows_desc(t: torch.Tensor, inner: int, rows: int) -> Tensor:
    """ggml [inner, rows] view of a 2-D (rows, >=inner) tensor with unit inner stride."""
    if t.dim() != 2 or t.shape[0] != rows or t.shape[1] != inner or t.stride(1) != 1:
        raise M4Error(EINVAL, f"expected a ({rows}, {inner}) row view, got {tuple(t.shape)} "
                              f"strides {tuple(t.stride())}")
    es = t.element_size()
    rs = t.stride(0) * es
    return gtensor(t, [inner, rows, 1, 1], [es, rs, rs * rows, rs * rows])


def _heads_desc(t: torch.Tensor, inner: int) -> Tensor:
    """ggml [inner, 1, heads] view of a 2-D (heads, >=inner) tensor (the g_kqv / kqv_mla shape)."""
    if t.dim() != 2 or t.shape[1] != inner or t.stride(1) != 1:
        raise M4Error(EINVAL, f"expected a (heads, {inner}) view, got {tuple(t.shape)}")
    es = t.element_size()
    hs = t.stride(0) * es
    return gtensor(t, [inner, 1, t.shape[0], 1], [es, inner * es, hs, hs * t.shape[0]])


def weight_desc(w: torch.Tensor) -> Tensor:
    """A weight tensor: f16 (heads, rows, K) -> F16 [K, rows, heads]; uint8 Q8_0 bytes
    (heads, rows, K / 32 * 34) or (rows, K / 32 * 34) -> Q8_0 [K, rows, heads]."""
    if w.dtype == torch.uint8:
        if w.shape[-1] % Q8_BLOCK or not w.is_contiguous():
            raise M4Error(EINVAL, "Q8_0 weights: contiguous uint8 rows of 34-byte blocks")
        K = w.shape[-1] // Q8_BLOCK * 32
        rows = w.shape[-2]
        heads = w.shape[0] if w.dim() == 3 else 1
        row = w.shape[-1]
        return gtensor(w, [K, rows, heads, 1], [Q8_BLOCK, row, row * rows, row * rows * heads],
                       type_id=Q8_0)
    return gtensor(w, list(reversed(w.shape)))


def latent_of(kcache: torch.Tensor) -> int:
    """The latent width R of a KV cache (rows of R + 64)."""
    return kcache.shape[-1] - ROPE


def _tokens_desc(t: torch.Tensor, inner: int, token_dim: int) -> Tensor:
    """ggml view of a (T, heads, >=inner) tensor with unit inner stride: [inner, heads, T] when
    token_dim == 2 (q, q_abs), [inner, T, heads] when token_dim == 1 (g_kqv, W_UV in/out)."""
    if t.dim() != 3 or t.shape[2] != inner or t.stride(2) != 1:
        raise M4Error(EINVAL, f"expected a (tokens, heads, {inner}) view, got {tuple(t.shape)}")
    es = t.element_size()
    T, Hh = t.shape[0], t.shape[1]
    ts, hs = t.stride(0) * es, t.stride(1) * es
    if token_dim == 2:
        return gtensor(t, [inner, Hh, T, 1], [es, hs, ts, ts * T])
    return gtensor(t, [inner, T, Hh, 1], [es, ts, hs, hs * Hh])


def _need_cuda(name: str, *ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise M4Error(EINVAL, f"{name} has no CPU handler (GPU-only op); got a host tensor")


def _stream():
    return c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(rc: int, what: str):
    if rc != OK:
        if rc == ECUDA:   # name the CUDA error behind it
            name = ctypes.c_char_p()
            code = _lib.m4b_last_cuda_error(ctypes.byref(name))
            if code:
                what = f"{what} [{(name.value or b'?').decode()} ({code})]"
        raise M4Error(rc, what)


# ---------------------------------------------------------------------------------------------
# ops
# ---------------------------------------------------------------------------------------------
def wkb(w_uk: torch.Tensor, q_nope: torch.Tensor, out: torch.Tensor | None = None,
        flags: int = 0) -> torch.Tensor:
    """GGML_OP_M4_WKB: out[h] = W_UK[h] . q_nope[h].  w_uk f16 (32, 512, 128) contiguous;
    q_nope f32 (32, 128) with any row stride; out f32 (32, 512), any row stride (may be a view
    of Qcur)."""
    _need_cuda("GGML_OP_M4_WKB", w_uk, q_nope, out)
    R = w_uk.shape[1]
    if out is None:
        shape = (HEADS, R) if q_nope.dim() == 2 else (q_nope.shape[0], HEADS, R)
        out = torch.empty(shape, device=w_uk.device, dtype=torch.float32)
    a = WkbArgs()
    a.src0 = weight_desc(w_uk)
    if q_nope.dim() == 3:   # a batch of tokens (T, 32, 128) -> (T, 32, 512)
        a.src1 = _tokens_desc(q_nope, q_nope.shape[2], 2)
        a.dst = _tokens_desc(out, out.shape[2], 2)
    else:
        a.src1 = _rows_desc(q_nope, q_nope.shape[1], q_nope.shape[0])
        a.dst = _rows_desc(out, out.shape[1], out.shape[0])
    a.flags = flags
    _check(_lib.m4b_wkb(ctypes.byref(a), _stream()), "m4b_wkb")
    return out


def kqkv_scratch_bytes(n_kv: int, latent: int = LATENT) -> int:
    return int(_lib.m4b_kqkv_scratch_bytes(0 if latent == LATENT else 1, n_kv))


def default_splits(n_kv: int) -> int:
    return int(_lib.m4b_kqkv_default_splits(n_kv))


def _kqkv_args(kcache, q, mask, kq_scale, flags) -> KqkvArgs:
    a = KqkvArgs()
    a.src0 = _rows_desc(kcache, kcache.shape[1], kcache.shape[0])
    a.src1 = _rows_desc(q, q.shape[1], q.shape[0])
    if mask is not None:
        if mask.dim() != 1 or mask.stride(0) != 1:
            raise M4Error(EINVAL, "mask must be a contiguous 1-D f32 tensor of n_kv elements")
        a.src2 = gtensor(mask, [mask.shape[0], 1, 1, 1])
    a.kq_scale = float(kq_scale)
    a.flags = flags
    return a


def kqkv(kcache: torch.Tensor, q: torch.Tensor, mask: torch.Tensor | None, kq_scale: float,
         out: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
         flags: int = 0) -> torch.Tensor:
    """GGML_OP_M4_KQKV: softmax(K.q * kq_scale + mask) . V per head.  kcache f16 (N, 576) with
    any 16-byte-multiple row stride; q f32 (32, 576); mask f32 (N,) of 0/-inf or None;
    out f32 (32, 512).  ``scratch``: a byte tensor of at least kqkv_scratch_bytes(N)."""
    _need_cuda("GGML_OP_M4_KQKV", kcache, q, mask, out, scratch)
    R = latent_of(kcache)
    if out is None:
        out = torch.empty(HEADS, R, device=q.device, dtype=torch.float32)
    if scratch is None:
        scratch = torch.empty(max(kqkv_scratch_bytes(kcache.shape[0], R), 16), device=q.device,
                              dtype=torch.uint8)
    a = _kqkv_args(kcache, q, mask, kq_scale, flags)
    a.dst = _heads_desc(out, R)
    a.scratch = scratch.data_ptr()
    a.scratch_bytes = scratch.numel() * scratch.element_size()
    _check(_lib.m4b_kqkv(ctypes.byref(a), _stream()), "m4b_kqkv")
    return out


def kqkv_partials(kcache: torch.Tensor, q: torch.Tensor, mask: torch.Tensor | None,
                  kq_scale: float, splits: int | None = None, out: torch.Tensor | None = None,
                  flags: int = 0) -> torch.Tensor:
    """Split-K partial records (S, 32, R + 4): o[R], m (log2 units), l per (split, head)."""
    _need_cuda("GGML_OP_M4_KQKV", kcache, q, mask, out)
    P = latent_of(kcache) + 4
    if out is None:
        s = splits if splits is not None else default_splits(kcache.shape[0])
        out = torch.empty(s, HEADS, P, device=q.device, dtype=torch.float32)
    a = _kqkv_args(kcache, q, mask, kq_scale, flags)
    a.dst = gtensor(out, [P, HEADS, out.shape[0], 1])
    _check(_lib.m4b_kqkv_partials(ctypes.byref(a), _stream()), "m4b_kqkv_partials")
    return out


def kqkv_ragged_scratch_bytes(n_tokens: int) -> int:
    return int(_lib.m4b_kqkv_ragged_scratch_bytes(n_tokens))


def kqkv_ragged(kcache: torch.Tensor, q: torch.Tensor, seq_base: torch.Tensor,
                seq_len: torch.Tensor, kq_scale: float, out: torch.Tensor | None = None,
                scratch: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """Ragged batch KQKV (additive op): token t attends to cache rows
    [seq_base[t], seq_base[t] + seq_len[t]).  kcache f16 (R, 576); q f32 (T, 32, 576);
    seq_base / seq_len int32 (T,) on the device; out f32 (T, 32, 512)."""
    _need_cuda("m4b_kqkv_ragged", kcache, q, seq_base, seq_len, out, scratch)
    T = q.shape[0]
    R = latent_of(kcache)
    if out is None:
        out = torch.empty(T, HEADS, R, device=q.device, dtype=torch.float32)
    if scratch is None:
        scratch = torch.empty(max(kqkv_ragged_scratch_bytes(T), 16), device=q.device,
                              dtype=torch.uint8)
    a = RaggedArgs()
    a.kcache = _rows_desc(kcache, kcache.shape[1], kcache.shape[0])
    a.q = _tokens_desc(q, q.shape[2], 2)
    for name, t in (("seq_base", seq_base), ("seq_len", seq_len)):
        if t.dtype != torch.int32 or t.dim() != 1 or t.stride(0) != 1:
            raise M4Error(EINVAL, f"{name} must be a contiguous 1-D int32 tensor")
        setattr(a, name, gtensor(t, [t.shape[0], 1, 1, 1]))
    a.dst = _tokens_desc(out, R, 1)
    a.kq_scale = float(kq_scale)
    a.flags = flags
    a.scratch = scratch.data_ptr()
    a.scratch_bytes = scratch.numel() * scratch.element_size()
    _check(_lib.m4b_kqkv_ragged(ctypes.byref(a), _stream()), "m4b_kqkv_ragged")
    return out


def _phase(phase: int, srcs, dst: Tensor, flags: int, scratch=None) -> None:
    a = PhaseArgs()
    for i, s in enumerate(srcs):
        if s is not None:
            a.src[i] = s
    a.dst = dst
    a.op_params[0] = phase
    a.flags = flags
    if scratch is not None:
        a.scratch = scratch.data_ptr()
        a.scratch_bytes = scratch.numel() * scratch.element_size()
    _check(_lib.m4b_phase(ctypes.byref(a), _stream()), f"m4b_phase({phase})")


def phase_wvb(w_uv: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None,
              flags: int = 0) -> torch.Tensor:
    """GGML_OP_M4_PHASE selector 1: out[h] = W_UV[h] . x[h].  w_uv f16 (32, 128, 512) or Q8_0
    bytes (32, 128, 272); x f32 (32, R) (any row stride) or a token batch (T, 32, R);
    out f32 (32, 128) / (T, 32, 128)."""
    _need_cuda("GGML_OP_M4_PHASE", w_uv, x, out)
    R = x.shape[-1]
    if out is None:
        shape = (HEADS, VHEAD) if x.dim() == 2 else (x.shape[0], HEADS, VHEAD)
        out = torch.empty(shape, device=x.device, dtype=torch.float32)
    if x.dim() == 3:   # a batch of tokens (T, 32, R) -> (T, 32, 128)
        xd, od = _tokens_desc(x, R, 1), _tokens_desc(out, VHEAD, 1)
    else:
        xd, od = _heads_desc(x, R), _heads_desc(out, VHEAD)
    _phase(PHASE_WVB, [weight_desc(w_uv), xd], od, flags)
    return out


def phase_combine_wvb(w_uv: torch.Tensor, partials: torch.Tensor,
                      out: torch.Tensor | None = None, attn_out: torch.Tensor | None = None,
                      scratch: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """GGML_OP_M4_PHASE selector 2 (additive): merge (S, 32, R + 4) partial records, then W_UV.
    ``attn_out`` (32, R) optionally receives the merged attention output."""
    _need_cuda("GGML_OP_M4_PHASE", w_uv, partials, out, attn_out, scratch)
    P = partials.shape[-1]
    if out is None:
        out = torch.empty(HEADS, VHEAD, device=partials.device, dtype=torch.float32)
    if attn_out is None and scratch is None:
        scratch = torch.empty(int(_lib.m4b_phase_scratch_bytes(2)), device=partials.device,
                              dtype=torch.uint8)
    srcs = [weight_desc(w_uv), gtensor(partials, [P, HEADS, partials.shape[0], 1]),
            _heads_desc(attn_out, P - 4) if attn_out is not None else None]
    _phase(PHASE_COMBINE_WVB, srcs, _heads_desc(out, VHEAD), flags, scratch)
    return out


def phase_merge_records(partials: torch.Tensor, out: torch.Tensor | None = None,
                        flags: int = 0) -> torch.Tensor:
    """GGML_OP_M4_PHASE selector 3 (additive): merge (S, 32, R + 4) partial records into one
    unnormalised record per head, (1, 32, R + 4) -- the payload of the multi-GPU exchange."""
    _need_cuda("GGML_OP_M4_PHASE", partials, out)
    P = partials.shape[-1]
    if out is None:
        out = torch.empty(1, HEADS, P, device=partials.device, dtype=torch.float32)
    srcs = [None, gtensor(partials, [P, HEADS, partials.shape[0], 1])]
    _phase(PHASE_MERGE, srcs, gtensor(out, [P, HEADS, 1, 1]), flags)
    return out


def _f32_bits(x: float) -> int:
    import struct
    return struct.unpack("<i", struct.pack("<f", float(x)))[0]


# the engine's attention scalars for the Mistral-Small-4 geometry (engine/m1_layer.cpp:60-95,
# m1_layer.h:56-67): YaRN factor 128 over an 8192 original context
MISTRAL_ROPE = {"freq_base": 10000.0, "freq_scale": 1.0 / 128.0, "ext_factor": 1.0,
                "attn_factor": 1.0 / (1.0 + 0.1 * math.log(128.0)), "beta_fast": 32.0,
                "beta_slow": 1.0, "eps": 9.999999974752427e-07, "n_dims": 64,
                "n_ctx_orig": 8192}


def phase_kvwrite(cur: torch.Tensor, w_kva: torch.Tensor, norm_w: torch.Tensor,
                  kcache: torch.Tensor, kidx: torch.Tensor, pos: torch.Tensor,
                  rope: dict | None = None, out: torch.Tensor | None = None,
                  flags: int = 0, slab_base: int | None = None) -> torch.Tensor:
    """GGML_OP_M4_PHASE selector 0, the KV-write (Mistral-Small-4 geometry): Kcur = norm(W_kva .
    cur) with YaRN rope on the last 64 values, written as f16 into kcache row kidx[0] (in place).
    cur f32 (4096,); w_kva Q8_0 bytes (320, 4352); norm_w f32 (256,); kcache f16 (N, 320);
    kidx int64 (1,) and pos int32 (1,) on the device; rope: the rope / norm scalars (default the
    engine's, MISTRAL_ROPE).  Returns Kcur f32 (320,).
    slab_base (additive, m4b_phase_kvwrite_slab): kcache is this GPU's slab of a sharded cache,
    holding rows [slab_base, slab_base + N) of it, and kidx[0] indexes the whole cache: the row is
    written only if this slab holds it."""
    _need_cuda("GGML_OP_M4_PHASE", cur, w_kva, norm_w, kcache, kidx, pos, out)
    rp = dict(MISTRAL_ROPE, **(rope or {}))
    if out is None:
        out = torch.empty(320, device=cur.device, dtype=torch.float32)
    a = PhaseArgs()
    a.src[0] = gtensor(cur, [cur.shape[0], 1, 1, 1])
    a.src[1] = weight_desc(w_kva)
    a.src[2] = gtensor(norm_w, [norm_w.shape[0], 1, 1, 1])
    a.src[3] = _rows_desc(kcache, kcache.shape[1], kcache.shape[0])
    a.src[4] = gtensor(kidx, [1, 1, 1, 1])
    a.src[5] = gtensor(pos, [1, 1, 1, 1])
    a.dst = gtensor(out, [out.shape[0], 1, 1, 1])
    a.op_params[0] = PHASE_KVWRITE
    for i, k in enumerate(("freq_base", "freq_scale", "ext_factor", "attn_factor", "beta_fast",
                           "beta_slow", "eps"), start=1):
        a.op_params[i] = _f32_bits(rp[k])
    a.op_params[8] = int(rp["n_dims"])
    a.op_params[9] = int(rp["n_ctx_orig"])
    a.flags = flags
    if slab_base is None:
        _check(_lib.m4b_phase(ctypes.byref(a), _stream()), "m4b_phase(0)")
    else:
        _check(_lib.m4b_phase_kvwrite_slab(ctypes.byref(a), c_int64(int(slab_base)), _stream()),
               "m4b_phase_kvwrite_slab")
    return out


# ---------------------------------------------------------------------------------------------
# supports_op, the tri-state flag, device status
# ---------------------------------------------------------------------------------------------
def supports_op(op: int, srcs: list[Tensor], dst: Tensor, op_params=None) -> bool:
    arr = (Tensor * len(srcs))(*srcs)
    p = None
    if op_params is not None:
        p = (c_int32 * 16)(*op_params)
    return bool(_lib.m4b_supports_op(op, arr, len(srcs), ctypes.byref(dst), p))


def resolve_flag(flag: int, gpu_core: bool, nt: int = 1, ragged_ok: bool = False) -> bool:
    """LoopArgs::m4_* tri-state (-1 AUTO, 0 off, 1 explicit) -> on/off; raises M4Error for the
    combinations the reference engine refuses (explicit 1 without --gpu-core, or at nt > 1)."""
    en = c_int(0)
    _check(_lib.m4b_resolve_flag(int(flag), int(bool(gpu_core)), int(nt), int(bool(ragged_ok)),
                                 ctypes.byref(en)), "m4b_resolve_flag")
    return bool(en.value)


def device_status() -> int:
    """Synchronise the current stream and return (and clear) the device status word."""
    return int(_lib.m4b_device_status(_stream()))


def set_wait_limit_cycles(cycles: int) -> None:
    """How long the kernels' bounded waits last before giving up, in SM cycles, on the current
    device (<= 0 restores the default, about 1 s).  Synchronises the device: not capturable."""
    _check(_lib.m4b_set_wait_limit_cycles(c_int64(int(cycles))), "m4b_set_wait_limit_cycles")
