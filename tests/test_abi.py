"""CPU tests of the C ABI and the host-side mirror: the library loads and exports every symbol
include/m4b.h declares, contract checks reject bad operands before any CUDA call, supports_op
mirrors the reference's per-op contract, and the tri-state flag resolves as the engine does.
No test here launches anything."""
import ctypes
import os
import re

import pytest
import torch

from aubier_b200 import m4
from aubier_b200.shard import kv_slabs, lpt_assign, rank_loads

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "m4b.h")
FAKE = 0x7F0000000000   # a 4 KB-aligned non-null address; never dereferenced by these tests


def declared_symbols():
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"M4B_API\s+[\w\s\*]+?\b(m4b_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 13
    lib = ctypes.CDLL(m4.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/m4b.h but not exported"


def test_abi_version_and_strerror():
    assert m4.abi_version() == 1
    for code in range(7):
        assert m4.strerror(code).startswith("ok") or m4.strerror(code).startswith("m4b")
    assert "unknown" in m4.strerror(99)


def T(type_id, ne, nb, addr=FAKE):
    t = m4.Tensor()
    t.data = addr
    t.type = type_id
    for i in range(4):
        t.ne[i] = ne[i]
        t.nb[i] = nb[i]
    return t


def contiguous(type_id, ne, esz):
    nb = [esz]
    for i in range(1, 4):
        nb.append(nb[-1] * ne[i - 1])
    return T(type_id, ne, nb)


N = 1000
WUK = contiguous(m4.F16, [128, 512, 32, 1], 2)
QNOPE = T(m4.F32, [128, 32, 1, 1], [4, 768, 768 * 32, 768 * 32])
QABS = contiguous(m4.F32, [512, 32, 1, 1], 4)
KC = contiguous(m4.F16, [576, N, 1, 1], 2)
QCUR = contiguous(m4.F32, [576, 32, 1, 1], 4)
MASK = contiguous(m4.F32, [N, 1, 1, 1], 4)
ATTN = T(m4.F32, [512, 1, 32, 1], [4, 2048, 2048, 2048 * 32])
WUV = contiguous(m4.F16, [512, 128, 32, 1], 2)
OUT = T(m4.F32, [128, 1, 32, 1], [4, 512, 512, 512 * 32])
PARTS = contiguous(m4.F32, [516, 32, 7, 1], 4)


def test_supports_op_accepts_the_baseline_contract():
    assert m4.supports_op(m4.OP_WKB, [WUK, QNOPE], QABS)
    assert m4.supports_op(m4.OP_KQKV, [KC, QCUR, MASK], ATTN)
    assert m4.supports_op(m4.OP_KQKV, [KC, QCUR], ATTN)              # mask optional
    assert m4.supports_op(m4.OP_PHASE, [WUV, ATTN], OUT, [1] + [0] * 15)
    assert m4.supports_op(m4.OP_PHASE, [WUV, PARTS], OUT, [2] + [0] * 15)
    assert m4.supports_op(m4.OP_PHASE, [WUV, PARTS], contiguous(m4.F32, [516, 32, 1, 1], 4),
                          [3] + [0] * 15)
    assert not m4.supports_op(m4.OP_PHASE, [WUV, PARTS], contiguous(m4.F32, [516, 32, 2, 1], 4),
                              [3] + [0] * 15)


def test_supports_op_rejects_contract_violations():
    bad_kc = contiguous(m4.F32, [576, N, 1, 1], 4)                     # cache must be F16
    assert not m4.supports_op(m4.OP_KQKV, [bad_kc, QCUR, MASK], ATTN)
    bad_mask = contiguous(m4.F32, [N - 1, 1, 1, 1], 4)                 # mask ne0 != n_kv
    assert not m4.supports_op(m4.OP_KQKV, [KC, QCUR, bad_mask], ATTN)
    odd_row = T(m4.F16, [576, N, 1, 1], [2, 1160, 1160 * N, 1160 * N])  # row not 16-B multiple
    assert not m4.supports_op(m4.OP_KQKV, [odd_row, QCUR, MASK], ATTN)
    unaligned = contiguous(m4.F16, [576, N, 1, 1], 2)
    unaligned.data = FAKE + 8                                          # TMA needs 16-B alignment
    assert not m4.supports_op(m4.OP_KQKV, [unaligned, QCUR, MASK], ATTN)
    assert not m4.supports_op(m4.OP_WKB, [WUK, contiguous(m4.F32, [128, 16, 1, 1], 4)], QABS)
    assert not m4.supports_op(m4.OP_PHASE, [WUV, ATTN], OUT, [3] + [0] * 15)   # unknown phase
    assert not m4.supports_op(m4.OP_PHASE, [WUV, ATTN], OUT, [0] + [0] * 15)   # kvwrite operands
    assert not m4.supports_op(m4.OP_WKB, [Q8_WUK, QNOPE], QABS)        # Q8_0 W_UK, BASELINE q
    assert not m4.supports_op(m4.OP_KQKV, [KC_M, QCUR, MASK_M], ATTN)  # mixed geometries
    bad_kvw = _kvwrite_srcs()
    bad_kvw[1] = contiguous(m4.Q8_0, [4096, 320, 1, 1], 34)            # ggml strides of Q8_0
    bad_kvw[1].nb[0] = 32
    assert not m4.supports_op(m4.OP_PHASE, bad_kvw, KCUR, KVW_PARAMS)
    assert not m4.supports_op(m4.OP_PHASE, _kvwrite_srcs(), KCUR, [0] + [0] * 7 + [32, 8192] + [0] * 6)


# Mistral-Small-4 geometry (engine/m1_layer.h:47-55): latent 256, row 320, Q8_0 weights
def q8(ne):
    """A packed Q8_0 tensor: ne[0] values per row in 34-byte blocks of 32."""
    row = ne[0] // 32 * 34
    return T(m4.Q8_0, ne, [34, row, row * ne[1], row * ne[1] * ne[2]])


Q8_WUK = q8([64, 256, 32, 1])
Q8_WUV = q8([256, 128, 32, 1])
QNOPE_M = T(m4.F32, [64, 32, 1, 1], [4, 512, 512 * 32, 512 * 32])     # head stride 128 floats
QABS_M = contiguous(m4.F32, [256, 32, 1, 1], 4)
KC_M = contiguous(m4.F16, [320, N, 1, 1], 2)
QCUR_M = contiguous(m4.F32, [320, 32, 1, 1], 4)
MASK_M = MASK
ATTN_M = T(m4.F32, [256, 1, 32, 1], [4, 1024, 1024, 1024 * 32])
PARTS_M = contiguous(m4.F32, [260, 32, 7, 1], 4)
KCUR = contiguous(m4.F32, [320, 1, 1, 1], 4)
KVW_PARAMS = [0, 0, 0, 0, 0, 0, 0, 0, 64, 8192] + [0] * 6


def _kvwrite_srcs():
    return [contiguous(m4.F32, [4096, 1, 1, 1], 4), q8([4096, 320, 1, 1]),
            contiguous(m4.F32, [256, 1, 1, 1], 4), contiguous(m4.F16, [320, N, 1, 1], 2),
            contiguous(m4.I64, [1, 1, 1, 1], 8), contiguous(m4.I32, [1, 1, 1, 1], 4)]


def test_supports_op_accepts_the_mistral_contract():
    assert m4.supports_op(m4.OP_WKB, [Q8_WUK, QNOPE_M], QABS_M)
    assert m4.supports_op(m4.OP_KQKV, [KC_M, QCUR_M, MASK_M], ATTN_M)
    assert m4.supports_op(m4.OP_PHASE, [Q8_WUV, ATTN_M], OUT, [1] + [0] * 15)
    assert m4.supports_op(m4.OP_PHASE, [Q8_WUV, PARTS_M], OUT, [2] + [0] * 15)
    assert m4.supports_op(m4.OP_PHASE, [m4.Tensor(), PARTS_M], contiguous(m4.F32, [260, 32, 1, 1], 4),
                          [3] + [0] * 15)
    assert m4.supports_op(m4.OP_PHASE, _kvwrite_srcs(), KCUR, KVW_PARAMS)
    assert not m4.supports_op(m4.OP_PHASE, [Q8_WUV, PARTS], OUT, [2] + [0] * 15)   # 516 records


def _call(fn, args):
    return fn(ctypes.byref(args), ctypes.c_void_p(0))


def test_entry_points_refuse_bad_operands_before_any_cuda_call():
    lib = m4.lib()
    a = m4.KqkvArgs()
    a.src0, a.src1, a.src2, a.dst = contiguous(m4.F32, [576, N, 1, 1], 4), QCUR, MASK, ATTN
    a.kq_scale = 0.07
    assert _call(lib.m4b_kqkv, a) == m4.EINVAL
    a.src0 = KC
    a.kq_scale = float("nan")
    assert _call(lib.m4b_kqkv, a) == m4.EINVAL
    w = m4.WkbArgs()
    w.src0, w.src1, w.dst = WUK, QNOPE, contiguous(m4.F32, [256, 32, 1, 1], 4)
    assert _call(lib.m4b_wkb, w) == m4.EINVAL
    p = m4.PhaseArgs()
    p.src[0], p.src[1], p.dst = WUV, ATTN, OUT
    p.op_params[0] = 7
    assert _call(lib.m4b_phase, p) == m4.EINVAL
    p.op_params[0] = 0                       # KV-write with W_UV / attn operands: malformed
    assert _call(lib.m4b_phase, p) == m4.EINVAL
    kv = m4.PhaseArgs()                      # a KV-write over a BASELINE-row cache: no such op
    kv.src[3] = KC
    assert _call(lib.m4b_phase, kv) == m4.ENOTSUP
    assert lib.m4b_phase_kvwrite_slab(None, 0, None) == m4.EINVAL
    assert lib.m4b_phase_kvwrite_slab(ctypes.byref(kv), -1, None) == m4.EINVAL
    p.op_params[0] = 1                       # the slab entry is the KV-write only
    assert lib.m4b_phase_kvwrite_slab(ctypes.byref(p), 0, None) == m4.EINVAL
    assert lib.m4b_kqkv(None, None) == m4.EINVAL


def test_static_scratch_entry_refuses_bad_operands_before_any_cuda_call():
    """m4b_kqkv_static_scratch validates like m4b_kqkv before it touches the runtime (no device
    check, no symbol lookup, no launch)."""
    lib = m4.lib()
    fn = lib.m4b_kqkv_static_scratch
    fn.argtypes = [ctypes.POINTER(m4.KqkvArgs), ctypes.c_void_p]
    assert lib.m4b_kqkv_static_scratch(None, None) == m4.EINVAL
    a = m4.KqkvArgs()
    a.src0, a.src1, a.src2, a.dst = KC, QCUR, MASK, ATTN
    a.kq_scale = 0.07
    a.dst = T(m4.F32, [256, 1, 32, 1], [4, 1024, 1024, 1024 * 32])   # latent 256 vs a 576 row
    assert _call(fn, a) == m4.EINVAL
    a.dst = ATTN
    a.src2 = contiguous(m4.F32, [N - 1, 1, 1, 1], 4)                 # mask shorter than n_kv
    assert _call(fn, a) == m4.EINVAL
    a.src2 = MASK
    a.src0 = contiguous(m4.F32, [576, N, 1, 1], 4)                   # f32 cache
    assert _call(fn, a) == m4.EINVAL
    a.src0 = KC
    a.kq_scale = float("nan")
    assert _call(fn, a) == m4.EINVAL
    a.kq_scale = 0.07
    a.dst = T(m4.F32, [512, 1, 32, 1], [4, 2048, 2048, 2048 * 32], addr=0)   # no output
    assert _call(fn, a) == m4.EINVAL


def test_wkb_qcat_needs_room_for_the_rope_half():
    """M4B_FLAG_QCAT copies 64 rope values behind q_nope into dst behind the latent: both head rows
    must be long enough, checked before any CUDA call (without a GPU a valid call then fails on the
    device check, not on the arguments)."""
    lib = m4.lib()
    w = m4.WkbArgs()
    w.src0, w.flags = WUK, m4.FLAG_QCAT
    w.src1, w.dst = QNOPE, QABS                      # dst head stride 512 floats: no room
    assert _call(lib.m4b_wkb, w) == m4.EINVAL
    w.src1 = contiguous(m4.F32, [128, 32, 1, 1], 4)   # q_nope alone: no rope values behind it
    w.dst = T(m4.F32, [512, 32, 1, 1], [4, 2304, 2304 * 32, 2304 * 32])
    assert _call(lib.m4b_wkb, w) == m4.EINVAL
    w.src1 = QNOPE                                    # head rows of 192 and 576 floats: accepted
    assert _call(lib.m4b_wkb, w) != m4.EINVAL


def test_exchange_refuses_bad_arguments_before_any_cuda_call():
    from aubier_b200 import exchange  # noqa: F401  (declares the argument types)
    lib = m4.lib()
    h = ctypes.c_void_p()
    for world, rank in ((0, 0), (9, 0), (2, 2), (2, -1)):
        assert lib.m4b_exchange_create(world, rank, ctypes.byref(h)) == m4.EINVAL
    assert lib.m4b_exchange_create(2, 0, None) == m4.EINVAL
    assert lib.m4b_exchange_detach(None) == m4.OK
    assert lib.m4b_exchange_destroy(None) == m4.OK
    assert lib.m4b_exchange_ipc_handle(None, None) == m4.EINVAL
    assert lib.m4b_exchange_open(None, None) == m4.EINVAL
    assert lib.m4b_exchange_open_local(None, None, 0) == m4.EINVAL
    p = m4.PhaseArgs()
    assert lib.m4b_exchange_publish(None, ctypes.byref(p), None) == m4.EINVAL
    assert lib.m4b_exchange_combine_wvb(None, ctypes.byref(p), None) == m4.EINVAL


def test_scratch_sizes():
    assert m4.kqkv_scratch_bytes(262144) == 148 * 32 * 516 * 4
    assert m4.kqkv_scratch_bytes(4096) == 32 * 32 * 516 * 4
    assert m4.kqkv_scratch_bytes(1) == 32 * 516 * 4
    assert m4.lib().m4b_phase_scratch_bytes(2) == 32 * 512 * 4
    assert m4.lib().m4b_kqkv_max_splits() == 148


@pytest.mark.parametrize("flag,gpu,nt,ragged,want", [
    (-1, 1, 1, 0, True), (-1, 0, 1, 0, False), (0, 1, 1, 0, False), (1, 1, 1, 0, True),
    (-1, 1, 4, 0, False), (-1, 1, 4, 1, True), (0, 0, 1, 0, False)])
def test_tristate_flag_resolution(flag, gpu, nt, ragged, want):
    assert m4.resolve_flag(flag, gpu, nt, ragged) is want


@pytest.mark.parametrize("flag,gpu,nt", [(1, 0, 1), (1, 1, 4), (2, 1, 1), (-2, 1, 1)])
def test_tristate_flag_refusals(flag, gpu, nt):
    with pytest.raises(m4.M4Error) as e:
        m4.resolve_flag(flag, gpu, nt)
    assert e.value.code == m4.EINVAL


def test_host_tensors_have_no_cpu_handler():
    kc = torch.zeros(16, 576, dtype=torch.float16)
    q = torch.zeros(32, 576)
    with pytest.raises(m4.M4Error, match="no CPU handler"):
        m4.kqkv(kc, q, None, 0.07)
    with pytest.raises(m4.M4Error, match="no CPU handler"):
        m4.wkb(torch.zeros(32, 512, 128, dtype=torch.float16), torch.zeros(32, 192)[:, :128])


def test_kv_slabs_cover_the_context():
    for n, w in [(262144, 1), (262144, 2), (262144, 8), (1000, 3), (5, 4), (0, 2)]:
        slabs = kv_slabs(n, w)
        assert len(slabs) == w and slabs[0][0] == 0 and slabs[-1][1] == n
        for (b0, e0), (b1, e1) in zip(slabs, slabs[1:]):
            assert e0 == b1
        tiles = [(e - b + 127) // 128 for b, e in slabs]
        assert max(tiles) - min(tiles) <= 1          # balanced to one 128-key tile


def test_lpt_balances_ragged_batches():
    lengths = [512, 65536, 4000, 30000, 777, 12345, 65000, 2048, 9999, 40000, 600, 31000,
               8000, 15000, 50000, 1234]
    for w in (1, 2, 4, 8):
        a = lpt_assign(lengths, w)
        assert sorted(i for r in a for i in r) == list(range(len(lengths)))
        loads = rank_loads(lengths, a)
        # LPT bound: makespan <= 4/3 OPT; OPT >= max(total / w, max length)
        opt_lb = max(sum(lengths) / w, max(lengths))
        assert max(loads) <= 4 / 3 * opt_lb + 1
    assert lpt_assign(lengths, 4) == lpt_assign(list(lengths), 4)   # deterministic
