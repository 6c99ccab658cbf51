"""GPU parity of the Mistral-Small-4 geometry (engine/m1_layer.h:47-55): Q8_0 W_UK / W_UV with the
fused reference kernels' Q8_1 activation numerics, the 320-wide KV row (latent 256) on the same
tcgen05 KQKV pipeline, and PHASE selector 0, the KV-write (Q8_0 gemv + RMS norm + YaRN rope + f16
scatter at a device-resident row).

Checks against the oracle restatement in both numerics: FUSED (the reference's fused kernels,
m4-wkb.cu / m4-phase.cu; tight, same rounding points, different float association) and CPU (the
unfused CPU graph the reference's ggml-cpu runs; the north-star gate), and against the golden
fixtures the reference's own ggml-cpu produced (tests/golden/mistral_*, kvwrite_*).
"""
import json
import os

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, rel_to_max
from mla_inputs import (MISTRAL as G, MISTRAL_ROPE, make_kvwrite, make_layer_q8, normal,
                        packed_bases, window_mask)
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FUSED_TOL = 1e-5     # same quantization and rounding points as the fused reference; float order
# W_UV output downstream of a Q8 activation: an attention output that differs in its last bits
# (~1e-4, inside the 2e-3 gate) flips single int8 roundings of the Q8 activation, each moving a
# block's contribution by d = amax/127; the reference documents the same for its own fused ops
# (m4-phase.cu:35-40: "never output equality").  Each stage is gated on the reference's own input
# to it (2e-3), and the end to end output of the chain is held to this bound.
Q8_CHAIN_TOL = 1e-2


@pytest.fixture(scope="module")
def m4():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from aubier_b200 import m4 as mod
    return mod


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


# ------------------------------------------------------------------------------------- WKB Q8
def test_wkb_q8_matches_fused_and_cpu_numerics(m4):
    q, w_uk, _, _ = make_layer_q8(31, 1)
    qd = dev(q)                                # (32, 128): the engine's head stride of 128 floats
    got = host(m4.wkb(dev(w_uk), qd[:, :G.nope]))
    assert got.shape == (G.H, G.R)
    assert rel_to_max(got, O.wkb_q8(w_uk, q, G.nope, G.R, O.FUSED)) <= FUSED_TOL
    assert rel_to_max(got, O.wkb_q8(w_uk, q, G.nope, G.R, O.CPU)) <= ATTN_TOL


def test_wkb_q8_token_batch_and_zero_block(m4):
    _, w_uk, _, _ = make_layer_q8(32, 1)
    T = 3
    q = normal(33, T * G.H * G.dq).astype(np.float32).reshape(T, G.H, G.dq)
    q[1, 5, :32] = 0.0                         # an all-zero activation block quantizes to 0
    got = host(m4.wkb(dev(w_uk), dev(q)[:, :, :G.nope]))
    for t in range(T):
        assert rel_to_max(got[t], O.wkb_q8(w_uk, q[t], G.nope, G.R, O.FUSED)) <= FUSED_TOL


# ------------------------------------------------------------------------------------- W_UV Q8
def test_wvb_q8_matches_fused_and_cpu_numerics(m4):
    _, _, _, w_uv = make_layer_q8(34, 1)
    x = normal(35, G.H * G.R).astype(np.float32).reshape(G.H, G.R) * 0.1
    got = host(m4.phase_wvb(dev(w_uv), dev(x)))
    assert rel_to_max(got, O.wvb_q8(w_uv, x, G.V, O.FUSED)) <= FUSED_TOL
    assert rel_to_max(got, O.wvb_q8(w_uv, x, G.V, O.CPU)) <= ATTN_TOL


def test_wvb_q8_token_batch(m4):
    _, _, _, w_uv = make_layer_q8(36, 1)
    x = normal(37, 4 * G.H * G.R).astype(np.float32).reshape(4, G.H, G.R)
    got = host(m4.phase_wvb(dev(w_uv), dev(x)))
    for t in range(4):
        assert rel_to_max(got[t], O.wvb_q8(w_uv, x[t], G.V, O.FUSED)) <= FUSED_TOL


# ------------------------------------------------------------------------------------- KQKV
@pytest.mark.parametrize("N,window", [(1, None), (256, None), (300, (37, 253)), (4096, (100, 3900)),
                                      (20000, None)])
def test_kqkv_320_row_matches_oracle(m4, N, window):
    q, w_uk, kc, _ = make_layer_q8(40 + N % 97, N)
    qcur = np.concatenate([O.wkb_q8(w_uk, q, G.nope, G.R, O.FUSED), q[:, G.nope:]], axis=1)
    mask = None if window is None else window_mask(N, *window)
    got = host(m4.kqkv(dev(kc), dev(qcur), None if mask is None else dev(mask), G.scale))
    assert got.shape == (G.H, G.R)
    assert rel_to_max(got, O.kqkv(kc, qcur, mask, G.scale, G.R)) <= ATTN_TOL


def test_partials_merge_and_combine_wvb_q8(m4):
    N = 9000
    q, w_uk, kc, w_uv = make_layer_q8(41, N)
    qcur = np.concatenate([O.wkb_q8(w_uk, q, G.nope, G.R, O.FUSED), q[:, G.nope:]], axis=1)
    parts = m4.kqkv_partials(dev(kc), dev(qcur), None, G.scale)
    assert parts.shape[-1] == G.R + 4
    attn = torch.empty(G.H, G.R, device="cuda")
    out = host(m4.phase_combine_wvb(dev(w_uv), parts, attn_out=attn))
    ref_attn = O.kqkv(kc, qcur, None, G.scale, G.R)
    assert rel_to_max(host(attn), ref_attn) <= ATTN_TOL
    assert rel_to_max(out, O.wvb_q8(w_uv, host(attn), G.V, O.FUSED)) <= FUSED_TOL
    rec = m4.phase_merge_records(parts)                      # selector 3 on 260-float records
    o, mm, ll = host(rec)[0, :, :G.R], host(rec)[0, :, G.R], host(rec)[0, :, G.R + 1]
    assert np.all(ll > 0) and np.all(np.isfinite(mm))
    assert rel_to_max(o / ll[:, None], ref_attn) <= ATTN_TOL


def test_ragged_320_row_windows(m4):
    lengths = [0, 1, 129, 700, 3000]
    bases = packed_bases(lengths, gap=5)
    rows = int(bases[-1] + lengths[-1])
    kc = normal(42, rows * G.D).astype(np.float16).reshape(rows, G.D)
    qcur = normal(43, 5 * G.H * G.D).astype(np.float32).reshape(5, G.H, G.D)
    got = host(m4.kqkv_ragged(dev(kc), dev(qcur), dev(np.asarray(bases, np.int32)),
                              dev(np.asarray(lengths, np.int32)), G.scale))
    assert m4.device_status() == m4.OK
    for t, (b, n) in enumerate(zip(bases, lengths)):
        if n == 0:
            assert not got[t].any()
        else:
            assert rel_to_max(got[t], O.kqkv(kc[b:b + n], qcur[t], None, G.scale, G.R)) <= ATTN_TOL


@pytest.mark.parametrize("name", ["mistral_n256", "mistral_window_n700"])
def test_layer_step_matches_reference_golden(m4, name):
    with open(os.path.join(GOLDEN, "index.json")) as f:
        case = json.load(f)["cases"][name]
    N = case["N"]
    q, w_uk, kc, w_uv = make_layer_q8(case["seed"], N)
    mask = window_mask(N, case["mask"][1], case["mask"][2])
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    qd = dev(q)
    qcur = torch.empty(G.H, G.D, device="cuda")
    qcur[:, G.R:] = qd[:, G.nope:]
    m4.wkb(dev(w_uk), qd[:, :G.nope], out=qcur[:, :G.R])
    attn = m4.kqkv(dev(kc), qcur, dev(mask), G.scale)
    out = host(m4.phase_wvb(dev(w_uv), attn))
    assert rel_to_max(host(qcur)[:, :G.R], gold["q_abs"]) <= ATTN_TOL
    assert rel_to_max(host(attn), gold["attn"]) <= ATTN_TOL            # the north-star gate
    # the W_UV stage on the reference's own attention output
    stage = host(m4.phase_wvb(dev(w_uv), dev(gold["attn"])))
    assert rel_to_max(stage, gold["out"]) <= ATTN_TOL
    assert rel_to_max(out, gold["out"]) <= Q8_CHAIN_TOL


def test_wkb_q8_qcat_writes_the_rope_half(m4):
    """M4B_FLAG_QCAT at the Mistral geometry: q (32, 128) = nope 64 + rope 64; Qcur (32, 320)."""
    q, w_uk, _, _ = make_layer_q8(73, 1)
    qd, wk = dev(q), dev(w_uk)
    plain = host(m4.wkb(wk, qd[:, :G.nope]))
    qcur = torch.full((G.H, G.D), 7.0, device="cuda")
    m4.wkb(wk, qd[:, :G.nope], out=qcur[:, :G.R], flags=m4.FLAG_QCAT)
    got = host(qcur)
    assert np.array_equal(got[:, :G.R], plain)
    assert np.array_equal(got[:, G.R:], q[:, G.nope:])


# ------------------------------------------------------------------------------------- KV-write
def _kvwrite_gpu(m4, cur, w, nw, kc, kidx, pos, rope=None):
    kcd = dev(kc)
    kcur = m4.phase_kvwrite(dev(cur), dev(w), dev(nw), kcd, dev(np.array([kidx], np.int64)),
                            dev(np.array([pos], np.int32)), rope)
    return host(kcur), host(kcd)


@pytest.mark.parametrize("pos", [0, 7, 900, 6000])
def test_kvwrite_matches_fused_numerics(m4, pos):
    cur, w, nw, kc = make_kvwrite(50 + pos % 13, 40)
    kcur, cache = _kvwrite_gpu(m4, cur, w, nw, kc, 11, pos)
    ref = O.kvwrite(cur, w, nw, None, 11, pos, MISTRAL_ROPE, O.FUSED)
    assert rel_to_max(kcur[:G.R], ref[:G.R]) <= FUSED_TOL               # gemv + RMS norm
    # the rope angle pos * powf(theta_scale, p): the device and host powf / cosf / sinf may
    # differ in the last bit, which the angle scales by pos
    assert rel_to_max(kcur[G.R:], ref[G.R:]) <= 1e-6 + 1e-7 * pos
    assert np.array_equal(cache[11], kcur.astype(np.float16))          # the row holds f16(Kcur)
    others = np.delete(np.arange(40), 11)
    assert np.array_equal(cache[others], kc[others])                    # nothing else written


@pytest.mark.parametrize("name", ["kvwrite_pos3", "kvwrite_pos4000"])
def test_kvwrite_matches_reference_golden(m4, name):
    with open(os.path.join(GOLDEN, "index.json")) as f:
        case = json.load(f)["kvwrite"][name]
    cur, w, nw, kc = make_kvwrite(case["seed"], case["N"])
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    kcur, cache = _kvwrite_gpu(m4, cur, w, nw, kc, case["kidx"], case["pos"], case["rope"])
    assert rel_to_max(kcur, gold["kcur"]) <= 1e-3
    row = cache[case["kidx"]].astype(np.float32)
    gold_row = gold["row"].view(np.float16).astype(np.float32)
    assert rel_to_max(row, gold_row) <= 2e-3


def test_kvwrite_row_outside_cache_writes_nothing(m4):
    cur, w, nw, kc = make_kvwrite(60, 16)
    kcur, cache = _kvwrite_gpu(m4, cur, w, nw, kc, 16, 5)               # rows are 0..15
    assert m4.device_status() == m4.EINVAL
    assert np.array_equal(cache, kc)
    ref = O.kvwrite(cur, w, nw, None, 0, 5, MISTRAL_ROPE, O.FUSED)
    assert rel_to_max(kcur, ref) <= 1e-5                                # Kcur is still produced
    assert m4.device_status() == m4.OK


@pytest.mark.parametrize("kidx", [0, 9, 23, 39])
def test_kvwrite_into_sharded_slabs_equals_one_cache(m4, kidx):
    """m4b_phase_kvwrite_slab: a 40-row cache split into slabs of 16 / 16 / 8 rows (one per GPU in
    a sharded deployment, emulated here on one GPU).  Every slab computes the same Kcur as the
    one-cache KV-write; only the slab holding global row kidx writes it, at kidx - slab_base, and
    the others are untouched and report no error."""
    cur, w, nw, kc = make_kvwrite(62, 40)
    kcur_ref, cache_ref = _kvwrite_gpu(m4, cur, w, nw, kc, kidx, 77)
    assert m4.device_status() == m4.OK
    idx, pos = dev(np.array([kidx], np.int64)), dev(np.array([77], np.int32))
    args = [dev(cur), dev(w), dev(nw)]
    slabs = [(0, 16), (16, 32), (32, 40)]
    for base, end in slabs:
        part = dev(kc[base:end])
        kcur = host(m4.phase_kvwrite(*args, part, idx, pos, slab_base=base))
        assert np.array_equal(kcur, kcur_ref)
        assert np.array_equal(host(part), cache_ref[base:end])           # own row written, no other
        assert m4.device_status() == m4.OK


def test_kvwrite_slab_refusals(m4):
    cur, w, nw, kc = make_kvwrite(63, 8)
    args = [dev(cur), dev(w), dev(nw), dev(kc)]
    pos = dev(np.array([1], np.int32))
    with pytest.raises(m4.M4Error):
        m4.phase_kvwrite(*args, dev(np.array([0], np.int64)), pos, slab_base=-1)
    part = args[3]
    m4.phase_kvwrite(*args[:3], part, dev(np.array([-3], np.int64)), pos, slab_base=8)
    assert m4.device_status() == m4.EINVAL                              # a negative row is an error
    assert np.array_equal(host(part), kc)
    assert m4.device_status() == m4.OK


def test_kvwrite_graph_replay_reads_row_and_position_on_device(m4):
    cur, w, nw, kc = make_kvwrite(61, 32)
    kcd = dev(kc)
    args = [dev(cur), dev(w), dev(nw), kcd]
    kidx = dev(np.array([3], np.int64))
    pos = dev(np.array([10], np.int32))
    out = torch.empty(G.D, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        m4.phase_kvwrite(*args, kidx, pos, out=out, flags=m4.FLAG_PDL)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        m4.phase_kvwrite(*args, kidx, pos, out=out, flags=m4.FLAG_PDL)
    for row, p in ((7, 100), (30, 2500)):
        kidx.fill_(row)
        pos.fill_(p)
        g.replay()
        ref = O.kvwrite(cur, w, nw, None, row, p, MISTRAL_ROPE, O.FUSED)
        assert rel_to_max(host(out), ref) <= 1e-6 + 1e-7 * p
        assert np.array_equal(host(kcd)[row], host(out).astype(np.float16))
    assert m4.device_status() == m4.OK


def test_layer_step_with_kvwrite_matches_oracle(m4):
    """The whole fused layer at this geometry: KV-write of the new token's row, then WKB, KQKV
    over the cache including that row, W_UV -- against the oracle doing the same."""
    N, new_row, pos = 2000, 1500, 1500
    q, w_uk, kc, w_uv = make_layer_q8(62, N)
    cur, w_kva, nw, _ = make_kvwrite(62, N)
    mask = window_mask(N, 0, new_row + 1)
    kcd = dev(kc)
    kcur = m4.phase_kvwrite(dev(cur), dev(w_kva), dev(nw), kcd, dev(np.array([new_row], np.int64)),
                            dev(np.array([pos], np.int32)))
    qd = dev(q)
    qcur = torch.empty(G.H, G.D, device="cuda")
    qcur[:, G.R:] = qd[:, G.nope:]
    m4.wkb(dev(w_uk), qd[:, :G.nope], out=qcur[:, :G.R])
    attn = m4.kqkv(kcd, qcur, dev(mask), G.scale)
    out = host(m4.phase_wvb(dev(w_uv), attn))
    kc_ref = kc.copy()
    O.kvwrite(cur, w_kva, nw, kc_ref, new_row, pos, MISTRAL_ROPE, O.FUSED)
    assert np.array_equal(host(kcd)[new_row], host(kcur).astype(np.float16))
    qcur_ref = np.concatenate([O.wkb_q8(w_uk, q, G.nope, G.R, O.FUSED), q[:, G.nope:]], axis=1)
    attn_ref = O.kqkv(kc_ref, qcur_ref, mask, G.scale, G.R)
    assert rel_to_max(host(attn), attn_ref) <= ATTN_TOL
    assert rel_to_max(out, O.wvb_q8(w_uv, host(attn), G.V, O.FUSED)) <= FUSED_TOL
    assert rel_to_max(out, O.wvb_q8(w_uv, attn_ref, G.V, O.CPU)) <= Q8_CHAIN_TOL
