"""GPU parity tests: the sm_100a kernels, called through the C ABI (libm4b.so via aubier_b200.m4),
against the CPU oracle (oracle/: the reference's unfused ggml graph, restated in C, and the
reference's own ggml-cpu for the committed golden fixtures).

Gate: max |out - ref| / max |ref| <= 2e-3 on the attention and W_UV outputs (fp32 accumulation),
1e-5 on the absorption gemv.  Sizes the oracle finishes in seconds are compared directly; the
262,144-key case is checked through size-independent properties (masking locality, split
invariance) and against a float64 evaluation on the GPU.
"""
import json
import os

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, QABS_TOL, elementwise_ok, rel_to_max
from mla_inputs import BASELINE, make_layer, normal, window_mask
from oracle import oracle as O

pytestmark = pytest.mark.gpu

G = BASELINE
SCALE = G.scale
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


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


def qcur_of(q, w_uk):
    return np.concatenate([O.wkb(w_uk, q, G.nope), q[:, G.nope:]], axis=1).astype(np.float32)


# ------------------------------------------------------------------------------------- WKB
def test_wkb_matches_oracle(m4):
    q, w_uk, _, _ = make_layer(11, 1)
    ref = O.wkb(w_uk, q, G.nope)
    qd = dev(q)
    out = m4.wkb(dev(w_uk), qd[:, :G.nope])
    assert rel_to_max(host(out), ref) <= QABS_TOL


def test_wkb_writes_into_qcur_view(m4):
    q, w_uk, _, _ = make_layer(12, 1)
    qd = dev(q)
    qcur = torch.full((G.H, G.D), 7.0, device="cuda")
    qcur[:, G.R:] = qd[:, G.nope:]
    m4.wkb(dev(w_uk), qd[:, :G.nope], out=qcur[:, :G.R])
    got = host(qcur)
    assert rel_to_max(got[:, :G.R], O.wkb(w_uk, q, G.nope)) <= QABS_TOL
    assert np.array_equal(got[:, G.R:], q[:, G.nope:])


@pytest.mark.parametrize("nt", [1, 3])
def test_wkb_qcat_writes_the_rope_half(m4, nt):
    """M4B_FLAG_QCAT: WKB also copies each head's 64 rope values behind the latent, so dst holds
    Qcur = concat(q_abs, q_pe); q_abs is bit-identical to a call without the flag."""
    _, w_uk, _, _ = make_layer(71, 1)
    q = normal(72, nt * G.H * G.dq).astype(np.float32).reshape(nt, G.H, G.dq)
    qd, wk = dev(q), dev(w_uk)
    plain = host(m4.wkb(wk, qd[:, :, :G.nope]))
    qcur = torch.full((nt, G.H, G.D), 7.0, device="cuda")
    m4.wkb(wk, qd[:, :, :G.nope], out=qcur[:, :, :G.R], flags=m4.FLAG_QCAT)
    got = host(qcur)
    assert np.array_equal(got[:, :, :G.R], plain)
    assert np.array_equal(got[:, :, G.R:], q[:, :, G.nope:])
    with pytest.raises(m4.M4Error):   # no room behind the latent in dst
        m4.wkb(wk, qd[:, :, :G.nope], out=torch.empty(nt, G.H, G.R, device="cuda"),
               flags=m4.FLAG_QCAT)
    with pytest.raises(m4.M4Error):   # no rope values behind q_nope in src1
        m4.wkb(wk, qd[:, :, :G.nope].contiguous(), out=qcur[:, :, :G.R], flags=m4.FLAG_QCAT)


# ------------------------------------------------------------------------------------- KQKV
@pytest.mark.parametrize("N", [1, 7, 127, 128, 129, 255, 256, 257, 640, 1000, 4096])
def test_kqkv_matches_oracle(m4, N):
    q, w_uk, kc, _ = make_layer(100 + N, N)
    qcur = qcur_of(q, w_uk)
    mask = np.zeros(N, np.float32)
    ref = O.kqkv(kc, qcur, mask, SCALE, G.R)
    out = host(m4.kqkv(dev(kc), dev(qcur), dev(mask), SCALE))
    assert np.isfinite(out).all()
    assert rel_to_max(out, ref) <= ATTN_TOL
    assert elementwise_ok(out, ref, rtol=2e-2, atol_frac=2e-3)


def test_kqkv_no_mask_equals_zero_mask(m4):
    N = 700
    q, w_uk, kc, _ = make_layer(5, N)
    qcur = dev(qcur_of(q, w_uk))
    a = host(m4.kqkv(dev(kc), qcur, None, SCALE))
    b = host(m4.kqkv(dev(kc), qcur, dev(np.zeros(N, np.float32)), SCALE))
    assert np.array_equal(a, b)


@pytest.mark.parametrize("base,length,N", [(37, 253, 300), (0, 1, 512), (500, 12, 512),
                                           (130, 1000, 1400), (0, 129, 129)])
def test_kqkv_window_mask(m4, base, length, N):
    q, w_uk, kc, _ = make_layer(7 + base, N)
    qcur = qcur_of(q, w_uk)
    mask = window_mask(N, base, length)
    ref = O.kqkv(kc, qcur, mask, SCALE, G.R)
    out = host(m4.kqkv(dev(kc), dev(qcur), dev(mask), SCALE))
    assert rel_to_max(out, ref) <= ATTN_TOL


def test_kqkv_mask_holes_and_fully_masked_tiles(m4):
    N = 1300
    q, w_uk, kc, _ = make_layer(21, N)
    qcur = qcur_of(q, w_uk)
    mask = np.zeros(N, np.float32)
    mask[np.arange(N) % 3 == 0] = -np.inf
    mask[128:512] = -np.inf      # whole tiles masked, in the middle of a split
    ref = O.kqkv(kc, qcur, mask, SCALE, G.R)
    out = host(m4.kqkv(dev(kc), dev(qcur), dev(mask), SCALE))
    assert rel_to_max(out, ref) <= ATTN_TOL


def test_kqkv_all_masked_is_zero(m4):
    N = 300
    q, w_uk, kc, _ = make_layer(22, N)
    out = host(m4.kqkv(dev(kc), dev(qcur_of(q, w_uk)), dev(np.full(N, -np.inf, np.float32)), SCALE))
    assert np.array_equal(out, np.zeros_like(out))


def test_kqkv_padded_row_stride(m4):
    N = 777
    q, w_uk, kc, _ = make_layer(23, N)
    qcur = qcur_of(q, w_uk)
    big = torch.zeros(N, 640, dtype=torch.float16, device="cuda")   # 1280-byte rows
    big[:, :G.D] = dev(kc)
    ref = O.kqkv(kc, qcur, None, SCALE, G.R)
    out = host(m4.kqkv(big[:, :G.D], dev(qcur), None, SCALE))
    assert rel_to_max(out, ref) <= ATTN_TOL


def test_kqkv_lazy_rescale_growing_scores(m4):
    """Scores that grow tile after tile force the running max up by >> 2^8 several times, so
    the O-in-TMEM rescale path runs; the result must still match the oracle."""
    N = 64 * 24
    q, w_uk, kc, _ = make_layer(24, N)
    qcur = qcur_of(q, w_uk)
    kc32 = kc.astype(np.float32)
    ramp = np.repeat(np.linspace(0.2, 3.0, 24), 64)[:, None]
    kc_r = (kc32 * ramp).astype(np.float16)
    ref = O.kqkv(kc_r, qcur, None, SCALE, G.R)
    out = host(m4.kqkv(dev(kc_r), dev(qcur), None, SCALE))
    assert rel_to_max(out, ref) <= ATTN_TOL


# ------------------------------------------------------------------------------ partials/merge
@pytest.mark.parametrize("N,S", [(1000, 3), (4096, 32), (4096, 7), (300, 1)])
def test_partials_merge_matches_exact(m4, N, S):
    q, w_uk, kc, _ = make_layer(31 + S, N)
    qcur = qcur_of(q, w_uk)
    part = host(m4.kqkv_partials(dev(kc), dev(qcur), None, SCALE, splits=S))
    assert part.shape == (S, G.H, G.R + 4)
    tk = m4.TILE_KEYS
    n_tiles = (N + tk - 1) // tk
    base, rem = divmod(n_tiles, S)
    for s in range(S):
        t0 = s * base + min(s, rem)
        t1 = t0 + base + (1 if s < rem else 0)
        ex = O.kqkv_partial(kc, t0 * tk, min(t1 * tk, N), qcur, None, SCALE, G.R)
        m, l, o = part[s, :, G.R], part[s, :, G.R + 1], part[s, :, :G.R]
        # the kernel's running max is lazy (within 2^8 of the true max): compare invariants
        em, el, eo = ex[:, G.R], ex[:, G.R + 1], ex[:, :G.R]
        assert np.all(m <= em + 1e-3) and np.all(m >= em - 8.0 - 1e-3)
        mass = l * np.exp2(m.astype(np.float64) - em)
        assert np.allclose(mass, el, rtol=1e-3)
        assert rel_to_max(o / l[:, None], eo / el[:, None]) <= ATTN_TOL
    merged = O.combine(part)
    ref = O.kqkv(kc, qcur, None, SCALE, G.R)
    assert rel_to_max(merged, ref) <= ATTN_TOL


def test_combine_wvb_matches_oracle(m4):
    N = 2048
    q, w_uk, kc, w_uv = make_layer(41, N)
    qcur = qcur_of(q, w_uk)
    part = m4.kqkv_partials(dev(kc), dev(qcur), None, SCALE, splits=5)
    attn = torch.empty(G.H, G.R, device="cuda")
    out = host(m4.phase_combine_wvb(dev(w_uv), part, attn_out=attn))
    ref_attn = O.kqkv(kc, qcur, None, SCALE, G.R)
    assert rel_to_max(host(attn), ref_attn) <= ATTN_TOL
    assert rel_to_max(out, O.wvb(w_uv, ref_attn)) <= ATTN_TOL
    out2 = host(m4.phase_combine_wvb(dev(w_uv), part))    # scratch instead of attn_out
    assert np.array_equal(out, out2)


def test_combine_wvb_one_launch_equals_two_steps(m4):
    """PHASE selector 2 merges and applies W_UV in one launch: its attn is bit-identical to the
    single-window op's merge of the same records, and its output matches W_UV applied to that attn
    (only the order of W_UV's additions differs)."""
    N = 30000
    q, w_uk, kc, w_uv = make_layer(43, N)
    qcur, kcd = dev(qcur_of(q, w_uk)), dev(kc)
    mask = dev(window_mask(N, 700, 25000))
    part = m4.kqkv_partials(kcd, qcur, mask, SCALE)
    attn = torch.empty(G.H, G.R, device="cuda")
    wuv = dev(w_uv)
    out = host(m4.phase_combine_wvb(wuv, part, attn_out=attn))
    assert np.array_equal(host(attn), host(m4.kqkv(kcd, qcur, mask, SCALE)))
    assert rel_to_max(out, host(m4.phase_wvb(wuv, attn))) <= 1e-5


def test_merge_records_two_level_equals_direct(m4):
    """PHASE selector 3 (the multi-GPU exchange payload): merging groups of partial records into
    one record each, then merging those, equals merging all records at once."""
    N = 30000
    q, w_uk, kc, w_uv = make_layer(42, N)
    qcur = dev(qcur_of(q, w_uk))
    mask = window_mask(N, 1000, 20000)          # some splits fully masked
    part = m4.kqkv_partials(dev(kc), qcur, dev(mask), SCALE, splits=148)
    groups = [part[:50], part[50:51], part[51:]]   # uneven "ranks"
    merged = torch.cat([m4.phase_merge_records(g) for g in groups])
    wuv = dev(w_uv)
    a1, a2 = torch.empty(G.H, G.R, device="cuda"), torch.empty(G.H, G.R, device="cuda")
    o1 = host(m4.phase_combine_wvb(wuv, part, attn_out=a1))
    o2 = host(m4.phase_combine_wvb(wuv, merged, attn_out=a2))
    assert rel_to_max(host(a2), host(a1)) <= 1e-5
    assert rel_to_max(o2, o1) <= 1e-4
    ref = O.kqkv(kc, qcur_of(q, w_uk), mask, SCALE, G.R)
    assert rel_to_max(host(a2), ref) <= ATTN_TOL
    # a record set where one group is fully masked merges to m = -inf, l = 0 and is ignored
    empty = m4.phase_merge_records(m4.kqkv_partials(dev(kc[:300]), qcur, dev(np.full(300, -np.inf, np.float32)), SCALE))
    e = host(empty)
    assert np.all(e[0, :, G.R] == -np.inf) and not e[0, :, G.R + 1].any()
    a3 = torch.empty(G.H, G.R, device="cuda")
    m4.phase_combine_wvb(wuv, torch.cat([merged, empty]), attn_out=a3)
    assert rel_to_max(host(a3), host(a2)) <= 1e-6


def test_phase_wvb_matches_oracle(m4):
    _, _, _, w_uv = make_layer(51, 1)
    x = normal(5151, G.H * G.R).astype(np.float32).reshape(G.H, G.R)
    out = host(m4.phase_wvb(dev(w_uv), dev(x)))
    assert rel_to_max(out, O.wvb(w_uv, x)) <= QABS_TOL * 10


# ------------------------------------------------------------------------ the whole layer step
def _layer_step(m4, q, w_uk, kc, mask, w_uv):
    qd = dev(q)
    qcur = torch.empty(G.H, G.D, device="cuda")
    qcur[:, G.R:] = qd[:, G.nope:]
    m4.wkb(dev(w_uk), qd[:, :G.nope], out=qcur[:, :G.R])
    attn = m4.kqkv(dev(kc), qcur, dev(mask) if mask is not None else None, SCALE)
    out = m4.phase_wvb(dev(w_uv), attn)
    return host(qcur[:, :G.R]), host(attn), host(out)


def _golden_cases():
    """The BASELINE-geometry fixtures (the Mistral ones are tested in test_gpu_mistral.py)."""
    with open(os.path.join(GOLDEN, "index.json")) as f:
        cases = json.load(f)["cases"]
    return {k: v for k, v in cases.items() if v.get("weights", "f16") == "f16"}


@pytest.mark.parametrize("name", sorted(_golden_cases()))
def test_layer_step_matches_reference_golden(m4, name):
    """WKB -> KQKV -> PHASE(wvb) against the reference ggml-cpu graph's own outputs."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    case = _golden_cases()[name]
    N = case["N"]
    q, w_uk, kc, w_uv = make_layer(case["seed"], N)
    mask = mg.build_mask(N, case["mask"])
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    q_abs, attn, out = _layer_step(m4, q, w_uk, kc, mask, w_uv)
    assert rel_to_max(q_abs, gold["q_abs"]) <= QABS_TOL
    assert rel_to_max(attn, gold["attn"]) <= ATTN_TOL
    assert rel_to_max(out, gold["out"]) <= ATTN_TOL


@pytest.mark.parametrize("N", [32768])
def test_layer_step_config3_size(m4, N):
    q, w_uk, kc, w_uv = make_layer(3, N)
    mask = np.zeros(N, np.float32)
    _, _, attn_ref, out_ref = O.mla_step(w_uk, q, kc, mask, w_uv, SCALE, G.nope)
    _, attn, out = _layer_step(m4, q, w_uk, kc, mask, w_uv)
    assert rel_to_max(attn, attn_ref) <= ATTN_TOL
    assert rel_to_max(out, out_ref) <= ATTN_TOL


# ------------------------------------------------------------- full size (262,144 keys)
N_FULL = 262144


@pytest.fixture(scope="module")
def full_inputs(m4):
    g = torch.Generator(device="cuda").manual_seed(262144)
    kc = torch.randn(N_FULL, G.D, device="cuda", generator=g).half()
    q = torch.randn(G.H, G.D, device="cuda", generator=g) * 0.5
    return kc, q


def test_full_size_window_locality(m4, full_inputs):
    """A 300-key window deep inside a 262,144-key cache equals attention over the window alone."""
    kc, q = full_inputs
    k0 = 200_011
    mask = torch.full((N_FULL,), float("-inf"), device="cuda")
    mask[k0:k0 + 300] = 0.0
    out = host(m4.kqkv(kc, q, mask, SCALE))
    ref = O.kqkv(host(kc[k0:k0 + 300]), host(q), None, SCALE, G.R)
    assert rel_to_max(out, ref) <= ATTN_TOL


def test_full_size_split_invariance_and_fp64(m4, full_inputs):
    kc, q = full_inputs
    full = host(m4.kqkv(kc, q, None, SCALE))
    for S in (1, 37):
        part = m4.kqkv_partials(kc, q, None, SCALE, splits=S)
        w = torch.empty(G.H, G.V, G.R, device="cuda", dtype=torch.float16)
        attn = torch.empty(G.H, G.R, device="cuda")
        m4.phase_combine_wvb(w.zero_(), part, attn_out=attn)
        # one split accumulates 2048 tiles into one TMEM accumulator (f32 drift ~1e-4); the
        # production split count keeps ~14 tiles per accumulator
        assert rel_to_max(host(attn), full) <= (1e-3 if S == 1 else 1e-4)
    # float64 evaluation on the GPU (q rounded to f16 as the kernel and the oracle do)
    q64 = q.half().double()
    s = (kc.double() @ q64.T) * SCALE                     # (N, H)
    p = torch.softmax(s, dim=0)
    ref = host((p.T @ kc[:, :G.R].double()).float())
    assert rel_to_max(full, ref) <= ATTN_TOL


# ------------------------------------------------------------------------ graph capture, errors
def test_cuda_graph_capture_replays(m4):
    N = 4096
    q, w_uk, kc, w_uv = make_layer(61, N)
    qd, wk, kcd, wv = dev(q), dev(w_uk), dev(kc), dev(w_uv)
    qcur = torch.empty(G.H, G.D, device="cuda")
    part = torch.empty(m4.default_splits(N), G.H, G.R + 4, device="cuda")
    out = torch.empty(G.H, G.V, device="cuda")
    attn = torch.empty(G.H, G.R, device="cuda")

    def step():
        qcur[:, G.R:] = qd[:, G.nope:]
        m4.wkb(wk, qd[:, :G.nope], out=qcur[:, :G.R], flags=m4.FLAG_PDL)
        m4.kqkv_partials(kcd, qcur, None, SCALE, out=part, flags=m4.FLAG_PDL | m4.FLAG_KV_STATIC)
        m4.phase_combine_wvb(wv, part, out=out, attn_out=attn, flags=m4.FLAG_PDL)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    eager = host(out).copy()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    out.zero_()
    graph.replay()
    assert np.array_equal(host(out), eager)
    _, _, _, out_ref = O.mla_step(w_uk, q, kc, None, w_uv, SCALE, G.nope)
    assert rel_to_max(eager, out_ref) <= ATTN_TOL
    assert m4.device_status() == m4.OK


def test_contract_violations_raise(m4):
    kc = torch.zeros(256, G.D, dtype=torch.float16, device="cuda")
    q = torch.zeros(G.H, G.D, device="cuda")
    with pytest.raises(m4.M4Error) as e:
        m4.kqkv(kc.float(), q, None, SCALE)                 # wrong cache type
    assert e.value.code == m4.EINVAL
    with pytest.raises(m4.M4Error):
        m4.kqkv(kc, q[:16], None, SCALE)                     # wrong head count
    with pytest.raises(m4.M4Error):
        m4.kqkv(kc, q, torch.zeros(255, device="cuda"), SCALE)   # mask length != n_kv
    with pytest.raises(m4.M4Error) as e:
        m4.kqkv(kc, q, None, SCALE, scratch=torch.empty(16, dtype=torch.uint8, device="cuda"))
    assert e.value.code == m4.ESCRATCH
    with pytest.raises(m4.M4Error):
        m4.kqkv(kc.cpu(), q.cpu(), None, SCALE)              # no CPU handler


def test_early_release_chain_is_bit_identical(m4):
    """M4B_FLAG_EARLY_RELEASE only moves the point at which the next launch may start: a chain of
    layers (WKB -> KQKV partials -> merge + W_UV) replayed from a CUDA graph gives the same bits
    with and without it, and each layer still matches the oracle.  (Set on KQKV as well, it is
    ignored there: releasing the cluster-launched merge from KQKV early made the merge read the
    records too soon in graph replay.)"""
    import torch
    L, N = 4, 5000
    layers = [make_layer(600 + l, N) for l in range(L)]
    d = [tuple(dev(a) for a in lay) for lay in layers]
    S = m4.default_splits(N)

    def run(extra):
        part = torch.empty(S, G.H, G.R + 4, device="cuda")
        outs = torch.empty(L, G.H, G.V, device="cuda")
        qcur = [torch.empty(G.H, G.D, device="cuda") for _ in range(L)]

        def chain():
            for l, (q, w_uk, kc, w_uv) in enumerate(d):
                m4.wkb(w_uk, q[:, :G.nope], out=qcur[l][:, :G.R], flags=m4.FLAG_PDL | m4.FLAG_QCAT)
                m4.kqkv_partials(kc, qcur[l], None, SCALE, out=part,
                                 flags=m4.FLAG_PDL | m4.FLAG_KV_STATIC | extra)   # ignored
                m4.phase_combine_wvb(w_uv, part, out=outs[l], flags=m4.FLAG_PDL | extra)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            chain()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            chain()
        for _ in range(3):
            g.replay()
        return host(outs)

    plain, early = run(0), run(m4.FLAG_EARLY_RELEASE)
    assert m4.device_status() == m4.OK
    assert np.array_equal(plain, early)
    for l, (q, w_uk, kc, w_uv) in enumerate(layers):
        _, _, _, ref = O.mla_step(w_uk, q, kc, None, w_uv, SCALE, G.nope)
        assert rel_to_max(early[l], ref) <= ATTN_TOL
