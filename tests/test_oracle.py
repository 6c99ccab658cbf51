"""CPU tests of the oracle: the C restatement against the reference's own ggml-cpu outputs (the
committed golden fixtures), the reference library itself when present, and the split-K
partial/merge rule."""
import hashlib
import json
import os

import numpy as np
import pytest

from helpers import rel_to_max
from mla_inputs import (BASELINE as G, MISTRAL as GM, MISTRAL_ROPE, make_kvwrite, make_layer,
                        make_layer_q8, window_mask)
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _index():
    with open(os.path.join(GOLDEN, "index.json")) as f:
        return json.load(f)


def _cases(weights="f16"):
    return {k: v for k, v in _index()["cases"].items() if v.get("weights", "f16") == weights}


def _mask(N, spec):
    import importlib.util
    sp = importlib.util.spec_from_file_location("mg", os.path.join(GOLDEN, "make_golden.py"))
    mg = importlib.util.module_from_spec(sp)
    sp.loader.exec_module(mg)
    return mg.build_mask(N, spec)


def _digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


@pytest.mark.parametrize("name", sorted(_cases()))
def test_restatement_matches_reference_golden(name):
    case = _cases()[name]
    N = case["N"]
    q, w_uk, kc, w_uv = make_layer(case["seed"], N)
    assert _digest(q, w_uk, kc, w_uv) == case["inputs_sha256_16"], "input generator drifted"
    mask = _mask(N, case["mask"])
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    q_abs, qcur, attn, out = O.mla_step(w_uk, q, kc, mask, w_uv, G.scale, G.nope)
    assert rel_to_max(q_abs, gold["q_abs"]) <= 1e-6
    assert rel_to_max(qcur, gold["qcur"]) <= 1e-6
    # the reference rounds P = e / sum to f16 after a SIMD exp; single f16 ulp flips remain
    assert rel_to_max(attn, gold["attn"]) <= 5e-4
    assert rel_to_max(out, gold["out"]) <= 5e-4


@pytest.mark.skipif(O.ref_library_path() is None, reason="oracle/_ref not built")
def test_reference_library_reproduces_golden():
    name = "config1_n256"
    case = _cases()[name]
    N = case["N"]
    q, w_uk, kc, w_uv = make_layer(case["seed"], N)
    ref = O.RefMLA(G.H, G.nope, G.rope, G.R, G.V, N, G.scale, n_threads=2)
    ref.set_inputs(q=q, w_uk=w_uk, kc=kc, mask=_mask(N, case["mask"]), w_uv=w_uv)
    ref.compute()
    q_abs, _, attn, out = ref.outputs()
    assert ref.n_nodes() == case["graph_nodes"]
    ref.close()
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    assert rel_to_max(q_abs, gold["q_abs"]) <= 1e-6
    assert rel_to_max(attn, gold["attn"]) <= 1e-4
    assert rel_to_max(out, gold["out"]) <= 1e-4


def test_partials_merge_equals_single_pass():
    N = 1000
    q, w_uk, kc, _ = make_layer(77, N)
    qcur = np.concatenate([O.wkb(w_uk, q, G.nope), q[:, G.nope:]], axis=1)
    mask = window_mask(N, 10, 950)
    bounds = [(0, 100), (100, 101), (101, 640), (640, 1000), (1000, 1000)]
    parts = np.stack([O.kqkv_partial(kc, a, b, qcur, mask, G.scale, G.R) for a, b in bounds])
    merged = O.combine(parts)
    single = O.combine(O.kqkv_partial(kc, 0, N, qcur, mask, G.scale, G.R)[None])
    assert rel_to_max(merged, single) <= 1e-5          # the merge rule is exact up to rounding
    assert rel_to_max(O.kqkv(kc, qcur, mask, G.scale, G.R), single) <= 1e-3


def test_all_masked_head_is_zero_and_empty_partial():
    N = 64
    q, w_uk, kc, _ = make_layer(78, N)
    qcur = np.concatenate([O.wkb(w_uk, q, G.nope), q[:, G.nope:]], axis=1)
    mask = np.full(N, -np.inf, np.float32)
    assert not O.kqkv(kc, qcur, mask, G.scale, G.R).any()
    part = O.kqkv_partial(kc, 0, N, qcur, mask, G.scale, G.R)
    assert np.all(part[:, G.R] == -np.inf) and not part[:, G.R + 1].any()
    assert not O.combine(part[None]).any()


def test_softmax_is_shift_invariant_in_the_mask():
    """soft_max_ext(kq*scale + mask): adding a constant to every unmasked key changes nothing."""
    N = 300
    q, w_uk, kc, _ = make_layer(79, N)
    qcur = np.concatenate([O.wkb(w_uk, q, G.nope), q[:, G.nope:]], axis=1)
    a = O.kqkv(kc, qcur, np.zeros(N, np.float32), G.scale, G.R, exact=True)
    b = O.kqkv(kc, qcur, np.full(N, 3.0, np.float32), G.scale, G.R, exact=True)
    assert rel_to_max(a, b) <= 1e-6


# ---- the Mistral-Small-4 geometry: Q8_0 weights (the restatement's CPU-graph numerics) ------
@pytest.mark.parametrize("name", sorted(_cases("q8_0")))
def test_q8_restatement_matches_reference_golden(name):
    case = _cases("q8_0")[name]
    N = case["N"]
    q, w_uk, kc, w_uv = make_layer_q8(case["seed"], N)
    assert _digest(q, w_uk, kc, w_uv) == case["inputs_sha256_16"], "input generator drifted"
    mask = _mask(N, case["mask"])
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    q_abs = O.wkb_q8(w_uk, q, GM.nope, GM.R, O.CPU)
    qcur = np.concatenate([q_abs, q[:, GM.nope:]], axis=1)
    attn = O.kqkv(kc, qcur, mask, GM.scale, GM.R)
    out = O.wvb_q8(w_uv, attn, GM.V, O.CPU)
    assert rel_to_max(q_abs, gold["q_abs"]) <= 1e-6
    assert rel_to_max(qcur, gold["qcur"]) <= 1e-6
    assert rel_to_max(attn, gold["attn"]) <= 5e-4
    # each stage pinned on the reference's own input to it: W_UV of the reference's attention
    assert rel_to_max(O.wvb_q8(w_uv, gold["attn"], GM.V, O.CPU), gold["out"]) <= 1e-5
    # end to end, the attention's last-bit differences flip single int8 roundings of the Q8
    # activation (a flip moves a product by d = amax/127): the north-star gate
    assert rel_to_max(out, gold["out"]) <= 2e-3
    # the fused reference kernels' Q8_1 activation form stays within the north-star gate
    q_abs_f = O.wkb_q8(w_uk, q, GM.nope, GM.R, O.FUSED)
    assert rel_to_max(q_abs_f, gold["q_abs"]) <= 2e-3
    assert rel_to_max(O.wvb_q8(w_uv, attn, GM.V, O.FUSED), gold["out"]) <= 2e-3


@pytest.mark.parametrize("name", sorted(_index()["kvwrite"]))
def test_kvwrite_restatement_matches_reference_golden(name):
    case = _index()["kvwrite"][name]
    cur, w, nw, kc = make_kvwrite(case["seed"], case["N"])
    assert _digest(cur, w, nw, kc) == case["inputs_sha256_16"], "input generator drifted"
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    cache = kc.copy()
    kcur = O.kvwrite(cur, w, nw, cache, case["kidx"], case["pos"], case["rope"], O.CPU)
    assert rel_to_max(kcur, gold["kcur"]) <= 1e-6
    row = cache[case["kidx"]].astype(np.float32)
    gold_row = gold["row"].view(np.float16).astype(np.float32)
    assert np.mean(row == gold_row) >= 0.99                           # f16 rounding flips only
    # one f16 ulp, with an absolute floor for values in the f16 subnormal range
    assert np.all(np.abs(row - gold_row) <= 2.0 ** -10 * np.abs(gold_row) +
                  1e-6 * np.abs(gold_row).max())
    others = np.delete(np.arange(case["N"]), case["kidx"])
    assert np.array_equal(cache[others], kc[others])                  # only row kidx written
    # the fused tail's angle (pos * powf(theta_scale, p)) differs from the CPU's iterated one by
    # float rounding that grows with the position
    fused = O.kvwrite(cur, w, nw, None, case["kidx"], case["pos"], case["rope"], O.FUSED)
    assert rel_to_max(fused, gold["kcur"]) <= 1e-3


def test_yarn_corr_dims_of_the_engine_rope():
    # n_dims 64, original context 8192, base 1e4, beta_fast 32, beta_slow 1 (m1_layer.h:56-67)
    lo, hi = O.rope_corr_dims(64, 8192, 10000.0, 32.0, 1.0)
    assert (lo, hi) == (12.0, 25.0)


@pytest.mark.skipif(O.ref_library_path() is None, reason="oracle/_ref not built")
def test_reference_library_reproduces_q8_golden():
    name = "mistral_n256"
    case = _cases("q8_0")[name]
    N = case["N"]
    q, w_uk, kc, w_uv = make_layer_q8(case["seed"], N)
    ref = O.RefMLA(GM.H, GM.nope, GM.rope, GM.R, GM.V, N, GM.scale, n_threads=2, weights="q8_0")
    ref.set_inputs(q=q, w_uk=w_uk, kc=kc, mask=_mask(N, case["mask"]), w_uv=w_uv)
    ref.compute()
    q_abs, _, attn, out = ref.outputs()
    ref.close()
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    assert rel_to_max(q_abs, gold["q_abs"]) <= 1e-6
    assert rel_to_max(out, gold["out"]) <= 1e-4
