"""GPU parity at the sizes the bench measures, against the reference's own CPU graph.

* Config 4: one seeded layer at 262,144 keys, run as the bench runs it (WKB with the rope half
  written into Qcur, KQKV split-K partials with the engine's mask, merge + W_UV in one launch) and
  through the reference-shaped single op m4b_kqkv.
* Config 5: the bench's whole ragged batch -- 16 sequences, lengths uniform on [512, 65536]
  (467,089 keys) -- through the token-batched WKB, the ragged KQKV and the token-batched W_UV.

Each output is compared with oracle/_ref (the reference's unfused ggml-cpu graph of
engine/m1_layer.cpp:437-502, compiled from its own sources) and with a float64 evaluation on the
host, which also bounds the reference graph itself.  Gate: max |out - ref| / max |ref| <= 2e-3
(north star).  Inputs come from numpy's PCG64 streams (fast at these sizes), not from the
splitmix64 generator of the small fixtures.
"""
import json

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, fp64_layer, rel_to_max
from mla_inputs import BASELINE as G
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _weights(rng):
    w_uk = (0.02 * rng.standard_normal((G.H, G.R, G.nope), dtype=np.float32)).astype(np.float16)
    w_uv = (0.02 * rng.standard_normal((G.H, G.V, G.R), dtype=np.float32)).astype(np.float16)
    return w_uk, w_uv


def _reference(q, w_uk, kc, w_uv, mask):
    ref = O.RefMLA(G.H, G.nope, G.rope, G.R, G.V, kc.shape[0], G.scale)
    try:
        ref.set_inputs(q=q, w_uk=w_uk, kc=kc, mask=mask, w_uv=w_uv)
        ref.compute()
        _, _, attn, out = ref.outputs()
    finally:
        ref.close()
    return attn, out


def _gaps(tag, attn, out, r_attn, r_out, x_attn, x_out):
    g = {"case": tag,
         "attn_vs_ref": rel_to_max(attn, r_attn), "out_vs_ref": rel_to_max(out, r_out),
         "attn_vs_fp64": rel_to_max(attn, x_attn), "out_vs_fp64": rel_to_max(out, x_out),
         "ref_attn_vs_fp64": rel_to_max(r_attn, x_attn), "ref_out_vs_fp64": rel_to_max(r_out, x_out)}
    print("parity", json.dumps(g))
    return g


def test_config4_layer_matches_reference_graph_and_fp64():
    from aubier_b200 import m4
    N = 262144
    rng = np.random.default_rng(4242)
    q = rng.standard_normal((G.H, G.dq), dtype=np.float32)
    w_uk, w_uv = _weights(rng)
    kc = rng.standard_normal((N, G.D), dtype=np.float32).astype(np.float16)
    mask = np.zeros(N, np.float32)     # the engine's mask for the window [0, N)

    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    qd, kcd, md = d(q), d(kc), d(mask)
    qcur = torch.empty(G.H, G.D, device="cuda")
    m4.wkb(d(w_uk), qd[:, :G.nope], out=qcur[:, :G.R], flags=m4.FLAG_QCAT)
    part = m4.kqkv_partials(kcd, qcur, md, G.scale)
    attn = torch.empty(G.H, G.R, device="cuda")
    out = m4.phase_combine_wvb(d(w_uv), part, attn_out=attn)
    attn_op = m4.kqkv(kcd, qcur, md, G.scale)          # GGML_OP_M4_KQKV as the engine calls it
    torch.cuda.synchronize()
    assert m4.device_status() == m4.OK
    attn, out, attn_op = attn.cpu().numpy(), out.cpu().numpy(), attn_op.cpu().numpy()
    del kcd, part
    assert np.isfinite(out).all() and np.isfinite(attn).all()

    r_attn, r_out = _reference(q, w_uk, kc, w_uv, mask)
    x_attn, x_out = fp64_layer(q, w_uk, kc, w_uv, mask, G.nope)
    g = _gaps("config4 n=262144", attn, out, r_attn, r_out, x_attn, x_out)
    assert g["ref_attn_vs_fp64"] <= ATTN_TOL and g["ref_out_vs_fp64"] <= ATTN_TOL
    for k in ("attn_vs_ref", "out_vs_ref", "attn_vs_fp64", "out_vs_fp64"):
        assert g[k] <= ATTN_TOL, (k, g[k])
    assert rel_to_max(attn_op, r_attn) <= ATTN_TOL
    assert rel_to_max(attn_op, attn) <= 1e-5          # same records, same merge rule


def test_config5_ragged_batch_matches_reference_graph_and_fp64():
    from aubier_b200 import m4
    from aubier_b200.shard import packed_bases, ragged_lengths
    lengths = ragged_lengths()                          # the bench's batch (seed 5)
    T, rows = len(lengths), sum(lengths)
    rng = np.random.default_rng(5005)
    q = rng.standard_normal((T, G.H, G.dq), dtype=np.float32)
    w_uk, w_uv = _weights(rng)
    kc = rng.standard_normal((rows, G.D), dtype=np.float32).astype(np.float16)
    base = packed_bases(lengths)

    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    qd = d(q)
    qcur = torch.empty(T, G.H, G.D, device="cuda")
    m4.wkb(d(w_uk), qd[:, :, :G.nope], out=qcur[:, :, :G.R], flags=m4.FLAG_QCAT)
    attn = m4.kqkv_ragged(d(kc), qcur, d(np.array(base, np.int32)),
                          d(np.array(lengths, np.int32)), G.scale)
    out = m4.phase_wvb(d(w_uv), attn)
    torch.cuda.synchronize()
    assert m4.device_status() == m4.OK
    attn, out = attn.cpu().numpy(), out.cpu().numpy()
    assert np.isfinite(out).all() and np.isfinite(attn).all()

    r_attn, r_out = np.empty_like(attn), np.empty_like(out)
    x_attn, x_out = np.empty_like(attn, dtype=np.float64), np.empty_like(out, dtype=np.float64)
    for t in range(T):
        kt = kc[base[t]:base[t] + lengths[t]]
        r_attn[t], r_out[t] = _reference(q[t], w_uk, kt, w_uv, np.zeros(lengths[t], np.float32))
        x_attn[t], x_out[t] = fp64_layer(q[t], w_uk, kt, w_uv, None, G.nope)
        for k, v in _gaps(f"config5 token {t} n={lengths[t]}", attn[t], out[t], r_attn[t],
                          r_out[t], x_attn[t], x_out[t]).items():
            if k != "case":
                assert v <= ATTN_TOL, (t, k, v)
    _gaps(f"config5 all {T} tokens, {rows} keys", attn, out, r_attn, r_out, x_attn, x_out)
