"""Generate the golden fixtures for the MLA decode-attention parity tests.

Each fixture is the output of the REFERENCE'S OWN unfused CPU ggml graph (oracle/_ref: the
vendored ggml + ggml-cpu sources of jmars/aubier compiled by oracle/ref.mk, graph built by
oracle/ref_harness.c following engine/m1_layer.cpp:437-502) on seeded synthetic inputs from
tests/mla_inputs.py.  Only the outputs and the case description are stored; the inputs are
regenerated bit-for-bit from the seed at test time.

Run from the repository root (needs oracle/_ref built):  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from mla_inputs import (BASELINE, MISTRAL, MISTRAL_ROPE, make_kvwrite, make_layer,  # noqa: E402
                        make_layer_q8, window_mask)
from oracle.oracle import RefKVWrite, RefMLA  # noqa: E402

# name -> (seed, N, mask spec)   mask spec: None = no mask tensor semantics (all zero),
# ("window", base, len), ("holes", base, len, period) = window with every period-th key masked.
CASES = {
    "config1_n256": (1, 256, ("window", 0, 256)),
    "window_n300": (2, 300, ("window", 37, 253)),
    "single_n1": (3, 1, ("window", 0, 1)),
    "tile_n129": (4, 129, ("window", 0, 129)),
    "holes_n520": (5, 520, ("holes", 3, 500, 7)),
}

# The Mistral-Small-4 geometry (Q8_0 W_UK / W_UV, KV row 320): same layout of fixtures.
CASES_Q8 = {
    "mistral_n256": (11, 256, ("window", 0, 256)),
    "mistral_window_n700": (12, 700, ("window", 45, 600)),
}

# The KV-write (PHASE selector 0): name -> (seed, cache rows N, kidx, pos)
CASES_KVW = {
    "kvwrite_pos3": (21, 64, 17, 3),
    "kvwrite_pos4000": (22, 64, 63, 4000),
}


def build_mask(N: int, spec) -> np.ndarray:
    kind = spec[0]
    if kind == "window":
        return window_mask(N, spec[1], spec[2])
    if kind == "holes":
        m = window_mask(N, spec[1], spec[2])
        m[np.arange(N) % spec[3] == 0] = -np.inf
        return m
    raise ValueError(kind)


def main() -> None:
    g = BASELINE
    out_dir = os.path.dirname(os.path.abspath(__file__))
    index = {}
    for name, (seed, N, spec) in CASES.items():
        q, w_uk, kc, w_uv = make_layer(seed, N, g)
        mask = build_mask(N, spec)
        ref = RefMLA(g.H, g.nope, g.rope, g.R, g.V, N, g.scale, n_threads=4)
        ref.set_inputs(q=q, w_uk=w_uk.view(np.uint16), kc=kc.view(np.uint16), mask=mask,
                       w_uv=w_uv.view(np.uint16))
        ref.compute()
        q_abs, qcur, attn, out = ref.outputs()
        n_nodes = ref.n_nodes()
        ref.close()
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), q_abs=q_abs, qcur=qcur,
                            attn=attn, out=out)
        h = hashlib.sha256()
        for a in (q, w_uk, kc, w_uv):
            h.update(np.ascontiguousarray(a).tobytes())
        index[name] = {"seed": seed, "N": N, "mask": list(spec), "graph_nodes": n_nodes,
                       "inputs_sha256_16": h.hexdigest()[:16],
                       "geometry": {"H": g.H, "nope": g.nope, "rope": g.rope, "R": g.R, "V": g.V},
                       "scale": g.scale}
        print(name, N, "nodes", n_nodes, "max|out|", float(np.abs(out).max()))
    gm = MISTRAL
    for name, (seed, N, spec) in CASES_Q8.items():
        q, w_uk, kc, w_uv = make_layer_q8(seed, N, gm)
        mask = build_mask(N, spec)
        ref = RefMLA(gm.H, gm.nope, gm.rope, gm.R, gm.V, N, gm.scale, n_threads=4, weights="q8_0")
        ref.set_inputs(q=q, w_uk=w_uk, kc=kc.view(np.uint16), mask=mask, w_uv=w_uv)
        ref.compute()
        q_abs, qcur, attn, out = ref.outputs()
        n_nodes = ref.n_nodes()
        ref.close()
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), q_abs=q_abs, qcur=qcur,
                            attn=attn, out=out)
        h = hashlib.sha256()
        for a in (q, w_uk, kc, w_uv):
            h.update(np.ascontiguousarray(a).tobytes())
        index[name] = {"seed": seed, "N": N, "mask": list(spec), "graph_nodes": n_nodes,
                       "inputs_sha256_16": h.hexdigest()[:16], "weights": "q8_0",
                       "geometry": {"H": gm.H, "nope": gm.nope, "rope": gm.rope, "R": gm.R,
                                    "V": gm.V},
                       "scale": gm.scale}
        print(name, N, "nodes", n_nodes, "max|out|", float(np.abs(out).max()))
    kvw = {}
    for name, (seed, N, kidx, pos) in CASES_KVW.items():
        cur, w, nw, kc = make_kvwrite(seed, N)
        ref = RefKVWrite(cur.shape[0], gm.R, gm.rope, N, MISTRAL_ROPE, n_threads=4)
        kcur, cache = ref.run(cur, w, nw, kc, kidx, pos)
        ref.close()
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), kcur=kcur,
                            row=cache[kidx].view(np.uint16))
        h = hashlib.sha256()
        for a in (cur, w, nw, kc):
            h.update(np.ascontiguousarray(a).tobytes())
        kvw[name] = {"seed": seed, "N": N, "kidx": kidx, "pos": pos,
                     "inputs_sha256_16": h.hexdigest()[:16], "rope": MISTRAL_ROPE}
        print(name, "max|kcur|", float(np.abs(kcur).max()))
    with open(os.path.join(out_dir, "index.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "oracle": "oracle/_ref (reference ggml-cpu, llama.cpp @ 50e3e3e4)",
                   "cases": index, "kvwrite": kvw}, f, indent=1)


if __name__ == "__main__":
    main()
