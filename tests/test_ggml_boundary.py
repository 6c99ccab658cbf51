"""CPU tests of the ggml side of the drop-in boundary (aubier_b200/ggml/).

The reference's vendored ggml (which carries its M4 patch, patches/ggml-m4/custom-op-m4.patch) is
copied into a build folder and patched with m4b-ggml.patch: the builders ggml_m4_wkb / ggml_m4_kqkv /
ggml_m4_phase_wvb take both head geometries (the reference asserts the Mistral-Small-4 shapes only,
ggml.c:3409-3413, 3433-3438, 3524-3527), WKB / WVB take token batches, ggml_m4_kqkv_ragged adds the
ragged form, and ggml-cuda's supports_op asks libm4b.  aubier_b200/ggml/ggml.mk builds it:
  * the patched ggml-cuda.cu (dispatch ggml-cuda.cu:2504-2512, supports_op :5848-5885) and the
    launcher shims m4-b200.cu compile with nvcc for sm_100a against ggml-cuda's own headers;
  * m4b_ggml_check, linked with the patched ggml core + ggml-cpu and libm4b, builds the nodes the
    engine builds (engine/m1_layer.cpp:415-502) through ggml's builders and runs libm4b's
    supports_op on them exactly as ggml-cuda does, before any memory exists;
  * a graph with an M4 node computed on ggml-cpu aborts (ggml-cpu.c:2064-2082), in a subprocess;
  * the engine's layer graph with m1-layer-batch.patch (fused ops kept for token batches) compiles.
No GPU is involved: supports_op makes no CUDA call and the CPU backend never reaches libm4b.
"""
import os
import re
import signal
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OUT = os.path.join(ROOT, "aubier_b200", "ggml", "_build")
CHECK = os.path.join(OUT, "m4b_ggml_check")


@pytest.fixture(scope="module")
def check():
    sys.path.insert(0, ROOT)
    from __graft_entry__ import REFERENCE
    if os.path.isdir(os.path.join(REFERENCE, "vendor", "llama.cpp", "ggml")):
        subprocess.check_call(["make", "-s", "-f", "aubier_b200/ggml/ggml.mk", f"REF={REFERENCE}",
                               f"OUT={OUT}", f"-j{os.cpu_count() or 4}"], cwd=ROOT)
    if not os.path.exists(CHECK):
        pytest.skip("the reference's ggml tree is not mounted and the boundary build is absent")
    return CHECK


def run(check, mode):
    return subprocess.run([check, mode], cwd=ROOT, capture_output=True, text=True, timeout=120)


def table(stdout):
    rows = {}
    for line in stdout.strip().splitlines():
        name, n0, n1, n2, n3, op, ok = line.split()
        rows[name] = ((int(n0), int(n1), int(n2), int(n3)), op, int(ok))
    return rows


def test_builders_take_both_geometries_and_supports_op_accepts_them(check):
    r = run(check, "graphs")
    assert r.returncode == 0, r.stderr
    want = {
        # f16 geometry: q_nope 128, latent 512, KV row 576
        "f16.wkb": ((512, 32, 1, 1), "M4_WKB"),
        "f16.kqkv": ((512, 1, 32, 1), "M4_KQKV"),        # the g_kqv layout (ggml.c:3445-3448)
        "f16.wvb": ((128, 1, 32, 1), "M4_PHASE"),
        "f16.wkb_batch": ((512, 32, 16, 1), "M4_WKB"),
        "f16.kqkv_ragged": ((512, 16, 32, 1), "M4_KQKV"),
        "f16.wvb_batch": ((128, 16, 32, 1), "M4_PHASE"),
        # the reference's own Mistral-Small-4 shapes (engine/m1_layer.h:47-55)
        "q8.wkb": ((256, 32, 1, 1), "M4_WKB"),
        "q8.kqkv": ((256, 1, 32, 1), "M4_KQKV"),
        "q8.wvb": ((128, 1, 32, 1), "M4_PHASE"),
        "q8.kvwrite": ((320, 1, 1, 1), "M4_PHASE"),
    }
    got = table(r.stdout)
    assert set(got) == set(want)
    for name, (ne, op) in want.items():
        assert got[name] == (ne, op, 1), (name, got[name])


def test_supports_op_refuses_other_shapes(check):
    r = run(check, "unsupported")
    assert r.returncode == 0, r.stderr
    got = table(r.stdout)
    for name in ("mask_len", "q_type", "w_uk_shape", "phase_7"):
        assert got[name][2] == 0, name          # ggml keeps the stock op sequence for the node
    for name in ("restored_kqkv", "restored_wkb", "restored_wvb"):
        assert got[name][2] == 1, name


@pytest.mark.parametrize("op,name", [("wkb", "GGML_OP_M4_WKB"), ("kqkv", "GGML_OP_M4_KQKV"),
                                     ("phase", "GGML_OP_M4_PHASE")])
def test_cpu_backend_aborts_on_the_fused_ops(check, op, name):
    r = run(check, f"abort:{op}")
    assert r.returncode == -signal.SIGABRT, (r.returncode, r.stderr[-400:])
    assert f"{name} has no CPU handler" in r.stderr
    assert "no abort" not in r.stderr


@pytest.mark.parametrize("case", ["wkb", "kqkv", "wvb"])
def test_builders_assert_on_shapes_of_neither_geometry(check, case):
    r = run(check, f"assert:{case}")
    assert r.returncode == -signal.SIGABRT, (r.returncode, r.stderr[-400:])
    assert "GGML_ASSERT" in r.stderr and "no assert" not in r.stderr


def test_ggml_cuda_dispatch_and_shims_compile_for_sm100(check):
    """The patched ggml-cuda.cu calls the launchers and supports_op that m4-b200.o defines."""
    def syms(obj):
        out = subprocess.run(["nm", "-C", os.path.join(OUT, "cuda", obj)], capture_output=True,
                             text=True, check=True).stdout
        rows = set()
        for line in out.splitlines():     # "<addr> T name" or "         U name"
            m = re.match(r"^[0-9a-fA-F]*\s+([A-Za-z])\s+(.+)$", line)
            if m:
                rows.add(f"{m.group(1)} {m.group(2)}")
        return rows
    shim, backend = syms("m4-b200.o"), syms("ggml-cuda.o")
    for fn in ("ggml_cuda_m4_wkb(ggml_backend_cuda_context&, ggml_tensor*)",
               "ggml_cuda_m4_kqkv(ggml_backend_cuda_context&, ggml_tensor*)",
               "ggml_cuda_m4_phase(ggml_backend_cuda_context&, ggml_tensor*)",
               "ggml_cuda_m4_supports_op(ggml_tensor const*)"):
        assert f"T {fn}" in shim, fn             # defined by the shim
        assert f"U {fn}" in backend, fn          # called by the backend's dispatch / supports_op
    for fn in ("m4b_wkb", "m4b_kqkv", "m4b_kqkv_ragged", "m4b_phase", "m4b_supports_op"):
        assert f"U {fn}" in shim, fn             # resolved by libm4b at link time


def test_engine_layer_keeps_the_fused_ops_for_batches(check):
    """m1-layer-batch.patch: engine/m1_layer.cpp's gate (m1_layer.cpp:283-297) keeps WKB, KQKV and
    W_UV on for up to 64 tokens, and at nt > 1 builds KQKV with ggml_m4_kqkv_ragged over each row's
    window (the cells its mask opens, m1_layer.cpp:756-773), staged as two I32 inputs.  The patched
    file compiles against the patched ggml headers."""
    obj = os.path.join(OUT, "engine", "m1_layer.o")
    out = subprocess.run(["nm", "-C", obj], capture_output=True, text=True, check=True).stdout
    used = {l.split()[-1] for l in out.splitlines() if l.strip().startswith("U ")}
    for fn in ("ggml_m4_wkb", "ggml_m4_kqkv", "ggml_m4_kqkv_ragged", "ggml_m4_phase_wvb",
               "ggml_m4_phase_kvwrite"):
        assert fn in used, fn
