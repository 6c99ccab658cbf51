"""GPU test of m4b_kqkv_static_scratch, the KQKV entry point for callers that cannot allocate
device memory: a plugin inside an application that owns every device allocation, or a decode
loop that must not stall or fail on cudaMalloc after start-up.  Its split-K records live in a
fixed array inside the library instead of caller scratch.

Every case calls the entry point through the C ABI twice in a row (the second call reuses the
array the first one filled) and compares both outputs with the regular entry point m4b_kqkv.  Both
run the same two kernels with the same split count, so the outputs must be bit-identical.  One
case is also held to the CPU oracle within the attention tolerance.  The cases run large first,
then small, then at the Mistral-Small-4 geometry (latent 256), so later calls find the array full
of an earlier, larger call's records.  Named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, rel_to_max
from mla_inputs import BASELINE, MISTRAL, make_layer, normal, window_mask

pytestmark = pytest.mark.gpu


def _static_call(m4, kc, q, mask, scale, out):
    lib = m4.lib()
    lib.m4b_kqkv_static_scratch.argtypes = [ctypes.POINTER(m4.KqkvArgs), ctypes.c_void_p]
    a = m4._kqkv_args(kc, q, mask, scale, 0)
    a.dst = m4._heads_desc(out, m4.latent_of(kc))
    rc = lib.m4b_kqkv_static_scratch(ctypes.byref(a), m4._stream())
    assert rc == m4.OK, m4.strerror(rc)
    return out


def _case(seed, N, mask, g):
    if g is BASELINE:
        _, _, kc, _ = make_layer(300 + seed, N)
    else:
        kc = normal(500 + seed, N * g.D).astype(np.float16).reshape(N, g.D)
    q = (0.3 * normal(400 + seed, g.H * g.D)).astype(np.float32).reshape(g.H, g.D)
    return kc, q


def test_static_scratch_matches_regular_entry_twice():
    assert torch.cuda.is_available()
    from aubier_b200 import m4
    from oracle import oracle as O
    cases = [(20000, None, BASELINE), (777, window_mask(777, 40, 700), BASELINE),
             (3001, None, MISTRAL)]
    for seed, (N, mask, g) in enumerate(cases):
        kc, q = _case(seed, N, mask, g)
        kcd, qd = torch.from_numpy(kc).cuda(), torch.from_numpy(q).cuda()
        md = torch.from_numpy(mask).cuda() if mask is not None else None
        ref = m4.kqkv(kcd, qd, md, g.scale).cpu().numpy()
        for _ in range(2):
            out = torch.full((g.H, g.R), float("nan"), device="cuda")
            got = _static_call(m4, kcd, qd, md, g.scale, out).cpu().numpy()
            assert np.array_equal(got, ref), f"case {seed}: differs from m4b_kqkv"
        if seed == 1:   # the windowed case against the CPU oracle as well
            assert rel_to_max(got, O.kqkv(kc, q, mask, g.scale, g.R)) <= ATTN_TOL
    assert m4.device_status() == m4.OK
