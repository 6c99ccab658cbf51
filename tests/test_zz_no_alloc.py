"""GPU test of m4b_kqkv_static_scratch, the KQKV entry point for callers that cannot allocate
(a plugin inside an application that owns all device memory, a loop that must not stall on
cudaMalloc): its split-K records live in a fixed array inside the library instead of caller
scratch.  Called through the C ABI twice in a row -- the second call reuses the array the first
one filled -- and compared with the regular entry point m4b_kqkv.  Named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, rel_to_max
from mla_inputs import BASELINE as G, make_layer, normal, window_mask

pytestmark = pytest.mark.gpu


def _static_call(m4, kc, q, mask, out):
    a = m4._kqkv_args(kc, q, mask, G.scale, 0)
    a.dst = m4._heads_desc(out, G.R)
    rc = m4.lib().m4b_kqkv_static_scratch(ctypes.byref(a), ctypes.c_void_p(
        torch.cuda.current_stream().cuda_stream))
    assert rc == m4.OK, m4.strerror(rc)
    return out


def test_static_scratch_matches_regular_entry_twice():
    assert torch.cuda.is_available()
    from aubier_b200 import m4
    m4.lib().m4b_kqkv_static_scratch.argtypes = [ctypes.POINTER(m4.KqkvArgs), ctypes.c_void_p]
    cases = [(20000, None), (777, window_mask(777, 40, 700))]   # big first, then small
    for seed, (N, mask) in enumerate(cases):
        _, _, kc, _ = make_layer(300 + seed, N)
        kcd = torch.from_numpy(kc).cuda()
        q = (0.3 * normal(400 + seed, G.H * G.D)).astype(np.float32).reshape(G.H, G.D)
        qd = torch.from_numpy(q).cuda()
        md = torch.from_numpy(mask).cuda() if mask is not None else None
        ref = m4.kqkv(kcd, qd, md, G.scale)
        got = _static_call(m4, kcd, qd, md, torch.full((G.H, G.R), float("nan"), device="cuda"))
        torch.cuda.synchronize()
        assert np.isfinite(got.cpu().numpy()).all()
        assert rel_to_max(got.cpu().numpy(), ref.cpu().numpy()) <= ATTN_TOL
    assert m4.device_status() == m4.OK
