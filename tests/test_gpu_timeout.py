"""The KV-slab exchange on one GPU, with every rank's exchange in this process
(m4b_exchange_open_local), and a bounded device wait that runs out without faulting or hanging.

* Two ranks on one GPU, two-launch form: both ranks publish their slab's merged record, then both
  combine.  No kernel waits for another (every record is in place before any combine starts), and
  the result matches the oracle over the whole cache, in three consecutive exchanges so both
  halves of the double-buffered receive area are used.
* The one-launch form (m4b_exchange_merge_wvb) as rank 0 of 2 and 8 ranks: the other ranks
  publish first, so rank 0's polls find every record in place; matches the oracle.
* Rank 1 never publishes: rank 0's one-launch exchange (m4b_exchange_merge_wvb) stores its record,
  then polls for rank 1's, which never comes.  With the wait limit shortened to a few milliseconds
  the kernel gives up, returns and reports M4B_ETIMEOUT through m4b_device_status(); the context
  stays usable (a regular KQKV launched right after matches the oracle).  The wait is the
  kernel's own bounded poll of local memory: nothing faults and no other kernel is involved.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, rel_to_max
from mla_inputs import BASELINE as G, make_layer

pytestmark = pytest.mark.gpu

LIMIT_CYCLES = 1 << 23   # ~4 ms at 2 GHz


@pytest.fixture(scope="module")
def m4():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from aubier_b200 import exchange  # noqa: F401  (declares the exchange argtypes)
    from aubier_b200 import m4 as mod
    return mod


def _local_exchange(m4, world):
    lib = m4.lib()
    hs = []
    for r in range(world):
        h = ctypes.c_void_p()
        m4._check(lib.m4b_exchange_create(world, r, ctypes.byref(h)), "m4b_exchange_create")
        hs.append(h)
    arr = (ctypes.c_void_p * world)(*[h.value for h in hs])
    for h in hs:
        m4._check(lib.m4b_exchange_open_local(h, arr, world), "m4b_exchange_open_local")
    return hs


def _close(m4, hs):
    torch.cuda.synchronize()
    for h in hs:
        m4.lib().m4b_exchange_detach(h)
    for h in hs:
        m4.lib().m4b_exchange_destroy(h)


def _args(m4, part=None, w_uv=None, out=None, attn=None):
    a = m4.PhaseArgs()
    if w_uv is not None:
        a.src[0] = m4.gtensor(w_uv, list(reversed(w_uv.shape)))
    if part is not None:
        a.src[1] = m4.gtensor(part, [m4.PART_STRIDE, m4.HEADS, part.shape[0], 1])
    if attn is not None:
        a.src[2] = m4._heads_desc(attn, m4.LATENT)
    if out is not None:
        a.dst = m4._heads_desc(out, m4.VHEAD)
    return a


def _layer(seed, N):
    from oracle import oracle as O
    q, w_uk, kc, w_uv = make_layer(seed, N)
    qcur = np.concatenate([O.wkb(w_uk, q, G.nope), q[:, G.nope:]], axis=1).astype(np.float32)
    return q, w_uk, kc, w_uv, qcur


def test_in_process_exchange_on_one_gpu_matches_oracle(m4):
    from oracle import oracle as O
    lib = m4.lib()
    N, world = 6144, 2
    hs = _local_exchange(m4, world)
    try:
        for k in range(3):   # epochs 1, 2, 3: both receive halves, the first one twice
            q, w_uk, kc, w_uv, qcur = _layer(90 + k, N)
            kcd, qd, wuvd = (torch.from_numpy(a).cuda() for a in (kc, qcur, w_uv))
            slabs = [kcd[: N // 2], kcd[N // 2:]]
            parts = [m4.kqkv_partials(s, qd, None, G.scale) for s in slabs]
            for h, part in zip(hs, parts):
                rc = lib.m4b_exchange_publish(h, ctypes.byref(_args(m4, part=part)), m4._stream())
                assert rc == m4.OK, m4.strerror(rc)
            outs, attns = [], []
            for h in hs:
                out = torch.full((G.H, G.V), float("nan"), device="cuda")
                attn = torch.full((G.H, G.R), float("nan"), device="cuda")
                a = _args(m4, w_uv=wuvd, out=out, attn=attn)
                rc = lib.m4b_exchange_combine_wvb(h, ctypes.byref(a), m4._stream())
                assert rc == m4.OK, m4.strerror(rc)
                outs.append(out)
                attns.append(attn)
            assert m4.device_status() == m4.OK
            o0, o1 = outs[0].cpu().numpy(), outs[1].cpu().numpy()
            assert np.array_equal(o0, o1)
            _, _, attn_ref, out_ref = O.mla_step(w_uk, q, kc, None, w_uv, G.scale, G.nope)
            assert rel_to_max(attns[0].cpu().numpy(), attn_ref) <= ATTN_TOL
            assert rel_to_max(o0, out_ref) <= ATTN_TOL
    finally:
        _close(m4, hs)


@pytest.mark.parametrize("world", [2, 8])
def test_one_launch_exchange_in_process_matches_oracle(m4, world):
    """m4b_exchange_merge_wvb (merge, store into every rank's buffer, poll, merge, W_UV in one
    launch) as rank 0 of `world` ranks in this process: ranks 1.. publish first (plain launches
    that wait for nothing), so rank 0's polls find every record already in place and no kernel
    waits for a later one.  Slabs of 19,000 keys give every rank the full 148 split records.
    Three consecutive exchanges use both halves of the receive area."""
    from oracle import oracle as O
    lib = m4.lib()
    slab = 19000
    N = world * slab
    hs = _local_exchange(m4, world)
    try:
        for k in range(3):
            q, w_uk, kc, w_uv, qcur = _layer(130 + 7 * world + k, N)
            kcd, qd, wuvd = (torch.from_numpy(a).cuda() for a in (kc, qcur, w_uv))
            parts = [m4.kqkv_partials(kcd[r * slab:(r + 1) * slab], qd, None, G.scale)
                     for r in range(world)]
            for r in range(1, world):
                rc = lib.m4b_exchange_publish(hs[r], ctypes.byref(_args(m4, part=parts[r])),
                                              m4._stream())
                assert rc == m4.OK, m4.strerror(rc)
            out = torch.full((G.H, G.V), float("nan"), device="cuda")
            attn = torch.full((G.H, G.R), float("nan"), device="cuda")
            a = _args(m4, part=parts[0], w_uv=wuvd, out=out, attn=attn)
            rc = lib.m4b_exchange_merge_wvb(hs[0], ctypes.byref(a), m4._stream())
            assert rc == m4.OK, m4.strerror(rc)
            assert m4.device_status() == m4.OK
            _, _, attn_ref, out_ref = O.mla_step(w_uk, q, kc, None, w_uv, G.scale, G.nope)
            assert rel_to_max(attn.cpu().numpy(), attn_ref) <= ATTN_TOL
            assert rel_to_max(out.cpu().numpy(), out_ref) <= ATTN_TOL
    finally:
        _close(m4, hs)


def test_exchange_wait_for_a_missing_peer_times_out(m4):
    from oracle import oracle as O
    lib = m4.lib()
    assert m4.device_status() == m4.OK
    N = 3000
    q, w_uk, kc, w_uv, qcur = _layer(77, N)
    kcd, qd, wuvd = (torch.from_numpy(a).cuda() for a in (kc, qcur, w_uv))
    part = m4.kqkv_partials(kcd, qd, None, G.scale)
    hs = _local_exchange(m4, 2)
    try:
        m4.set_wait_limit_cycles(LIMIT_CYCLES)
        out = torch.full((G.H, G.V), float("nan"), device="cuda")
        a = _args(m4, part=part, w_uv=wuvd, out=out)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rc = lib.m4b_exchange_merge_wvb(hs[0], ctypes.byref(a), m4._stream())   # rank 1: nothing
        assert rc == m4.OK, m4.strerror(rc)
        status = m4.device_status()      # synchronises: the kernel has returned
        elapsed = time.perf_counter() - t0
        assert status == m4.ETIMEOUT, m4.strerror(status)
        assert elapsed < 5.0, f"the bounded wait took {elapsed:.2f} s"
        assert m4.device_status() == m4.OK   # reading cleared it
    finally:
        m4.set_wait_limit_cycles(0)          # back to the default
        _close(m4, hs)

    # the context is still usable: a regular layer's attention matches the oracle
    got = m4.kqkv(kcd, qd, None, G.scale)
    torch.cuda.synchronize()
    assert m4.device_status() == m4.OK
    assert rel_to_max(got.cpu().numpy(), O.kqkv(kc, qcur, None, G.scale, G.R)) <= ATTN_TOL
