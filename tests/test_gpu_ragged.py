"""GPU parity of the ragged batched decode path: a batch of tokens, each attending to its own
window [base, base + len) of one packed KV cache (the engine's per-row mask,
engine/m1_layer.cpp:756-773), with the token-batched absorption gemvs around it.

Checked against the oracle (the reference's unfused CPU graph restated: one single-token layer
step per window) at sizes it finishes in seconds, and at config-5 size (16 windows, lengths
uniform on [512, 65536]) against the single-token GPU op on each window.  Edge cases: empty
windows, windows shorter than a tile, windows not on tile boundaries, gaps and shared rows in
the packed cache, more windows than tiles, a window outside the cache, graph replay with
windows changed in device memory.
"""
import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, QABS_TOL, rel_to_max
from mla_inputs import BASELINE as G, make_layer, normal, packed_bases, ragged_lengths
from oracle import oracle as O

pytestmark = pytest.mark.gpu


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


def tokens(seed, T):
    """T queries (T, 32, 192) f32."""
    return normal(seed, T * G.H * G.dq).astype(np.float32).reshape(T, G.H, G.dq)


def cache(seed, rows):
    return normal(seed, rows * G.D).astype(np.float16).reshape(rows, G.D)


def oracle_attn(kc, qcur, base, length):
    if length == 0:
        return np.zeros((G.H, G.R), np.float32)
    return O.kqkv(kc[base:base + length], qcur, None, G.scale, G.R)


def i32(a):
    return dev(np.asarray(a, np.int32))


# ------------------------------------------------------------------ token-batched gemvs
def test_wkb_token_batch_matches_oracle(m4):
    _, w_uk, _, _ = make_layer(61, 1)
    q = tokens(62, 5)
    out = m4.wkb(dev(w_uk), dev(q)[:, :, :G.nope])
    got = host(out)
    for t in range(5):
        assert rel_to_max(got[t], O.wkb(w_uk, q[t], G.nope)) <= QABS_TOL


def test_wkb_token_batch_writes_into_qcur(m4):
    _, w_uk, _, _ = make_layer(63, 1)
    q = tokens(64, 3)
    qd = dev(q)
    qcur = torch.full((3, G.H, G.D), 5.0, device="cuda")
    m4.wkb(dev(w_uk), qd[:, :, :G.nope], out=qcur[:, :, :G.R])
    got = host(qcur)
    assert np.all(got[:, :, G.R:] == 5.0)
    for t in range(3):
        assert rel_to_max(got[t, :, :G.R], O.wkb(w_uk, q[t], G.nope)) <= QABS_TOL


def test_wvb_token_batch_matches_oracle(m4):
    _, _, _, w_uv = make_layer(65, 1)
    x = normal(66, 7 * G.H * G.R).astype(np.float32).reshape(7, G.H, G.R)
    got = host(m4.phase_wvb(dev(w_uv), dev(x)))
    for t in range(7):
        assert rel_to_max(got[t], O.wvb(w_uv, x[t])) <= ATTN_TOL


@pytest.mark.parametrize("nt", [2, 4, 16, 17, 64])
def test_token_batch_equals_single_token_calls(m4, nt):
    """The batched gemvs stage the tokens in shared memory and reduce several (row, token) dots
    per butterfly; the per-lane dot and the pairing of the reduction are the single-token
    kernels', so every token's result is bit-identical to a one-token call."""
    _, w_uk, _, w_uv = make_layer(68, 1)
    qd = dev(tokens(69, nt))
    wk = dev(w_uk)
    batch = host(m4.wkb(wk, qd[:, :, :G.nope]))
    for t in range(nt):
        assert np.array_equal(batch[t], host(m4.wkb(wk, qd[t, :, :G.nope])))
    xd = dev(normal(70, nt * G.H * G.R).astype(np.float32).reshape(nt, G.H, G.R))
    wv = dev(w_uv)
    b2 = host(m4.phase_wvb(wv, xd))
    for t in range(nt):
        assert np.array_equal(b2[t], host(m4.phase_wvb(wv, xd[t])))


def test_token_batch_limits(m4):
    _, w_uk, _, w_uv = make_layer(67, 1)
    with pytest.raises(m4.M4Error):
        m4.wkb(dev(w_uk), torch.zeros(65, G.H, G.nope, device="cuda"))
    with pytest.raises(m4.M4Error):
        m4.phase_wvb(dev(w_uv), torch.zeros(65, G.H, G.R, device="cuda"))


# ------------------------------------------------------------------ ragged KQKV vs oracle
def _ragged_vs_oracle(m4, seed, lengths, bases, rows):
    T = len(lengths)
    kc = cache(seed, rows)
    qcur = normal(seed + 1, T * G.H * G.D).astype(np.float32).reshape(T, G.H, G.D)
    out = m4.kqkv_ragged(dev(kc), dev(qcur), i32(bases), i32(lengths), G.scale)
    got = host(out)
    assert m4.device_status() == m4.OK
    for t in range(T):
        ref = oracle_attn(kc, qcur[t], bases[t], lengths[t])
        if lengths[t] == 0:
            assert np.all(got[t] == 0.0)
        else:
            assert rel_to_max(got[t], ref) <= ATTN_TOL, (t, lengths[t])


def test_ragged_edge_windows(m4):
    # empty, 1 key, tile-1, tile, tile+1, odd lengths; packed with gaps
    lengths = [0, 1, 127, 128, 129, 1000, 3001, 77]
    bases = packed_bases(lengths, gap=13)
    _ragged_vs_oracle(m4, 71, lengths, bases, int(bases[-1] + lengths[-1] + 50))


def test_ragged_shared_and_unordered_windows(m4):
    # windows may overlap, repeat and come in any order in the cache
    lengths = [4096, 4096, 500, 9000, 300]
    bases = [5000, 5000, 0, 100, 13000]
    _ragged_vs_oracle(m4, 72, lengths, bases, 14000)


def test_ragged_more_windows_than_tiles(m4):
    # 64 short windows: fewer tiles than SMs, many windows per CTA range in the balanced cut
    lengths = [int(x) for x in (np.arange(64) * 7) % 190]
    bases = packed_bases(lengths)
    _ragged_vs_oracle(m4, 73, lengths, bases, int(sum(lengths)) + 1)


def test_ragged_many_windows_per_cta(m4):
    # 64 windows of 1-2 tiles on 148 SMs: segments cross CTA boundaries in both directions
    lengths = [int(x) for x in 100 + (np.arange(64) * 37) % 200]
    bases = packed_bases(lengths)
    _ragged_vs_oracle(m4, 74, lengths, bases, int(sum(lengths)))


def test_ragged_short_first_segments(m4):
    # 64 windows of 11-14 tiles over 148 SMs (~5.5 tiles per CTA): 10 or 11 CTAs each start with
    # the last 1, 2, 3 or 4 tiles of one window and then go on to the next.  A segment that ends
    # after 1-2 tiles reads its accumulator while the matrix unit may still be two tiles behind.
    lengths = [1400 + (i * 97) % 300 for i in range(64)]
    bases = packed_bases(lengths)
    _ragged_vs_oracle(m4, 80, lengths, bases, int(sum(lengths)))


def test_ragged_one_window_equals_single_token_op(m4):
    N = 20000
    kc = dev(cache(75, N))
    q = normal(76, G.H * G.D).astype(np.float32).reshape(1, G.H, G.D)
    a = host(m4.kqkv_ragged(kc, dev(q), i32([0]), i32([N]), G.scale))[0]
    b = host(m4.kqkv(kc, dev(q[0]), None, G.scale))
    assert rel_to_max(a, b) <= 1e-5


def test_ragged_config5_size_against_single_token_op(m4):
    # config 5: 16 sequences, lengths U[512, 65536] by seed, packed; each token's output must
    # equal the single-token op on its window (same numerics, different split structure)
    lengths = ragged_lengths(5)
    bases = packed_bases(lengths)
    rows = int(lengths.sum())
    kc = torch.randn(rows, G.D, device="cuda", generator=torch.Generator("cuda").manual_seed(5)).half()
    q = torch.randn(16, G.H, G.D, device="cuda", generator=torch.Generator("cuda").manual_seed(6))
    got = host(m4.kqkv_ragged(kc, q, i32(bases), i32(lengths), G.scale))
    assert m4.device_status() == m4.OK
    for t in range(16):
        b, n = int(bases[t]), int(lengths[t])
        ref = host(m4.kqkv(kc[b:b + n], q[t], None, G.scale))
        assert rel_to_max(got[t], ref) <= 1e-3, t


def test_ragged_window_outside_cache_is_reported(m4):
    lengths = [300, 200, 400]
    bases = [0, 900, 300]            # token 1 runs past the 1000-row cache
    kc = cache(77, 1000)
    qcur = normal(78, 3 * G.H * G.D).astype(np.float32).reshape(3, G.H, G.D)
    got = host(m4.kqkv_ragged(dev(kc), dev(qcur), i32(bases), i32(lengths), G.scale))
    assert m4.device_status() == m4.EINVAL
    assert np.all(got[1] == 0.0)
    for t in (0, 2):
        assert rel_to_max(got[t], oracle_attn(kc, qcur[t], bases[t], lengths[t])) <= ATTN_TOL
    assert m4.device_status() == m4.OK   # the status word was cleared by the read


def test_ragged_contract_violations(m4):
    kc = dev(cache(79, 256))
    q = torch.zeros(2, G.H, G.D, device="cuda")
    with pytest.raises(m4.M4Error):   # int64 windows
        m4.kqkv_ragged(kc, q, dev(np.zeros(2, np.int64)), dev(np.zeros(2, np.int64)), G.scale)
    with pytest.raises(m4.M4Error):   # window arrays shorter than the batch
        m4.kqkv_ragged(kc, q, i32([0]), i32([1]), G.scale)
    with pytest.raises(m4.M4Error):   # more than 64 tokens
        m4.kqkv_ragged(kc, torch.zeros(65, G.H, G.D, device="cuda"), i32([0] * 65),
                       i32([1] * 65), G.scale)
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(m4.M4Error):   # scratch too small
        m4.kqkv_ragged(kc, q, i32([0, 0]), i32([1, 1]), G.scale, scratch=small)


def test_ragged_graph_replay_follows_windows_in_device_memory(m4):
    rows = 12000
    kc_np = cache(80, rows)
    kc = dev(kc_np)
    qcur = normal(81, 4 * G.H * G.D).astype(np.float32).reshape(4, G.H, G.D)
    qd = dev(qcur)
    base = i32([0, 3000, 6000, 9000])
    length = i32([3000, 3000, 3000, 3000])
    out = torch.empty(4, G.H, G.R, device="cuda")
    scratch = torch.empty(m4.kqkv_ragged_scratch_bytes(4), dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        m4.kqkv_ragged(kc, qd, base, length, G.scale, out=out, scratch=scratch,
                       flags=m4.FLAG_PDL)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        m4.kqkv_ragged(kc, qd, base, length, G.scale, out=out, scratch=scratch,
                       flags=m4.FLAG_PDL)
    for lens, bases in (([3000, 1, 0, 2999], [0, 3000, 6000, 9000]),
                        ([12000, 129, 5000, 64], [0, 11000, 7000, 11936])):
        length.copy_(i32(lens))
        base.copy_(i32(bases))
        g.replay()
        got = host(out)
        for t in range(4):
            ref = oracle_attn(kc_np, qcur[t], bases[t], lens[t])
            if lens[t] == 0:
                assert np.all(got[t] == 0.0)
            else:
                assert rel_to_max(got[t], ref) <= ATTN_TOL, (lens, t)
    assert m4.device_status() == m4.OK


def test_ragged_layer_step_matches_oracle(m4):
    # WKB (batched) -> Qcur -> ragged KQKV -> W_UV (batched): one layer for 6 tokens
    q, w_uk, _, w_uv = make_layer(82, 1)
    T = 6
    qs = tokens(83, T)
    lengths = [700, 0, 2048, 129, 5000, 1]
    bases = packed_bases(lengths, gap=3)
    rows = int(bases[-1] + lengths[-1])
    kc = cache(84, rows)
    qd = dev(qs)
    qcur = torch.empty(T, G.H, G.D, device="cuda")
    qcur[:, :, G.R:] = qd[:, :, G.nope:]
    m4.wkb(dev(w_uk), qd[:, :, :G.nope], out=qcur[:, :, :G.R])
    attn = m4.kqkv_ragged(dev(kc), qcur, i32(bases), i32(lengths), G.scale)
    out = host(m4.phase_wvb(dev(w_uv), attn))
    for t in range(T):
        if lengths[t] == 0:
            assert np.all(out[t] == 0.0)
            continue
        _, _, _, ref = O.mla_step(w_uk, qs[t], kc[bases[t]:bases[t] + lengths[t]], None, w_uv,
                                  G.scale, G.nope)
        assert rel_to_max(out[t], ref) <= ATTN_TOL, t
