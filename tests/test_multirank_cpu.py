"""World-size-2 gloo tests (CPU) of the multi-GPU host logic: the KV-slab sharding with the
partial-record all-gather + merge gives the single-rank result, and a rank that dies before the
exchange makes its peer's collective fail with an error instead of hanging.  No GPU involved:
the partial records come from the oracle, the exchange is gloo."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from aubier_b200.shard import kv_slabs


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _slab_worker(rank, world, port, result_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests")]
    from mla_inputs import BASELINE as G, make_layer
    from oracle import oracle as O
    _init(rank, world, port)
    N = 3000
    q, w_uk, kc, w_uv = make_layer(91, N)
    qcur = np.concatenate([O.wkb(w_uk, q, G.nope), q[:, G.nope:]], axis=1)
    b, e = kv_slabs(N, world)[rank]
    # this rank's slab as two local splits, like the kernel's split-K records
    mid = (b + e) // 2
    local = np.stack([O.kqkv_partial(kc, b, mid, qcur, None, G.scale, G.R),
                      O.kqkv_partial(kc, mid, e, qcur, None, G.scale, G.R)])
    t = torch.from_numpy(local)
    gathered = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(gathered, t)
    merged = O.combine(torch.cat(gathered).numpy())
    out = O.wvb(w_uv, merged)
    if rank == 0:
        single = O.wvb(w_uv, O.combine(O.kqkv_partial(kc, 0, N, qcur, None, G.scale, G.R)[None]))
        np.save(result_path, np.stack([out, single]))
    dist.barrier()
    dist.destroy_process_group()


def test_kv_slab_exchange_matches_single_rank(tmp_path):
    path = str(tmp_path / "res.npy")
    mp.spawn(_slab_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    out, single = np.load(path)
    # W_UV rounds the merged attention to f16 (as the reference's mul_mat does), so a merge that
    # differs in the last f32 bits can flip single f16 roundings: 1e-4 of max
    assert np.abs(out - single).max() / np.abs(single).max() <= 1e-4


def _dead_peer_worker(rank, world, port, result_path):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(0)             # leaves between steps, before the exchange
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as e:     # gloo reports the lost peer / timeout as an error
        outcome = "error:" + type(e).__name__
    with open(result_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_lost_rank_fails_the_exchange_instead_of_hanging(tmp_path):
    path = str(tmp_path / "outcome.txt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, path)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung on a lost peer")
    with open(path) as f:
        assert f.read().startswith("error:")


def _ragged_worker(rank, world, port, result_path):
    """Config 5's sharding on gloo ranks: whole sequences per rank by LPT on key counts, each rank
    packs its own sequences' caches back to back and runs every token over its window [base,
    base + len) of that packed cache (the engine's batch mask, m1_layer.cpp:756-773; the batch rig's
    per-sequence regions, tools/m1_batch_test.cpp:19-24), then rank 0 gathers the outputs."""
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests")]
    from aubier_b200.shard import lpt_assign, packed_bases
    from mla_inputs import BASELINE as G, make_layer
    from oracle import oracle as O
    _init(rank, world, port)
    lengths = [300, 1000, 129, 2000, 50, 700, 1, 1500]
    _, w_uk, _, w_uv = make_layer(95, 1)
    mine = lpt_assign(lengths, world)[rank]
    # sequence i's cache and query depend on i only, not on the rank that holds it
    caches = {i: make_layer(200 + i, lengths[i])[2] for i in mine}
    queries = {i: make_layer(200 + i, 1)[0] for i in mine}
    packed = np.concatenate([caches[i] for i in mine]) if mine else None
    bases = packed_bases([lengths[i] for i in mine])
    outs = {}
    for i, base in zip(mine, bases):
        window = packed[base:base + lengths[i]]
        _, _, _, out = O.mla_step(w_uk, queries[i], window, None, w_uv, G.scale, G.nope)
        outs[i] = out
    gathered = [None] * world
    dist.all_gather_object(gathered, outs)
    if rank == 0:
        got = {}
        for part in gathered:
            for i, out in part.items():
                assert i not in got, f"sequence {i} ran on two ranks"
                got[i] = out
        assert sorted(got) == list(range(len(lengths))), "a sequence ran nowhere"
        single = [O.mla_step(w_uk, make_layer(200 + i, 1)[0], make_layer(200 + i, n)[2], None,
                             w_uv, G.scale, G.nope)[3] for i, n in enumerate(lengths)]
        np.save(result_path, np.stack([np.stack([got[i] for i in range(len(lengths))]),
                                       np.stack(single)]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ragged_batch_sharded_by_sequence_matches_single_rank(tmp_path, world):
    path = str(tmp_path / "ragged.npy")
    mp.spawn(_ragged_worker, args=(world, _free_port(), path), nprocs=world, join=True)
    sharded, single = np.load(path)
    assert np.array_equal(sharded, single)   # same per-token arithmetic, only the placement moved
