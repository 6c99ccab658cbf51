"""Multi-GPU parity of the fused KV-slab exchange (m4b_exchange_*): each rank owns one GPU and one
contiguous slab of the cache, computes split-K records over it, publishes one merged record per
head into every peer over NVLink and merges all ranks' records before W_UV.  The result must
match the oracle's single-GPU layer step on the whole cache (the reference runs on one GPU,
engine/m1_engine.cpp:2165).  Covers repeated exchanges (the double-buffered receive halves),
a CUDA-graph replay of several layers, a mask under which one rank's slab is fully masked, and the
one-launch form of the exchange (m4b_exchange_merge_wvb) against the two-launch form.

Needs at least 2 GPUs; skipped otherwise.  Handles travel over a gloo group on 127.0.0.1; the
data path uses no library collective.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from helpers import ATTN_TOL, rel_to_max
from mla_inputs import BASELINE as G, make_layer, window_mask
from oracle import oracle as O

pytestmark = pytest.mark.gpu

N_KEYS = 6144
SEEDS = (401, 402, 403)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _masks():
    """Per-layer masks: none, a window inside the first slab only (later slabs fully masked),
    and a window straddling every slab boundary."""
    return [None, window_mask(N_KEYS, 100, 1500), window_mask(N_KEYS, 1000, 4000)]


def _worker(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests")]
    import torch.distributed as dist
    from aubier_b200 import m4
    from aubier_b200.exchange import PeerExchange
    from aubier_b200.shard import kv_slabs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    b, e = kv_slabs(N_KEYS, world)[rank]
    layers = []
    for seed, mask in zip(SEEDS, _masks()):
        q, w_uk, kc, w_uv = make_layer(seed, N_KEYS)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        qd = t(q)
        qcur = torch.empty(G.H, G.D, device=dev)
        qcur[:, G.R:] = qd[:, G.nope:]
        layers.append(dict(q=qd, w_uk=t(w_uk), kc=t(kc[b:e]), w_uv=t(w_uv), qcur=qcur,
                           mask=None if mask is None else t(mask[b:e])))
    x = PeerExchange(world, rank)
    S = m4.default_splits(e - b)
    part = torch.empty(S, G.H, m4.PART_STRIDE, device=dev)
    attn = torch.empty(len(layers), G.H, G.R, device=dev)
    out = torch.empty(len(layers), G.H, G.V, device=dev)

    def layer_step(i, flags, fused):
        L = layers[i]
        m4.wkb(L["w_uk"], L["q"][:, :G.nope], out=L["qcur"][:, :G.R], flags=flags)
        m4.kqkv_partials(L["kc"], L["qcur"], L["mask"], G.scale, out=part, flags=flags)
        if fused:   # one launch: merge, publish, wait, merge, W_UV
            x.merge_wvb(part, L["w_uv"], out=out[i], attn_out=attn[i], flags=flags)
        else:
            x.publish(part, flags=flags)
            x.combine_wvb(L["w_uv"], out=out[i], attn_out=attn[i], flags=flags)

    results = {}
    for mode, fused in (("two", False), ("one", True)):   # both share the exchange's epochs
        dist.barrier()
        # eager: 7 exchanges cycle both receive halves; keep the last result per layer
        for k in range(7):
            layer_step(k % 3, 0, fused)
        torch.cuda.synchronize()
        results[f"{mode}_eager_attn"], results[f"{mode}_eager_out"] = attn.cpu().numpy(), out.cpu().numpy()
        attn.zero_()
        out.zero_()
        # one CUDA graph over the three layers with PDL, replayed three times
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(3):
                layer_step(i, m4.FLAG_PDL, fused)
        dist.barrier()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        results[f"{mode}_graph_attn"], results[f"{mode}_graph_out"] = attn.cpu().numpy(), out.cpu().numpy()
        del g
    results["status"] = np.array(m4.device_status())
    x.close()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **results)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_matches_single_gpu_oracle(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, have {torch.cuda.device_count()}")
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    refs = []
    for seed, mask in zip(SEEDS, _masks()):
        q, w_uk, kc, w_uv = make_layer(seed, N_KEYS)
        _, _, a, o = O.mla_step(w_uk, q, kc, mask, w_uv, G.scale, G.nope)
        refs.append((a, o))
    for r in range(world):
        res = np.load(tmp_path / f"rank{r}.npz")
        assert int(res["status"]) == 0, f"rank {r}: device status {int(res['status'])}"
        for mode in ("two", "one"):
            for kind in ("eager", "graph"):
                for i, (a, o) in enumerate(refs):
                    assert rel_to_max(res[f"{mode}_{kind}_attn"][i], a) <= ATTN_TOL, (r, mode, kind, i)
                    assert rel_to_max(res[f"{mode}_{kind}_out"][i], o) <= ATTN_TOL, (r, mode, kind, i)
        # the one-launch exchange merges with the two launches' arithmetic; only W_UV's order differs
        for kind in ("eager", "graph"):
            assert np.array_equal(res[f"one_{kind}_attn"], res[f"two_{kind}_attn"]), (r, kind)
            assert rel_to_max(res[f"one_{kind}_out"], res[f"two_{kind}_out"]) <= 1e-5, (r, kind)
