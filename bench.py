#!/usr/bin/env python
"""bench.py -- MLA decode-attention layer-steps/s on B200 for aubier's fused M4 path.

Workload (the default): one decode token over a 262,144-key latent+rope f16 KV
cache, 36 layers, each with its own seeded W_UK / W_UV / cache and its own f32 window mask (the
engine's, resident on the device); 32 heads, q_nope 128, rope 64, latent 512, V head 128,
kq_scale 1/sqrt(192).  One step = the 36 layer-steps WKB -> KQKV -> PHASE(combine + W_UV),
captured in one CUDA graph.  With N GPUs the 262,144 keys of every layer are split into N
contiguous slabs (strong scaling): each rank computes split-K partials over its slab, merges them
into one record per head and stores it into every peer over NVLink (fused exchange; --exchange
nccl uses an NCCL all-gather instead), then merges all ranks' records and applies W_UV.

--config 2 / 3: the same step at 4,096 / 32,768 keys (at N=1 the default run also measures both
and reports them under "other_configs"; at every N it also measures config 5 there).
--config 5: ragged batched decode, 16 sequences with one new token each, lengths uniform on
[512, 65536] by seed, one packed cache per layer with per-sequence base/length; whole sequences
per rank (LPT on keys), no exchange.  A layer-step covers all 16 sequences.

Printed JSON line (rank 0): value = layer-steps/s of the whole job, timed on the device (max over
ranks) around exactly --steps graph replays; e2e = the same metric with the step's queries copied
host->device and its outputs device->host inside the timed region; roofline = the KQKV kernel's
algorithmic bytes per launch over its CUDA-event-timed average launch, against the measured HBM
copy peak; cpu_baseline = the reference's own unfused CPU ggml graph (oracle/_ref) on this host,
median of >= 20 layer-steps; parity = the last layer of one more step against a float64
evaluation of the same inputs (slabs gathered from every rank), outside the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|4|5]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, NOPE, ROPE, R, V = 32, 128, 64, 512, 128
D, DQ = R + ROPE, NOPE + ROPE
SCALE = 1.0 / math.sqrt(DQ)
PART = R + 4
METRIC = "MLA decode attn layer-steps/s (262144 keys, 36 layers)"
METRIC_KEYS = "MLA decode attn layer-steps/s ({keys} keys, 36 layers)"
CONFIG_KEYS = {2: 4096, 3: 32768, 4: 262144}
METRIC5 = "MLA decode attn layer-steps/s (16 ragged sequences, 36 layers)"
METRIC_M = "MLA decode attn layer-steps/s (262144 keys, 36 layers, Mistral-Small-4 geometry)"
UNIT = "layer-steps/s"


def layer_bytes(n_keys: int, mask: bool = True) -> int:
    """Algorithmic bytes of one layer-step: KV once, the f32 mask when the op consumes it, weights
    once, q and the output."""
    return (1152 + (4 if mask else 0)) * n_keys + 2 * (H * R * NOPE * 2) + H * DQ * 4 + H * V * 4


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(name: str):
    """Per-launch DRAM bytes of the KQKV kernel from a committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1].split()[0]))
                    mx = float(parts[2].split()[0])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        load = [x for x in sm if mx is None or x > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# reference arm / CPU baseline: the reference's unfused CPU ggml graph (oracle/_ref)
# ---------------------------------------------------------------------------------------------
def _ref_graph(n_keys: int, threads: int, seed: int):
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    ref = O.RefMLA(H, NOPE, ROPE, R, V, n_keys, SCALE, n_threads=threads)
    ref.set_inputs(q=rng.standard_normal((H, DQ), dtype=np.float32),
                   w_uk=(0.02 * rng.standard_normal((H, R, NOPE), dtype=np.float32)).astype(np.float16),
                   kc=rng.standard_normal((n_keys, D), dtype=np.float32).astype(np.float16),
                   mask=np.zeros(n_keys, np.float32),
                   w_uv=(0.02 * rng.standard_normal((H, V, R), dtype=np.float32)).astype(np.float16))
    return ref


def cpu_reference(lengths, reps: int = 20, warmup: int = 1, budget_s: float = 30.0):
    """The reference's CPU graph for one layer-step of the workload: one single-token graph per
    sequence (config 4: one sequence of 262,144 keys), all host threads.  At least ``reps``
    layer-steps when they fit in about ``budget_s`` seconds (never fewer than 3); the value is
    the median over the timed layer-steps."""
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    refs = [_ref_graph(n, threads, 4 + i) for i, n in enumerate(lengths)]
    for _ in range(warmup):
        for r in refs:
            r.compute()
    times = []
    t_all = time.perf_counter()
    while len(times) < reps:
        t0 = time.perf_counter()
        for r in refs:
            r.compute()
        times.append(time.perf_counter() - t0)
        if len(times) >= 3 and time.perf_counter() - t_all > budget_s:
            break
    for r in refs:
        r.close()
    med = statistics.median(times)
    what = (f"{lengths[0]} keys" if len(lengths) == 1 else
            f"{len(lengths)} sequences, {sum(lengths)} keys in all")
    return {"value": 1.0 / med, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"median of {len(times)} x 1 layer-step ({what}; unfused ggml-cpu graph of "
                      f"engine/m1_layer.cpp:437-502, {O.ref_library_path().rsplit('/', 1)[-1]})",
            "s_per_layer_step": med, "reps": len(times)}


def workload_lengths(args):
    if args.config == 5:
        from aubier_b200.shard import ragged_lengths
        return ragged_lengths()
    return [args.keys]


def metric_of(args):
    if args.config == 5:
        return METRIC5
    return METRIC if args.keys == 262144 else METRIC_KEYS.format(keys=args.keys)


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    try:
        cb = cpu_reference(workload_lengths(args), reps=max(20, args.steps), warmup=args.warmup,
                           budget_s=120.0)
    except Exception as e:   # the oracle library travels prebuilt; report if it does not load
        print(json.dumps({"impl": "reference", "unavailable": f"oracle/_ref not loadable: {e}"}))
        return
    line = {"impl": "reference", "metric": metric_of(args), "value": cb["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": cb["reps"], "warmup": args.warmup,
            "ms_per_step": 1e3 / cb["value"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"BASELINE config {args.config}, 1 layer per step",
                       "keys": sum(workload_lengths(args)), "layers_per_step": 1},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# our arm: the two workloads
# ---------------------------------------------------------------------------------------------
class Workload:
    """Per-rank device state of one workload: ``step()`` enqueues the L layer-steps (WKB also
    writes each query's rope half into Qcur, so the device-timed and the e2e graphs do the same
    work), ``kq()`` the L launches of the dominant kernel alone; ``q``/``out`` are the per-step
    input / output buffers the e2e timing copies from / to the host."""

    def close(self):
        pass


def _layer_weights(L, dev):
    import torch
    g = torch.Generator(device=dev)
    wuk, wuv = [], []
    for layer in range(L):
        g.manual_seed(1000 * layer + 7)
        wuk.append((0.02 * torch.randn(H, R, NOPE, device=dev, generator=g)).half())
        wuv.append((0.02 * torch.randn(H, V, R, device=dev, generator=g)).half())
    return wuk, wuv, g


def slab_workload(args, rank, world, dev):
    """Configs 2-4: one token, N keys per layer (4,096 / 32,768 / 262,144), cut into one
    contiguous slab per rank; the per-head records cross GPUs once per layer (fused NVLink
    exchange, or NCCL).  Every layer's KQKV consumes its own f32 mask -- the engine's mask for the
    window [0, N) (m1_layer.cpp:756-773), resident on the device -- as the engine's graph does."""
    import torch
    import torch.distributed as dist
    from aubier_b200 import m4
    L, N = args.layers, args.keys
    assert N % world == 0, "keys must split evenly across ranks"
    n_loc = N // world
    S = m4.default_splits(n_loc)
    wuk, wuv, g = _layer_weights(L, dev)
    kc, qcur, mask = [], [], []
    q = torch.empty(L, H, DQ, device=dev)
    for layer in range(L):
        g.manual_seed(1000 * layer + 11 + 100003 * rank)   # weights replicated, slabs differ
        kc.append(torch.randn(n_loc, D, device=dev, generator=g).half())
        g.manual_seed(1000 * layer + 13)
        q[layer] = torch.randn(H, DQ, device=dev, generator=g)
        qc = torch.empty(H, D, device=dev)
        qc[:, R:] = q[layer][:, NOPE:]
        qcur.append(qc)
        mask.append(torch.zeros(n_loc, device=dev))
    w = Workload()
    part = torch.empty(S, H, PART, device=dev)
    merged = torch.empty(1, H, PART, device=dev)
    gathered = torch.empty(world, H, PART, device=dev) if world > 1 else part
    attn = torch.empty(H, R, device=dev)
    w.q, w.out = q, torch.empty(L, H, V, device=dev)
    xchg = None
    if world > 1 and args.exchange == "p2p":
        from aubier_b200.exchange import PeerExchange
        xchg = PeerExchange(world, rank)
        torch.cuda.synchronize()            # every rank's inputs exist before the first exchange
        dist.barrier()
    flags = m4.FLAG_PDL
    # the merge releases the next layer's launch once its W_UV loads are issued (with the
    # two-issuer KQKV this gains at every slab size, 262,144 keys included)
    early = m4.FLAG_EARLY_RELEASE

    def step():
        for layer in range(L):
            # WKB writes q_abs and (QCAT) the query's rope half: Qcur = concat(q_abs, q_pe)
            m4.wkb(wuk[layer], q[layer][:, :NOPE], out=qcur[layer][:, :R], flags=flags | m4.FLAG_QCAT)
            m4.kqkv_partials(kc[layer], qcur[layer], mask[layer], SCALE, out=part,
                             flags=flags | m4.FLAG_KV_STATIC)
            if xchg is not None:   # one launch: merge, NVLink stores into every peer, wait, merge, W_UV
                xchg.merge_wvb(part, wuv[layer], out=w.out[layer], attn_out=attn, flags=flags | early)
                continue
            if world > 1:   # library collective: merge the local splits, all-gather 66 KB per rank
                m4.phase_merge_records(part, out=merged, flags=flags)
                dist.all_gather_into_tensor(gathered, merged)
            m4.phase_combine_wvb(wuv[layer], gathered, out=w.out[layer], attn_out=attn,
                                 flags=flags | early)

    def kq():
        for layer in range(L):
            m4.kqkv_partials(kc[layer], qcur[layer], mask[layer], SCALE, out=part,
                             flags=m4.FLAG_PDL | m4.FLAG_KV_STATIC)

    def parity():
        """The last layer of the step just run (its attention is still in ``attn``) against a
        float64 evaluation of the same inputs on rank 0, the slabs gathered from every rank."""
        layer = L - 1
        if world > 1:
            full = torch.empty(world * n_loc, D, dtype=kc[layer].dtype, device=dev)
            dist.all_gather_into_tensor(full, kc[layer])
        else:
            full = kc[layer]
        if rank != 0:
            return None
        xa, xo = fp64_layer_torch(q[layer], wuk[layer], full, wuv[layer])
        return {"layer": layer, "keys": N,
                "rel_err_out": _rel_to_max(w.out[layer], xo),
                "rel_err_attn": _rel_to_max(attn, xa), "tol": 2e-3,
                "ref": "float64 torch evaluation of the same inputs (q and Qcur rounded to f16 "
                       "as the tensor cores and the CPU graph's mul_mat round them; attention "
                       "rounded to f16 before W_UV)"}

    w.step, w.kq, w.parity = step, kq, parity
    w.kq_kernel = "kqkv_partial_kernel"
    w.kq_bytes = (1152 + 4) * n_loc + H * D * 4
    w.job_layer_bytes = layer_bytes(N)
    # WKB, partials, merge + W_UV (one launch; with the fused exchange, the exchange too); the
    # NCCL variant adds the local record merge (NCCL's own kernel is not counted)
    w.launches_per_step = (3 if (world == 1 or xchg is not None) else 4) * L
    w.traffic = profiled_traffic("kqkv_partial_n262144.md") if N == 262144 else None
    if w.traffic is not None and world > 1:
        w.traffic = w.traffic / world        # the committed capture is of the 1-GPU slab
    cfg = {4096: 2, 32768: 3, 262144: 4}.get(N)
    w.metric = METRIC if N == 262144 else METRIC_KEYS.format(keys=N)
    w.config = {"workload": (f"BASELINE config {cfg}: " if cfg else "") +
                            f"1 decode token, {N}-key f16 latent+rope KV cache, {L} layers, 32 "
                            "heads, nope 128 / rope 64 / latent 512 / V 128",
                "keys": N, "layers": L, "keys_per_gpu": n_loc, "splits_per_gpu": S,
                "mask": "f32 [N] per layer, the engine's window mask, resident on the device "
                        "and read by every KQKV launch",
                "parallelism": f"kv-slab x{world}" + (
                    "" if world == 1 else
                    " + fused NVLink record exchange" if xchg is not None else
                    " + nccl all-gather of merged records"),
                "l2": f"inputs larger than L2 ({L} layers x {1156 * N / 1e6:.1f} MB KV + mask "
                      "per step)",
                "step": "WKB -> KQKV split-K partials -> PHASE combine+W_UV per layer, "
                        "one CUDA graph per step",
                "early_release": bool(early)}
    w.close = (lambda: xchg.close()) if xchg is not None else (lambda: None)
    w.lengths = [N]
    return w


def fp64_layer_torch(q, w_uk, kc, w_uv):
    """One layer step in float64 on the device, the arbiter of the bench's parity line: q_nope
    and Qcur rounded to f16 (the tensor-core operands; the reference CPU graph's mul_mat rounds
    its f32 src1 to f16 the same way), the attention rounded to f16 before W_UV, all sums in
    float64.  q (H, 192) f32, w_uk (H, 512, 128) f16, kc (N, 576) f16, w_uv (H, 128, 512) f16."""
    import torch
    f64 = torch.float64
    qn = q[:, :NOPE].half().to(f64)
    qabs = torch.einsum("hrk,hk->hr", w_uk.to(f64), qn)
    qc = torch.cat([qabs, q[:, NOPE:].to(f64)], 1).half().to(f64)
    K = kc.to(f64)
    p = torch.softmax((K @ qc.T) * SCALE, dim=0)       # (N, H)
    attn = p.T @ K[:, :R]
    out = torch.einsum("hvr,hr->hv", w_uv.to(f64), attn.half().to(f64))
    return attn, out


def _rel_to_max(x, ref) -> float:
    import torch
    d = (x.to(torch.float64) - ref).abs().max()
    return float(d / ref.abs().max().clamp_min(1e-300))


def _q8_bytes(rows: int, K: int, g, dev):
    """Q8_0 weights drawn on the device: int8 quants uniform on [-127, 127], f16 block scales
    around 4e-4 (the size N(0, 0.02) weights quantize to); ggml's 34-byte block layout."""
    import torch
    nb = K // 32
    quants = torch.randint(-127, 128, (rows, nb, 32), device=dev, generator=g, dtype=torch.int32)
    scales = (4e-4 * (0.5 + torch.rand(rows, nb, 1, device=dev, generator=g))).half()
    out = torch.empty(rows, nb, 34, dtype=torch.uint8, device=dev)
    out[:, :, :2] = scales.view(torch.uint8)
    out[:, :, 2:] = quants.to(torch.int8).view(torch.uint8)
    return out.view(rows, nb * 34)


def mistral_workload(args, rank, world, dev):
    """Config 4 at the reference's own geometry (Mistral-Small-4: latent 256, KV row 320, Q8_0
    weights), one GPU: per layer the engine's fused sequence -- KV-write of the new token's row
    (PHASE 0), WKB, KQKV split-K partials, merge + W_UV (PHASE 2)."""
    import torch
    from aubier_b200 import m4
    assert world == 1, "the Mistral-geometry line is a single-GPU measurement"
    L, N = args.layers, args.keys
    RM, DM, NOPEM, DQM = 256, 320, 64, 128
    S = m4.default_splits(N)
    g = torch.Generator(device=dev)
    wuk, wuv, wkv, nw, kc, cur, qcur = [], [], [], [], [], [], []
    q = torch.empty(L, H, DQM, device=dev)
    for layer in range(L):
        g.manual_seed(2000 * layer + 7)
        wuk.append(_q8_bytes(H * RM, NOPEM, g, dev).view(H, RM, -1))
        wuv.append(_q8_bytes(H * V, RM, g, dev).view(H, V, -1))
        wkv.append(_q8_bytes(DM, 4096, g, dev))
        nw.append(1.0 + 0.1 * torch.randn(RM, device=dev, generator=g))
        kc.append(torch.randn(N, DM, device=dev, generator=g).half())
        cur.append(torch.randn(4096, device=dev, generator=g))
        q[layer] = torch.randn(H, DQM, device=dev, generator=g)
        qc = torch.empty(H, DM, device=dev)
        qc[:, RM:] = q[layer][:, NOPEM:]
        qcur.append(qc)
    kidx = torch.tensor([N - 1], dtype=torch.int64, device=dev)   # the new token's row
    pos = torch.tensor([N - 1], dtype=torch.int32, device=dev)
    kcur = torch.empty(DM, device=dev)
    part = torch.empty(S, H, RM + 4, device=dev)
    attn = torch.empty(H, RM, device=dev)
    scale = 1.0 / math.sqrt(DQM)
    w = Workload()
    w.q, w.out = q, torch.empty(L, H, V, device=dev)
    flags = m4.FLAG_PDL   # no KV_STATIC: the KV-write two launches earlier writes the cache

    def step():
        for layer in range(L):
            m4.phase_kvwrite(cur[layer], wkv[layer], nw[layer], kc[layer], kidx, pos, out=kcur,
                             flags=flags)
            m4.wkb(wuk[layer], q[layer][:, :NOPEM], out=qcur[layer][:, :RM],
                   flags=flags | m4.FLAG_QCAT)
            m4.kqkv_partials(kc[layer], qcur[layer], None, scale, out=part, flags=flags)
            m4.phase_combine_wvb(wuv[layer], part, out=w.out[layer], attn_out=attn, flags=flags)

    def kq():
        for layer in range(L):
            m4.kqkv_partials(kc[layer], qcur[layer], None, scale, out=part,
                             flags=m4.FLAG_PDL | m4.FLAG_KV_STATIC)

    def parity():
        """The last layer's attention (after its KV-write) against a float64 evaluation from the
        same Qcur; the Q8_0 gemvs around it follow the fused reference's Q8_1 numerics and are
        checked against their restatement by the test suite, not here."""
        import torch
        layer = L - 1
        f64 = torch.float64
        qc = qcur[layer].half().to(f64)
        K = kc[layer].to(f64)
        p = torch.softmax((K @ qc.T) * scale, dim=0)
        xa = p.T @ K[:, :RM]
        return {"layer": layer, "keys": N, "rel_err_attn": _rel_to_max(attn, xa), "tol": 2e-3,
                "ref": "float64 torch evaluation of the attention from the same Qcur (rounded to "
                       "f16) and the cache after the KV-write"}

    w.step, w.kq, w.parity = step, kq, parity
    w.kq_kernel = "kqkv_partial_kernel<Geo<256>>"
    w.kq_bytes = 640 * N + H * DM * 4
    w.job_layer_bytes = (640 * N + H * RM * 68 + H * V * 272 + DM * 4352 + 4096 * 4 + H * DQM * 4
                         + H * V * 4)
    w.launches_per_step = 6 * L   # KV-write (2), WKB, partials, merge + W_UV (2)
    w.traffic = None
    w.metric = METRIC_M
    w.config = {"workload": "BASELINE config 4 at the Mistral-Small-4 geometry of the reference "
                            "(engine/m1_layer.h:47-55): 1 decode token, 262144-key f16 KV cache of "
                            "320-wide rows, 36 layers, 32 heads, nope 64 / rope 64 / latent 256 / "
                            "V 128, Q8_0 W_UK / W_UV / W_kva",
                "keys": N, "layers": L, "keys_per_gpu": N, "splits_per_gpu": S,
                "parallelism": "kv-slab x1",
                "l2": f"inputs larger than L2 ({L} layers x {640 * N / 1e6:.0f} MB KV per step)",
                "step": "KV-write -> WKB -> KQKV split-K partials -> PHASE combine+W_UV per layer, "
                        "one CUDA graph per step"}
    w.lengths = None
    return w


def ragged_workload(args, rank, world, dev):
    """Config 5: 16 sequences, one new token each, lengths uniform on [512, 65536] by seed, each
    layer's cache packed with per-sequence base/length; whole sequences per rank (LPT on keys),
    no exchange."""
    import torch
    import torch.distributed as dist
    from aubier_b200 import m4
    from aubier_b200.shard import lpt_assign, packed_bases, ragged_lengths
    L = args.layers
    lengths = ragged_lengths()
    mine = lpt_assign(lengths, world)[rank]
    assert mine, "more ranks than sequences"
    my_len = [lengths[i] for i in mine]
    T, rows = len(mine), sum(my_len)
    base = torch.tensor(packed_bases(my_len), dtype=torch.int32, device=dev)
    length = torch.tensor(my_len, dtype=torch.int32, device=dev)
    wuk, wuv, g = _layer_weights(L, dev)
    kc, qcur = [], []
    q = torch.empty(L, T, H, DQ, device=dev)
    for layer in range(L):
        parts = []
        for i in mine:      # sequence i's cache and query depend on (layer, i), not on the rank
            g.manual_seed(1000 * layer + 17 + 7919 * i)
            parts.append(torch.randn(lengths[i], D, device=dev, generator=g).half())
            q[layer, len(parts) - 1] = torch.randn(H, DQ, device=dev, generator=g)
        kc.append(torch.cat(parts))
        del parts
        qc = torch.empty(T, H, D, device=dev)
        qc[:, :, R:] = q[layer][:, :, NOPE:]
        qcur.append(qc)
    w = Workload()
    w.q, w.out = q, torch.empty(L, T, H, V, device=dev)
    attn = torch.empty(T, H, R, device=dev)
    scratch = torch.empty(m4.kqkv_ragged_scratch_bytes(T), dtype=torch.uint8, device=dev)
    flags = m4.FLAG_PDL

    def step():
        for layer in range(L):
            m4.wkb(wuk[layer], q[layer][:, :, :NOPE], out=qcur[layer][:, :, :R],
                   flags=flags | m4.FLAG_QCAT)
            m4.kqkv_ragged(kc[layer], qcur[layer], base, length, SCALE, out=attn, scratch=scratch,
                           flags=flags | m4.FLAG_KV_STATIC)
            m4.phase_wvb(wuv[layer], attn, out=w.out[layer], flags=flags)

    def kq():
        for layer in range(L):
            m4.kqkv_ragged(kc[layer], qcur[layer], base, length, SCALE, out=attn, scratch=scratch,
                           flags=m4.FLAG_PDL | m4.FLAG_KV_STATIC)

    def parity():
        """Every token of this rank in the last layer of the step just run against a float64
        evaluation of its window; the worst gap over all ranks is reported by rank 0."""
        layer = L - 1
        worst = torch.zeros(4, dtype=torch.float64, device=dev)   # max|d attn|, max|attn|, out ...
        bases = packed_bases(my_len)
        for t in range(T):
            kt = kc[layer][bases[t]:bases[t] + my_len[t]]
            xa, xo = fp64_layer_torch(q[layer][t], wuk[layer], kt, wuv[layer])
            v = torch.stack([(attn[t].double() - xa).abs().max(), xa.abs().max(),
                             (w.out[layer][t].double() - xo).abs().max(), xo.abs().max()])
            worst = torch.maximum(worst, v)
        if world > 1:
            dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        if rank != 0:
            return None
        wv = worst.tolist()
        return {"layer": layer, "tokens": len(lengths), "keys": sum(lengths),
                "rel_err_out": wv[2] / wv[3], "rel_err_attn": wv[0] / wv[1], "tol": 2e-3,
                "ref": "float64 torch evaluation of every token's window (q and Qcur rounded to "
                       "f16 as the tensor cores and the CPU graph's mul_mat round them; attention "
                       "rounded to f16 before W_UV); max gap over all tokens and ranks over the "
                       "max reference value"}

    w.step, w.kq, w.parity = step, kq, parity
    w.kq_kernel = "kqkv_partial_kernel (ragged) + kqkv_ragged_combine_kernel"
    w.kq_bytes = 1152 * rows + T * H * D * 4
    w.job_layer_bytes = 1152 * sum(lengths) + 2 * (H * R * NOPE * 2) + len(lengths) * (
        H * DQ * 4 + H * V * 4)
    w.launches_per_step = 4 * L
    w.traffic = profiled_traffic("kqkv_ragged_config5.md")
    w.metric = METRIC5
    w.config = {"workload": "BASELINE config 5: ragged batched decode, 16 sequences x 1 token, "
                            "KV lengths uniform on [512, 65536] (seed 5), packed f16 latent+rope "
                            "cache with per-sequence base/length, 36 layers, 32 heads",
                "keys": sum(lengths), "layers": L, "sequences": len(lengths),
                "keys_per_gpu": rows, "sequences_per_gpu": T,
                "parallelism": f"sequences x{world} (LPT on keys), no exchange",
                "l2": f"inputs larger than L2 ({L} layers x {1152 * sum(lengths) / 1e6:.0f} MB KV "
                      "per step)",
                "step": "WKB(16 tokens) -> ragged KQKV -> W_UV(16 tokens) per layer, "
                        "one CUDA graph per step"}
    w.lengths = lengths
    return w


def measure(w, args, rank: int, world: int, dev, sample_clocks: bool = True) -> dict:
    """Warm up, capture one CUDA graph per step, time exactly --steps replays (barrier and
    synchronize on both sides, max over ranks), then the e2e variant, the dominant kernel alone
    and the parity check of one freshly computed step.  Every rank takes the same collective
    steps in the same order."""
    import torch
    import torch.distributed as dist
    from aubier_b200 import m4
    L = args.layers

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(ms):
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- eager warm-up, then one CUDA graph per step
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            w.step()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        w.step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    status = m4.device_status()
    assert status == m4.OK, f"device status {status}"

    # ---- timed region: exactly --steps replays, barrier + synchronize on both sides
    sampler = ClockSampler(torch.cuda.current_device()) if (rank == 0 and sample_clocks) else None
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms_max = max_over_ranks(e0.elapsed_time(e1))
    r = {"ms_per_step": ms_max / args.steps, "value": L * args.steps / (ms_max * 1e-3),
         "clocks": clocks}

    # ---- end to end: host queries in, host outputs back, every step (the same seeded queries on
    # every rank: the ranks of one job share each token's query)
    q_dev = w.q.clone()
    q_host = torch.randn((args.steps,) + tuple(w.q.shape),
                         generator=torch.Generator().manual_seed(1234), pin_memory=True)
    out_host = torch.empty((args.steps,) + tuple(w.out.shape), pin_memory=True)
    graph_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_e2e):
        w.step()
    graph_e2e.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for k in range(args.steps):
        w.q.copy_(q_host[k], non_blocking=True)
        graph_e2e.replay()
        out_host[k].copy_(w.out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    r["e2e"] = {"value": L * args.steps / (max_over_ranks(e0.elapsed_time(e1)) * 1e-3),
                "unit": UNIT,
                "h2d_bytes_per_step": w.q.numel() * 4 * world,   # every rank copies its queries
                "d2h_bytes_per_step": w.out.numel() * 4 * world}

    # ---- the dominant kernel alone: one graph of its L launches, CUDA events around it
    graph_kq = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_kq):
        w.kq()
    graph_kq.replay()
    torch.cuda.synchronize()
    kreps = max(3, args.steps // 4)
    e0.record()
    for _ in range(kreps):
        graph_kq.replay()
    e1.record()
    torch.cuda.synchronize()
    kq_us = e0.elapsed_time(e1) * 1e3 / (kreps * L)
    peak, peak_kind = measured_peak()
    achieved = w.kq_bytes / (kq_us * 1e-6) / 1e9
    r["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": w.traffic, "peak_kind": peak_kind,
                     "kernel": w.kq_kernel, "kernel_us": kq_us,
                     "bytes_per_launch": w.kq_bytes,
                     "frac_of_nominal_8000": achieved / 8000.0}
    r["hbm_gbs_step"] = L * w.job_layer_bytes / (r["ms_per_step"] * 1e-3) / 1e9
    assert m4.device_status() == m4.OK
    del graph, graph_e2e, graph_kq           # release graphs before the process group

    # ---- parity: one eager step, its last layer against a float64 evaluation (outside timing)
    w.q.copy_(q_dev)
    w.step()
    torch.cuda.synchronize()
    assert m4.device_status() == m4.OK
    par = w.parity()
    if par is not None:   # the headline figure: the larger of the output's and attention's gaps
        par["rel_err"] = max(v for k, v in par.items() if k.startswith("rel_err_"))
        par["pass"] = par["rel_err"] <= par["tol"]
    r["parity"] = par
    return r


def cpu_baseline_of(lengths, reps):
    try:
        cb = cpu_reference(lengths, reps=reps)
        return {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    except Exception as e:
        return {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                "sample": f"unavailable: {e}"}


def run_ours(args, rank: int, world: int) -> None:
    import copy

    import torch

    dev = torch.device("cuda", torch.cuda.current_device())
    if args.geometry == "mistral":
        w = mistral_workload(args, rank, world, dev)
    else:
        w = (ragged_workload if args.config == 5 else slab_workload)(args, rank, world, dev)
    r = measure(w, args, rank, world, dev)
    w.close()                                # collective where the workload exchanges
    lengths, metric, config = w.lengths, w.metric, w.config
    launches = w.launches_per_step * args.steps
    del w
    torch.cuda.empty_cache()

    # beside the headline: configs 2 and 3 (4,096 and 32,768 keys, 36 layers) on one GPU, and
    # config 5 (16 ragged sequences, sharded by sequence over the ranks) at every GPU count
    others = []
    if (args.config == 4 and args.geometry == "baseline" and args.keys == 262144
            and not args.no_other_configs):
        for cfg in ((2, 3, 5) if world == 1 else (5,)):
            a2 = copy.copy(args)
            a2.config = cfg
            a2.keys = CONFIG_KEYS.get(cfg, args.keys)
            try:   # a failure that every rank meets alike costs this entry, not the headline line
                w2 = (ragged_workload if cfg == 5 else slab_workload)(a2, rank, world, dev)
                r2 = measure(w2, a2, rank, world, dev, sample_clocks=False)
                w2.close()
            except Exception as e:     # noqa: BLE001 -- reported in the JSON line
                others.append({"config": cfg, "error": f"{type(e).__name__}: {e}"[:300]})
                torch.cuda.empty_cache()
                continue
            r2 = {"config": cfg, "metric": w2.metric, "value": r2["value"], "unit": UNIT,
                  "ms_per_step": r2["ms_per_step"], "e2e": r2["e2e"], "roofline": r2["roofline"],
                  "hbm_gbs_step": r2["hbm_gbs_step"], "parity": r2["parity"],
                  "workload": w2.config["workload"], "parallelism": w2.config.get("parallelism"),
                  "gpu_launches": w2.launches_per_step * a2.steps}
            if world == 1 and not args.no_cpu_baseline:
                r2["cpu_baseline"] = cpu_baseline_of(w2.lengths, 20)
            others.append(r2)
            del w2
            torch.cuda.empty_cache()

    if rank != 0:
        return
    _restore_stdout()
    cpu_baseline = None
    if world == 1 and not args.no_cpu_baseline and lengths is not None:
        cpu_baseline = cpu_baseline_of(lengths, args.cpu_reps)
        if args.config == 4 and args.geometry == "baseline":
            # config 1: the reference's own CPU-runnable case, 256 keys, 1 layer-step
            cpu_baseline["config1"] = cpu_baseline_of([256], 200)
    line = {
        "metric": metric, "value": r["value"], "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": config, "hbm_gbs_step": r["hbm_gbs_step"],
        "roofline": r["roofline"], "cpu_baseline": cpu_baseline, "e2e": r["e2e"],
        "gpu_launches": launches, "clocks": r["clocks"], "parity": r["parity"],
    }
    if others:
        line["other_configs"] = others
    print(json.dumps(line), flush=True)


_SAVED_STDOUT = None


def _redirect_stdout():
    """Libraries (torch's NCCL process group, NCCL) print banners on fd 1; the contract is one JSON
    line on rank 0's stdout, so fd 1 points at stderr until that line is printed."""
    global _SAVED_STDOUT
    sys.stdout.flush()
    _SAVED_STDOUT = os.dup(1)
    os.dup2(2, 1)


def _restore_stdout():
    global _SAVED_STDOUT
    if _SAVED_STDOUT is not None:
        sys.stdout.flush()
        os.dup2(_SAVED_STDOUT, 1)
        os.close(_SAVED_STDOUT)
        _SAVED_STDOUT = None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=150)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--keys", type=int, default=None,
                    help="keys per layer (default: the config's, 262,144 for config 4)")
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--cpu-reps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="config 4: skip the lines beside the headline (configs 2 and 3 at N=1, "
                         "config 5 at every N)")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="config 4, N>1: fused NVLink exchange in the merge kernels, or NCCL")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=4,
                    help="2/3/4: 4,096 / 32,768 / 262,144-key slabs (4 is the headline); "
                         "5: 16 ragged sequences")
    ap.add_argument("--geometry", choices=["baseline", "mistral"], default="baseline",
                    help="mistral: config 4 at the reference's own model geometry (1 GPU)")
    args = ap.parse_args()
    if args.keys is None:
        args.keys = CONFIG_KEYS.get(args.config, 262144)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    _redirect_stdout()
    import datetime

    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        run_ours(args, rank, world)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
