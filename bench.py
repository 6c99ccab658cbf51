#!/usr/bin/env python
"""bench.py -- MLA decode-attention layer-steps/s on B200 for aubier's fused M4 path.

Workload: one decode token over a 262,144-key latent+rope f16 KV cache, 36
layers, each with its own seeded W_UK / W_UV / cache; 32 heads, q_nope 128, rope 64, latent 512,
V head 128, kq_scale 1/sqrt(192).  One step = the 36 layer-steps WKB -> KQKV -> PHASE(combine +
W_UV), captured in one CUDA graph.  With N GPUs the 262,144 keys of every layer are split into N
contiguous slabs (strong scaling); each rank computes split-K partials over its slab and the
each rank's partials are merged into one record per head (66 KB), all-gathered over NCCL, and
merged again with W_UV applied.

Printed JSON line (rank 0): value = layer-steps/s of the whole job, timed on the device (max over
ranks) around exactly --steps graph replays; e2e = the same metric with the step's queries copied
host->device and its outputs device->host inside the timed region; roofline = the KQKV kernel's
algorithmic bytes per launch over its CUDA-event-timed average launch, against the measured HBM
copy peak; cpu_baseline = the reference's own unfused CPU ggml graph (oracle/_ref) on this host.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
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
UNIT = "layer-steps/s"


def layer_bytes(n_keys: int) -> int:
    """Algorithmic bytes of one layer-step: KV once, weights once, q and the output (no mask)."""
    return 1152 * n_keys + 2 * (H * R * NOPE * 2) + H * DQ * 4 + H * V * 4


def kqkv_bytes(n_keys: int) -> int:
    """Algorithmic bytes of one KQKV launch: its KV slab once plus the f32 query."""
    return 1152 * n_keys + H * D * 4


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the KQKV kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "kqkv_partial_n262144.md")
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
def cpu_reference(n_keys: int, reps: int, warmup: int = 1, budget_s: float = 60.0):
    import numpy as np
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(4)
    ref = O.RefMLA(H, NOPE, ROPE, R, V, n_keys, SCALE, n_threads=threads)
    ref.set_inputs(q=rng.standard_normal((H, DQ), dtype=np.float32),
                   w_uk=(0.02 * rng.standard_normal((H, R, NOPE), dtype=np.float32)).astype(np.float16),
                   kc=rng.standard_normal((n_keys, D), dtype=np.float32).astype(np.float16),
                   mask=np.zeros(n_keys, np.float32),
                   w_uv=(0.02 * rng.standard_normal((H, V, R), dtype=np.float32)).astype(np.float16))
    for _ in range(warmup):
        ref.compute()
    t0 = time.perf_counter()
    done = 0
    while done < reps:        # bounded: at most `reps` layer-steps or about budget_s seconds
        ref.compute()
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    reps = done
    ref.close()
    kind = "reference"
    return {"value": reps / dt, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{reps} x 1 layer-step at {n_keys} keys (unfused ggml-cpu graph of "
                      f"engine/m1_layer.cpp:437-502, {O.ref_library_path().rsplit('/', 1)[-1]})",
            "s_per_layer_step": dt / reps, "reps": reps}


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    try:
        cb = cpu_reference(args.keys, reps=args.steps, warmup=args.warmup)
    except Exception as e:   # the oracle library travels prebuilt; report if it does not load
        print(json.dumps({"impl": "reference", "unavailable": f"oracle/_ref not loadable: {e}"}))
        return
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": cb["reps"], "warmup": args.warmup,
            "ms_per_step": 1e3 / cb["value"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"BASELINE config 4: 1 token, {args.keys} keys, 1 layer per step",
                       "keys": args.keys, "layers_per_step": 1},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def run_ours(args, rank: int, world: int) -> None:
    import torch
    import torch.distributed as dist
    from aubier_b200 import m4

    dev = torch.device("cuda", torch.cuda.current_device())
    L, N = args.layers, args.keys
    assert N % world == 0, "keys must split evenly across ranks"
    n_loc = N // world
    S = m4.default_splits(n_loc)

    # ---- per-layer state, generated on the device from fixed seeds (weights replicated, KV slabs
    # differ per rank); q_pe is part of the per-layer query input and is pre-placed into Qcur
    g = torch.Generator(device=dev)
    kc, wuk, wuv, q, qcur = [], [], [], [], []
    for layer in range(L):
        g.manual_seed(1000 * layer + 7)
        wuk.append((0.02 * torch.randn(H, R, NOPE, device=dev, generator=g)).half())
        wuv.append((0.02 * torch.randn(H, V, R, device=dev, generator=g)).half())
        q.append(torch.randn(H, DQ, device=dev, generator=g))
        g.manual_seed(1000 * layer + 11 + 100003 * rank)
        kc.append(torch.randn(n_loc, D, device=dev, generator=g).half())
        qc = torch.empty(H, D, device=dev)
        qc[:, R:] = q[-1][:, NOPE:]
        qcur.append(qc)
    part = torch.empty(S, H, PART, device=dev)
    merged = torch.empty(1, H, PART, device=dev)                 # this rank's record per head
    gathered = torch.empty(world, H, PART, device=dev) if world > 1 else part
    xchg = None
    if world > 1 and args.exchange == "p2p":
        from aubier_b200.exchange import PeerExchange
        xchg = PeerExchange(world, rank)
        torch.cuda.synchronize()            # every rank's inputs exist before the first exchange
        dist.barrier()
    attn = torch.empty(H, R, device=dev)
    out = torch.empty(L, H, V, device=dev)
    flags = m4.FLAG_PDL

    def step(with_rope_copy: bool = False):
        for layer in range(L):
            if with_rope_copy:   # e2e: the fresh query's rope half goes into Qcur as well
                qcur[layer][:, R:].copy_(q[layer][:, NOPE:])
            m4.wkb(wuk[layer], q[layer][:, :NOPE], out=qcur[layer][:, :R], flags=flags)
            m4.kqkv_partials(kc[layer], qcur[layer], None, SCALE, out=part,
                             flags=flags | m4.FLAG_KV_STATIC)
            if xchg is not None:   # fused: merge + NVLink stores into every peer, then wait+merge
                xchg.publish(part, flags=flags)
                xchg.combine_wvb(wuv[layer], out=out[layer], attn_out=attn, flags=flags)
                continue
            if world > 1:   # library collective: merge the local splits, all-gather 66 KB per rank
                m4.phase_merge_records(part, out=merged, flags=flags)
                dist.all_gather_into_tensor(gathered, merged)
            m4.phase_combine_wvb(wuv[layer], gathered, out=out[layer], attn_out=attn, flags=flags)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- eager warm-up, then one CUDA graph per step
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    status = m4.device_status()
    assert status == m4.OK, f"device status {status}"

    # ---- timed region: exactly --steps replays, barrier + synchronize on both sides
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
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
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = L * args.steps / (ms_max * 1e-3)

    # ---- end to end: host queries in, host outputs back, every step
    q_host = torch.randn(args.steps, L, H, DQ, pin_memory=True)
    out_host = torch.empty(args.steps, L, H, V, pin_memory=True)
    qbuf = torch.stack(q)                         # graph inputs are views of these buffers
    for layer in range(L):
        q[layer].data = qbuf[layer]
    graph_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_e2e):
        step(with_rope_copy=True)
    graph_e2e.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for k in range(args.steps):
        qbuf.copy_(q_host[k], non_blocking=True)
        graph_e2e.replay()
        out_host[k].copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = L * args.steps / (float(te.item()) * 1e-3)

    # ---- the dominant kernel alone: one graph of the L KQKV launches, CUDA events around it
    graph_kq = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_kq):
        for layer in range(L):
            m4.kqkv_partials(kc[layer], qcur[layer], None, SCALE, out=part,
                             flags=m4.FLAG_PDL | m4.FLAG_KV_STATIC)
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
    achieved = kqkv_bytes(n_loc) / (kq_us * 1e-6) / 1e9
    traffic = profiled_traffic()
    if traffic is not None and world > 1:
        traffic = traffic / world        # the committed capture is of the 1-GPU slab

    assert m4.device_status() == m4.OK
    del graph, graph_e2e, graph_kq           # release graphs before the process group
    if xchg is not None:
        xchg.close()                         # collective: detach, meet, free

    if rank != 0:
        return
    cpu_baseline = None
    _restore_stdout()
    if world == 1 and not args.no_cpu_baseline:
        try:
            cb = cpu_reference(N, reps=args.cpu_reps)
            cpu_baseline = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as e:
            cpu_baseline = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                            "sample": f"unavailable: {e}"}
    step_gbs = L * layer_bytes(N) / (ms_per_step * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "BASELINE config 4: 1 decode token, 262144-key f16 latent+rope KV "
                               "cache, 36 layers, 32 heads, nope 128 / rope 64 / latent 512 / V 128",
                   "keys": N, "layers": L, "keys_per_gpu": n_loc, "splits_per_gpu": S,
                   "parallelism": f"kv-slab x{world}" + (
                       "" if world == 1 else
                       " + fused NVLink record exchange" if args.exchange == "p2p" else
                       " + nccl all-gather of merged records"),
                   "l2": "inputs larger than L2 (36 layers x 302 MB KV per step)",
                   "step": "WKB -> KQKV split-K partials -> PHASE combine+W_UV per layer, "
                           "one CUDA graph per step"},
        "hbm_gbs_step": step_gbs,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": "kqkv_partial_kernel", "kernel_us": kq_us,
                     "frac_of_nominal_8000": achieved / 8000.0},
        "cpu_baseline": cpu_baseline,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": L * H * DQ * 4,
                "d2h_bytes_per_step": L * H * V * 4},
        "gpu_launches": (4 + (1 if world > 1 else 0)) * L * args.steps,   # p2p: publish+gather
                                                                             # replace merge+combine
        "clocks": clocks,
    }
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
    ap.add_argument("--keys", type=int, default=262144)
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--cpu-reps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: fused NVLink exchange in the merge kernels, or NCCL all-gather")
    args = ap.parse_args()

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
