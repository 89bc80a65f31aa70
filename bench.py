#!/usr/bin/env python3
"""Benchmark: SMat block-sparse causal softmax attention fwd+bwd on B200.

Workload: B=4, H=32, T=16384, D=128, block 128, local
window 4, stride-8 summary blocks, 2 sink blocks, bf16 inputs with fp32 LSE
and accumulators; Q/K/V/dO i.i.d. N(0,1) (seed 2 + rank), scale 1/sqrt(D).
A step is one forward (O, LSE) plus one backward (dQ, dK, dV) over the batch.

Metric: effective TFLOP/s counting only unmasked (i, j) pairs,
F = 3.5 * 4 * D * pairs * B * H per step (pairs per head from the layout).
Multi-GPU (torchrun): every rank processes its own batch of the same shape
((batch, head) partition, no collective on the data path; "weak" scaling);
value = N * F / max-over-ranks time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --workload c5 [--shard heads|queries] ...   (long context)

``--workload c5`` runs BASELINE config 5 (B=1, H=32, T=131072) with the
total work fixed ("strong" scaling): ``--shard heads`` gives every rank
H / N heads (no collective); ``--shard queries`` gives every rank a zig-zag
share of the query tiles of every head, with the K/V exchange before the
forward and the dK/dV return after the backward inside the timed step
(smat_attention_b200.sharding).

``--impl reference`` times the reference's CPU dense-masked path (the oracle
port in ``oracle/``) on this host's cores on a bounded sample of the same
workload and prints the same JSON line with ``"impl": "reference"``.
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
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

WORKLOADS = {
    "c3": dict(name="c3", B=4, H=32, T=16384, D=128, block=128, window=4, stride=8, sinks=2,
               seed=2),
    # long context: B=1 leaves 32 (b, h) pairs; sharded by heads or by query blocks
    "c5": dict(name="c5", B=1, H=32, T=131072, D=128, block=128, window=8, stride=32, sinks=4,
               seed=4),
    # LM training step, batch 8 x 8192 per rank
    "c4": dict(name="c4", B=8, seed=3),
    # decode over a c3-shaped KV cache
    "decode": dict(name="decode", seed=2),
    # the reference's kernelised op (pooled schedule) on B200 kernels
    "kattn": dict(name="kattn", seed=5),
    # the reference's own mask family on the c3 shapes: M^(3) at chunk 128
    # (n = 8192 landmarks, C 552 x 529), tiled by 128 as a pattern layout
    "md3": dict(name="md3", B=4, H=32, T=16384, D=128, block=128, d=3, chunk=128, seed=2),
}
WORKLOAD = dict(WORKLOADS["c3"])
METRIC = "SMat attn fwd+bwd effective TFLOP/s (unmasked FLOPs)"
UNIT = "TFLOP/s"


def _layout_pairs():
    """The workload's mask (a block layout, or an M^(d) spec) and its unmasked
    pairs per head."""
    from smat_attention_b200.mask import block_layout_stats, build_block_mask, build_mask
    w = WORKLOAD
    if "d" in w:
        spec = build_mask(w["T"], w["d"], chunk=w["chunk"])
    else:
        spec = build_block_mask(w["T"], w["block"], w["window"], w["stride"], w["sinks"])
    return spec, block_layout_stats(spec)["pairs"]


def _describe(H=None):
    w = WORKLOAD
    H = w["H"] if H is None else H
    head = f"{w['name']}: B={w['B']} H={H} T={w['T']} D={w['D']} bs={w['block']} "
    if "d" in w:
        return head + f"M^({w['d']}) chunk={w['chunk']} (reference build_mask) fwd+bwd per rank"
    return head + f"W={w['window']} S={w['stride']} sinks={w['sinks']} fwd+bwd per rank"


def _flops(pairs):
    w = WORKLOAD
    fwd = 4.0 * w["D"] * pairs * w["B"] * w["H"]
    return {"fwd": fwd, "dkdv": 2.0 * fwd, "dq": 1.5 * fwd, "bwd": 2.5 * fwd, "step": 3.5 * fwd}


def _tensor_mib():
    w = WORKLOAD
    return w["B"] * w["H"] * w["T"] * w["D"] * 2 // (1 << 20)


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"tflops": float(p["bf16_tflops_sustained"]), "hbm": float(p["hbm_gbs"]),
                "source": "measured (MEASURED_PEAKS.json, bf16_tflops_sustained)"}
    except (OSError, KeyError, ValueError):
        return {"tflops": 1400.0, "hbm": 6650.0,
                "source": "fallback (1.4 PFLOP/s sustained, 6.65 TB/s)"}


def _traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/), if one is present."""
    path = os.path.join(ROOT, "profiles", "traffic_c3.txt")
    out = {}
    try:
        for line in open(path):
            m = re.match(r"\s*(\w+)\s+dram_bytes_per_launch\s*=\s*([0-9.eE+]+)", line)
            if m:
                out[m.group(1)] = float(m.group(2))
    except OSError:
        pass
    return out


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        load = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        rank = int(os.environ["RANK"])
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        return dist, rank, ws, local
    return None, 0, 1, 0


def _barrier(dist, device):
    if dist is not None:
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


def _max_over_ranks(dist, value, device):
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------
# CPU baseline: the reference's dense-masked path (oracle port) on host cores
# ----------------------------------------------------------------------------

def cpu_sample(reps=1):
    """Time the oracle's dense-masked fp32 forward + backward on one (batch,
    head) of the workload at the full sequence length; returns the effective
    TFLOP/s of that head and a description."""
    from oracle import layout as OL
    from oracle.dense_softmax import rowchunked_masked_softmax
    w = WORKLOAD
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    spec, pairs = _layout_pairs()
    g = torch.Generator().manual_seed(w["seed"])
    q, k, v, do = (torch.randn(1, w["T"], w["D"], generator=g).to(torch.bfloat16).float()
                   for _ in range(4))
    if "d" in w:
        from smat_attention_b200.mask import materialise
        dense = torch.from_numpy(materialise(spec, np.uint8))
        rows = lambda r0, r1: dense[r0:r1]
    else:
        rows = OL.block_mask_rows(w["T"], w["block"], w["window"], w["stride"], w["sinks"])
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        rowchunked_masked_softmax(q, k, v, do, rows, 1 / math.sqrt(w["D"]), rows=2048)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    f_head = 3.5 * 4.0 * w["D"] * pairs
    return {"value": f_head / t / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"one (b,h) head of {w['name']} (T={w['T']}, D={w['D']}) dense-masked "
                      f"fp32 fwd+bwd, oracle port, median of {reps}: {t:.2f} s/head"}


def _config(ws, strong, H_rank):
    """The `config` of the attention workloads' JSON line (both arms):
    H_rank is the heads each rank runs."""
    w = WORKLOAD
    return {"workload": _describe(H_rank),
            "global_batch": w["B"] * (1 if strong else ws), "seq_len": w["T"],
            "heads": H_rank * (ws if strong else 1), "head_dim": w["D"],
            "parallelism": (f"head partition x{ws}" if strong
                            else f"(batch,head) partition x{ws}"),
            "l2": f"inputs larger than L2 ({w['B'] * H_rank * w['T'] * w['D'] * 2 >> 20} MiB "
                  f"per tensor); no flush"}


def run_reference(args):
    dist, rank, ws, local = _dist()
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    for _ in range(max(0, args.warmup)):
        pass   # the CPU sample needs no device warm-up; each step is a full sample
    vals = []
    t0 = time.perf_counter()
    steps = max(1, args.steps)
    base = None
    for _ in range(steps):
        base = cpu_sample(reps=1)
        vals.append(base["value"])
    elapsed = time.perf_counter() - t0
    v = statistics.median(vals)
    base["value"] = v
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
            "warmup": args.warmup, "ms_per_step": elapsed / steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": _config(args.gpus, WORKLOAD["name"] == "c5",
                              WORKLOAD["H"] // args.gpus if WORKLOAD["name"] == "c5"
                              else WORKLOAD["H"]),
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------

def _e2e(host, shape, device, spec, scale, K, dist, stream):
    """Same step through the public autograd API with pinned host buffers:
    per step H2D of q, k, v, dO and D2H of o, dq, dk, dv inside the timed
    region.  The batch goes through in slices of one sequence, pipelined the
    way a caller streaming from host memory would: the H2D of slice b + 1 (a
    copy stream) and the D2H of slice b - 1 (another) overlap the attention
    of slice b (slices of 8 heads measured slower: the smaller launches do
    not fill the GPU).  Returns (ms per step, bytes each way per step)."""
    from smat_attention_b200.attention import smat_softmax_attention
    pinned = [x.pin_memory() for x in host]
    outs = [torch.empty(shape, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    E = max(1, min(K, 3))
    h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def e2e_step():
        for b in range(shape[0]):
            sl = slice(b, b + 1)
            with torch.cuda.stream(h2d):
                ins = [x[sl].to(device, non_blocking=True) for x in pinned]
            stream.wait_stream(h2d)
            for t in ins:
                t.record_stream(stream)
            qd, kd, vd, dod = ins
            qd.requires_grad_(True)
            kd.requires_grad_(True)
            vd.requires_grad_(True)
            od, _ = smat_softmax_attention(qd, kd, vd, spec, scale)
            od.backward(dod)
            d2h.wait_stream(stream)
            with torch.cuda.stream(d2h):
                for dst, src in zip(outs, (od.detach(), qd.grad, kd.grad, vd.grad)):
                    dst[sl].copy_(src, non_blocking=True)
                    src.record_stream(d2h)
        stream.wait_stream(d2h)   # the step ends when its last result is on the host

    e2e_step()
    torch.cuda.synchronize(device)
    _barrier(dist, device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(E):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(dist, e0.elapsed_time(e1) / E, device)
    nbytes = sum(x.numel() * x.element_size() for x in host)

    return e2e_ms, nbytes


def run_gpu(args):
    from smat_attention_b200 import _lib
    from smat_attention_b200.attention import (bwd, check_device_errors, fwd,
                                               layout_device_args, smat_softmax_attention)
    dist, rank, ws, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = WORKLOAD
    strong = w["name"] == "c5"
    if strong:
        # total work fixed: this rank's share of the heads
        if w["H"] % ws:
            raise SystemExit(f"H={w['H']} does not split over {ws} ranks")
        w["H"] //= ws
    spec, pairs = _layout_pairs()
    fl = _flops(pairs)
    scale = 1.0 / math.sqrt(w["D"])
    g = torch.Generator().manual_seed(w["seed"] + rank)
    shape = (w["B"], w["H"], w["T"], w["D"])
    host = [torch.randn(*shape, generator=g).to(torch.bfloat16) for _ in range(4)]
    q, k, v, do = (x.to(device) for x in host)
    L = _lib.lib()
    lay = layout_device_args(spec, device)
    o = torch.empty_like(q)
    lse = torch.empty(w["B"], w["H"], w["T"], dtype=torch.float32, device=device)
    delta = torch.empty_like(lse)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    sp = _lib.strides3
    B, H, T, D = shape

    def launch_fwd():
        _lib.check("smat_fwd", L.smat_fwd(
            1, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v), o.data_ptr(), sp(o),
            lse.data_ptr(), B, H, T, D, lay["indptr"].data_ptr(), lay["indices"].data_ptr(),
            lay["kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"],
            scale, err.data_ptr(), stream.cuda_stream))

    def launch_pre():
        _lib.check("smat_bwd_preprocess", L.smat_bwd_preprocess(
            1, o.data_ptr(), sp(o), do.data_ptr(), sp(do), delta.data_ptr(), B, H, T, D,
            stream.cuda_stream))

    def launch_dkdv():
        _lib.check("smat_bwd_dkdv", L.smat_bwd_dkdv(
            1, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v), do.data_ptr(),
            sp(do), lse.data_ptr(), delta.data_ptr(), dk.data_ptr(), sp(dk), dv.data_ptr(),
            sp(dv), B, H, T, D, lay["t_indptr"].data_ptr(), lay["t_indices"].data_ptr(),
            lay["t_kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"],
            lay["t_max_row"], scale, err.data_ptr(), stream.cuda_stream))

    def launch_dq():
        _lib.check("smat_bwd_dq", L.smat_bwd_dq(
            1, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v), do.data_ptr(),
            sp(do), lse.data_ptr(), delta.data_ptr(), dq.data_ptr(), sp(dq), B, H, T, D,
            lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
            lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"], scale, err.data_ptr(),
            stream.cuda_stream))

    def launch_fwd_pattern():
        _lib.check("smat_fwd_pattern", L.smat_fwd_pattern(
            1, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v), o.data_ptr(), sp(o),
            lse.data_ptr(), B, H, T, D, lay["indptr"].data_ptr(), lay["indices"].data_ptr(),
            lay["kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"],
            lay["pattern"], scale, err.data_ptr(), stream.cuda_stream))

    def launch_bwd_pattern():
        _lib.check("smat_bwd_pattern", L.smat_bwd_pattern(
            1, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v), o.data_ptr(), sp(o),
            do.data_ptr(), sp(do), lse.data_ptr(), delta.data_ptr(), dq.data_ptr(), sp(dq),
            dk.data_ptr(), sp(dk), dv.data_ptr(), sp(dv), B, H, T, D,
            lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
            lay["t_indptr"].data_ptr(), lay["t_indices"].data_ptr(), lay["t_kind"].data_ptr(),
            lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"], lay["t_max_row"],
            lay["pattern"], scale, err.data_ptr(), stream.cuda_stream))

    if lay["pattern"] is None:
        kernels = [("fwd", launch_fwd), ("bwd_pre", launch_pre), ("dkdv", launch_dkdv),
                   ("dq", launch_dq)]
        launches_per_step = 4
    else:
        # M^(d): the pattern entry points (the backward launches its three passes)
        kernels = [("fwd", launch_fwd_pattern), ("bwd", launch_bwd_pattern)]
        launches_per_step = 4
    for _ in range(max(3, args.warmup)):
        for _, fn in kernels:
            fn()
    _barrier(dist, device)

    # ---- device-resident timed region --------------------------------------
    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(kernels) + 1)]
          for _ in range(K)]
    clocks = ClockSampler(device)
    _barrier(dist, device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(K):
        ev[s][0].record(stream)
        for i, (_, fn) in enumerate(kernels):
            fn()
            ev[s][i + 1].record(stream)
    stop.record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    _barrier(dist, device)
    total_ms = start.elapsed_time(stop)
    per_kernel = {name: sum(ev[s][i].elapsed_time(ev[s][i + 1]) for s in range(K)) / K
                  for i, (name, _) in enumerate(kernels)}
    dev_err = int(err.item())
    ms_step = _max_over_ranks(dist, total_ms / K, device)
    value = ws * fl["step"] / (ms_step * 1e-3) / 1e12

    # ---- end to end through the public API with host buffers ---------------
    e2e_ms, nbytes = None, 0
    if not args.no_e2e:
        e2e_ms, nbytes = _e2e(host, shape, device, spec, scale, K, dist, stream)
    dev_err |= check_device_errors(device)

    if rank == 0:
        peaks = _peaks()
        dom = max(per_kernel, key=per_kernel.get)
        achieved = fl[dom if dom in fl else "fwd"] / (per_kernel[dom] * 1e-3) / 1e12 \
            if dom != "bwd_pre" else None
        traffic = _traffic().get(dom)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": K,
            "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": _config(ws, strong, w["H"]),
            "tokens_per_s": (1 if strong else ws) * w["B"] * w["T"] / (ms_step * 1e-3),
            "frac_of_peak": value / ws / peaks["tflops"],
            "peak_source": peaks["source"],
            "per_kernel_ms": per_kernel,
            "roofline": {"bound": "tensor", "kernel": dom, "achieved": achieved,
                         "peak": peaks["tflops"], "unit": UNIT,
                         "frac": None if achieved is None else achieved / peaks["tflops"],
                         "traffic": traffic},
            "e2e": None if e2e_ms is None else {
                "value": ws * fl["step"] / (e2e_ms * 1e-3) / 1e12, "unit": UNIT,
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": nbytes,
                "d2h_bytes_per_step": nbytes},
            "gpu_launches": K * launches_per_step,
            "device_errors": dev_err,
            "clocks": clk,
        }
        if ws == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_sample(reps=1)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_lm(args):
    """training steps (forward, backward, AdamW on fp32
    masters) of the 12-layer LM with the block-sparse arm in every layer, on
    uniform synthetic token IDs.  Data parallel over the ranks: every rank
    runs the full per-rank batch and the bf16 gradients are all-reduced
    (one NCCL call over a flat buffer) before the optimizer step."""
    from smat_attention_b200.attention import check_device_errors
    from smat_attention_b200.lm import C4, LM, MasterAdamW, allreduce_grads, train_step
    dist, rank, ws, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = WORKLOAD
    cfg = C4
    B, T = w["B"], cfg.seq_len
    model = LM(cfg, device=device, seed=w["seed"])
    opt = MasterAdamW(model.parameters(), lr=6e-4)
    g = torch.Generator().manual_seed(w["seed"] + rank)
    host = torch.randint(0, cfg.vocab, (B, T + 1), generator=g).pin_memory()
    tokens = host.to(device)
    hook = (lambda: allreduce_grads(model, dist)) if dist is not None else None

    def step(tok):
        return train_step(model, opt, tok, before_step=hook)

    for _ in range(max(3, args.warmup)):
        step(tokens)
    _barrier(dist, device)
    K = args.steps
    clocks = ClockSampler(device)
    stream = torch.cuda.current_stream(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    ev[0].record(stream)
    for i in range(K):
        loss = step(tokens)
        ev[i + 1].record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(K)]
    ms_step = _max_over_ranks(dist, sum(ms) / K, device)
    # end to end: token IDs from pinned host memory, the loss read back, per step
    E = max(1, min(K, 3))
    _barrier(dist, device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    losses = []
    for _ in range(E):
        loss_e = step(host.to(device, non_blocking=True))
        losses.append(loss_e.to("cpu", non_blocking=True))
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(dist, e0.elapsed_time(e1) / E, device)
    dev_err = check_device_errors(device)
    if rank == 0:
        tok_step = ws * B * T
        attn = cfg.n_layers * 3.5 * 4.0 * cfg.head_dim * _lm_pairs(cfg) * B * cfg.n_heads
        dense = 6.0 * cfg.n_params() * B * T
        line = {
            "metric": "LM training tokens/s (fwd+bwd+AdamW)", "value": tok_step / (ms_step * 1e-3),
            "unit": "tokens/s", "n_gpus": ws, "steps": K, "warmup": max(3, args.warmup),
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"c4: {cfg.n_layers} layers d_model {cfg.d_model} "
                                   f"{cfg.n_heads}x{cfg.head_dim} heads SwiGLU {cfg.mlp_hidden} "
                                   f"vocab {cfg.vocab}, batch {B} x {T} per rank, bs "
                                   f"{cfg.block} W={cfg.window} S={cfg.stride} "
                                   f"sinks={cfg.n_sink}, bf16 + fp32 master AdamW",
                       "global_batch": B * ws, "seq_len": T,
                       "parallelism": f"data parallel x{ws} (NCCL gradient all-reduce)",
                       "params": cfg.n_params(),
                       "l2": "activations far larger than L2; no flush"},
            "model_tflops": (dense + attn) * ws / (ms_step * 1e-3) / 1e12,
            "attention_tflops_per_step": attn / 1e12,
            "loss": float(losses[-1].item()),
            "e2e": {"value": tok_step / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": host.numel() * 8,
                    "d2h_bytes_per_step": 4},
            "device_errors": dev_err,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_decode(args):
    """Decode on the c3 shapes: every (batch, head) row attends from the last
    position (t = T - 1, the longest CSR row) over a KV cache of the whole
    sequence; L2 is flushed (a 256 MiB read) between timed steps.  Algorithmic
    bytes per step: the visible keys and values (2 D bytes each, bf16) plus q
    and o."""
    from smat_attention_b200.attention import check_device_errors
    from smat_attention_b200.decode import decode_attention
    from smat_attention_b200.mask import build_block_mask
    dist, rank, ws, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = WORKLOADS["c3"]
    B, H, T, D = w["B"], w["H"], w["T"], w["D"]
    spec = build_block_mask(T, w["block"], w["window"], w["stride"], w["sinks"])
    g = torch.Generator().manual_seed(w["seed"] + rank)
    k = torch.randn(B, H, T, D, generator=g).to(device, torch.bfloat16)
    v = torch.randn(B, H, T, D, generator=g).to(device, torch.bfloat16)
    q = torch.randn(B, H, D, generator=g).to(device, torch.bfloat16)
    pos = torch.full((B,), T - 1, dtype=torch.int32, device=device)
    qb = (T - 1) // w["block"]
    row = spec.indices[spec.indptr[qb]:spec.indptr[qb + 1]]
    keys = sum(min(w["block"], T - int(kb) * w["block"]) for kb in row)
    nbytes = B * H * (keys * 2 * D * 2 + 2 * D * 2)
    # read-only flush: a 256 MiB read evicts the cache's contents without
    # leaving dirty lines whose write-back would land inside the timed step
    flush = torch.ones(64 << 20, dtype=torch.float32, device=device)
    sink = torch.empty((), dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(max(3, args.warmup)):
        decode_attention(q, k, v, pos, spec)
    _barrier(dist, device)
    K = max(args.steps, 10)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(K)]
    clocks = ClockSampler(device)
    for i in range(K):
        torch.sum(flush, 0, out=sink)
        ev[i][0].record(stream)
        o, _ = decode_attention(q, k, v, pos, spec)
        ev[i][1].record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    ms = sorted(a.elapsed_time(b) for a, b in ev)
    ms_step = _max_over_ranks(dist, statistics.median(ms), device)
    # end to end: q from pinned host memory in, o out, every step
    qh = q.cpu().pin_memory()
    oh = torch.empty(B, H, D, dtype=torch.bfloat16).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        o, _ = decode_attention(qh.to(device, non_blocking=True), k, v, pos, spec)
        oh.copy_(o, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(dist, e0.elapsed_time(e1) / K, device)
    dev_err = check_device_errors(device)
    if rank == 0:
        peaks = _peaks()
        gbs = nbytes / (ms_step * 1e-3) / 1e9
        line = {
            "metric": "decode tokens/s (one query per sequence, c3 shapes)",
            "value": ws * B / (ms_step * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": K,
            "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"decode at t = T - 1 over a KV cache: B={B} H={H} T={T} "
                                   f"D={D} bs={w['block']} W={w['window']} S={w['stride']} "
                                   f"sinks={w['sinks']} ({len(row)} blocks, {keys} keys)",
                       "global_batch": B * ws, "seq_len": T,
                       "parallelism": f"(batch) partition x{ws}",
                       "l2": "flushed (256 MiB read) between timed steps"},
            "roofline": {"bound": "hbm", "kernel": "decode_partial", "achieved": gbs,
                         "peak": peaks["hbm"], "unit": "GB/s", "frac": gbs / peaks["hbm"],
                         "traffic": None, "algorithmic_bytes": nbytes},
            "e2e": {"value": ws * B / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": B * H * D * 2, "d2h_bytes_per_step": B * H * D * 2},
            "gpu_launches": 2 * K, "device_errors": dev_err, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def _import_reference():
    """The reference package installed under baseline/_ref (its own code,
    unmodified), or None when it is absent."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "smat")):
        return None
    if ref not in sys.path:
        sys.path.insert(0, ref)
    try:
        import smat.attention as RA
        import smat.kernels.triton_bwd as RB
        import smat.mask as RM
        return RA, RB, RM
    except Exception:
        return None


def run_kattn(args):
    """The reference's kernelised op (smat_attention, pooled schedule, M^(3) at
    chunk 128) forward + backward on nb = 32 sequences of T = 16384 with r = 64
    features and d_v = 64: ours (kernel_attention, tcgen05 TF32 chunk pass)
    against the reference's own Triton kernels (baseline/_ref, scan and
    incidence backends "triton", triton_bwd.patch() for the backward) on the
    same inputs and GPU."""
    from smat_attention_b200 import kernel_attention as KA
    from smat_attention_b200.attention import check_device_errors
    from smat_attention_b200.mask import build_mask
    dist, rank, ws, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    nb, T, r, dv, d = 32, 16384, 64, 64, 3
    g = torch.Generator().manual_seed(5 + rank)
    Phi = (torch.nn.functional.elu(torch.randn(nb, T, r, generator=g)) + 1).to(device)
    Psi = (torch.nn.functional.elu(torch.randn(nb, T, r, generator=g)) + 1).to(device)
    V = torch.randn(nb, T, dv, generator=g).to(device)
    dout = torch.randn(nb, T, dv, generator=g).to(device)
    spec = build_mask(T, d, chunk=128)
    stream = torch.cuda.current_stream(device)

    def timed(fn, K):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(device)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(K)]
        for a, b in ev:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(device)
        return statistics.median(a.elapsed_time(b) for a, b in ev)

    def ours(backward):
        def fn():
            ins = [x.requires_grad_(backward) for x in (Phi.detach(), Psi.detach(), V.detach())]
            Vb = torch.cat([ins[2], torch.ones(nb, T, 1, device=device)], dim=-1)
            out = KA.smat_attention(ins[0], ins[1], Vb, spec, chunk=128)
            if backward:
                out.backward(dout)
        return fn

    K = max(args.steps, 5)
    t_fwd = timed(ours(False), K)
    t_step = timed(ours(True), K)
    # one forward's chunk pass alone (the fused kernel), as the roofline line
    C = 128
    nc = T // C
    Phi_c, Psi_c = Phi.reshape(nb, nc, C, r), Psi.reshape(nb, nc, C, r)
    Vb_c = torch.cat([V, torch.ones(nb, T, 1, device=device)], -1).reshape(nb, nc, C, dv + 1)
    Sin = torch.rand(nb, nc, r, dv + 1, device=device)
    t_chunk = timed(lambda: KA.chunk_local(Phi_c, Psi_c, Vb_c, Sin), K)
    chunk_bytes = nb * T * (2 * r + 2 * (dv + 1)) * 4 + nb * nc * r * (dv + 1) * 4
    # streaming decode (SmatDecoder): prefill with the first n columns, then
    # 64 tokens n, n + 1, ... (nb sequences per step), each step's inputs
    # contiguous as a model would produce them; 64 steps back to back between
    # two events, per step
    Vb_all = torch.cat([V, torch.ones(nb, T, 1, device=device)], -1)
    n0 = spec.n
    ND = 64
    step_in = [x[:, n0:n0 + ND].transpose(0, 1).contiguous() for x in (Phi, Psi, Vb_all)]

    def timed_decode(make):
        d = make()
        for i in range(ND):            # warm-up pass over the tokens
            d.step(*(x[i] for x in step_in))
        d = make()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(ND):
            d.step(*(x[i] for x in step_in))
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / ND
    t_dec = timed_decode(lambda: KA.SmatDecoder(Psi[:, :n0], Vb_all[:, :n0], spec))
    ref_line = None
    R = _import_reference()
    if R is not None:
        RA, RB, RM = R
        try:
            rspec = RM.build_mask(T, d, chunk=128)
            RA.to_device(rspec, device)
            RB.patch()

            def theirs(backward):
                def fn():
                    ins = [x.requires_grad_(backward)
                           for x in (Phi.detach(), Psi.detach(), V.detach())]
                    Vb = torch.cat([ins[2], torch.ones(nb, T, 1, device=device)], dim=-1)
                    out = RA.smat_attention(ins[0], ins[1], Vb, rspec, chunk=128,
                                            scan_backend="triton", incidence_backend="triton")
                    if backward:
                        out.backward(dout)
                return fn
            ref_line = {"fwd_ms": timed(theirs(False), K), "step_ms": timed(theirs(True), K),
                        "source": "reference smat (baseline/_ref), Triton backends, patched "
                                  "differentiable kernels"}
            ref_line["decode_step_us"] = timed_decode(
                lambda: RA.SmatDecoder(Psi[:, :n0], Vb_all[:, :n0], rspec)) * 1e3
        except Exception as e:   # noqa: BLE001 -- reported, not fatal
            ref_line = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    dev_err = check_device_errors(device)
    if rank == 0:
        peaks = _peaks()
        line = {
            "metric": "kernelised SMat attention fwd+bwd tokens/s (reference op, M^(3))",
            "value": ws * nb * T / (t_step * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": K, "warmup": max(3, args.warmup), "ms_per_step": t_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"kattn: nb={nb} T={T} r={r} d_v={dv} M^({d}) chunk 128, "
                                   f"fp32 features elu+1", "global_batch": nb * ws,
                       "seq_len": T, "parallelism": f"(sequence) partition x{ws}",
                       "l2": "inputs larger than L2; no flush"},
            "fwd_ms": t_fwd,
            "decode_step_us": t_dec * 1e3,
            "roofline": {"bound": "hbm", "kernel": "kattn_chunk_fwd", "achieved":
                         chunk_bytes / (t_chunk * 1e-3) / 1e9, "peak": peaks["hbm"],
                         "unit": "GB/s", "frac": chunk_bytes / (t_chunk * 1e-3) / 1e9 /
                         peaks["hbm"], "traffic": None, "kernel_ms": t_chunk},
            "reference_triton": ref_line,
            "device_errors": dev_err,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def _lm_pairs(cfg):
    from smat_attention_b200.mask import block_layout_stats
    return block_layout_stats(cfg.mask())["pairs"]


def run_sharded(args):
    """c5 with query-block sharding: every rank runs its zig-zag share of the
    query tiles of all heads; the timed step includes both exchanges."""
    from smat_attention_b200.attention import check_device_errors
    from smat_attention_b200.mask import block_layout_stats, build_block_mask
    from smat_attention_b200.sharding import make_plan, sharded_bwd, sharded_fwd
    dist, rank, ws, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = WORKLOAD
    spec = build_block_mask(w["T"], w["block"], w["window"], w["stride"], w["sinks"])
    pairs = block_layout_stats(spec)["pairs"]
    fl = _flops(pairs)
    plan = make_plan(spec, ws, rank)
    scale = 1.0 / math.sqrt(w["D"])
    shape = (w["B"], w["H"], w["T"], w["D"])
    # the same global inputs on every rank; rows a rank does not own are
    # zeroed so that what it reads of them arrives through the exchange
    g = torch.Generator(device=device).manual_seed(w["seed"])
    q, k, v, do = (torch.randn(*shape, generator=g, device=device, dtype=torch.bfloat16)
                   for _ in range(4))
    own = torch.from_numpy(plan.owned_row_mask()).to(device)
    for x in (q, k, v, do):
        x[:, :, ~own] = 0
    o = torch.empty_like(q)
    lse = torch.empty(w["B"], w["H"], w["T"], dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    groups = args.kv_groups

    def step(ev=None):
        rec = (lambda i: ev[i].record(stream)) if ev else (lambda i: None)
        rec(0)
        sharded_fwd(plan, spec, q, k, v, scale, o=o, lse=lse, groups=groups)
        rec(1)
        sharded_bwd(plan, spec, q, k, v, o, lse, do, scale, overlap=not args.no_overlap)
        rec(2)

    for _ in range(max(3, args.warmup)):
        step()
    _barrier(dist, device)
    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    clocks = ClockSampler(device)
    _barrier(dist, device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(K):
        step(evs[s])
    stop.record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    _barrier(dist, device)
    names = ["fwd_with_kv_exchange", "bwd_with_dkdv_return"]
    phases = {n: sum(evs[s][i].elapsed_time(evs[s][i + 1]) for s in range(K)) / K
              for i, n in enumerate(names)}
    phases_max = {n: _max_over_ranks(dist, t, device) for n, t in phases.items()}
    ms_step = _max_over_ranks(dist, start.elapsed_time(stop) / K, device)
    dev_err = check_device_errors(device)
    value = fl["step"] / (ms_step * 1e-3) / 1e12
    if rank == 0:
        peaks = _peaks()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": K,
            "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{w['name']}: B={w['B']} H={w['H']} T={w['T']} D={w['D']} "
                                   f"bs={w['block']} W={w['window']} S={w['stride']} "
                                   f"sinks={w['sinks']} fwd+bwd, whole job",
                       "global_batch": w["B"], "seq_len": w["T"], "heads": w["H"],
                       "head_dim": w["D"], "parallelism": f"query-block shards x{ws} (zig-zag"
                                      + f", kv groups {args.kv_groups}, dK/dV return "
                                      + ("after dQ)" if args.no_overlap else "beside dQ)"),
                       "l2": f"inputs larger than L2 ({_tensor_mib()} MiB per tensor); "
                             f"no flush"},
            "tokens_per_s": w["B"] * w["T"] / (ms_step * 1e-3),
            "frac_of_peak": value / ws / peaks["tflops"], "peak_source": peaks["source"],
            "phase_ms_max_over_ranks": phases_max,
            "kv_rows_received_rank0": int(sum(r.size for r in plan.recv_rows)),
            "gpu_launches": K * ((3 + len(plan.runs)) if ws == 1 else
                                 (groups + 2 + len(plan.runs) + 2 * groups + 2)),
            "device_errors": dev_err, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the host-buffer end-to-end leg (profiling runs)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override B (smaller cases for ncu captures)")
    ap.add_argument("--heads", type=int, default=None, help="override H")
    ap.add_argument("--workload", default="c3", choices=sorted(WORKLOADS))
    ap.add_argument("--no-overlap", action="store_true",
                    help="c5 --shard queries: run the dK/dV return after dQ, not beside it")
    ap.add_argument("--kv-groups", type=int, default=1,
                    help="c5 --shard queries: head groups of the K/V exchange / forward")
    ap.add_argument("--shard", default="heads", choices=["heads", "queries"],
                    help="c5 only: split the heads, or the query blocks, over the ranks")
    args = ap.parse_args()
    WORKLOAD.clear()
    WORKLOAD.update(WORKLOADS[args.workload])
    if args.workload == "c5":
        # the host-buffer leg and the CPU sample are taken on the default workload
        args.no_e2e = True
        args.no_cpu_baseline = True
    if args.batch:
        WORKLOAD["B"] = args.batch
    if args.heads:
        WORKLOAD["H"] = args.heads
    if args.workload in ("c4", "decode", "kattn"):
        args.no_cpu_baseline = True
    if args.impl == "reference" and args.workload not in ("c4", "decode", "kattn"):
        run_reference(args)
    elif args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the "
                          "dense-masked attention step on host cores; this workload has no "
                          "CPU counterpart there"}))
    elif args.workload == "c4":
        run_lm(args)
    elif args.workload == "decode":
        run_decode(args)
    elif args.workload == "kattn":
        run_kattn(args)
    elif args.workload == "c5" and args.shard == "queries":
        run_sharded(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
