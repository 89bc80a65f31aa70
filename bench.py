#!/usr/bin/env python3
"""Benchmark: SMat block-sparse causal softmax attention fwd+bwd on B200.

Workload: B=4, H=32, T=16384, D=128, block 128, local
window 4, stride-8 summary blocks, 2 sink blocks, bf16 inputs with fp32 LSE
and accumulators; Q/K/V/dO i.i.d. N(0,1) (seed 2 + rank), scale 1/sqrt(D).
A step is one forward (O, LSE) plus one backward (dQ, dK, dV) over the batch.

Metric: effective TFLOP/s counting only unmasked (i, j) pairs,
F = 3.5 * 4 * D * pairs * B * H per step (pairs per head from the layout).
Multi-GPU (torchrun): the global problem stays B=4 x H=32 and its heads are
divided over the ranks ((batch, head) partition, no collective on the data
path; "strong" scaling); value = F / max-over-ranks time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --workload c5 [--shard heads|queries] ...   (long context)
    python bench.py --workload c4|decode|kattn|md3|c2|c1 ...    (one line each)

The default line carries, besides the c3 numbers:
* ``e2e``: the same step through the public autograd op with pinned host
  buffers, and ``e2e_floor``: the same copies alone (no kernels);
* ``c5_queries`` / ``c5_parity`` (every N): config 5 (B=1, H=32, T=131072)
  sharded by query blocks with the NCCL K/V exchange and the dK/dV return in
  the timed step, its single-GPU time measured in the same run, and a parity
  check of the sharded outputs against the single-GPU kernels on a 4-head
  slice;
* at N=1 only, compact keys for the other workloads (``c1``, ``c2``, ``c4``,
  ``kattn``, ``decode``, ``md3``) and the CPU baseline.

``--impl reference`` times the reference's CPU dense-masked path (the oracle
port in ``oracle/``) on this host's cores on a bounded sample of the same
workload and prints the same JSON line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import contextlib
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
    # the reference's CPU-runnable case, fp32 fwd+bwd
    "c1": dict(name="c1", B=1, H=4, T=1024, D=64, block=64, window=4, stride=0, sinks=1,
               seed=0, dtype="f32"),
    # forward only, O + fp32 LSE, inputs scaled by 0.5
    "c2": dict(name="c2", B=8, H=16, T=4096, D=64, block=64, window=8, stride=16, sinks=1,
               seed=1, scale_in=0.5, fwd_only=True),
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


def _layout_pairs(w=None):
    """The workload's mask (a block layout, or an M^(d) spec) and its unmasked
    pairs per head."""
    from smat_attention_b200.mask import block_layout_stats, build_block_mask, build_mask
    w = WORKLOAD if w is None else w
    if "d" in w:
        spec = build_mask(w["T"], w["d"], chunk=w["chunk"])
    else:
        spec = build_block_mask(w["T"], w["block"], w["window"], w["stride"], w["sinks"])
    return spec, block_layout_stats(spec)["pairs"]


def _describe(w, H):
    head = f"{w['name']}: B={w['B']} H={H} T={w['T']} D={w['D']} bs={w['block']} "
    what = "fwd" if w.get("fwd_only") else "fwd+bwd"
    if "d" in w:
        return head + f"M^({w['d']}) chunk={w['chunk']} (reference build_mask) {what} per rank"
    return head + f"W={w['window']} S={w['stride']} sinks={w['sinks']} {what} per rank"


def _flops(pairs, w, H):
    fwd = 4.0 * w["D"] * pairs * w["B"] * H
    # dkdv_dq: the fused backward kernel (dK/dV plus the dQ accumulation)
    return {"fwd": fwd, "dkdv": 2.0 * fwd, "dq": 1.5 * fwd, "dkdv_dq": 2.5 * fwd,
            "bwd": 2.5 * fwd, "step": 3.5 * fwd}


def _peaks():
    """Roofline denominators: the measured burst bf16 GEMM rate (the kernels
    are timed in sub-second regions at full clock) and, for reference, the
    sustained one; the measured copy bandwidth."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"tflops": float(p["bf16_tflops"]),
                "tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "hbm": float(p["hbm_gbs"]),
                "source": "of measured (MEASURED_PEAKS.json bf16_tflops, burst)"}
    except (OSError, KeyError, ValueError):
        return {"tflops": 1590.0, "tflops_sustained": 1400.0, "hbm": 6650.0,
                "source": "of fallback (1.59 PFLOP/s burst, 6.65 TB/s)"}


def _traffic():
    """Per-launch DRAM bytes of the kernels from the committed ncu summary
    (profiles/), if one is present."""
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
    """SM clock and clock-event reasons sampled every ~2 ms while the timed
    region runs (NVML read-only queries from a background thread; nothing is
    set).  Falls back to an `nvidia-smi` poll when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        import threading
        self.samples, self.proc, self.thread = [], None, None
        self.stop_flag = threading.Event()
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(ident)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            time.sleep(0.01)
            return
        except Exception:
            self.nv = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def _poll(self):
        nv, h = self.nv, self.handle
        while not self.stop_flag.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(mhz), int(bits)))
            except Exception:
                return
            time.sleep(0.002)

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=2)
            if not self.samples:
                return None
            sm = [m for m, _ in self.samples]
            reasons = set()
            for name, attr in self.REASONS:
                bit = getattr(self.nv, attr, 0)
                if any(b & bit for _, b in self.samples):
                    reasons.add(name)
            load = [x for x in sm if x > 0.5 * max(sm)] or sm
            return {"sm_mhz": statistics.median(load), "sm_max_mhz": float(self.max_mhz),
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 2 ms"}
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
        names = [n for n, _ in self.REASONS]
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
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi 100 ms"}


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


def _reduce(dist, value, device, op="max"):
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


def _max_over_ranks(dist, value, device):
    return _reduce(dist, value, device, "max")


def _events(n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


# ----------------------------------------------------------------------------
# host memory placement
# ----------------------------------------------------------------------------

def _gpu_numa_cpus(device):
    """(CPUs of the NUMA node the GPU's PCIe function sits on, or None; a note
    saying what was found)."""
    try:
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None, f"{bus}: no NUMA node reported"
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None, f"{bus}: node {node} has none of this process's CPUs"
        return cpus, f"{bus}: node {node}, {len(cpus)} CPUs"
    except (OSError, ValueError, AttributeError) as e:
        return None, f"no placement ({type(e).__name__})"


@contextlib.contextmanager
def _near_gpu(device):
    """Run the body on the CPUs of the GPU's NUMA node, so that pinned host
    buffers allocated inside it are placed in that node's memory (the driver
    allocates and touches the pages from the calling thread).  Yields a note
    on the placement."""
    cpus, note = _gpu_numa_cpus(device)
    old = os.sched_getaffinity(0)
    if cpus:
        os.sched_setaffinity(0, cpus)
    try:
        yield note
    finally:
        if cpus:
            os.sched_setaffinity(0, old)


# ----------------------------------------------------------------------------
# CPU baseline: the reference's dense-masked path (oracle port) on host cores
# ----------------------------------------------------------------------------

def cpu_sample(reps=1, w=None):
    """Time the oracle's dense-masked fp32 forward + backward on one (batch,
    head) of the workload at the full sequence length; returns the effective
    TFLOP/s of that head and a description."""
    from oracle import layout as OL
    from oracle.dense_softmax import rowchunked_masked_softmax
    w = WORKLOAD if w is None else w
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    spec, pairs = _layout_pairs(w)
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


def cpu_c1_full(reps=5):
    """Config 1 in full on the host (fp32 fwd+bwd, all threads): the oracle
    port of the dense-masked softmax, and beside it the reference's own
    ``dense_masked_kernel_attention`` (baseline/_ref, its einsum path,
    ``src/smat/attention.py:485-489``) on the same shapes with positive
    features and the same dense mask, as the reference's prefill benchmark
    times it (``analysis/bench_prefill.py:275-281``)."""
    from oracle import layout as OL
    from oracle.dense_softmax import rowchunked_masked_softmax
    w = WORKLOADS["c1"]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    B, H, T, D = w["B"], w["H"], w["T"], w["D"]
    g = torch.Generator().manual_seed(w["seed"])
    q, k, v, do = (torch.randn(B * H, T, D, generator=g) for _ in range(4))
    rows = OL.block_mask_rows(T, w["block"], w["window"], w["stride"], w["sinks"])

    def med(fn):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts) * 1e3

    out = {"cores": threads, "port_ms": med(lambda: rowchunked_masked_softmax(
        q, k, v, do, rows, 1 / math.sqrt(D), rows=T))}
    R = _import_reference()
    if R is None:
        out["reference_dense_masked_ms"] = None
        out["reference_note"] = "baseline/_ref not installed"
        return out
    RA = R[0]
    M = rows(0, T).float()
    Phi = torch.nn.functional.elu(torch.randn(B * H, T, D, generator=g)) + 1
    Psi = torch.nn.functional.elu(torch.randn(B * H, T, D, generator=g)) + 1
    Vb = torch.cat([v, torch.ones(B * H, T, 1)], -1)
    dout = torch.randn(B * H, T, D, generator=g)

    def ref_step():
        ins = [x.detach().requires_grad_(True) for x in (Phi, Psi, Vb)]
        RA.dense_masked_kernel_attention(*ins, M).backward(dout)

    out["reference_dense_masked_ms"] = med(ref_step)
    out["reference_note"] = ("reference dense_masked_kernel_attention (kernelised, fp32, "
                             "autograd fwd+bwd) on c1 shapes, same mask")
    return out


def _config(ws, w=None, H_total=None):
    """The `config` of the attention workloads' JSON line (both arms): the
    global problem and how it is split over `ws` ranks."""
    w = WORKLOAD if w is None else w
    H_total = w["H"] if H_total is None else H_total
    H_rank = H_total // ws
    return {"workload": _describe(w, H_rank),
            "global_batch": w["B"], "seq_len": w["T"], "heads": H_total, "head_dim": w["D"],
            "parallelism": f"head partition x{ws}",
            "l2": f"step inputs larger than L2 (4 x {w['B'] * H_rank * w['T'] * w['D'] * 2 >> 20} "
                  f"MiB per rank); no flush"}


def run_reference(args):
    dist, rank, ws, local = _dist()
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
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
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": _config(args.gpus),
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# GPU arm: one attention workload
# ----------------------------------------------------------------------------

class AttnCase:
    """The kernels of one attention workload on one rank: inputs, layout and
    the launches of a step through the C ABI (fwd, bwd preprocess, dK/dV, dQ
    for block layouts; the pattern entry points for M^(d) masks; the forward
    alone for forward-only configs)."""

    def __init__(self, w, H, device, seed, keep_host=False):
        from smat_attention_b200 import _lib
        from smat_attention_b200.attention import layout_device_args
        self.w, self.H, self.device = w, H, device
        self.spec, self.pairs = _layout_pairs(w)
        self.fl = _flops(self.pairs, w, H)
        self.scale = 1.0 / math.sqrt(w["D"])
        self.dtype = torch.float32 if w.get("dtype") == "f32" else torch.bfloat16
        self.dt_code = _lib.DTYPE_F32 if self.dtype == torch.float32 else _lib.DTYPE_BF16
        g = torch.Generator().manual_seed(seed)
        self.shape = (w["B"], H, w["T"], w["D"])
        s_in = w.get("scale_in", 1.0)
        host = [(torch.randn(*self.shape, generator=g) * s_in).to(self.dtype) for _ in range(4)]
        self.q, self.k, self.v, self.do = (x.to(device) for x in host)
        self.host = host if keep_host else None
        self.lay = layout_device_args(self.spec, device)
        self.o = torch.empty_like(self.q)
        B, H_, T, D = self.shape
        self.lse = torch.empty(B, H_, T, dtype=torch.float32, device=device)
        self.delta = torch.empty_like(self.lse)
        self.dq, self.dk, self.dv = (torch.empty_like(self.q) for _ in range(3))
        # the opt-in fused backward: dQ accumulated by the dK/dV kernel in fp32
        # (only with SMAT_FUSED_DQ=1, as in the library)
        from smat_attention_b200 import attention as A
        self.fused = (A.fused_dq_applies(self.dtype, D) and not w.get("fwd_only")
                      and A.FUSED_DQ)
        self.dq_acc = (torch.empty(B * H_ * T * D, dtype=torch.float32, device=device)
                       if self.fused else None)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.stream = torch.cuda.current_stream(device)
        self.L = _lib.lib()
        self.kernels = self._kernels()

    def _kernels(self):
        from smat_attention_b200 import _lib
        L, lay, sp, st = self.L, self.lay, _lib.strides3, self.stream.cuda_stream
        q, k, v, do, o = self.q, self.k, self.v, self.do, self.o
        lse, delta, dq, dk, dv, err = self.lse, self.delta, self.dq, self.dk, self.dv, self.err
        B, H, T, D = self.shape
        dt, scale = self.dt_code, self.scale

        def launch_fwd():
            _lib.check("smat_fwd", L.smat_fwd(
                dt, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                o.data_ptr(), sp(o), lse.data_ptr(), B, H, T, D, lay["indptr"].data_ptr(),
                lay["indices"].data_ptr(), lay["kind"].data_ptr(), lay["nblocks"], lay["nnzb"],
                lay["block"], lay["max_row"], scale, err.data_ptr(), st))

        def launch_pre():
            _lib.check("smat_bwd_preprocess", L.smat_bwd_preprocess(
                dt, o.data_ptr(), sp(o), do.data_ptr(), sp(do), delta.data_ptr(), B, H, T, D,
                st))

        def launch_dkdv():
            _lib.check("smat_bwd_dkdv", L.smat_bwd_dkdv(
                dt, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                do.data_ptr(), sp(do), lse.data_ptr(), delta.data_ptr(), dk.data_ptr(), sp(dk),
                dv.data_ptr(), sp(dv), B, H, T, D, lay["t_indptr"].data_ptr(),
                lay["t_indices"].data_ptr(), lay["t_kind"].data_ptr(), lay["nblocks"],
                lay["nnzb"], lay["block"], lay["t_max_row"], scale, err.data_ptr(), st))

        def launch_dq():
            _lib.check("smat_bwd_dq", L.smat_bwd_dq(
                dt, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                do.data_ptr(), sp(do), lse.data_ptr(), delta.data_ptr(), dq.data_ptr(), sp(dq),
                B, H, T, D, lay["indptr"].data_ptr(), lay["indices"].data_ptr(),
                lay["kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"],
                lay["max_row"], scale, err.data_ptr(), st))

        def launch_dkdv_dq():
            acc = self.dq_acc
            _lib.check("smat_bwd_dkdv_dq", L.smat_bwd_dkdv_dq(
                dt, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                do.data_ptr(), sp(do), lse.data_ptr(), delta.data_ptr(), acc.data_ptr(),
                acc.numel(), dk.data_ptr(), sp(dk), dv.data_ptr(), sp(dv), B, H, T, D,
                lay["t_indptr"].data_ptr(), lay["t_indices"].data_ptr(),
                lay["t_kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"],
                lay["t_max_row"], scale, err.data_ptr(), st))

        def launch_dq_finish():
            acc = self.dq_acc
            _lib.check("smat_bwd_dq_finish", L.smat_bwd_dq_finish(
                dt, acc.data_ptr(), acc.numel(), dq.data_ptr(), sp(dq), B, H, T, D, scale, st))

        def launch_bwd_acc_pattern():
            acc = self.dq_acc
            _lib.check("smat_bwd_acc", L.smat_bwd_acc(
                dt, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                o.data_ptr(), sp(o), do.data_ptr(), sp(do), lse.data_ptr(), delta.data_ptr(),
                dq.data_ptr(), sp(dq), dk.data_ptr(), sp(dk), dv.data_ptr(), sp(dv),
                B, H, T, D, lay["indptr"].data_ptr(), lay["indices"].data_ptr(),
                lay["kind"].data_ptr(), lay["t_indptr"].data_ptr(), lay["t_indices"].data_ptr(),
                lay["t_kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"],
                lay["max_row"], lay["t_max_row"], lay["pattern"], acc.data_ptr(), acc.numel(),
                scale, err.data_ptr(), st))

        def launch_fwd_pattern():
            _lib.check("smat_fwd_pattern", L.smat_fwd_pattern(
                dt, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                o.data_ptr(), sp(o), lse.data_ptr(), B, H, T, D, lay["indptr"].data_ptr(),
                lay["indices"].data_ptr(), lay["kind"].data_ptr(), lay["nblocks"], lay["nnzb"],
                lay["block"], lay["max_row"], lay["pattern"], scale, err.data_ptr(), st))

        def launch_bwd_pattern():
            _lib.check("smat_bwd_pattern", L.smat_bwd_pattern(
                dt, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                o.data_ptr(), sp(o), do.data_ptr(), sp(do), lse.data_ptr(), delta.data_ptr(),
                dq.data_ptr(), sp(dq), dk.data_ptr(), sp(dk), dv.data_ptr(), sp(dv),
                B, H, T, D, lay["indptr"].data_ptr(), lay["indices"].data_ptr(),
                lay["kind"].data_ptr(), lay["t_indptr"].data_ptr(), lay["t_indices"].data_ptr(),
                lay["t_kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"],
                lay["max_row"], lay["t_max_row"], lay["pattern"], scale, err.data_ptr(), st))

        if self.w.get("fwd_only"):
            # (name, launch, kernel launches it makes)
            return [("fwd", launch_fwd, 1)]
        if lay["pattern"] is None and self.fused:
            # the fused backward: dK/dV/dQ-accumulate (after zeroing the
            # accumulator), then dQ's conversion
            return [("fwd", launch_fwd, 1), ("bwd_pre", launch_pre, 1),
                    ("dkdv_dq", launch_dkdv_dq, 1), ("dq_finish", launch_dq_finish, 1)]
        if lay["pattern"] is None:
            return [("fwd", launch_fwd, 1), ("bwd_pre", launch_pre, 1),
                    ("dkdv", launch_dkdv, 1), ("dq", launch_dq, 1)]
        # M^(d): the pattern entry points (the backward launches its three passes)
        if self.fused:
            return [("fwd", launch_fwd_pattern, 1), ("bwd", launch_bwd_acc_pattern, 3)]
        return [("fwd", launch_fwd_pattern, 1), ("bwd", launch_bwd_pattern, 3)]

    @property
    def step_flops(self):
        return self.fl["fwd"] if self.w.get("fwd_only") else self.fl["step"]

    @property
    def launches_per_step(self):
        return sum(n for _, _, n in self.kernels)

    def warm(self, n):
        for _ in range(max(3, n)):
            for _, fn, _ in self.kernels:
                fn()

    def timed(self, K, dist=None, clocks=False):
        """K steps between events (per-kernel events inside); returns
        (ms per step, per-kernel ms, clock record)."""
        ev = [_events(len(self.kernels) + 1) for _ in range(K)]
        _barrier(dist, self.device)
        sampler = ClockSampler(self.device) if clocks else None
        _barrier(dist, self.device)
        start, stop = _events(2)
        start.record(self.stream)
        for s in range(K):
            ev[s][0].record(self.stream)
            for i, (_, fn, _) in enumerate(self.kernels):
                fn()
                ev[s][i + 1].record(self.stream)
        stop.record(self.stream)
        torch.cuda.synchronize(self.device)
        clk = sampler.stop() if sampler else None
        _barrier(dist, self.device)
        per_kernel = {name: sum(ev[s][i].elapsed_time(ev[s][i + 1]) for s in range(K)) / K
                      for i, (name, _, _) in enumerate(self.kernels)}
        return start.elapsed_time(stop) / K, per_kernel, clk

    def free(self):
        for name in ("q", "k", "v", "do", "o", "lse", "delta", "dq", "dk", "dv", "dq_acc"):
            setattr(self, name, None)
        self.kernels = []


def _e2e(case, K, dist, heads_per_slice=None):
    """The step through the public autograd API with pinned host buffers:
    per step H2D of q, k, v, dO and D2H of o, dq, dk, dv inside the timed
    region.  The batch goes through in slices of one sequence (and, if asked,
    `heads_per_slice` heads),
    pipelined the way a caller streaming from host memory would: the H2D of
    slice s + 1 (a copy stream) and the D2H of slice s - 1 (another) overlap
    the attention of slice s, so the step costs the transfers plus one slice's
    H2D at the start and one slice's D2H at the end.  The pinned buffers are
    allocated from the CPUs of the GPU's NUMA node.  Also times the copy
    floor: the same copies on the same streams with no kernels (all H2D on one
    stream, all D2H on the other).  Returns (e2e ms per step, floor ms per
    step, bytes each way per step, placement note, heads per slice)."""
    from smat_attention_b200.attention import smat_softmax_attention
    device, stream, shape, spec, scale = case.device, case.stream, case.shape, case.spec, \
        case.scale
    with _near_gpu(device) as note:
        pinned = [x.pin_memory() for x in case.host]
        outs = [torch.empty(shape, dtype=case.dtype).pin_memory() for _ in range(4)]
    E = max(1, min(K, 3))
    h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    B, H = shape[0], shape[1]
    hs = H if not heads_per_slice else max(1, min(H, heads_per_slice))
    slices = [(slice(b, b + 1), slice(h, min(H, h + hs))) for b in range(B)
              for h in range(0, H, hs)]

    def e2e_step():
        for sl in slices:
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

    dev_bufs = [torch.empty(shape, dtype=case.dtype, device=device) for _ in range(4)]

    def floor_step():
        h2d.wait_stream(stream)
        d2h.wait_stream(stream)
        for sl in slices:
            with torch.cuda.stream(h2d):
                for src, dst in zip(pinned, dev_bufs):
                    dst[sl].copy_(src[sl], non_blocking=True)
            with torch.cuda.stream(d2h):
                for dst, src in zip(outs, dev_bufs):
                    dst[sl].copy_(src[sl], non_blocking=True)
        stream.wait_stream(h2d)
        stream.wait_stream(d2h)

    def timed(fn):
        fn()
        torch.cuda.synchronize(device)
        _barrier(dist, device)
        e0, e1 = _events(2)
        e0.record(stream)
        for _ in range(E):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(device)
        return _max_over_ranks(dist, e0.elapsed_time(e1) / E, device)

    e2e_ms = timed(e2e_step)
    floor_ms = timed(floor_step)
    nbytes = sum(x.numel() * x.element_size() for x in case.host)
    del dev_bufs, pinned, outs
    return e2e_ms, floor_ms, nbytes, note, hs


# ----------------------------------------------------------------------------
# secondary workloads: each returns a dict (one JSON line of its own when run
# with --workload, a compact key of the default line at N=1)
# ----------------------------------------------------------------------------

def measure_attn(w, device, K, warmup, dist=None, rank=0, ws=1, clocks=False):
    """A block-layout or M^(d) attention workload split by heads: device
    timing, per-kernel times and the roofline of every kernel."""
    if w["H"] % ws:
        raise SystemExit(f"H={w['H']} does not split over {ws} ranks")
    H_rank = w["H"] // ws
    case = AttnCase(w, H_rank, device, w["seed"] + rank)
    case.warm(warmup)
    ms, per_kernel, clk = case.timed(K, dist, clocks)
    ms_step = _max_over_ranks(dist, ms, device)
    peaks = _peaks()
    total_fl = case.step_flops * ws
    kern = {}
    for name, t in per_kernel.items():
        f = case.fl.get(name) if name != "bwd" else case.fl["bwd"]
        kern[name] = {"ms": t, "tflops": None if f is None else f / (t * 1e-3) / 1e12}
        if f is not None:
            kern[name]["frac"] = kern[name]["tflops"] / peaks["tflops"]
    out = {"value": total_fl / (ms_step * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms_step,
           "steps": K, "per_kernel": kern, "config": _config(ws, w), "clocks": clk,
           "frac_of_peak": total_fl / ws / (ms_step * 1e-3) / 1e12 / peaks["tflops"],
           "gpu_launches": K * case.launches_per_step}
    return out, case


def measure_c1(device, K=20):
    """Config 1 (fp32 CUDA-core kernels) on the GPU, and c1 in full on the
    host (the oracle port and the reference's own dense-masked op)."""
    out, case = measure_attn(WORKLOADS["c1"], device, K, 3)
    case.free()
    out["cpu_full"] = cpu_c1_full()
    out["gpu_vs_cpu_port"] = out["cpu_full"]["port_ms"] / out["ms_per_step"]
    return out


def measure_lm(args, device, dist=None, rank=0, ws=1, K=None):
    """training steps (forward, backward, AdamW on fp32
    masters) of the 12-layer LM with the block-sparse arm in every layer, on
    uniform synthetic token IDs; data parallel over the ranks (bf16 gradients
    all-reduced in one NCCL call before the optimizer step)."""
    from smat_attention_b200.attention import check_device_errors
    from smat_attention_b200.lm import C4, LM, MasterAdamW, allreduce_grads, train_step
    w = WORKLOADS["c4"]
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
    K = args.steps if K is None else K
    clocks = ClockSampler(device)
    stream = torch.cuda.current_stream(device)
    ev = _events(K + 1)
    ev[0].record(stream)
    for i in range(K):
        step(tokens)
        ev[i + 1].record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(K)]
    ms_step = _max_over_ranks(dist, sum(ms) / K, device)
    # end to end: token IDs from pinned host memory, the loss read back, per step
    E = max(1, min(K, 3))
    _barrier(dist, device)
    e0, e1 = _events(2)
    e0.record(stream)
    losses = []
    for _ in range(E):
        loss_e = step(host.to(device, non_blocking=True))
        losses.append(loss_e.to("cpu", non_blocking=True))
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(dist, e0.elapsed_time(e1) / E, device)
    dev_err = check_device_errors(device)
    tok_step = ws * B * T
    attn = cfg.n_layers * 3.5 * 4.0 * cfg.head_dim * _lm_pairs(cfg) * B * cfg.n_heads
    dense = 6.0 * cfg.n_params() * B * T
    out = {"value": tok_step / (ms_step * 1e-3), "unit": "tokens/s", "ms_per_step": ms_step,
           "steps": K, "model_tflops": (dense + attn) * ws / (ms_step * 1e-3) / 1e12,
           "attention_tflops_per_step": attn / 1e12, "loss": float(losses[-1].item()),
           "e2e": {"value": tok_step / (e2e_ms * 1e-3), "unit": "tokens/s",
                   "ms_per_step": e2e_ms, "h2d_bytes_per_step": host.numel() * 8,
                   "d2h_bytes_per_step": 4},
           "device_errors": dev_err, "clocks": clk,
           "config": {"workload": f"c4: {cfg.n_layers} layers d_model {cfg.d_model} "
                                  f"{cfg.n_heads}x{cfg.head_dim} heads SwiGLU {cfg.mlp_hidden} "
                                  f"vocab {cfg.vocab}, batch {B} x {T} per rank, bs "
                                  f"{cfg.block} W={cfg.window} S={cfg.stride} "
                                  f"sinks={cfg.n_sink}, bf16 + fp32 master AdamW",
                      "global_batch": B * ws, "seq_len": T,
                      "parallelism": f"data parallel x{ws} (NCCL gradient all-reduce)",
                      "params": cfg.n_params(),
                      "l2": "activations far larger than L2; no flush"}}
    del model, opt
    return out


def measure_decode(args, device, dist=None, rank=0, ws=1, K=None):
    """Decode on the c3 shapes: every (batch, head) row attends from the last
    position (t = T - 1, the longest CSR row) over a KV cache of the whole
    sequence; L2 is flushed (a 256 MiB read) between timed steps.  Algorithmic
    bytes per step: the visible keys and values (2 D bytes each, bf16) plus q
    and o."""
    from smat_attention_b200.attention import check_device_errors
    from smat_attention_b200.decode import decode_attention
    from smat_attention_b200.mask import build_block_mask
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
    K = max(args.steps, 10) if K is None else K
    ev = [_events(2) for _ in range(K)]
    clocks = ClockSampler(device)
    for i in range(K):
        torch.sum(flush, 0, out=sink)
        ev[i][0].record(stream)
        decode_attention(q, k, v, pos, spec)
        ev[i][1].record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    ms = sorted(a.elapsed_time(b) for a, b in ev)
    ms_step = _max_over_ranks(dist, statistics.median(ms), device)
    # end to end: q from pinned host memory in, o out, every step
    qh = q.cpu().pin_memory()
    oh = torch.empty(B, H, D, dtype=torch.bfloat16).pin_memory()
    e0, e1 = _events(2)
    e0.record(stream)
    for _ in range(K):
        o, _ = decode_attention(qh.to(device, non_blocking=True), k, v, pos, spec)
        oh.copy_(o, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(dist, e0.elapsed_time(e1) / K, device)
    dev_err = check_device_errors(device)
    peaks = _peaks()
    gbs = nbytes / (ms_step * 1e-3) / 1e9
    return {
        "value": ws * B / (ms_step * 1e-3), "unit": "tokens/s", "ms_per_step": ms_step,
        "us_per_step": ms_step * 1e3, "steps": K,
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
        "gpu_launches": K, "device_errors": dev_err, "clocks": clk,
    }


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


def measure_kattn(args, device, dist=None, rank=0, ws=1, K=None, with_reference=True):
    """The reference's kernelised op (smat_attention, pooled schedule, M^(3) at
    chunk 128) forward + backward on nb = 32 sequences of T = 16384 with r = 64
    features and d_v = 64: ours (kernel_attention, tcgen05 TF32 chunk pass)
    against the reference's own Triton kernels (baseline/_ref, scan and
    incidence backends "triton", triton_bwd.patch() for the backward) on the
    same inputs and GPU."""
    from smat_attention_b200 import kernel_attention as KA
    from smat_attention_b200.attention import check_device_errors
    from smat_attention_b200.mask import build_mask
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
        ev = [_events(2) for _ in range(K)]
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

    K = max(args.steps, 5) if K is None else K
    t_fwd = timed(ours(False), K)
    t_step = timed(ours(True), K)
    # the forward's phases (the reference's timer hook), mean of K forwards
    Vb_ph = torch.cat([V, torch.ones(nb, T, 1, device=device)], dim=-1)
    tm = KA.PhaseTimer(device)
    for _ in range(K):
        KA.smat_attention(Phi, Psi, Vb_ph, spec, chunk=128, timer=tm)
    phases = {k: v / K for k, v in tm.results().items()}
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
        dec = make()
        for i in range(ND):            # warm-up pass over the tokens
            dec.step(*(x[i] for x in step_in))
        dec = make()
        torch.cuda.synchronize(device)
        a, b = _events(2)
        a.record(stream)
        for i in range(ND):
            dec.step(*(x[i] for x in step_in))
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / ND
    t_dec = timed_decode(lambda: KA.SmatDecoder(Psi[:, :n0], Vb_all[:, :n0], spec))
    ref_line = None
    R = _import_reference() if with_reference else None
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
            ref_line["speedup_step"] = ref_line["step_ms"] / t_step
            ref_line["speedup_fwd"] = ref_line["fwd_ms"] / t_fwd
        except Exception as e:   # noqa: BLE001 -- reported, not fatal
            ref_line = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    elif with_reference:
        ref_line = {"unavailable": "baseline/_ref not installed"}
    dev_err = check_device_errors(device)
    peaks = _peaks()
    return {
        "value": ws * nb * T / (t_step * 1e-3), "unit": "tokens/s", "ms_per_step": t_step,
        "steps": K, "fwd_ms": t_fwd, "fwd_phase_ms": phases, "decode_step_us": t_dec * 1e3,
        "config": {"workload": f"kattn: nb={nb} T={T} r={r} d_v={dv} M^({d}) chunk 128, "
                               f"fp32 features elu+1", "global_batch": nb * ws,
                   "seq_len": T, "parallelism": f"(sequence) partition x{ws}",
                   "l2": "inputs larger than L2; no flush"},
        "roofline": {"bound": "hbm", "kernel": "kattn_chunk_fwd", "achieved":
                     chunk_bytes / (t_chunk * 1e-3) / 1e9, "peak": peaks["hbm"],
                     "unit": "GB/s", "frac": chunk_bytes / (t_chunk * 1e-3) / 1e9 /
                     peaks["hbm"], "traffic": None, "kernel_ms": t_chunk},
        "reference_triton": ref_line,
        "device_errors": dev_err,
    }


def _lm_pairs(cfg):
    from smat_attention_b200.mask import block_layout_stats
    return block_layout_stats(cfg.mask())["pairs"]


# ----------------------------------------------------------------------------
# c5: query-block sharding with the NCCL exchanges
# ----------------------------------------------------------------------------

def measure_c5_queries(dist, rank, ws, device, K=5, warmup=3, kv_groups=1, overlap=True):
    """Config 5 sharded by query blocks over the ranks: each rank its zig-zag
    share of the query tiles of every head, the K/V exchange before the
    forward and the dK/dV return after the backward inside the timed step.
    The whole problem is also timed on one GPU with the unsharded kernels
    (every rank at once, on the same inputs) for the scaling efficiency."""
    from smat_attention_b200.attention import bwd, check_device_errors, fwd
    from smat_attention_b200.mask import block_layout_stats, build_block_mask
    from smat_attention_b200.sharding import make_plan, sharded_bwd, sharded_fwd
    w = WORKLOADS["c5"]
    spec = build_block_mask(w["T"], w["block"], w["window"], w["stride"], w["sinks"])
    pairs = block_layout_stats(spec)["pairs"]
    fl = _flops(pairs, w, w["H"])
    plan = make_plan(spec, ws, rank)
    scale = 1.0 / math.sqrt(w["D"])
    shape = (w["B"], w["H"], w["T"], w["D"])
    stream = torch.cuda.current_stream(device)
    # the same global inputs on every rank
    g = torch.Generator(device=device).manual_seed(w["seed"])
    q, k, v, do = (torch.randn(*shape, generator=g, device=device, dtype=torch.bfloat16)
                   for _ in range(4))

    # the whole problem on this one GPU (the N = 1 reference of the curve)
    def single():
        o1, lse1 = fwd(q, k, v, spec, scale)
        bwd(q, k, v, o1, lse1, do, spec, scale)
    for _ in range(2):
        single()
    _barrier(dist, device)
    a, b = _events(2)
    a.record(stream)
    for _ in range(3):
        single()
    b.record(stream)
    torch.cuda.synchronize(device)
    t1 = _max_over_ranks(dist, a.elapsed_time(b) / 3, device)

    # rows this rank does not own are zeroed: what it reads of them arrives
    # through the exchange
    own = torch.from_numpy(plan.owned_row_mask()).to(device)
    for x in (q, k, v, do):
        x[:, :, ~own] = 0
    o = torch.empty_like(q)
    lse = torch.empty(w["B"], w["H"], w["T"], dtype=torch.float32, device=device)

    def step(ev=None):
        rec = (lambda i: ev[i].record(stream)) if ev else (lambda i: None)
        rec(0)
        sharded_fwd(plan, spec, q, k, v, scale, o=o, lse=lse, groups=kv_groups)
        rec(1)
        sharded_bwd(plan, spec, q, k, v, o, lse, do, scale, overlap=overlap)
        rec(2)

    for _ in range(max(3, warmup)):
        step()
    _barrier(dist, device)
    evs = [_events(3) for _ in range(K)]
    clocks = ClockSampler(device)
    _barrier(dist, device)
    start, stop = _events(2)
    start.record(stream)
    for s in range(K):
        step(evs[s])
    stop.record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    _barrier(dist, device)
    names = ["fwd_with_kv_exchange", "bwd_with_dkdv_return"]
    phases = {n: _max_over_ranks(dist, sum(evs[s][i].elapsed_time(evs[s][i + 1])
                                           for s in range(K)) / K, device)
              for i, n in enumerate(names)}
    ms_step = _max_over_ranks(dist, start.elapsed_time(stop) / K, device)
    dev_err = int(_max_over_ranks(dist, check_device_errors(device), device))
    peaks = _peaks()
    value = fl["step"] / (ms_step * 1e-3) / 1e12
    del q, k, v, do, o, lse
    return {
        "value": value, "unit": UNIT, "ms_per_step": ms_step, "steps": K,
        "single_gpu_ms": t1, "single_gpu_tflops": fl["step"] / (t1 * 1e-3) / 1e12,
        "speedup": t1 / ms_step, "efficiency": t1 / (ws * ms_step),
        "frac_of_peak": value / ws / peaks["tflops"],
        "phase_ms_max_over_ranks": phases,
        "kv_rows_received_rank0": int(sum(r.size for r in plan.recv_rows)),
        "config": {"workload": f"c5: B={w['B']} H={w['H']} T={w['T']} D={w['D']} "
                               f"bs={w['block']} W={w['window']} S={w['stride']} "
                               f"sinks={w['sinks']} fwd+bwd, whole job",
                   "parallelism": f"query-block shards x{ws} (zig-zag, NCCL all_to_all of "
                                  f"K/V rows, dK/dV return " +
                                  ("beside dQ)" if overlap else "after dQ)")},
        "scaling": "strong", "device_errors": dev_err, "clocks": clk,
        "gpu_launches": K * ((3 + len(plan.runs)) if ws == 1 else
                             (kv_groups + 2 + len(plan.runs) + 2 * kv_groups + 2)),
    }


def measure_c5_parity(dist, rank, ws, device, H=4):
    """The query-sharded path against the single-GPU kernels on a slice of
    config 5 (its first H heads at the full T): every rank runs the sharded
    forward + backward with NaN in every row it does not own (so a row read
    without the exchange poisons the result) and the unsharded kernels on the
    full inputs; O, LSE and dQ of its owned rows must be equal bit for bit.
    dK and dV of an imported key block are sums of bf16 partials from several
    ranks (each rounded once before the owner adds them in fp32), so they may
    differ from the single-GPU value by a rounding or two: the bound is 2e-2
    or two bf16 units in the last place of the single-GPU value, whichever is
    larger."""
    from smat_attention_b200.attention import bwd, check_device_errors, fwd
    from smat_attention_b200.mask import build_block_mask
    from smat_attention_b200.sharding import make_plan, sharded_bwd, sharded_fwd
    w = WORKLOADS["c5"]
    spec = build_block_mask(w["T"], w["block"], w["window"], w["stride"], w["sinks"])
    plan = make_plan(spec, ws, rank)
    scale = 1.0 / math.sqrt(w["D"])
    shape = (w["B"], H, w["T"], w["D"])
    g = torch.Generator(device=device).manual_seed(w["seed"] + 100)
    q, k, v, do = (torch.randn(*shape, generator=g, device=device, dtype=torch.bfloat16)
                   for _ in range(4))
    o1, lse1 = fwd(q, k, v, spec, scale)
    dq1, dk1, dv1 = bwd(q, k, v, o1, lse1, do, spec, scale)
    own = torch.from_numpy(plan.owned_row_mask()).to(device)
    qs, ks, vs, dos = (x.clone() for x in (q, k, v, do))
    for x in (qs, ks, vs, dos):
        x[:, :, ~own] = float("nan")
    o, lse = sharded_fwd(plan, spec, qs, ks, vs, scale)
    dq, dk, dv = sharded_bwd(plan, spec, qs, ks, vs, o, lse, dos, scale)
    torch.cuda.synchronize(device)
    errs = int(check_device_errors(device))
    exact = {name: bool(torch.equal(a[:, :, own], b[:, :, own]))
             for name, a, b in (("o", o, o1), ("lse", lse, lse1), ("dq", dq, dq1))}
    dmax, ulps = {}, {}
    for name, a, b in (("dk", dk, dk1), ("dv", dv, dv1)):
        diff = (a[:, :, own].float() - b[:, :, own].float()).abs()
        ref = b[:, :, own].float().abs()
        # one bf16 unit in the last place of |ref| (8 significant bits)
        ulp = torch.exp2(torch.floor(torch.log2(ref.clamp_min(2.0 ** -126))) - 7)
        dmax[name] = float(diff.max().item())
        # worst element against its own bound max(2e-2, 2 ulp): <= 1 passes
        ulps[name] = float((diff / torch.clamp(2.0 * ulp, min=2e-2)).max().item())
        del diff, ref, ulp
    ok = all(exact.values()) and errs == 0 and all(u <= 1.0 for u in ulps.values())
    ok_all = _reduce(dist, 1.0 if ok else 0.0, device, "min") == 1.0
    exact_all = {n: _reduce(dist, 1.0 if e else 0.0, device, "min") == 1.0
                 for n, e in exact.items()}
    dmax_all = {n: _max_over_ranks(dist, x, device) for n, x in dmax.items()}
    ulps_all = {n: _max_over_ranks(dist, x, device) for n, x in ulps.items()}
    errs_all = int(_max_over_ranks(dist, errs, device))
    return {"pass": ok_all, "bit_exact_owned_rows": exact_all, "dkdv_max_abs": dmax_all,
            "dkdv_worst_over_bound": ulps_all,
            "tolerance_dkdv": "per element max(2e-2, 2 bf16 ulps of the single-GPU value)",
            "device_errors": errs_all,
            "slice": f"c5 first {H} heads (B=1, T={w['T']}), {ws} rank(s), non-owned rows NaN"}


# ----------------------------------------------------------------------------
# the default line
# ----------------------------------------------------------------------------

def _secondary(name, fn):
    """Run one N=1 side measurement; its failure is reported in the line
    instead of ending the run."""
    t0 = time.perf_counter()
    try:
        out = fn()
    except Exception as e:   # noqa: BLE001
        out = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    out["wall_s"] = round(time.perf_counter() - t0, 2)
    torch.cuda.empty_cache()
    return out


def run_gpu(args):
    from smat_attention_b200.attention import check_device_errors
    dist, rank, ws, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = WORKLOAD
    if w["H"] % ws:
        raise SystemExit(f"H={w['H']} does not split over {ws} ranks")
    H_rank = w["H"] // ws
    case = AttnCase(w, H_rank, device, w["seed"] + rank, keep_host=not args.no_e2e)
    case.warm(args.warmup)
    _barrier(dist, device)

    # ---- device-resident timed region --------------------------------------
    K = args.steps
    ms, per_kernel, clk = case.timed(K, dist, clocks=True)
    dev_err = int(case.err.item())
    ms_step = _max_over_ranks(dist, ms, device)
    total_fl = case.step_flops * ws
    value = total_fl / (ms_step * 1e-3) / 1e12
    per_kernel_max = {n: _max_over_ranks(dist, t, device) for n, t in per_kernel.items()}

    # ---- end to end through the public API with host buffers ---------------
    e2e = None
    if not args.no_e2e and not w.get("fwd_only") and case.dtype == torch.bfloat16:
        e2e_ms, floor_ms, nbytes, numa, hs = _e2e(case, K, dist, args.e2e_heads)
        e2e = {"value": total_fl / (e2e_ms * 1e-3) / 1e12, "unit": UNIT,
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": nbytes,
               "d2h_bytes_per_step": nbytes,
               "floor_ms_per_step": floor_ms, "e2e_over_floor": e2e_ms / floor_ms,
               "host_gbs_floor": 2 * nbytes * ws / (floor_ms * 1e-3) / 1e9,
               "host_placement": numa, "slice": f"1 sequence x {hs} heads"}
    dev_err |= check_device_errors(device)
    launches = K * case.launches_per_step
    case.free()
    torch.cuda.empty_cache()

    peaks = _peaks()
    kern = {}
    for name, t in per_kernel_max.items():
        f = case.fl.get(name)
        kern[name] = {"ms": t}
        if f is not None and name != "bwd_pre":
            tf = f / (t * 1e-3) / 1e12
            kern[name].update({"tflops": tf, "frac": tf / peaks["tflops"],
                               "frac_sustained": tf / peaks["tflops_sustained"]})
    dom = max((n for n in per_kernel_max if n not in ("bwd_pre", "dq_finish")),
              key=per_kernel_max.get)
    achieved = case.fl[dom] / (per_kernel_max[dom] * 1e-3) / 1e12
    traffic = _traffic().get(dom)
    if traffic is not None and H_rank != WORKLOADS["c3"]["H"]:
        traffic *= H_rank / WORKLOADS["c3"]["H"]   # per-head traffic, this rank's heads
    sm_mhz = clk["sm_mhz"] if clk else None
    line = {
        "metric": METRIC if not w.get("fwd_only") else "SMat attn fwd effective TFLOP/s",
        "value": value, "unit": UNIT, "n_gpus": ws, "steps": K,
        "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "f32" if case.dtype == torch.float32 else "bf16", "data": "synthetic",
        "config": _config(ws, w),
        "tokens_per_s": w["B"] * w["T"] / (ms_step * 1e-3),
        "frac_of_peak": value / ws / peaks["tflops"],
        "frac_of_peak_sustained": value / ws / peaks["tflops_sustained"],
        "peak_source": peaks["source"], "sm_mhz": sm_mhz,
        "per_kernel": kern,
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": achieved,
                     "peak": peaks["tflops"], "unit": UNIT, "frac": achieved / peaks["tflops"],
                     "peak_sustained": peaks["tflops_sustained"],
                     "frac_sustained": achieved / peaks["tflops_sustained"],
                     "traffic": traffic, "sm_mhz": sm_mhz},
        "e2e": e2e,
        "gpu_launches": launches,
        "device_errors": dev_err,
        "clocks": clk,
    }

    # ---- c5 sharded by query blocks (every N) -------------------------------
    if not args.no_c5 and w["name"] == "c3":
        line["c5_queries"] = _secondary("c5_queries", lambda: measure_c5_queries(
            dist, rank, ws, device, K=args.c5_steps))
        line["c5_parity"] = _secondary("c5_parity", lambda: measure_c5_parity(
            dist, rank, ws, device))

    # ---- N = 1: the CPU baseline and the other workloads -------------------
    if ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(reps=1)
    if ws == 1 and not args.no_extras and w["name"] == "c3":
        sub = argparse.Namespace(steps=5, warmup=3)
        line["c2"] = _secondary("c2", lambda: _strip(measure_attn(
            WORKLOADS["c2"], device, 20, 3)[0]))
        line["c1"] = _secondary("c1", lambda: _strip(measure_c1(device)))
        line["md3"] = _secondary("md3", lambda: _strip(measure_attn(
            WORKLOADS["md3"], device, 5, 3)[0]))
        line["decode"] = _secondary("decode", lambda: _strip(measure_decode(
            sub, device, K=20)))
        line["c4"] = _secondary("c4", lambda: _strip(measure_lm(sub, device, K=5)))
        line["kattn"] = _secondary("kattn", lambda: _strip(measure_kattn(sub, device, K=5)))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def _strip(d):
    """A side measurement as a compact key (its config kept as one string)."""
    d = dict(d)
    cfg = d.pop("config", None)
    if isinstance(cfg, dict):
        d["workload"] = cfg.get("workload")
    d.pop("clocks", None)
    return d


def _print_line(out, args, ws, metric, dtype, scaling="weak", launches=None):
    line = {"metric": metric, "value": out["value"], "unit": out["unit"], "n_gpus": ws,
            "steps": out.get("steps", args.steps), "warmup": max(3, args.warmup),
            "ms_per_step": out["ms_per_step"], "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": dtype, "data": "synthetic"}
    line.update({k: v for k, v in out.items() if k not in line})
    if launches is not None:
        line["gpu_launches"] = launches
    print(json.dumps(line), flush=True)


def run_side(args):
    """One secondary workload as its own JSON line (``--workload X``)."""
    dist, rank, ws, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    name = WORKLOAD["name"]
    if name == "c4":
        out = measure_lm(args, device, dist, rank, ws)
        metric, dtype, scaling = "LM training tokens/s (fwd+bwd+AdamW)", "bf16", "weak"
    elif name == "decode":
        out = measure_decode(args, device, dist, rank, ws)
        metric, dtype, scaling = ("decode tokens/s (one query per sequence, c3 shapes)", "bf16",
                                  "weak")
    elif name == "kattn":
        out = measure_kattn(args, device, dist, rank, ws)
        metric, dtype, scaling = ("kernelised SMat attention fwd+bwd tokens/s (reference op, "
                                  "M^(3))", "f32", "weak")
    elif name == "c5" and args.shard == "queries":
        out = measure_c5_queries(dist, rank, ws, device, K=args.steps, warmup=args.warmup,
                                 kv_groups=args.kv_groups, overlap=not args.no_overlap)
        metric, dtype, scaling = METRIC, "bf16", "strong"
    else:   # c1, c2, md3, c5 by heads
        out, case = measure_attn(WORKLOAD, device, args.steps, args.warmup, dist, rank, ws,
                                 clocks=True)
        case.free()
        metric = "SMat attn fwd effective TFLOP/s" if WORKLOAD.get("fwd_only") else METRIC
        dtype, scaling = ("f32" if WORKLOAD.get("dtype") == "f32" else "bf16"), "strong"
        if name == "c1" and ws == 1:
            out["cpu_full"] = cpu_c1_full()
    if rank == 0:
        _print_line(out, args, ws, metric, dtype, scaling)
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
    ap.add_argument("--no-c5", action="store_true",
                    help="skip the c5 query-sharded keys of the default line")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the N=1 keys of the other workloads")
    ap.add_argument("--quick", action="store_true",
                    help="the c3 numbers only (= --no-e2e --no-c5 --no-extras "
                         "--no-cpu-baseline; profiling runs)")
    ap.add_argument("--c5-steps", type=int, default=5)
    ap.add_argument("--e2e-heads", type=int, default=None,
                    help="heads per slice of the host-buffer leg (default: whole sequences)")
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
    if args.quick:
        args.no_e2e = args.no_c5 = args.no_extras = args.no_cpu_baseline = True
    WORKLOAD.clear()
    WORKLOAD.update(WORKLOADS[args.workload])
    if args.batch:
        WORKLOAD["B"] = args.batch
    if args.heads:
        WORKLOAD["H"] = args.heads
    if args.impl == "reference" and args.workload in ("c3", "c5", "md3"):
        run_reference(args)
    elif args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the "
                          "dense-masked attention step on host cores; this workload has no "
                          "CPU counterpart there"}))
    elif args.workload == "c3":
        run_gpu(args)
    else:
        run_side(args)


if __name__ == "__main__":
    main()
