#!/usr/bin/env python
"""Benchmark of the B200 block-scaled quantized GEMM (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload auto|nvfp4_8192|nvfp4_256|mxfp8_ffn|colpar]

Workloads:
  nvfp4_8192  NVFP4 M=N=K=8192, bf16 out (configs[1]; the N=1 default)
  colpar      column-parallel NVFP4 M=16384, N=53248, K=8192: B sharded along
              N over the ranks, A broadcast once, bf16 output shards; the
              optional NCCL all-gather is timed separately (the N>1 default)
  mxfp8_ffn   MXFP8 4096 x 14336 x 4096, bf16 out
  nvfp4_256   NVFP4 256^3 fp32 out

A "step" is one GEMM launch over one problem whose quantised operands are
already resident in HBM.  `value` is whole-job TFLOP/s (all ranks' FLOPs over
the max-over-ranks device time of exactly K steps).  `e2e` is the same metric
through the public API with pinned HOST operands: per step the quantised
operands are copied host->device, the GEMM runs, and the bf16 result is
copied back.  The reference arm (--impl reference) times the reference's own
CPU path (oracle/_ref, else this repo's CPU restatement) on bounded samples.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent

WORKLOADS = {
    "nvfp4_8192": dict(fmt="nvfp4", m=8192, n=8192, k=8192, out="bf16", cfg=1),
    # the same GEMM with the output requantised to NVFP4 in the epilogue
    # (the reference's tc6 fused epilogue, GEMMsm110/include/backends/tc6_nvfp4.cuh:460-503)
    "nvfp4_8192_requant": dict(fmt="nvfp4", m=8192, n=8192, k=8192, out="nvfp4", cfg=1),
    # MXFP4 (e2m1, ue8m0 per 32 K; the reference's CUTLASS 72a rows) at 8192^3
    "mxfp4_8192": dict(fmt="mxfp4", m=8192, n=8192, k=8192, out="bf16", cfg=1),
    "nvfp4_256": dict(fmt="nvfp4", m=256, n=256, k=256, out="fp32", cfg=0),
    "mxfp8_ffn": dict(fmt="mxfp8", m=4096, n=14336, k=4096, out="bf16", cfg=2),
    "colpar": dict(fmt="nvfp4", m=16384, n=53248, k=8192, out="bf16", cfg=4),
    # decode GEMM with fused activation quantisation; HBM bound
    "skinny_m16": dict(fmt="nvfp4", m=16, n=28672, k=8192, out="bf16", cfg=3, skinny=True),
    "skinny_m64": dict(fmt="nvfp4", m=64, n=28672, k=8192, out="bf16", cfg=3, skinny=True),
    "skinny_m128": dict(fmt="nvfp4", m=128, n=28672, k=8192, out="bf16", cfg=3, skinny=True),
}
METRIC = "NVFP4/FP8 GEMM TFLOPS and % of B200 tensor peak (HBM GB/s for skinny M), 1/2/4/8 GPU"
SEED = 20260817


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profile_traffic(kernel_tag: str):
    """Per-launch DRAM bytes of `kernel_tag` from the committed ncu summary."""
    f = ROOT / "profiles" / "traffic_per_launch.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_tag:
            return int(parts[1])
    return None


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons sampled while the
    timed region runs: NVML polled every 5 ms from a thread (nvidia-smi
    needs ~1 s to start, longer than a short timed region); nvidia-smi -lms
    when NVML cannot be loaded.  Reads only; changes no GPU setting."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.nvml = None
        self.handle = None
        self.stop = threading.Event()
        self.thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            try:
                props = torch.cuda.get_device_properties(index)
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
        except Exception:
            self.nvml = None

    def __enter__(self):
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _poll_nvml(self):
        nv, h = self.nvml, self.handle
        bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        try:
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception:
            smax = 0
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                flags = ["Active" if rs & b else "Not Active" for b in bits]
                self.lines.append(", ".join([str(self.index), str(sm), str(smax), f"{pw:.1f}",
                                             hex(rs)] + flags))
            except Exception:
                break
            self.stop.wait(0.005)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread is not None and self.nvml is not None:
            self.thread.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        pmax = max(r[2] for r in rows)
        loaded = [r for r in rows if r[2] >= 0.5 * pmax] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in loaded:
            for nm, flag in zip(names, r[3][1:]):
                if flag.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r[0] for r in loaded),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": sorted(reasons),
                "samples": len(loaded), "power_w_max": pmax}


# --------------------------------------------------------------------- ours
def make_operands(q, torch, w, m_rows, n_rows, dev, gen, b_std=1.0):
    """Seeded synthetic fp32 inputs quantised on the device (untimed)."""
    k = w["k"]
    a = torch.randn(m_rows, k, generator=gen, device=dev, dtype=torch.float32)
    b = torch.randn(n_rows, k, generator=gen, device=dev, dtype=torch.float32) * b_std
    if w["fmt"] == "nvfp4":
        A, B = q.make_nvfp4(a), q.make_nvfp4(b)
    elif w["fmt"] == "mxfp4":
        A, B = q.make_mxfp4(a), q.make_mxfp4(b)
    else:
        A, B = q.make_mxfp8(a), q.make_mxfp8(b)
    del a, b
    return A, B


def run_ours(args, w, rank, world, dist, torch):
    from cuda_optimazation_b200 import qgemm as q
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    m, k = w["m"], w["k"]
    n_total = w["n"]
    colpar = args.workload_name == "colpar"
    from cuda_optimazation_b200 import colpar as cp
    if colpar:
        lo, hi = cp.shard_range(n_total, world, rank)
        n = hi - lo
    else:
        n = n_total
    out_dtype = torch.bfloat16 if w["out"] == "bf16" else torch.float32
    requant = w["out"] == "nvfp4"
    gen = torch.Generator(device=dev)
    b_std = 0.02 if w["fmt"] == "mxfp8" else 1.0
    # Operand sets rotate between steps so no step finds its inputs in L2.
    set_bytes = (m + n) * k * (1.0 if w["fmt"] == "mxfp8" else 0.5)
    out_bytes = m * n * {"bf16": 2, "fp32": 4, "nvfp4": 0.5625}[w["out"]]
    nsets = 1 if set_bytes + out_bytes > 3 * 126e6 else 3
    sets = []
    for s in range(nsets):
        if colpar:
            # A identical on every rank (seeded), B: this rank's N-slice.
            gen.manual_seed(SEED + s)
            A, _ = make_operands(q, torch, dict(w, n=0), m, 1, dev, gen)
            gen.manual_seed(SEED + 1000 + s * 97 + rank)
            _, B = make_operands(q, torch, w, 1, n, dev, gen, b_std)
        else:
            gen.manual_seed(SEED + s)
            A, B = make_operands(q, torch, w, m, n, dev, gen, b_std)
        sets.append((A, B))
    if colpar and world > 1:
        # A is broadcast once from rank 0 (untimed).
        for A, _ in sets:
            cp.broadcast_operand([A.quantized, A.block_scales, A.tensor_scale], src=0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    if requant:
        # NVFP4 output (values then REF_LINEAR scales in one buffer) under a
        # fixed output tensor scale, as tc6 takes it.
        qbytes = m * n // 2
        C = torch.empty(qbytes + m * n // 16, dtype=torch.uint8, device=dev)
        out_ts = torch.full((1,), 4.0, dtype=torch.float32, device=dev)
    else:
        C = torch.empty(m, n, dtype=out_dtype, device=dev)
    torch.cuda.synchronize()

    def gemm_into(aq, asf, ats, bq, bsf, bts, dst, layout):
        if requant:
            q.gemm_nvfp4_requant_raw(aq, asf, ats, bq, bsf, bts, out_ts, dst[:qbytes],
                                     dst[qbytes:], m, n, k, q.LAYOUT_REF_LINEAR, layout,
                                     status=status)
        elif w["fmt"] == "nvfp4":
            q.gemm_nvfp4_raw(aq, asf, ats, bq, bsf, bts, dst, m, n, k, layout, status)
        elif w["fmt"] == "mxfp4":
            q.gemm_mxfp4_raw(aq, asf, bq, bsf, dst, m, n, k, layout, status)
        else:
            q.gemm_mxfp8_raw(aq, asf, bq, bsf, dst, m, n, k, layout, status)

    def step(i):
        A, B = sets[i % nsets]
        if requant:
            gemm_into(A.quantized, A.block_scales, A.tensor_scale, B.quantized, B.block_scales,
                      B.tensor_scale, C, A.layout)
        else:
            q.block_scaled_gemm(A, B, out=C, status=status)

    flops_rank = 2.0 * m * n * k
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"device status {code} during warm-up")

    with ClockSampler(dev.index) as clocks:
        # keep the GPU busy briefly before the timed region so the sampler has
        # loaded samples even for short K
        for i in range(args.warmup):
            step(i)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        # Events only around the K steps: an event record between steps costs
        # ~2.6 us of device time, which a ~30 us decode step would carry.
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(stream)
        for i in range(args.steps):
            step(i)
        ev[-1].record(stream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
    total_ms = ev[0].elapsed_time(ev[-1])
    # Average launch time over the timed region (one GEMM launch per step).
    launch_ms = [total_ms / args.steps]
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"device status {code} in the timed region")
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    flops_job = 2.0 * m * n_total * k if colpar else flops_rank * world
    value_tflops = flops_job * args.steps / (total_ms * 1e-3) / 1e12

    # ---- optional all-gather of the bf16 output shards (colpar, N > 1)
    gather = None
    if colpar and world > 1 and not args.no_allgather:
        # colpar.gather_columns: NCCL all-gather of the shards + placement
        # into the full [M, N] matrix.
        for _ in range(2):
            full = cp.gather_columns(C, n_total)
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, min(args.steps, 10))
        g0.record(stream)
        for _ in range(reps):
            full = cp.gather_columns(C, n_total)
        g1.record(stream)
        torch.cuda.synchronize()
        gt = torch.tensor([g0.elapsed_time(g1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        gms = float(gt.item())
        recv = (n_total - n) * m * C.element_size()
        gather = {"ms": gms, "recv_bytes_per_rank": recv, "gbs_per_rank": recv / (gms * 1e-3) / 1e9,
                  "gemm_plus_gather_tflops": flops_job / ((ms_per_step + gms) * 1e-3) / 1e12}
        del full
        # The same gather fused into the GEMM: every tile is TMA-stored into
        # every rank's full C over peer memory (CUDA IPC), overlapping NVLink
        # with the math.  Device time per step, max over ranks.
        if w["fmt"] == "nvfp4":
            bufs = cp.GatherBuffers(m, n_total, dev)
            A, B = sets[0]
            for _ in range(2):
                q.gemm_nvfp4_gather(A, B, bufs.ptrs, lo, n_total, status=status)
            torch.cuda.synchronize()
            dist.barrier()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(reps):
                q.gemm_nvfp4_gather(A, B, bufs.ptrs, lo, n_total, status=status)
            f1.record(stream)
            torch.cuda.synchronize()
            dist.barrier()
            rc, code = q.read_status(status)
            if rc != q.OK:
                raise SystemExit(f"device status {code} in the fused gather")
            ft = torch.tensor([f0.elapsed_time(f1) / reps], dtype=torch.float64, device=dev)
            dist.all_reduce(ft, op=dist.ReduceOp.MAX)
            fms = float(ft.item())
            gather["fused"] = {"ms_per_step": fms,
                               "tflops": flops_job / (fms * 1e-3) / 1e12,
                               "kernel": "gemm_pair_kernel, epilogue TMA stores to all ranks"}
            bufs.close()

    # ---- end to end through the public API with host buffers
    A0, B0 = sets[0]
    host = {name: t_.cpu().pin_memory() for name, t_ in
            (("aq", A0.quantized), ("asf", A0.block_scales), ("bq", B0.quantized),
             ("bsf", B0.block_scales))}
    hts = [A0.tensor_scale.cpu().pin_memory() if hasattr(A0, "tensor_scale") else None,
           B0.tensor_scale.cpu().pin_memory() if hasattr(B0, "tensor_scale") else None]
    hout = [torch.empty_like(C, device="cpu").pin_memory() for _ in range(2)]
    # Two device buffer sets so step i's host->device copies (copy-in
    # stream) and step i-1's device->host read of the result (copy-out
    # stream) overlap step i's GEMM, as a serving loop would run them; every
    # step still moves its full inputs in and its full result out.
    dA = [{name: torch.empty_like(h, device=dev) for name, h in host.items()} for _ in range(2)]
    dts = [[None if h is None else torch.empty_like(h, device=dev) for h in hts] for _ in range(2)]
    dC = [torch.empty_like(C) for _ in range(2)]
    h2d = sum(h.numel() * h.element_size() for h in host.values()) + \
        sum(h.numel() * 4 for h in hts if h is not None)
    d2h = hout[0].numel() * hout[0].element_size()
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of buffer set landed
    ev_gemm = [torch.cuda.Event() for _ in range(2)]   # GEMM on buffer set done
    ev_out = [torch.cuda.Event() for _ in range(2)]    # result of buffer set read back
    for e_ in ev_gemm + ev_out:
        e_.record(stream)

    def e2e_step(i):
        b_ = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_gemm[b_])            # set b_ free (GEMM i-2 consumed it)
            for name in host:
                dA[b_][name].copy_(host[name], non_blocking=True)
            for d_, h_ in zip(dts[b_], hts):
                if h_ is not None:
                    d_.copy_(h_, non_blocking=True)
            ev_in[b_].record(s_in)
        stream.wait_event(ev_in[b_])
        stream.wait_event(ev_out[b_])               # C[b_] read back (step i-2)
        gemm_into(dA[b_]["aq"], dA[b_]["asf"], dts[b_][0], dA[b_]["bq"], dA[b_]["bsf"],
                  dts[b_][1], dC[b_], A0.layout)
        ev_gemm[b_].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_gemm[b_])
            hout[b_].copy_(dC[b_], non_blocking=True)
            ev_out[b_].record(s_out)

    e2e_steps = max(3, min(args.steps, 20))
    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_stream(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    et = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_ms = float(et.item())
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"device status {code} in the e2e region")

    if rank != 0:
        return None
    pk = peaks()
    ratio = 2.0 if w["fmt"] == "mxfp8" else 4.0
    peak_tflops = pk["bf16_tflops"] * ratio
    avg_launch_ms = statistics.mean(launch_ms)
    achieved = flops_rank / (avg_launch_ms * 1e-3) / 1e12
    tag = f"gemm_{w['fmt']}_{args.workload_name}"
    line = {
        "metric": METRIC,
        "value": round(value_tflops, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "strong" if colpar else "weak",
        "vs_baseline": None,
        "dtype": w["fmt"],
        "data": "synthetic (seeded torch.randn N(0,1); weights N(0,0.02) for mxfp8), quantised "
                "on the device before timing",
        "config": {
            "workload": f"{w['fmt']}_gemm_{m}x{n_total}x{k}_{w['out']}out",
            "baseline_config_index": w["cfg"], "m": m, "n": n_total, "k": k,
            "n_per_rank": n, "out": w["out"],
            "parallelism": f"colpar{world}" if colpar else (f"replica{world}" if world > 1 else "single"),
            "l2": (f"{nsets} rotating operand sets ({set_bytes / 1e6:.0f} MB each) + "
                   f"{out_bytes / 1e6:.0f} MB output per step vs 126 MB L2"),
        },
        "pct_peak": round(100.0 * value_tflops / world / peak_tflops, 2),
        "roofline": {
            "bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak_tflops, 1),
            "unit": "TFLOP/s", "frac": round(achieved / peak_tflops, 4),
            "traffic": profile_traffic(tag),
            "peak_basis": f"{pk['source']} cuBLAS bf16 burst {pk['bf16_tflops']} TF/s x {ratio:g} "
                          f"(dense {w['fmt']} : bf16 tensor rate on B200); nominal "
                          f"{9000 if ratio == 4 else 4500} TF/s -> frac "
                          f"{achieved / (9000 if ratio == 4 else 4500):.4f}",
            "algorithmic_flop_per_launch": flops_rank,
        },
        "e2e": {"value": round(flops_job / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": round(e2e_ms, 4),
                "pipeline": "H2D, GEMM and D2H on three streams over two buffer sets"},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if gather:
        line["allgather"] = gather
    if world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline(w, budget_s=args.cpu_budget)
        except ValueError as e:  # the reference's CPU path covers NVFP4 only
            line["cpu_baseline"] = {"unavailable": str(e)}
    return line


def run_skinny(args, w, rank, world, dist, torch):
    """Decode GEMM: bf16 activations with 0.1% outliers
    x50, pre-quantised NVFP4 weights N(0, 0.02); one step = one
    qg_gemm_nvfp4_skinny call (activation amax + quantise + stream-K GEMM +
    scale/convert).  Metric: algorithmic HBM bytes / step time."""
    from cuda_optimazation_b200 import qgemm as q
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    m, n, k = w["m"], w["n"], w["k"]
    gen = torch.Generator(device=dev)
    # Two weight sets (2 x 132 MB > 126 MB L2) alternate between steps.
    sets = []
    for s_ in range(2):
        gen.manual_seed(SEED + 500 + s_ + rank)
        W = q.make_nvfp4(torch.randn(n, k, generator=gen, device=dev) * 0.02)
        x = torch.randn(m, k, generator=gen, device=dev)
        x.view(-1)[::1000] *= 50.0
        sets.append((x.to(torch.bfloat16), W))
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ws = q.skinny_workspace(m, n, k, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def call(i):
        x, W = sets[i % 2]
        q.gemm_nvfp4_skinny(x, W, out=out, workspace=ws, status=status)

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    # A decode step is ~20 us of GPU work, less than the host needs to issue
    # one call (tensor-map encodes, 5 launches, Python/ctypes), so each step
    # is one CUDA-graph replay of the public call, as a decode loop runs it.
    graphs = []
    for i in range(2):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            call(i)
        graphs.append(g)
    torch.cuda.synchronize()

    def step(i):
        graphs[i % 2].replay()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        for i in range(args.warmup):
            step(i)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        # Events only around the K steps: an event record between steps costs
        # ~2.6 us of device time, which a ~30 us decode step would carry.
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(stream)
        for i in range(args.steps):
            step(i)
        ev[-1].record(stream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"device status {code}")
    total_ms = ev[0].elapsed_time(ev[-1])
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms = total_ms / args.steps
    bytes_step = n * k * (0.5 + 1 / 16) + m * k * 2 + m * n * 2
    value = bytes_step * world * args.steps / (total_ms * 1e-3) / 1e9

    # End to end: every step copies its activations in from pinned host
    # memory and its result out to pinned host memory.  Two buffer sets (and
    # the two weight sets) alternate so that step i's host->device copy and
    # step i-1's device->host copy overlap step i's call, on their own
    # streams, as a serving loop would run them.
    hx = [sets[b][0].cpu().pin_memory() for b in range(2)]
    hout = [torch.empty(m, n, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dx = [torch.empty_like(sets[b][0]) for b in range(2)]
    dout = [torch.empty(m, n, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    ge = []
    for b in range(2):
        g_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_):
            q.gemm_nvfp4_skinny(dx[b], sets[b][1], out=dout[b], workspace=ws, status=status)
        ge.append(g_)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_call = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for e_ in ev_call + ev_out:
        e_.record(stream)

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_call[b])        # dx[b] consumed by call i-2
            dx[b].copy_(hx[b], non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])           # dout[b] read back (step i-2)
        ge[b].replay()
        ev_call[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_call[b])
            hout[b].copy_(dout[b], non_blocking=True)
            ev_out[b].record(s_out)

    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(4, min(args.steps, 50))
    e0.record(stream)
    s_in.wait_stream(stream)
    for i in range(reps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / reps
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"device status {code} in the e2e region")
    if rank != 0:
        return None
    pk = peaks()
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4",
        "data": "synthetic (seeded torch.randn; activations N(0,1) with every 1000th x50, "
                "weights N(0,0.02)); weights quantised before timing",
        "config": {"workload": f"nvfp4_skinny_gemm_m{m}_n{n}_k{k}_fused_act_quant",
                   "baseline_config_index": 3, "m": m, "n": n, "k": k, "out": "bf16",
                   "parallelism": f"replica{world}" if world > 1 else "single",
                   "l2": "2 alternating 132 MB weight sets vs 126 MB L2",
                   "launch": "each step replays a CUDA graph of one qg_gemm_nvfp4_skinny call"},
        "tflops": round(2.0 * m * n * k / (ms * 1e-3) / 1e12, 2),
        "roofline": {"bound": "hbm", "achieved": round(bytes_step / (ms * 1e-3) / 1e9, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(bytes_step / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                     "traffic": profile_traffic(f"gemm_skinny_m{m}"),
                     "peak_basis": f"{pk['source']} STREAM copy GB/s; achieved counts the whole "
                                   "fused call (one cooperative launch: activation quantisation + GEMM) as the unit",
                     "algorithmic_bytes_per_call": int(bytes_step)},
        "e2e": {"value": round(bytes_step / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": int(m * k * 2), "d2h_bytes_per_step": int(m * n * 2),
                "ms_per_step": round(e2e_ms, 4),
                "pipeline": "H2D, call and D2H on three streams over two buffer sets"},
        "gpu_launches": args.steps,  # one kernel per call
        "clocks": clocks.summary(),
    }


# --------------------------------------------------------------------- CPU
def _cpu_impl():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as om
    o = om.Oracle()
    try:
        ref = om.Reference()
        return o, ref, "reference"
    except (FileNotFoundError, OSError):
        return o, None, "port"


class _CpuPath:
    """Cost model of the CPU path, measured on bounded samples.

    The job is: quantise A (M rows) and B (N rows) with the NVFP4 quantizer,
    dequantise, and run the double-accumulation O2 GEMM over M x N outputs.
    `sample()` times the quantise + dequantise of `qrows` rows and O2 over an
    `orows` x `ocols` block of outputs (threads split the rows), and returns
    the extrapolated job time (M + N) * t_row + M * N * t_out."""

    def __init__(self, o, ref, w, threads, seed=SEED):
        import numpy as np
        if w["fmt"] != "nvfp4" or w.get("skinny"):
            raise ValueError("the reference's CPU path (quantise + O2) exists for NVFP4 only")
        self.np, self.o, self.ref, self.w, self.threads, self.seed = np, o, ref, w, threads, seed

    def _quant(self, x, r):
        np, k = self.np, self.w["k"]
        if self.ref is not None:
            q, sf, _ = self.ref.nvfp4_reference(x)
            codes = np.stack([q >> 4, q & 0xF], axis=1).ravel()[: r * k]  # high nibble first
            mag = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float32)
            vals = np.where(codes & 8, -mag[codes & 7], mag[codes & 7]).astype(np.float32)
            lut = np.array([self.ref.L.qgr_decode_e4m3_positive(i) for i in range(256)], np.float32)
            return vals, lut[sf[: r * k // 16]]
        q, sf, _ = self.o.nvfp4_mma(x.reshape(r, k), 0)
        return self.o.nvfp4_decode(q, sf, r, k, 0)

    def sample(self, qrows, orows, ocols, seed_offset=0):
        m, n, k = self.w["m"], self.w["n"], self.w["k"]
        xa = self.o.normal(qrows * k, self.seed + seed_offset)
        xb = self.o.normal(ocols * k, (self.seed ^ 0xBB67AE85) + seed_offset)
        t0 = time.perf_counter()
        av, as_ = self._quant(xa, qrows)
        t_quant = time.perf_counter() - t0
        bv, bs = self._quant(xb, ocols)
        gemm = (self.ref or self.o).gemm
        t0 = time.perf_counter()
        gemm(av[: orows * k], bv, as_[: orows * (k // 16)], bs, orows, ocols, k, 16,
             rows=(0, orows), threads=self.threads)
        t_gemm = time.perf_counter() - t0
        t_row = t_quant / qrows
        t_out = t_gemm / (orows * ocols)
        t_job = (m + n) * t_row + m * n * t_out
        return t_job, t_quant + t_gemm, t_row, t_out


def cpu_baseline(w, budget_s: float = 20.0) -> dict:
    o, ref, kind = _cpu_impl()
    threads = os.cpu_count() or 1
    m, n, k = w["m"], w["n"], w["k"]
    path = _CpuPath(o, ref, w, threads)
    qrows, orows, ocols = min(m, 64), min(m, threads), min(n, 256)
    _, t_s, _, t_out = path.sample(qrows, orows, ocols)
    # Grow the O2 block toward the time budget.
    scale = max(1.0, (budget_s * 0.8) / max(t_s, 1e-6))
    orows = int(min(m, max(orows, (orows * scale) // threads * threads)))
    qrows = min(m, max(256, orows))
    t_job, t_s, t_row, t_out = path.sample(qrows, orows, ocols)
    flops = 2.0 * m * n * k
    return {"value": round(flops / t_job / 1e12, 8), "unit": "TFLOP/s", "cores": threads,
            "kind": kind,
            "sample": (f"{'oracle/_ref (reference headers)' if ref else 'oracle port'}: NVFP4 "
                       f"quantise+dequantise of {qrows} rows ({t_row * 1e3:.2f} ms/row, one thread, "
                       f"as the reference) and O2 GEMM of a {orows}x{ocols} output block "
                       f"({t_out * 1e6:.2f} us/output on {threads} threads); job time "
                       f"(M+N)*t_row + M*N*t_out = {t_job:.1f}s"),
            "job_seconds_extrapolated": round(t_job, 2)}


def run_reference_arm(args, w, rank, world):
    """Time the reference's own CPU implementation on bounded samples of the
    same workload (rank 0 only); each step is one sample."""
    if rank != 0:
        return None
    o, ref, kind = _cpu_impl()
    threads = os.cpu_count() or 1
    m, n, k = w["m"], w["n"], w["k"]
    path = _CpuPath(o, ref, w, threads)
    qrows, orows, ocols = min(m, 64), min(m, 4 * threads), min(n, 512)
    for i in range(min(args.warmup, 1)):
        path.sample(qrows, orows, ocols, seed_offset=i + 1)
    res = [path.sample(qrows, orows, ocols, seed_offset=i + 100) for i in range(args.steps)]
    t_job = statistics.mean(r[0] for r in res)
    t_step = statistics.mean(r[1] for r in res)
    value = 2.0 * m * n * k / t_job / 1e12
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 8), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t_step * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if args.workload_name == "colpar" else "weak", "vs_baseline": None,
        "dtype": w["fmt"], "data": "synthetic (seeded std::mt19937_64 N(0,1))",
        "config": {"workload": f"{w['fmt']}_gemm_{m}x{n}x{k}_{w['out']}out",
                   "baseline_config_index": w["cfg"], "m": m, "n": n, "k": k},
        "cpu_baseline": {"value": round(value, 8), "unit": "TFLOP/s", "cores": threads,
                         "kind": kind,
                         "sample": f"per step: NVFP4 quantise+dequantise of {qrows} rows (one "
                                   f"thread) and O2 over a {orows}x{ocols} output block "
                                   f"({threads} threads); job time (M+N)*t_row + M*N*t_out"},
        "e2e": {"value": round(value, 8), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="auto", choices=["auto", *WORKLOADS])
    ap.add_argument("--no-allgather", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.workload == "auto":
        args.workload = "colpar" if world > 1 else "nvfp4_8192"
    args.workload_name = args.workload
    w = WORKLOADS[args.workload]

    if args.impl == "reference":
        if w["fmt"] != "nvfp4" or w.get("skinny"):
            line = {"impl": "reference", "unavailable":
                    "the reference has no CPU path for this workload (MXFP8 / decode GEMM)"}
        else:
            line = run_reference_arm(args, w, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import torch
    dist = None
    if world > 1:
        import torch.distributed as td
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        td.init_process_group("nccl", device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
        dist = td
    line = (run_skinny if w.get("skinny") else run_ours)(args, w, rank, world, dist, torch)
    if line is not None:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
