#!/usr/bin/env python
"""Benchmark of the B200 block-scaled quantized GEMM (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload auto|colpar|nvfp4_8192|...] [--no-subrecords]

Headline workload (every N): the column-parallel NVFP4
GEMM M=16384, N=53248, K=8192.  B is quantised once and sharded along N over
the ranks (colpar.shard_rows of one K-major operand), A is quantised once and
broadcast, every rank runs its local GEMM with no communication; at N = 1 the
one rank owns all of B.  The output gather (NCCL, and fused into the GEMM
epilogue over peer memory) is timed separately at N > 1.

At N = 1 the line also carries `subrecords` for the other BASELINE configs,
each with its own steps, ms, roofline and clocks: NVFP4 8192^3,
the same GEMM with NVFP4 output (the tc6 row), MXFP4 8192^3, MXFP8
4096x14336x4096 and the decode GEMM at m = 16, 64, 128
(configs[3]).

A "step" is one GEMM launch over one problem whose quantised operands are
already resident in HBM.  `value` is whole-job TFLOP/s (all ranks' FLOPs over
the max-over-ranks device time of exactly K steps).  `e2e` is the same metric
through the public API starting from fp32 HOST data, as the reference's CPU
path does: per step A and B are copied host->device, quantised to NVFP4 on the
device, multiplied, and the bf16 result is copied back.  The reference arm
(--impl reference) times the reference's own CPU path (oracle/_ref, else this
repo's CPU restatement) on the same bounded sample blocks as `cpu_baseline`.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent

WORKLOADS = {
    "colpar": dict(fmt="nvfp4", m=16384, n=53248, k=8192, out="bf16", cfg=4),
    "nvfp4_8192": dict(fmt="nvfp4", m=8192, n=8192, k=8192, out="bf16", cfg=1),
    # the same GEMM with the output requantised to NVFP4 in the epilogue
    # (the reference's tc6 fused epilogue, GEMMsm110/include/backends/tc6_nvfp4.cuh:460-503)
    "nvfp4_8192_requant": dict(fmt="nvfp4", m=8192, n=8192, k=8192, out="nvfp4", cfg=1),
    # MXFP4 (e2m1, ue8m0 per 32 K; the reference's CUTLASS 72a rows) at 8192^3
    "mxfp4_8192": dict(fmt="mxfp4", m=8192, n=8192, k=8192, out="bf16", cfg=1),
    "nvfp4_256": dict(fmt="nvfp4", m=256, n=256, k=256, out="fp32", cfg=0),
    "mxfp8_ffn": dict(fmt="mxfp8", m=4096, n=14336, k=4096, out="bf16", cfg=2),
    # decode GEMM with fused activation quantisation; HBM bound
    "skinny_m16": dict(fmt="nvfp4", m=16, n=28672, k=8192, out="bf16", cfg=3, skinny=True),
    "skinny_m64": dict(fmt="nvfp4", m=64, n=28672, k=8192, out="bf16", cfg=3, skinny=True),
    "skinny_m128": dict(fmt="nvfp4", m=128, n=28672, k=8192, out="bf16", cfg=3, skinny=True),
}
SUBRECORDS = ["nvfp4_8192", "nvfp4_8192_requant", "mxfp4_8192", "mxfp8_ffn",
              "skinny_m16", "skinny_m64", "skinny_m128"]
METRIC = "NVFP4/FP8 GEMM TFLOPS and % of B200 tensor peak (HBM GB/s for skinny M), 1/2/4/8 GPU"
SEED = 20260817
L2_BYTES = 126e6
# Timed regions of the sub-records last at least this long, so the clock
# sampler sees the GPU under load.
SUB_MIN_TIMED_S = 0.25


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
    """Per-launch DRAM bytes of `kernel_tag` from the committed ncu summary
    (profiles/traffic_per_launch.txt: tag, bytes, how they were captured)."""
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
        import torch
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


# --------------------------------------------------------------------- config
def sample_rows(m: int, count: int) -> list:
    """The reference's sample rows s*131 % m (GEMMsm110/include/gemm_benchmark.cuh:51-53)."""
    return sorted({(s * 131) % m for s in range(count)} | {m - 1})


def sample_cols(n: int, count: int) -> list:
    """The reference's sample columns s*197 % n (gemm_benchmark.cuh:51-53)."""
    return sorted({(s * 197) % n for s in range(count)} | {n - 1})


def workload_config(name: str, w: dict, world: int, rank: int) -> dict:
    """The `config` object of the JSON line, identical in both arms."""
    from_colpar = name == "colpar"
    m, n_total, k = w["m"], w["n"], w["k"]
    if from_colpar:
        lo, hi = shard_range(n_total, world, rank)
        n_local = hi - lo
    else:
        n_local = n_total
    if w.get("skinny"):
        return {"workload": f"nvfp4_skinny_gemm_m{m}_n{n_total}_k{k}_fused_act_quant",
                "baseline_config_index": 3, "m": m, "n": n_total, "k": k, "out": "bf16",
                "parallelism": f"replica{world}" if world > 1 else "single",
                "l2": "2 alternating 132 MB weight sets vs 126 MB L2",
                "launch": "each step replays a CUDA graph of one qg_gemm_nvfp4_skinny call"}
    elem = 1.0 if w["fmt"] == "mxfp8" else 0.5
    set_bytes = (m + n_local) * k * elem
    out_bytes = m * n_local * {"bf16": 2, "fp32": 4, "nvfp4": 0.5625}[w["out"]]
    nsets = 1 if set_bytes + out_bytes > 3 * L2_BYTES else 3
    return {
        "workload": f"{w['fmt']}_gemm_{m}x{n_total}x{k}_{w['out']}out",
        "baseline_config_index": w["cfg"], "m": m, "n": n_total, "k": k,
        "n_per_rank": n_local, "out": w["out"],
        "parallelism": (f"colpar{world} (B sharded along N, A broadcast)" if from_colpar
                        else (f"replica{world}" if world > 1 else "single")),
        "l2": (f"{nsets} rotating operand set(s) ({set_bytes / 1e6:.0f} MB each) + "
               f"{out_bytes / 1e6:.0f} MB output per step vs 126 MB L2"),
        "operand_sets": nsets,
    }


def shard_range(n: int, world: int, rank: int, align: int = 256):
    """Same split as colpar.shard_range (importable without torch)."""
    blocks = (n + align - 1) // align
    per, extra = blocks // world, blocks % world
    b0 = rank * per + min(rank, extra)
    b1 = b0 + per + (1 if rank < extra else 0)
    return min(n, b0 * align), min(n, b1 * align)


def timed(torch, stream, fn, steps, dist=None):
    """Device time (ms) of exactly `steps` calls of fn(i), events on the
    launching stream at the two ends only (a record between steps costs
    ~2.6 us of device time), barrier + synchronise on both sides; max over
    ranks."""
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    for i in range(steps):
        fn(i)
    ev[1].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t = torch.tensor([ev[0].elapsed_time(ev[1])], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------- ours
def run_gemm(args, name, w, rank, world, dist, torch, steps, headline=True):
    """One GEMM workload: operands quantised on the device (untimed), the
    timed region, and for the headline the e2e leg, the gather legs (N > 1)
    and the sample the CPU checker compares against."""
    from cuda_optimazation_b200 import colpar as cp
    from cuda_optimazation_b200 import qgemm as q
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    stream = torch.cuda.current_stream()
    cfg = workload_config(name, w, world, rank)
    m, n_total, k = w["m"], w["n"], w["k"]
    is_colpar = name == "colpar"
    lo, hi = shard_range(n_total, world, rank) if is_colpar else (0, n_total)
    n = hi - lo
    nsets = cfg["operand_sets"]
    requant = w["out"] == "nvfp4"
    out_dtype = torch.bfloat16 if w["out"] == "bf16" else torch.float32
    b_std = 0.02 if w["fmt"] == "mxfp8" else 1.0
    layout = q.LAYOUT_MMA_KMAJOR if is_colpar else q.LAYOUT_MMA
    quant = {"nvfp4": lambda x: q.make_nvfp4(x, layout), "mxfp4": lambda x: q.make_mxfp4(x, layout),
             "mxfp8": lambda x: q.make_mxfp8(x, layout)}[w["fmt"]]
    gen = torch.Generator(device=dev)
    sets, check = [], None
    rows_s, cols_s = sample_rows(m, 16), sample_cols(n_total, 4096)
    for s in range(nsets):
        # A: identical on every rank (same seed), quantised once.  B: the
        # whole seeded B quantised once (one tensor scale), this rank keeps
        # its N-shard -- what a checkpoint loader does.
        gen.manual_seed(SEED + s)
        xa = torch.randn(m, k, generator=gen, device=dev)
        A = quant(xa)
        gen.manual_seed((SEED ^ 0xBB67AE85) + s)
        xb = torch.randn(n_total, k, generator=gen, device=dev)
        if b_std != 1.0:
            xb *= b_std
        B_full = quant(xb)
        B = cp.shard_rows(B_full, lo, hi) if is_colpar else B_full
        if s == 0 and headline and w["fmt"] == "nvfp4" and not requant and world == 1:
            # What the CPU checker needs (N = 1 only): the fp32 sample rows
            # of A and of B (= output columns), the tensors' amax, and the
            # quantised bytes of those rows.
            ri = torch.tensor(rows_s, device=dev)
            ci = torch.tensor(cols_s, device=dev)
            check = {"rows": rows_s, "cols": cols_s, "m": m, "n": n_total, "k": k,
                     "bf16": w["out"] == "bf16",
                     "layout_order": 1 if is_colpar else 0,
                     "xa_rows": xa[ri].cpu().numpy(), "xb_rows": xb[ci].cpu().numpy(),
                     "amax_a": float(xa.abs().max().item()), "amax_b": float(xb.abs().max().item()),
                     "ts_a": float(A.tensor_scale.item()), "ts_b": float(B_full.tensor_scale.item()),
                     "qa_rows": A.quantized.view(m, k // 2)[ri].cpu().numpy(),
                     "sfa": A.block_scales.cpu().numpy(),
                     "qb_rows": B_full.quantized.view(n_total, k // 2)[ci].cpu().numpy(),
                     "sfb": B_full.block_scales.cpu().numpy()}
        del xa, xb
        sets.append((A, B))
    if is_colpar and world > 1:
        # A is broadcast once from rank 0 (untimed); every rank already holds
        # the same bytes, the broadcast is the deployment's data path.
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

    def step(i):
        A, B = sets[i % nsets]
        if requant:
            q.gemm_nvfp4_requant_raw(A.quantized, A.block_scales, A.tensor_scale, B.quantized,
                                     B.block_scales, B.tensor_scale, out_ts, C[:qbytes],
                                     C[qbytes:], m, n, k, q.LAYOUT_REF_LINEAR, A.layout,
                                     status=status)
        else:
            q.block_scaled_gemm(A, B, out=C, status=status)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"{name}: device status {code} during warm-up")
    est_ms = timed(torch, stream, step, 2, dist) / 2
    if not headline:
        steps = max(steps, math.ceil(SUB_MIN_TIMED_S * 1e3 / max(est_ms, 1e-3)))
    with ClockSampler(dev.index) as clocks:
        # keep the GPU busy briefly before the timed region so the sampler
        # sees it loaded even for short K
        for i in range(args.warmup):
            step(i)
        total_ms = timed(torch, stream, step, steps, dist)
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"{name}: device status {code} in the timed region")
    ms_per_step = total_ms / steps
    flops_rank = 2.0 * m * n * k
    flops_job = 2.0 * m * n_total * k if is_colpar else flops_rank * world
    value = flops_job * steps / (total_ms * 1e-3) / 1e12

    pk = peaks()
    ratio = 2.0 if w["fmt"] == "mxfp8" else 4.0
    peak_tflops = pk["bf16_tflops"] * ratio
    # This rank's launches over the timed region (the max over ranks is in
    # ms_per_step); one GEMM launch per step.
    achieved = flops_rank / (ms_per_step * 1e-3) / 1e12
    tag = {"colpar": f"colpar_n{n}", "nvfp4_8192": "gemm_nvfp4_nvfp4_8192"}.get(
        name, f"gemm_{w['fmt']}_{name}")
    rec = {
        "value": round(value, 2), "unit": "TFLOP/s", "steps": steps,
        "ms_per_step": round(ms_per_step, 5), "dtype": w["fmt"], "config": cfg,
        "pct_peak": round(100.0 * value / world / peak_tflops, 2),
        "roofline": {
            "bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak_tflops, 1),
            "unit": "TFLOP/s", "frac": round(achieved / peak_tflops, 4),
            "traffic": profile_traffic(tag),
            "traffic_source": "profiles/traffic_per_launch.txt (ncu dram__bytes_read+write of one launch)",
            "peak_basis": f"{pk['source']} cuBLAS bf16 burst {pk['bf16_tflops']} TF/s x {ratio:g} "
                          f"(dense {w['fmt']} : bf16 tensor rate on B200); nominal "
                          f"{9000 if ratio == 4 else 4500} TF/s -> frac "
                          f"{achieved / (9000 if ratio == 4 else 4500):.4f}",
            "algorithmic_flop_per_launch": flops_rank,
            "kernel": "gemm_pair_kernel (cta_group::2, one launch per step)",
        },
        "gpu_launches": steps,
        "clocks": clocks.summary(),
    }
    if not headline:
        return rec

    # ---- output gather legs (column-parallel, N > 1)
    if is_colpar and world > 1 and not args.no_allgather:
        rec["allgather"] = gather_legs(args, torch, dist, q, cp, sets, step, C, m, n_total, lo,
                                       n, flops_job, ms_per_step, status, stream, dev)

    # ---- end to end through the public API from fp32 host data
    rec["e2e"] = e2e_leg(args, torch, dist, q, cp, w, dev, stream, m, n, k, b_std, layout,
                         flops_job, world)
    rec["_check"] = check
    if check is not None:
        step(0)  # C holds set 0's product for the checker
        torch.cuda.synchronize()
        ri = torch.tensor(check["rows"], device=dev)
        ci = torch.tensor(check["cols"], device=dev)
        check["c"] = C[ri][:, ci].float().cpu().numpy()
    return rec


def gather_legs(args, torch, dist, q, cp, sets, step, C, m, n_total, lo, n, flops_job,
                ms_per_step, status, stream, dev):
    """NCCL all-gather of the shards (rank-major, no placement copy) and the
    gather fused into the GEMM epilogue (row-major full C on every rank),
    each timed on the device (max over ranks); the fused result is compared
    bit for bit with the shards the NCCL leg moved."""
    step(0)  # C = set 0's shard
    torch.cuda.synchronize()
    world = dist.get_world_size()
    reps = max(3, min(args.steps, 10))
    gathered = None

    def nccl_gather(_):
        nonlocal gathered
        gathered = cp.gather_columns(C, n_total, rank_major=True)

    for i in range(2):
        nccl_gather(i)
    gms = timed(torch, stream, nccl_gather, reps, dist) / reps
    recv = (n_total - n) * m * C.element_size()
    out = {"nccl": {"ms": round(gms, 4), "layout": "rank-major [P, M, N/P]",
                    "recv_bytes_per_rank": recv, "gbs_per_rank": round(recv / (gms * 1e-3) / 1e9, 1),
                    "gemm_plus_gather_tflops": round(flops_job / ((ms_per_step + gms) * 1e-3) / 1e12, 2)}}
    bufs = cp.GatherBuffers(m, n_total, dev)
    A, B = sets[0]

    def fused(_):
        q.gemm_nvfp4_gather(A, B, bufs.ptrs, lo, n_total, status=status)

    # The timed loop calls the kernel back to back with identical inputs:
    # each step overwrites the peers' buffers with the same values, so no
    # reader is disturbed (colpar_gemm_fused orders ranks between steps).
    for i in range(2):
        fused(i)
    fms = timed(torch, stream, fused, reps, dist) / reps
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"device status {code} in the fused gather")
    # Every rank's full C must hold every rank's shard exactly as the local
    # GEMM wrote it (the shards the NCCL leg gathered).
    ok = True
    for r in range(world):
        a, b = cp.shard_range(n_total, world, r)
        ok &= bool(torch.equal(bufs.c[:, a:b], gathered[r, :, : b - a]))
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    out["fused"] = {"ms_per_step": round(fms, 4), "tflops": round(flops_job / (fms * 1e-3) / 1e12, 2),
                    "kernel": "gemm_pair_kernel, epilogue TMA stores to all ranks",
                    "nvlink_gbs_per_rank": round(recv / (fms * 1e-3) / 1e9, 1)}
    out["parity"] = ("ok: every rank's fused full C equals the NCCL-gathered local shards bit for bit"
                     if flag.item() == 1 else "FAIL: fused gather differs from the local shards")
    bufs.close()
    return out


def e2e_leg(args, torch, dist, q, cp, w, dev, stream, m, n, k, b_std, layout, flops_job, world):
    """The public API end to end from fp32 host data: per step H2D of A and
    this rank's B rows (pinned), qg_quantize_nvfp4 of both, the GEMM, D2H of
    the bf16 result.  Copies, quantisation and the GEMM run on three streams
    over two buffer sets, as a serving loop would run them; every step still
    moves its full inputs in and its full result out."""
    if w["fmt"] != "nvfp4" or w["out"] != "bf16":
        return None
    g = torch.Generator(device=dev).manual_seed(SEED + 77)
    ha = torch.randn(m, k, generator=g, device=dev).cpu().pin_memory()
    hb = (torch.randn(n, k, generator=g, device=dev) * b_std).cpu().pin_memory()
    hout = [torch.empty(m, n, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dA = [torch.empty_like(ha, device=dev) for _ in range(2)]
    dB = [torch.empty_like(hb, device=dev) for _ in range(2)]
    dC = [torch.empty(m, n, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    ws = [torch.empty(int(q.lib().qg_quantize_workspace_bytes()), dtype=torch.uint8, device=dev)
          for _ in range(2)]
    h2d = (ha.numel() + hb.numel()) * 4
    d2h = m * n * 2
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_gemm = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for e_ in ev_gemm + ev_out:
        e_.record(stream)

    def e2e_step(i):
        b_ = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_gemm[b_])            # set b_ free (step i-2 consumed it)
            dA[b_].copy_(ha, non_blocking=True)
            dB[b_].copy_(hb, non_blocking=True)
            ev_in[b_].record(s_in)
        stream.wait_event(ev_in[b_])
        stream.wait_event(ev_out[b_])               # C[b_] read back (step i-2)
        A = q.make_nvfp4(dA[b_], layout, workspace=ws[b_])
        B = q.make_nvfp4(dB[b_], layout, workspace=ws[b_])
        q.block_scaled_gemm(A, B, out=dC[b_])
        ev_gemm[b_].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_gemm[b_])
            hout[b_].copy_(dC[b_], non_blocking=True)
            ev_out[b_].record(s_out)

    steps = max(3, min(args.steps, 20))
    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_stream(stream)
    for i in range(steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    et = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_ms = float(et.item())
    return {"value": round(flops_job / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(e2e_ms, 4), "steps": steps,
            "work_per_step": "H2D fp32 A and this rank's B rows, qg_quantize_nvfp4 of both, "
                             "qg_gemm_nvfp4, D2H of the bf16 C"
                             + ("; at N > 1 each rank quantises its B rows under their own tensor "
                                "scale (same work; the timed `value` runs shards of one quantised B)"
                                if world > 1 else ""),
            "pipeline": "H2D, quantise+GEMM and D2H on three streams over two buffer sets",
            "gpu_launches_per_step": 5}


def run_skinny(args, name, w, rank, world, dist, torch, steps, headline=True):
    """Decode GEMM: bf16 activations with 0.1% outliers
    x50, pre-quantised NVFP4 weights N(0, 0.02); one step = one
    qg_gemm_nvfp4_skinny call (activation amax pass, quantiser, and the
    stream-K GEMM with its scale/convert epilogue: three launches, the last
    two with programmatic dependent launch).  Metric: algorithmic HBM bytes /
    step time."""
    from cuda_optimazation_b200 import qgemm as q
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
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
    # A decode step is ~30 us of GPU work, less than the host needs to issue
    # one call (tensor-map encodes, Python/ctypes), so each step is one
    # CUDA-graph replay of the public call, as a decode loop runs it.
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
    est_ms = timed(torch, stream, step, 4, dist) / 4
    if not headline:
        steps = max(steps, math.ceil(SUB_MIN_TIMED_S * 1e3 / max(est_ms, 1e-3)))
    with ClockSampler(dev.index) as clocks:
        for i in range(args.warmup):
            step(i)
        total_ms = timed(torch, stream, step, steps, dist)
    rc, code = q.read_status(status)
    if rc != q.OK:
        raise SystemExit(f"device status {code}")
    ms = total_ms / steps
    bytes_step = n * k * (0.5 + 1 / 16) + m * k * 2 + m * n * 2
    value = bytes_step * world * steps / (total_ms * 1e-3) / 1e9
    pk = peaks()
    rec = {
        "value": round(value, 1), "unit": "GB/s", "steps": steps, "ms_per_step": round(ms, 5),
        "dtype": "nvfp4", "config": workload_config(f"skinny_m{m}", w, world, rank),
        "tflops": round(2.0 * m * n * k / (ms * 1e-3) / 1e12, 2),
        "roofline": {"bound": "hbm", "achieved": round(bytes_step / (ms * 1e-3) / 1e9, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(bytes_step / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                     "traffic": profile_traffic(f"gemm_skinny_m{m}"),
                     "peak_basis": f"{pk['source']} STREAM copy GB/s; achieved counts the whole "
                                   "fused call (amax + quantiser + GEMM launches) as the unit",
                     "algorithmic_bytes_per_call": int(bytes_step),
                     # m in (32, 128] at this n runs on CTA pairs (the library's choice
                     # for decode shapes whose 512-row tiles nearly fill the SMs)
                     "kernel": ("gemm_skinny_pair_kernel" if m > 32 else "gemm_skinny_kernel")
                               + " (with skinny_amax_kernel and skinny_quant_kernel ahead of "
                                 "it in each call)"},
        "gpu_launches": 3 * steps,  # amax, quantiser, GEMM per call
        "clocks": clocks.summary(),
    }
    if not headline:
        return rec

    # End to end: every step copies its activations in from pinned host
    # memory and its result out to pinned host memory, on their own streams.
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
            s_in.wait_event(ev_call[b])
            dx[b].copy_(hx[b], non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])
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
    reps = max(4, min(steps, 50))
    e0.record(stream)
    s_in.wait_stream(stream)
    for i in range(reps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / reps
    rec["e2e"] = {"value": round(bytes_step / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                  "h2d_bytes_per_step": int(m * k * 2), "d2h_bytes_per_step": int(m * n * 2),
                  "ms_per_step": round(e2e_ms, 4),
                  "pipeline": "H2D, call and D2H on three streams over two buffer sets"}
    return rec


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


def cpu_block(w, threads):
    """The sample block both CPU legs time: NVFP4 quantise + dequantise of
    `qrows` rows (single-threaded, as the reference) and O2 over an
    orows x ocols output block (rows spread over the threads)."""
    return dict(qrows=min(w["m"], 256), orows=min(w["m"], 16 * threads), ocols=min(w["n"], 512))


class _CpuPath:
    """Cost model of the reference's CPU path, measured on bounded samples.

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
    blk = cpu_block(w, threads)
    res = [path.sample(**blk)]
    # Repeat the same block (new inputs) toward the time budget.
    while sum(r[1] for r in res) < budget_s * 0.8 and len(res) < 50:
        res.append(path.sample(**blk, seed_offset=len(res)))
    t_row = statistics.mean(r[2] for r in res)
    t_out = statistics.mean(r[3] for r in res)
    t_job = (m + n) * t_row + m * n * t_out
    flops = 2.0 * m * n * k
    # The same per-row and per-output costs carried to the other NVFP4
    # configs (both grow linearly in K): what the reference's CPU path would
    # take for each whole job on this host.
    per_config = {}
    for cname in ("nvfp4_256", "nvfp4_8192", "colpar", "skinny_m16", "skinny_m64", "skinny_m128"):
        cw = WORKLOADS[cname]
        f = cw["k"] / k
        tj = (cw["m"] + cw["n"]) * t_row * f + cw["m"] * cw["n"] * t_out * f
        per_config[cname] = {"job_seconds": round(tj, 3),
                             "tflops": round(2.0 * cw["m"] * cw["n"] * cw["k"] / tj / 1e12, 8)}
    return {"value": round(flops / t_job / 1e12, 8), "unit": "TFLOP/s", "cores": threads,
            "per_config_extrapolated": per_config,
            "kind": kind,
            "sample": (f"{'oracle/_ref (reference headers)' if ref else 'oracle port'}: "
                       f"{len(res)} samples of NVFP4 quantise+dequantise of {blk['qrows']} rows "
                       f"({t_row * 1e3:.2f} ms/row, one thread, as the reference) and O2 over a "
                       f"{blk['orows']}x{blk['ocols']} output block ({t_out * 1e6:.2f} us/output "
                       f"on {threads} threads); job time (M+N)*t_row + M*N*t_out = {t_job:.1f}s"),
            "job_seconds_extrapolated": round(t_job, 2)}


def cpu_check(chk: dict) -> dict:
    """The CPU checker on the headline GEMM (rank 0, N = 1): the tensor
    scales against amax/(448*6) (GEMMsm110/include/requant/nvfp4_reference.cuh:66-74),
    the quantised bytes of the sampled rows of A and B against O1's block
    rule under them (nvfp4_reference.cuh:84-111), and the GPU output on the
    sampled rows x sampled columns against O2
    (cutlass-gemm-cpp-guide/include/guide/block_scale_reference.hpp:10-37):
    relative Frobenius <= 1e-5 and per element
    |err| <= 1e-3 * ||oracle row over the sampled columns||_2, plus 2^-8
    (relative, per element and Frobenius) for bf16 output rounding."""
    import numpy as np
    o, _, _ = _cpu_impl()
    k, order = chk["k"], chk["layout_order"]
    out = {"rows": len(chk["rows"]), "cols": len(chk["cols"])}
    ok = True
    for tag, amax, ts in (("a", chk["amax_a"], chk["ts_a"]), ("b", chk["amax_b"], chk["ts_b"])):
        want = np.float32(amax) / np.float32(2688.0) if amax > 0 else np.float32(1.0)
        ok &= bool(np.float32(ts) == want)
    views = []
    for x, qrows, sf, rows, total, ts in (
            (chk["xa_rows"], chk["qa_rows"], chk["sfa"], chk["rows"], chk["m"], chk["ts_a"]),
            (chk["xb_rows"], chk["qb_rows"], chk["sfb"], chk["cols"], chk["n"], chk["ts_b"])):
        lq, lsf = o.nvfp4_with_ts(x, ts)
        qm, _ = o.linear_to_mma(lq, lsf, len(rows), k, 0)
        ok &= bool(np.array_equal(qrows.ravel(), qm))
        ok &= bool(np.array_equal(o.scale_rows(sf, rows, total, k, 16, order).ravel(), lsf))
        qfull = np.zeros((total, k // 2), np.uint8)
        qfull[rows] = qrows
        views.append(o.nvfp4_rows(qfull.ravel(), sf, rows, total, k, order))
    out["quantizer_bytes"] = "bit-exact" if ok else "MISMATCH"
    (av, asf), (bv, bsf) = views
    ref = o.gemm(av, bv, asf, bsf, len(chk["rows"]), len(chk["cols"]), k, 16,
                 threads=os.cpu_count() or 8)
    ref = (ref * np.float32(np.float32(chk["ts_a"]) * np.float32(chk["ts_b"]))).astype(np.float64)
    got = chk["c"].astype(np.float64)
    err = got - ref
    frob = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    bf16_rel = 2.0 ** -8 if chk["bf16"] else 0.0
    tol = 1e-3 * np.linalg.norm(ref, axis=1, keepdims=True) + bf16_rel * np.abs(ref)
    worst = float(np.max(np.abs(err) - tol))
    gemm_ok = bool(np.isfinite(got).all()) and frob <= 1e-5 + bf16_rel and worst <= 0.0
    out.update({"frob": frob, "worst_excess": worst,
                "gemm": "within tolerance" if gemm_ok else "OUT OF TOLERANCE"})
    out["status"] = "ok" if (ok and gemm_ok) else "FAIL"
    out["how"] = ("oracle O1 bytes of the sampled rows of A and B (rows s*131 % M, B rows = output "
                  "columns s*197 % N), O2 on the sampled block vs the GPU's bf16 output")
    return out


def run_reference_arm(args, name, w, rank, world):
    """Time the reference's own CPU implementation on the same sample block
    as the cpu_baseline leg (rank 0 only); each step is one sample."""
    if rank != 0:
        return None
    o, ref, kind = _cpu_impl()
    threads = os.cpu_count() or 1
    m, n, k = w["m"], w["n"], w["k"]
    path = _CpuPath(o, ref, w, threads)
    blk = cpu_block(w, threads)
    for i in range(min(args.warmup, 1)):
        path.sample(**blk, seed_offset=i + 1)
    res = [path.sample(**blk, seed_offset=i + 100) for i in range(args.steps)]
    t_job = statistics.mean(r[0] for r in res)
    t_step = statistics.mean(r[1] for r in res)
    value = 2.0 * m * n * k / t_job / 1e12
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 8), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t_step * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if name == "colpar" else "weak", "vs_baseline": None,
        "dtype": w["fmt"], "data": "synthetic (seeded std::mt19937_64 N(0,1))",
        "config": workload_config(name, w, world, rank),
        "cpu_baseline": {"value": round(value, 8), "unit": "TFLOP/s", "cores": threads,
                         "kind": kind,
                         "sample": f"per step: NVFP4 quantise+dequantise of {blk['qrows']} rows "
                                   f"(one thread, as the reference) and O2 over a "
                                   f"{blk['orows']}x{blk['ocols']} output block ({threads} "
                                   f"threads); job time (M+N)*t_row + M*N*t_out"},
        "e2e": {"value": round(value, 8), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="auto", choices=["auto", *WORKLOADS])
    ap.add_argument("--no-allgather", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    name = "colpar" if args.workload == "auto" else args.workload
    w = WORKLOADS[name]

    if args.impl == "reference":
        if w["fmt"] != "nvfp4" or w.get("skinny"):
            line = {"impl": "reference", "unavailable":
                    "the reference has no CPU path for this workload (MXFP8 / MXFP4 / decode GEMM)"}
        else:
            line = run_reference_arm(args, name, w, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import torch
    dist = None
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    if world > 1:
        import torch.distributed as td
        td.init_process_group("nccl", device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
        dist = td
    runner = run_skinny if w.get("skinny") else run_gemm
    rec = runner(args, name, w, rank, world, dist, torch, args.steps)
    check = rec.pop("_check", None)
    torch.cuda.empty_cache()
    subs = {}
    if world == 1 and not args.no_subrecords and name == "colpar":
        for sname in SUBRECORDS:
            sw = WORKLOADS[sname]
            fn = run_skinny if sw.get("skinny") else run_gemm
            subs[sname] = fn(args, sname, sw, rank, world, dist, torch, args.steps, headline=False)
            torch.cuda.empty_cache()
    if rank == 0:
        line = {"metric": METRIC, "value": rec.pop("value"), "unit": rec.pop("unit"),
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": rec.pop("ms_per_step"), "higher_is_better": True,
                "scaling": "strong" if name == "colpar" else "weak", "vs_baseline": None,
                "dtype": rec.pop("dtype"),
                "data": "synthetic (seeded torch.randn N(0,1); B N(0,0.02) for mxfp8), quantised "
                        "on the device before timing",
                "config": rec.pop("config")}
        line.update(rec)
        if subs:
            line["subrecords"] = subs
        if world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline(w, budget_s=args.cpu_budget)
            except ValueError as e:  # the reference's CPU path covers NVFP4 only
                line["cpu_baseline"] = {"unavailable": str(e)}
            if check is not None:
                line["parity"] = cpu_check(check)
        elif "allgather" in line:
            line["parity"] = line["allgather"].get("parity")
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
