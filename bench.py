"""Benchmark of the vq4 hot path on B200 (one JSON line on rank 0).

Default workload (the metric's configuration): packed
GEMV with coded weights, W = 11008 x 4096 FP32 N(0, 0.02^2) with every
16-value block L2-normalised, group 16, FP32 activations X of 1 x 4096 from
N(0, 1). To exercise HBM rather than L2 or launch latency, one step is one
grouped launch over E distinct coded matrices per GPU (E = 768: 1.08 GB of
codes per launch, far above the 126 MB L2, so no flush is needed). The
headline metric is coded-weight GB/s = (code bytes + codebook bytes) / time.

  value    device time of the grouped launch, inputs resident in HBM
  e2e      the same metric through VQDevice.matmul_dense_grouped with host
           (pinned) buffers: the inputs are copied to the device and Y back
           every step
  roofline the k_dense_lut launch against the measured HBM copy bandwidth
  cpu_baseline / --impl reference
           the CPU restatement (decode + dot product, all host threads) on a
           bounded sample of the same experts

Other workloads (`--workload`): cfg2-m4/m16/m64 (same, M rows), cfg3 (both
operands coded, 4096 x 4096 times 14336 x 4096, g32), cfg4 (fused VQAdamW,
8 experts of 3 x 4096 x 1024 g8 per GPU), encode / decode (2^30 values).

Multi-GPU (torchrun): every rank runs its own E experts (expert sharding,
no collective, weak scaling); the reported time is the max over ranks.
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

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "alelyon-compute-kit_b200"))

N_ROWS, K_COLS, GROUP = 11008, 4096, 16
CODE_BYTES = N_ROWS * K_COLS // GROUP // 2     # 1,409,024
BOOK_BYTES = 16 * GROUP * 4                    # 1,024


def measured_peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def profile_traffic(name: str):
    """Per-launch DRAM bytes recorded from an ncu capture (profiles/<name>.md,
    a line `traffic_bytes_per_launch: <int>`), or None."""
    path = ROOT / "profiles" / f"{name}.md"
    try:
        for line in path.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip().replace(",", ""))
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock and throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower() in ("active", "1", "yes"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        backend = "nccl" if args.impl == "ours" else "gloo"
        if backend == "nccl":
            import torch
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    return world, rank, local


# ------------------------------------------------------------------ workload --

def make_cfg2(torch, cuda, vq, experts: int, m: int, device):
    """E distinct coded 11008 x 4096 g16 matrices in HBM, built on the device:
    each W_e ~ N(0, 0.02^2) with 16-value blocks L2-normalised, encoded with
    one codebook fitted on the CPU from a sample of W_0; X_e ~ N(0, 1)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    w0 = torch.randn(N_ROWS * K_COLS, generator=gen, device=device) * 0.02
    blocks = w0.view(-1, GROUP)
    blocks /= blocks.norm(dim=1, keepdim=True)
    book = vq.fit_codebook(w0.view(N_ROWS, K_COLS).cpu().numpy(), group=GROUP)
    tbook = torch.from_numpy(book).to(device)
    words = CODE_BYTES // 4
    codes = torch.empty((experts, words), dtype=torch.int32, device=device)
    books = tbook.unsqueeze(0).repeat(experts, 1, 1).contiguous()
    status = cuda.status_word(device)
    for e in range(experts):
        if e:
            gen.manual_seed(7 + e)
            torch.randn(N_ROWS * K_COLS, generator=gen, device=device, out=w0)
            w0.mul_(0.02)
            blocks /= blocks.norm(dim=1, keepdim=True)
        cuda.encode(w0, tbook, GROUP, out=codes[e], status=status)
    cuda.check(status)
    del w0, blocks
    gen.manual_seed(8)
    x = torch.randn((experts, m, K_COLS), generator=gen, device=device)
    return codes, books, x, book


def bytes_per_expert(m: int) -> int:
    return CODE_BYTES + BOOK_BYTES + 4 * m * K_COLS + 4 * m * N_ROWS


def cpu_dense_sample(codes_np, books_np, x_np, budget_s: float):
    """C oracle (decode + dot, all host threads) over experts until the
    budget is spent; returns (coded GB/s, experts timed, threads)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vq_oracle_c as oc
    oc.lib()
    done, t0 = 0, time.perf_counter()
    while True:
        e = done % len(codes_np)
        oc.dense_nt(x_np[e], codes_np[e], books_np[e], N_ROWS, GROUP)
        done += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= budget_s or done >= 64:
            break
    return done * (CODE_BYTES + BOOK_BYTES) / elapsed / 1e9, done, oc.threads(), elapsed


def run_cfg2(args, world, rank, local):
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    m = args.m
    experts = args.experts
    codes, books, x, book = make_cfg2(torch, cuda, vq, experts, m, device)
    y = torch.empty((experts, m, N_ROWS), dtype=torch.float32, device=device)
    status = cuda.status_word(device)

    def step():
        cuda.dense(x, codes, books, N_ROWS, GROUP, out=y, status=status)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    cuda.check(status)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    cuda.check(status)
    ms_step = ms / args.steps
    coded = experts * (CODE_BYTES + BOOK_BYTES)
    value = world * coded / (ms_step / 1e3) / 1e9
    algorithmic = experts * bytes_per_expert(m)
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    achieved = algorithmic / (ms_step / 1e3) / 1e9
    traffic_name = f"dense_lut_cfg2_m{m}"
    traffic = profile_traffic(traffic_name)
    result = {
        "metric": f"vq4 packed GEMV coded-weight GB/s (cfg2 W 11008x4096 g16, M={m}, grouped)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded N(0,0.02^2) weights, 16-value blocks L2-normalised; X ~ N(0,1))",
        "config": {"workload": f"cfg2-grouped-gemv-m{m}", "experts_per_gpu": experts, "M": m, "N": N_ROWS,
                   "K": K_COLS, "group": GROUP, "coded_bytes_per_gpu_step": coded,
                   "l2": "inputs larger than L2 (codes of all experts exceed 126 MB per launch)",
                   "parallelism": f"expert-sharded x{world}, no collective"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak if peak else 6650.0, "unit": "GB/s",
                     "frac": round(achieved / (peak if peak else 6650.0), 4),
                     "traffic": traffic, "peak_source": "measured" if peak else "fallback",
                     "kernel": "k_dense_lut", "algorithmic_bytes_per_launch": algorithmic},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and not args.no_e2e:
        result["e2e"] = run_cfg2_e2e(args, torch, vq, codes, books, x, book, local)
    if rank == 0 and not args.no_cpu:
        sample = min(experts, 8)
        gbs, done, threads, elapsed = cpu_dense_sample(
            codes[:sample].cpu().numpy().view(np.uint32), books[:sample].cpu().numpy(), x[:sample].cpu().numpy(),
            args.cpu_budget)
        result["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                                  "sample": f"{done} experts of the workload (decode + dot, float64 sums), "
                                            f"{elapsed:.1f} s"}
    return result


def run_cfg2_e2e(args, torch, vq, codes, books, x, book, local):
    """Through the public API with host buffers: VQDevice.matmul_dense_grouped
    uploads X, codes and books and downloads Y every step."""
    from alelyon_compute_kit import ack
    experts, m = codes.shape[0], x.shape[1]
    pin_codes = torch.empty(codes.shape, dtype=torch.int32, pin_memory=True)
    pin_codes.copy_(codes)
    pin_books = torch.empty(books.shape, dtype=torch.float32, pin_memory=True)
    pin_books.copy_(books)
    pin_x = torch.empty(x.shape, dtype=torch.float32, pin_memory=True)
    pin_x.copy_(x)
    stack = vq.VQStack((N_ROWS, K_COLS), GROUP, pin_codes.numpy().view(np.uint32), pin_books.numpy())
    xs = pin_x.numpy()
    os.environ.setdefault("ACK_DEVICE", f"gpu:{local}")
    with ack.Device() as dev:
        backend = vq.VQDevice(dev)
        for _ in range(2):
            backend.matmul_dense_grouped(xs, stack)
        steps = max(3, min(args.steps, 10))
        t0 = time.perf_counter()
        for _ in range(steps):
            yv = backend.matmul_dense_grouped(xs, stack)
        elapsed = (time.perf_counter() - t0) / steps
    h2d = pin_codes.numel() * 4 + pin_books.numel() * 4 + pin_x.numel() * 4 + 4
    d2h = yv.nbytes + 4
    return {"value": round(experts * (CODE_BYTES + BOOK_BYTES) / elapsed / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(elapsed * 1e3, 3),
            "api": "VQDevice.matmul_dense_grouped (C ABI ack_vq2, host buffers)"}


def run_reference(args, world, rank):
    """The reference arm: the CPU restatement of the path (decode + dot
    product with all host threads) on a bounded sample of the workload."""
    if rank != 0:
        return None
    sys.path.insert(0, str(ROOT / "oracle"))
    import vq_oracle as o
    import vq_oracle_c as oc
    from alelyon_compute_kit import vq
    m = args.m
    rng = np.random.default_rng(7)
    sample = 2
    w = o.block_normalised(o.gaussian((N_ROWS, K_COLS), 0.02, 7), GROUP)
    book = vq.fit_codebook(w, group=GROUP)
    codes = [oc.encode(w, book, GROUP)]
    for e in range(1, sample):
        perm = rng.permutation(codes[0].size)
        codes.append(codes[0][perm])
    x = rng.standard_normal((sample, m, K_COLS)).astype(np.float32)
    per_step = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for e in range(sample):
            oc.dense_nt(x[e], codes[e], book, N_ROWS, GROUP)
        if i >= args.warmup:
            per_step.append(time.perf_counter() - t0)
    t = sum(per_step) / len(per_step)
    value = sample * (CODE_BYTES + BOOK_BYTES) / t / 1e9
    return {"impl": "reference", "metric": f"vq4 packed GEMV coded-weight GB/s (cfg2 W 11008x4096 g16, M={m}, grouped)",
            "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"cfg2-grouped-gemv-m{m}", "M": m, "N": N_ROWS, "K": K_COLS, "group": GROUP,
                       "sample_experts_per_step": sample},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": oc.threads(), "kind": "port",
                             "sample": f"{sample} experts per step (decode + dot, float64 sums)"},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="cfg2")
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--experts", type=int, default=768)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        result = run_reference(args, world, rank)
    elif args.workload == "cfg2":
        result = run_cfg2(args, world, rank, local)
    else:
        raise SystemExit(f"unknown workload {args.workload!r}")
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
