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
           (pinned) buffers and device-resident weights: X is copied to the
           device and Y back every step
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
    """Per-launch DRAM bytes recorded from an ncu capture (profiles/<name>.txt,
    a line `traffic_bytes_per_launch: <int>`), or None."""
    path = ROOT / "profiles" / f"{name}.txt"
    try:
        for line in path.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip().replace(",", ""))
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    50 ms during the timed region. Read-only: no setting is changed."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, local: int):
        self.local = local
        self.samples: list[tuple[int, int, int]] = []
        self._stop = threading.Event()
        self.handle = None
        self.error = None

    def _open(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.local).uuid)
        for candidate in (uuid, "GPU-" + uuid):
            try:
                return pynvml, pynvml.nvmlDeviceGetHandleByUUID(candidate)
            except pynvml.NVMLError:
                continue
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.local)

    def _run(self, nvml):
        while not self._stop.is_set():
            try:
                sm = nvml.nvmlDeviceGetClockInfo(self.handle, nvml.NVML_CLOCK_SM)
                mx = nvml.nvmlDeviceGetMaxClockInfo(self.handle, nvml.NVML_CLOCK_SM)
                reasons = nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((sm, mx, reasons))
            except Exception as exc:  # noqa: BLE001
                self.error = str(exc)
                return
            self._stop.wait(0.05)

    def __enter__(self):
        try:
            nvml, self.handle = self._open()
            self.thread = threading.Thread(target=self._run, args=(nvml,), daemon=True)
            self.thread.start()
        except Exception as exc:  # noqa: BLE001
            self.error = str(exc)
            self.handle = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.handle is not None:
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": self.error}
        reasons = set()
        for _, _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples)}


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
        if elapsed >= budget_s or done >= 4096:
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
    layout = args.layout if args.layout != "auto" else ("canonical" if m == 1 else "tile32")
    args.layout = layout
    if layout == "tile32":
        # resident weights are repacked once into the tile32 layout (outside the timed region)
        codes_canonical = codes
        codes, status = cuda.repack_tile32(codes_canonical, N_ROWS, K_COLS, GROUP, status=status)
        cuda.check(status)

    def step():
        cuda.dense(x, codes, books, N_ROWS, GROUP, layout=layout, out=y, status=status)

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
        torch.cuda.nvtx.range_push("timed")
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
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
    kernel = "k_dense_t32" if layout == "tile32" else ("k_dense_pair" if m == 1 else "k_dense_lut")
    traffic_name = f"{kernel}_cfg2_m{m}"
    traffic = profile_traffic(traffic_name)
    result = {
        "metric": f"vq4 packed GEMV coded-weight GB/s (cfg2 W 11008x4096 g16, M={m}, grouped)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded N(0,0.02^2) weights, 16-value blocks L2-normalised; X ~ N(0,1))",
        "config": {"workload": f"cfg2-grouped-gemv-m{m}", "experts_per_gpu": experts, "M": m, "N": N_ROWS,
                   "K": K_COLS, "group": GROUP, "coded_bytes_per_gpu_step": coded,
                   "l2": "inputs larger than L2 (codes of all experts exceed 126 MB per launch)",
                   "weight_layout": layout,
                   "parallelism": f"expert-sharded x{world}, no collective"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak if peak else 6650.0, "unit": "GB/s",
                     "frac": round(achieved / (peak if peak else 6650.0), 4),
                     "traffic": traffic, "peak_source": "measured" if peak else "fallback",
                     "kernel": kernel, "algorithmic_bytes_per_launch": algorithmic},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    canonical = codes_canonical if layout == "tile32" else codes
    if rank == 0 and not args.no_e2e:
        result["e2e"] = run_cfg2_e2e(args, torch, vq, canonical, books, x, book, local)
    if rank == 0 and not args.no_cpu:
        sample = min(experts, 8)
        gbs, done, threads, elapsed = cpu_dense_sample(
            canonical[:sample].cpu().numpy().view(np.uint32), books[:sample].cpu().numpy(), x[:sample].cpu().numpy(),
            args.cpu_budget)
        result["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                                  "sample": f"{done} experts of the workload (decode + dot, float64 sums), "
                                            f"{elapsed:.1f} s"}
    return result


def run_cfg2_e2e(args, torch, vq, codes, books, x, book, local):
    """Through the public API with host buffers. The weights are made
    resident once (VQDevice.resident: uploaded and repacked on the device,
    outside the timed region); every step copies X from pinned host memory,
    runs the grouped product and copies Y back into pinned host memory
    (VQDevice.matmul_dense_grouped on the ResidentStack)."""
    from alelyon_compute_kit import ack
    experts, m = codes.shape[0], x.shape[1]
    host_codes = codes.cpu().numpy().view(np.uint32)
    host_books = books.cpu().numpy()
    pin_x = torch.empty(x.shape, dtype=torch.float32, pin_memory=True)
    pin_x.copy_(x)
    pin_y = torch.empty((experts, m, N_ROWS), dtype=torch.float32, pin_memory=True)
    stack = vq.VQStack((N_ROWS, K_COLS), GROUP, host_codes, host_books)
    xs, ys = pin_x.numpy(), pin_y.numpy()
    os.environ.setdefault("ACK_DEVICE", f"gpu:{local}")
    with ack.Device() as dev:
        backend = vq.VQDevice(dev)
        with backend.resident(stack, layout=args.layout) as weights:
            del stack, host_codes
            for _ in range(3):
                backend.matmul_dense_grouped(xs, weights, out=ys)
            steps = max(5, args.steps)
            t0 = time.perf_counter()
            for _ in range(steps):
                backend.matmul_dense_grouped(xs, weights, out=ys)
            elapsed = (time.perf_counter() - t0) / steps
    h2d = xs.nbytes + 4          # X and the cleared status word
    d2h = ys.nbytes + 4          # Y and the status word
    return {"value": round(experts * (CODE_BYTES + BOOK_BYTES) / elapsed / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(elapsed * 1e3, 3),
            "api": "VQDevice.matmul_dense_grouped on a ResidentStack (C ABI ack_vq2; weights resident, "
                   "X in and Y out through pinned host memory every step)"}


def _timed(torch, fn, steps, warmup, world, device, local, label="timed"):
    """CUDA-event time of `steps` calls after `warmup`, max over ranks (ms/step).
    The timed calls run inside the NVTX range `label`."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push(label)
        start.record()
        for _ in range(steps):
            fn()
        stop.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = start.elapsed_time(stop)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms / steps, clocks.summary()


def _fit_from_device(vq, torch, values, group, sample_vectors=65536):
    """fit_codebook on the CPU from the strided sample of a device tensor
    (the sample is what fit_codebook would draw from the whole tensor)."""
    complete = values.numel() // group
    pos = np.linspace(0, complete - 1, min(complete, sample_vectors), dtype=np.int64)
    sample = values[: complete * group].view(complete, group)[torch.from_numpy(pos).to(values.device)]
    return vq.fit_codebook(sample.cpu().numpy().reshape(-1), group=group, sample_vectors=sample_vectors)


def run_codec(args, world, rank, local, which):
    """cfg 5: encode or decode of 2^30 FP32 values (args.dist: gauss or heavy)."""
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    group, n = args.group, args.values
    gen = torch.Generator(device=device)
    gen.manual_seed(10 + rank)
    if args.dist == "heavy":
        atoms = torch.from_numpy(np.random.default_rng(10).standard_normal((16, group)).astype(np.float32)).to(device)
        idx = torch.zeros(n // group, dtype=torch.int64, device=device)
        rare = int(round(idx.numel() * 0.15))
        idx[:rare] = 1 + torch.arange(rare, device=device) % 15
        idx = idx[torch.randperm(idx.numel(), generator=gen, device=device)]
        x = atoms[idx].reshape(-1)
        del idx
    else:
        x = torch.randn(n, generator=gen, device=device)
        blocks = x.view(-1, group)
        blocks /= blocks.norm(dim=1, keepdim=True)
    book = torch.from_numpy(_fit_from_device(vq, torch, x, group)).to(device)
    codes, status = cuda.encode(x, book, group)
    cuda.check(status)
    if which == "encode":
        fn = lambda: cuda.encode(x, book, group, out=codes, status=status)  # noqa: E731
    else:
        fn = lambda: cuda.decode(codes, book, n, group, out=x, status=status)  # noqa: E731
    ms, clocks = _timed(torch, fn, args.steps, args.warmup, world, device, local)
    cuda.check(status)
    code_bytes = codes.numel() * 4
    algorithmic = 4 * n + code_bytes + 64 * group
    peak = measured_peaks().get("hbm_gbs") or 6650.0
    achieved = algorithmic / (ms / 1e3) / 1e9
    # x from torch is 16-byte aligned: encode runs the tensor-core kernel
    kernel = "k_encode_tc" if which == "encode" else "k_decode"
    result = {
        "metric": f"vq4 {which} Gvalues/s (cfg5, 2^30 values, g{group}, {args.dist})",
        "value": round(world * n / (ms / 1e3) / 1e9, 3), "unit": "Gvalues/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": f"synthetic ({args.dist})",
        "config": {"workload": f"cfg5-{which}-g{group}-{args.dist}", "values_per_gpu": n, "group": group,
                   "l2": "inputs larger than L2", "parallelism": f"range-sharded x{world}, no collective"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": profile_traffic(f"{kernel}_cfg5_g{group}"),
                     "kernel": kernel, "algorithmic_bytes_per_launch": algorithmic},
        # encode: the book-staging kernel and the encode kernel per step
        "gpu_launches": args.steps * (2 if which == "encode" else 1), "clocks": clocks,
    }
    if rank == 0 and not args.no_cpu:
        sys.path.insert(0, str(ROOT / "oracle"))
        import vq_oracle_c as oc
        m = 1 << 24
        xs, cb, bk = x[:m].cpu().numpy(), codes[: m // group // 8].cpu().numpy().view(np.uint32), book.cpu().numpy()
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < args.cpu_budget:
            if which == "encode":
                oc.encode(xs, bk, group)
            else:
                oc.decode(cb, bk, m, group)
            reps += 1
        el = time.perf_counter() - t0
        result["cpu_baseline"] = {"value": round(reps * m / el / 1e9, 4), "unit": "Gvalues/s", "cores": oc.threads(),
                                  "kind": "port", "sample": f"{reps} x 2^24 values, {el:.1f} s"}
    return result


def run_cfg3(args, world, rank, local):
    """cfg 3: both operands coded, X 4096 x 4096 (g32, own book) times
    W 14336 x 4096 (g32) transposed; the 16x16 codebook inner-product table."""
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    m, n, k, group = 4096, 14336, 4096, 32
    gen = torch.Generator(device=device)
    gen.manual_seed(8)
    x = torch.randn(m * k, generator=gen, device=device)
    gen.manual_seed(7)
    w = torch.randn(n * k, generator=gen, device=device) * 0.02
    xb = torch.from_numpy(_fit_from_device(vq, torch, x, group, 4096)).to(device)
    wb = torch.from_numpy(_fit_from_device(vq, torch, w, group, 4096)).to(device)
    xc, status = cuda.encode(x, xb, group)
    wc, _ = cuda.encode(w, wb, group, status=status)
    cuda.check(status)
    del x, w
    y = torch.empty((m, n), dtype=torch.float32, device=device)
    fn = lambda: cuda.coded(xc, xb, wc, wb, m, n, k, group, flags=2, out=y, status=status)  # noqa: E731
    ms, clocks = _timed(torch, fn, args.steps, args.warmup, world, device, local)
    cuda.check(status)
    flops = 2.0 * m * n * k
    lookups = m * n * (k // group)
    byts = xc.numel() * 4 + wc.numel() * 4 + 2 * 64 * group + 4 * m * n
    peak = measured_peaks().get("hbm_gbs") or 6650.0
    return {
        "metric": "vq4 both-coded GEMM effective TFLOP/s (cfg3, 4096x4096 . (14336x4096)^T, g32)",
        "value": round(world * flops / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg3-coded-gemm", "M": m, "N": n, "K": k, "group": group,
                   "lut_lookups_per_s": lookups / (ms / 1e3), "parallelism": f"replicated x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(byts / (ms / 1e3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(byts / (ms / 1e3) / 1e9 / peak, 4), "traffic": None, "kernel": "k_coded_lut",
                     "note": "the table lookups on the shared-memory pipe bound this kernel, not HBM"},
        "gpu_launches": args.steps, "clocks": clocks,
    }


def run_cfg4(args, world, rank, local):
    """cfg 4: the VQAdamW step of 8 experts per GPU, each W, M, V of
    4096 x 1024 g8 with a coded gradient: the AdamW values of the
    calibration sample (op 18), fit_codebook of W', M', V' on the device
    (op 24, bit for bit the CPU fit), then decode -> AdamW -> encode of all
    three states (op 20). The whole step is device-timed; the encode pass
    alone is reported beside it."""
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    experts, rows, cols, group = args.experts_cfg4, 4096, 1024, 8
    count = rows * cols
    words = cuda.words_for(count, group)
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    codes = torch.empty((experts, 4, words), dtype=torch.int32, device=device)
    books = torch.empty((experts, 4, 16, group), dtype=torch.float32, device=device)
    status = cuda.status_word(device)
    scales = (0.02, 1e-4, 1e-7, 1e-3)
    for e in range(experts):
        for s, scale in enumerate(scales):
            v = torch.randn(count, generator=gen, device=device) * scale
            if s == 2:
                v = v.abs()
            b = torch.from_numpy(_fit_from_device(vq, torch, v, group, 4096)).to(device)
            books[e, s] = b
            cuda.encode(v, b, group, out=codes[e, s], status=status)
    coefs = torch.from_numpy(np.tile(np.array([1e-3, 0.9, 0.999, 1e-8, 0.01, 1 - 0.9 ** 2, 1 - 0.999 ** 2],
                                              np.float32), (experts, 1))).to(device)
    positions = torch.from_numpy(np.linspace(0, count // group - 1, 4096, dtype=np.int64).astype(np.uint32)
                                 .view(np.int32)).to(device)
    samples = torch.empty((experts, 3, 4096, group), dtype=torch.float32, device=device)
    new_books = torch.empty((experts, 3, 16, group), dtype=torch.float32, device=device)
    workspace = torch.empty(experts * 3 * cuda.fit_workspace_bytes(4096), dtype=torch.uint8, device=device)
    out = torch.empty((experts, 3, words), dtype=torch.int32, device=device)
    changed = torch.empty(experts, dtype=torch.int32, device=device)

    def step():
        cuda.adamw_sample(codes, books, coefs, positions, count, group, batch=experts, out=samples, status=status)
        cuda.adamw_fit(codes, books, coefs, samples, count, group, iterations=4, batch=experts, out=new_books,
                       workspace=workspace, status=status)
        cuda.adamw_encode(codes, books, coefs, new_books, count, group, batch=experts, out=out, changed=changed,
                          status=status)

    encode_pass = lambda: cuda.adamw_encode(codes, books, coefs, new_books, count, group,  # noqa: E731
                                            batch=experts, out=out, changed=changed, status=status)
    ms, clocks = _timed(torch, step, args.steps, args.warmup, world, device, local)
    cuda.check(status)
    ms_encode, _ = _timed(torch, encode_pass, args.steps, args.warmup, world, device, local, label="encode-pass")
    cuda.check(status)
    byts = codes.numel() * 4 + out.numel() * 4
    peak = measured_peaks().get("hbm_gbs") or 6650.0
    result = {
        "metric": "vq4 VQAdamW step Gvalues/s (cfg4, 3 x 4096x1024 g8 per expert: sample, device fit, re-encode)",
        "value": round(world * experts * count / (ms / 1e3) / 1e9, 3), "unit": "Gvalues/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg4-vqadamw-step", "experts_per_gpu": experts, "rows": rows, "cols": cols,
                   "group": group, "sample_vectors": 4096, "fit_iterations": 4, "fit": "device",
                   "parallelism": f"expert-sharded x{world}, no collective"},
        "encode_pass": {"ms": round(ms_encode, 4),
                        "gvalues_per_s": round(world * experts * count / (ms_encode / 1e3) / 1e9, 3)},
        "roofline": {"bound": "hbm", "achieved": round(byts / (ms_encode / 1e3) / 1e9, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(byts / (ms_encode / 1e3) / 1e9 / peak, 4), "traffic": None,
                     "kernel": "k_adamw_encode",
                     "note": "compute-bound (three certified 16-entry searches per value); coded bytes only"},
        # per step: sample 1, fit 1 + 4 x 3, encode pass 2 per expert (book staging + pass)
        "gpu_launches": args.steps * (1 + 13 + 2 * experts), "clocks": clocks,
    }
    if rank == 0 and not args.no_e2e:
        result["e2e"] = run_cfg4_e2e(args, torch, vq, codes, books, experts, count, group, local)
    return result


def run_cfg4_e2e(args, torch, vq, codes, books, experts, count, group, local):
    """VQAdamW.step through the public API with host VQArrays (every step
    uploads W, M, V, G and downloads W', M', V'): fit on the device, and one
    step with the CPU fit beside it."""
    from alelyon_compute_kit import ack
    host_codes = codes.cpu().numpy().view(np.uint32)
    host_books = books.cpu().numpy()
    shape = (4096, 1024)
    arrays = [[vq.VQArray(shape, group, host_codes[e, s], host_books[e, s]) for s in range(4)] for e in range(experts)]
    os.environ.setdefault("ACK_DEVICE", f"gpu:{local}")
    timings = {}
    with ack.Device() as dev:
        backend = vq.VQDevice(dev)
        for fit, steps in (("device", max(3, min(args.steps, 5))), ("host", 1)):
            opts = []
            for e in range(experts):
                opt = vq.VQAdamW(backend, arrays[e][0], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                                 fit=fit)
                opt.momentum, opt.variance, opt.steps = arrays[e][1], arrays[e][2], 1
                opts.append(opt)
            if fit == "device":
                for e in range(experts):
                    opts[e].step(arrays[e][3])
            t0 = time.perf_counter()
            for _ in range(steps):
                for e in range(experts):
                    opts[e].step(arrays[e][3])
            timings[fit] = (time.perf_counter() - t0) / steps
    h2d = experts * 4 * (host_codes[0, 0].nbytes + host_books[0, 0].nbytes)
    d2h = experts * 3 * (host_codes[0, 0].nbytes + host_books[0, 0].nbytes)
    return {"value": round(experts * count / timings["device"] / 1e9, 4), "unit": "Gvalues/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(timings["device"] * 1e3, 2),
            "api": "VQAdamW.step (fit='device') per expert, host VQArrays",
            "host_fit_ms_per_step": round(timings["host"] * 1e3, 1)}


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
    ap.add_argument("--group", type=int, default=16)
    ap.add_argument("--layout", choices=("auto", "tile32", "canonical"), default="auto",
                    help="auto: canonical for M = 1 (the byte-table kernel), tile32 otherwise")
    ap.add_argument("--values", type=int, default=1 << 30)
    ap.add_argument("--dist", choices=("gauss", "heavy"), default="gauss")
    ap.add_argument("--experts-cfg4", type=int, default=8)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        result = run_reference(args, world, rank)
    elif args.workload == "cfg2":
        result = run_cfg2(args, world, rank, local)
    elif args.workload in ("encode", "decode"):
        result = run_codec(args, world, rank, local, args.workload)
    elif args.workload == "cfg3":
        result = run_cfg3(args, world, rank, local)
    elif args.workload == "cfg4":
        result = run_cfg4(args, world, rank, local)
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
