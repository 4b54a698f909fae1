"""Benchmark of the vq4 hot path on B200 (one JSON line on rank 0).

Default workload (cfg2, the configuration the headline metric is quoted on): packed
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
  roofline the k_dense_pair launch against the measured HBM copy bandwidth
  cpu_baseline / --impl reference
           the CPU restatement (decode + dot product, all host threads) on a
           bounded sample of the same experts

Other workloads: cfg2 at M rows (`--m 4/16/64`), and `--workload` cfg3 (both
operands coded, 4096 x 4096 times 14336 x 4096, g32), cfg4 (fused VQAdamW,
8 experts of 3 x 4096 x 1024 g8 per GPU), encode / decode (2^30 values,
`--group`, `--dist`), nf4 (the NF4 comparator's GEMV on the cfg2 shape) and
profile (small cases of every kernel, for ncu captures; no timing). The
default run carries all of them in the line's `secondary` object.

Multi-GPU (torchrun): every rank runs its own E experts (expert sharding,
no collective, weak scaling); the reported time is the max over ranks. The
line's `sharded` object adds the row splits of cfg2 and cfg3 across ranks
(strong scaling) without and with the NCCL all-gather of the output, cfg2
with the GEMV storing its outputs into every rank's buffer over NVLink (CUDA
IPC peer stores) instead of the all-gather, and the cfg4 VQAdamW step at 8
experts per GPU.
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
    2 ms during the timed region (a few samples even for a region of a few
    milliseconds). Read-only: no setting is changed."""

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

    def _sample(self, nvml) -> bool:
        try:
            sm = nvml.nvmlDeviceGetClockInfo(self.handle, nvml.NVML_CLOCK_SM)
            mx = nvml.nvmlDeviceGetMaxClockInfo(self.handle, nvml.NVML_CLOCK_SM)
            reasons = nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
            self.samples.append((sm, mx, reasons))
            return True
        except Exception as exc:  # noqa: BLE001
            self.error = str(exc)
            return False

    def _run(self, nvml):
        while not self._stop.is_set() and self._sample(nvml):
            self._stop.wait(0.002)

    def __enter__(self):
        try:
            nvml, self.handle = self._open()
            self._sample(nvml)  # one sample as the region starts, then every 2 ms
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

def make_cfg2(torch, cuda, vq, experts: int, device):
    """E distinct coded 11008 x 4096 g16 matrices in HBM, built on the device:
    each W_e ~ N(0, 0.02^2) with 16-value blocks L2-normalised, encoded with
    one codebook fitted on the CPU from a sample of W_0."""
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
    return codes, books, book


def make_cfg2_x(torch, experts: int, m: int, device):
    """X_e ~ N(0, 1), (E, M, 4096)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(8)
    return torch.randn((experts, m, K_COLS), generator=gen, device=device)


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


def roofline(bound: str, achieved: float, kernel: str, algorithmic, traffic_name: str | None, **extra) -> dict:
    """The roofline object of one workload against the measured peak of its
    bound ("hbm": GB/s copy bandwidth; "tensor": cuBLAS bf16 TFLOP/s)."""
    peaks = measured_peaks()
    if bound == "hbm":
        peak, unit = peaks.get("hbm_gbs"), "GB/s"
        fallback = 6650.0
    else:
        peak, unit = peaks.get("bf16_tflops"), "TFLOP/s"
        fallback = 1590.0
    out = {"bound": bound, "achieved": round(achieved, 2), "peak": peak or fallback, "unit": unit,
           "frac": round(achieved / (peak or fallback), 4),
           "traffic": profile_traffic(traffic_name) if traffic_name else None,
           "peak_source": "measured" if peak else "fallback", "kernel": kernel,
           "algorithmic_per_launch": algorithmic}
    out.update(extra)
    return out


def time_cfg2(args, torch, cuda, codes, books, m, device, world, local, engine="auto", layout="auto"):
    """Device time of the grouped product for M activation rows over the
    resident experts (one launch per step; inputs exceed L2)."""
    experts = codes.shape[0]
    x = make_cfg2_x(torch, experts, m, device)
    y = torch.empty((experts, m, N_ROWS), dtype=torch.float32, device=device)
    status = cuda.status_word(device)
    engine = engine if engine != "auto" else cuda.dense_engine(m, K_COLS, GROUP)
    layout = layout if layout != "auto" else ("canonical" if m == 1 or engine == "tensor" else "tile32")
    if layout != "canonical":
        engine = "lut"
    run_codes = codes
    if layout == "tile32":
        # resident weights are repacked once into the tile32 layout (outside the timed region)
        run_codes, _ = cuda.repack_tile32(codes, N_ROWS, K_COLS, GROUP, status=status)
        cuda.check(status)
    workspace = (torch.empty(cuda.dense_tc_workspace_bytes(m, K_COLS, GROUP, experts), dtype=torch.uint8,
                             device=device) if engine == "tensor" else None)

    def step():
        cuda.dense(x, run_codes, books, N_ROWS, GROUP, layout=layout, out=y, status=status, engine=engine,
                   workspace=workspace)

    ms, clocks = _timed(torch, step, args.steps, args.warmup, world, device, local)
    cuda.check(status)
    coded = experts * (CODE_BYTES + BOOK_BYTES)
    kernel = ("k_dense_tc" if engine == "tensor" else
              "k_dense_t32" if layout == "tile32" else ("k_dense_pair" if m == 1 else "k_dense_lut"))
    algorithmic = experts * bytes_per_expert(m)
    flops = 2.0 * experts * m * N_ROWS * K_COLS
    achieved_hbm = algorithmic / (ms / 1e3) / 1e9
    if engine == "tensor":
        # the MMA runs 128 P rows (64 rows of X, bf16 hi and lo) per 64-row tile of X, each
        # 16 K / G long, against every W row
        mma_tflops = 2.0 * experts * 128 * ((m + 63) // 64) * N_ROWS * (16 * K_COLS // GROUP)
        mma_tflops /= (ms / 1e3) * 1e12
        roof = roofline("tensor", mma_tflops, kernel, flops, f"{kernel}_cfg2_m{m}",
                        hbm_gbs=round(achieved_hbm, 1), dense_equivalent_tflops=round(flops / (ms / 1e3) / 1e12, 2),
                        note="MMA TFLOP/s of the one-hot bf16 GEMM (hi and lo halves) against the cuBLAS bf16 peak")
    else:
        roof = roofline("hbm", achieved_hbm, kernel, algorithmic, f"{kernel}_cfg2_m{m}")
    del x, y, workspace
    if run_codes is not codes:
        del run_codes
    return {"ms": ms, "value": world * coded / (ms / 1e3) / 1e9, "coded": coded, "engine": engine,
            "layout": layout, "kernel": kernel, "roofline": roof, "clocks": clocks,
            "tflops_dense_equivalent": flops / (ms / 1e3) / 1e12}


def compact(result: dict) -> dict:
    """A secondary workload's entry: its metric, value, device time per
    step, roofline and clock record."""
    keep = ("metric", "value", "unit", "ms_per_step", "roofline", "clocks", "config")
    return {k: result[k] for k in keep if k in result}


def run_cfg2(args, world, rank, local):
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    m = args.m
    experts = args.experts
    codes, books, book = make_cfg2(torch, cuda, vq, experts, device)
    rec = time_cfg2(args, torch, cuda, codes, books, m, device, world, local, args.engine, args.layout)
    ms_step = rec["ms"]
    args.layout = rec["layout"]
    result = {
        "metric": f"vq4 packed GEMV coded-weight GB/s (cfg2 W 11008x4096 g16, M={m}, grouped)",
        "value": round(rec["value"], 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02^2) weights, 16-value blocks L2-normalised; X ~ N(0,1))",
        "config": {"workload": f"cfg2-grouped-gemv-m{m}", "experts_per_gpu": experts, "M": m, "N": N_ROWS,
                   "K": K_COLS, "group": GROUP, "coded_bytes_per_gpu_step": rec["coded"],
                   "l2": "inputs larger than L2 (codes of all experts exceed 126 MB per launch)",
                   "weight_layout": rec["layout"], "engine": rec["engine"],
                   "parallelism": f"expert-sharded x{world}, no collective"},
        "roofline": rec["roofline"],
        "gpu_launches": args.steps * (2 if rec["engine"] == "tensor" else 1),
        "clocks": rec["clocks"],
    }
    x = make_cfg2_x(torch, experts, m, device)
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
    del x
    if world == 1 and not args.no_secondary:
        result["secondary"] = run_secondary(args, torch, cuda, codes, books, device, world, rank, local)
    if world > 1 and not args.no_secondary:
        result["sharded"] = run_sharded(args, torch, cuda, codes, books, device, world, rank, local)
    return result


def run_sharded(args, torch, cuda, codes, books, device, world, rank, local) -> dict:
    """The partitions of the path across ranks (N > 1), beside the weak-scaling
    headline:

    * cfg2 split by W rows (output columns of Y): every rank holds rows
      [r0, r1) of each of the same E experts, X is replicated; strong
      scaling (the whole job is the E full products). Timed without and with
      the NCCL all-gather of the Y shards, which lands in place in a
      rank-major (world, E, M, rows) buffer.
    * cfg3 split the same way (rows of the coded W, columns of C), timed
      without and with the all-gather of C's column shards.
    * cfg4: the VQAdamW step of 8 experts per GPU (64 at 8 GPUs), experts
      split across ranks, no collective."""
    import copy

    import torch.distributed as dist

    from alelyon_compute_kit import parallel
    experts, m = codes.shape[0], 1
    ranges = parallel.row_ranges(N_ROWS, K_COLS, GROUP, world)
    r0, r1 = ranges[rank]
    width = max(b - a for a, b in ranges)
    row_words = K_COLS // GROUP // 8
    shard = codes.view(experts, N_ROWS, row_words)[:, r0:r1].contiguous().view(experts, -1)
    x = make_cfg2_x(torch, experts, m, device)
    y = torch.zeros((experts, m, r1 - r0), dtype=torch.float32, device=device)
    send = y if r1 - r0 == width else torch.zeros((experts, m, width), dtype=torch.float32, device=device)
    gathered = torch.empty((world, experts, m, width), dtype=torch.float32, device=device)
    status = cuda.status_word(device)

    def compute():
        cuda.dense(x, shard, books, r1 - r0, GROUP, out=y, status=status)

    def compute_gather():
        compute()
        if send is not y:  # a narrower last shard is padded to the common width
            send[..., : r1 - r0] = y
        dist.all_gather_into_tensor(gathered.view(-1), send.view(-1))

    ms_c, clocks = _timed(torch, compute, args.steps, args.warmup, world, device, local, label="sharded")
    ms_g, _ = _timed(torch, compute_gather, args.steps, args.warmup, world, device, local, label="sharded-gather")
    cuda.check(status)
    # the same gathered result by peer stores from the GEMV itself (equal shards only)
    ms_p, peer_error = None, None
    if r1 - r0 == width:
        try:
            slots = parallel.PeerSlots(experts, width)   # all ranks raise together if any cannot map
        except Exception as exc:  # noqa: BLE001
            slots, peer_error = None, str(exc)[:200]
        if slots is not None:
            pstatus = cuda.status_word(device)   # its own word: a stalled wait is reported, not fatal
            try:
                ms_p, _ = _timed(torch, lambda: slots.dense(x, shard, books, width, GROUP, pstatus), args.steps,
                                 args.warmup, world, device, local, label="sharded-peer")
                cuda.check(pstatus)
            except Exception as exc:  # noqa: BLE001
                ms_p, peer_error = None, str(exc)[:200]
            finally:
                slots.close()
                dist.barrier()
    coded_total = experts * (CODE_BYTES + BOOK_BYTES)
    out = {"cfg2-nsplit": {
        "metric": "vq4 packed GEMV coded-weight GB/s, W rows split across ranks (cfg2, M=1, strong scaling)",
        "unit": "GB/s", "experts": experts, "rows_per_rank": width, "scaling": "strong",
        "ms_per_step_compute": round(ms_c, 4), "value_compute": round(coded_total / (ms_c / 1e3) / 1e9, 2),
        "ms_per_step_with_allgather": round(ms_g, 4),
        "value_with_allgather": round(coded_total / (ms_g / 1e3) / 1e9, 2),
        "allgather_bytes_per_rank": send.numel() * 4, "allgather_share": round(max(0.0, ms_g - ms_c) / ms_g, 4),
        "ms_per_step_with_peer_stores": None if ms_p is None else round(ms_p, 4),
        "peer_stores_error": peer_error,
        "value_with_peer_stores": None if ms_p is None else round(coded_total / (ms_p / 1e3) / 1e9, 2),
        "peer_stores": "the GEMV stores each output into every rank's rank-major buffer over NVLink (CUDA IPC), "
                       "then step flags; the same bytes as the all-gather, bit for bit",
        "gather_layout": "rank-major (world, E, M, rows), in place", "clocks": clocks}}
    del shard, x, y, send, gathered
    torch.cuda.empty_cache()
    # cfg3: W rows (output columns of C) split across ranks, both operands coded
    from alelyon_compute_kit import vq
    xc, xb, wc, wb, m3, n3, k3, g3 = make_cfg3(torch, cuda, vq, device)
    ranges3 = parallel.row_ranges(n3, k3, g3, world)
    a3, b3 = ranges3[rank]
    width3 = max(b - a for a, b in ranges3)
    wshard = wc.view(n3, k3 // g3 // 8)[a3:b3].contiguous().view(-1)
    del wc
    y3 = torch.zeros((m3, b3 - a3), dtype=torch.float32, device=device)
    send3 = y3 if b3 - a3 == width3 else torch.zeros((m3, width3), dtype=torch.float32, device=device)
    gathered3 = torch.empty((world, m3, width3), dtype=torch.float32, device=device)

    def compute3():
        cuda.coded(xc, xb, wshard, wb, m3, b3 - a3, k3, g3, flags=2, out=y3, status=status)

    def compute3_gather():
        compute3()
        if send3 is not y3:
            send3[:, : b3 - a3] = y3
        dist.all_gather_into_tensor(gathered3.view(-1), send3.view(-1))

    ms3_c, clocks3 = _timed(torch, compute3, args.steps, args.warmup, world, device, local, label="sharded-cfg3")
    ms3_g, _ = _timed(torch, compute3_gather, args.steps, args.warmup, world, device, local,
                      label="sharded-cfg3-gather")
    cuda.check(status)
    flops3 = 2.0 * m3 * n3 * k3
    out["cfg3-nsplit"] = {
        "metric": "vq4 both-coded GEMM effective TFLOP/s, W rows split across ranks (cfg3, strong scaling)",
        "unit": "TFLOP/s", "rows_per_rank": width3, "scaling": "strong",
        "ms_per_step_compute": round(ms3_c, 4), "value_compute": round(flops3 / (ms3_c / 1e3) / 1e12, 2),
        "ms_per_step_with_allgather": round(ms3_g, 4),
        "value_with_allgather": round(flops3 / (ms3_g / 1e3) / 1e12, 2),
        "allgather_bytes_per_rank": send3.numel() * 4, "allgather_share": round(max(0.0, ms3_g - ms3_c) / ms3_g, 4),
        "gather_layout": "rank-major (world, M, rows), in place", "clocks": clocks3}
    del xc, wshard, y3, send3, gathered3
    torch.cuda.empty_cache()
    sub = copy.copy(args)
    sub.no_e2e = sub.no_cpu = True
    bank = run_cfg4(sub, world, rank, local)
    out["cfg4-bank"] = {"metric": bank["metric"], "value": bank["value"], "unit": bank["unit"],
                        "experts_total": world * args.experts_cfg4, "ms_per_step": bank["ms_per_step"],
                        "scaling": "weak", "clocks": bank["clocks"]}
    return out


def run_nf4(args, world, rank, local) -> dict:
    """The NF4 comparator on the headline's shape: 768 experts of an
    11008 x 4096 weight in bitsandbytes' NF4 stored form (random indices and
    absmax bytes, absmax2 in [0.004, 0.2]), one bf16 row of activations each,
    through nf4-gemv/v1 (bit for bit the reference's law). The law indexes
    values in 32 bits, so a step is 12 calls of 64 experts. `value` is NF4
    weight bytes (indices + absmax bytes + absmax2) per second, the same
    quantity as the headline's coded-weight bytes."""
    import torch

    from alelyon_compute_kit import nf4
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    experts, chunk = args.experts, 64
    per = N_ROWS * K_COLS
    calls = (experts + chunk - 1) // chunk
    experts = calls * chunk
    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    packed = torch.randint(0, 256, (experts * per // 2,), generator=gen, dtype=torch.uint8, device=device)
    absq = torch.randint(0, 256, (experts * per // 64,), generator=gen, dtype=torch.uint8, device=device)
    absmax2 = 0.004 + torch.randint(0, 997, (experts * per // 16384,), generator=gen, device=device).float() * 2e-4
    from statistics import NormalDist
    nd = NormalDist()
    code = sorted([nd.inv_cdf(q) for q in np.linspace(0.03, 0.97, 15)] + [0.0])
    code = np.array(code) / max(abs(c) for c in code)
    tables = torch.from_numpy(np.concatenate([code, (np.arange(256) - 127.5) / 128.0]).astype(np.float32)).to(device)
    starts = torch.arange(chunk, dtype=torch.int64, device=device) * per
    offsets = torch.zeros(chunk, dtype=torch.float32, device=device)
    a16 = (torch.randn((experts, K_COLS), generator=gen, device=device)).to(torch.bfloat16).view(torch.int16)
    table = torch.from_numpy(np.array([[i, 1, i * per] for i in range(chunk)], np.uint32).view(np.int32)).to(device)
    out = torch.empty((calls, chunk, N_ROWS), dtype=torch.float32, device=device)
    wb_per = per // 2 + per // 64 + 4 * (per // 16384)

    def step():
        for c in range(calls):
            e0 = c * chunk
            nf4.gemv(a16[e0: e0 + chunk], packed[e0 * per // 2: (e0 + chunk) * per // 2],
                     absq[e0 * per // 64: (e0 + chunk) * per // 64],
                     absmax2[e0 * per // 16384: (e0 + chunk) * per // 16384], tables, starts, offsets, table,
                     rows=chunk, n=N_ROWS, k=K_COLS, elem="bf16", max_rows=1, out=out[c])

    ms, clocks = _timed(torch, step, args.steps, args.warmup, world, device, local)
    weight = experts * wb_per
    algorithmic = weight + experts * (2 * K_COLS + 4 * N_ROWS)
    del packed, absq, absmax2, a16, out
    return {"metric": "NF4 comparator GEMV weight GB/s (cfg2 shape, 11008x4096, M=1, 768 experts, bf16 A)",
            "value": round(world * weight / (ms / 1e3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "config": {"workload": "nf4-gemv-cfg2-shape", "experts": experts, "calls_per_step": calls,
                       "weight_bytes_per_expert": wb_per},
            "roofline": roofline("hbm", algorithmic / (ms / 1e3) / 1e9, "k_nf4_gemv", algorithmic, None,
                                 note="the law's per-value rounding of the weight to 16 bits makes it "
                                      "instruction-bound before HBM"),
            "clocks": clocks}


def run_secondary(args, torch, cuda, codes, books, device, world, rank, local) -> dict:
    """Every other workload of the configs, measured in the same run: cfg2
    at M = 4, 16, 64 over the same experts; cfg3; the cfg4 VQAdamW step;
    decode and encode of 2^30 values for each group and distribution."""
    import copy
    sec = {}
    for m in (4, 16, 64):
        rec = time_cfg2(args, torch, cuda, codes, books, m, device, world, local)
        sec[f"cfg2-m{m}"] = {
            "metric": f"vq4 packed GEMM coded-weight GB/s (cfg2, M={m})", "value": round(rec["value"], 2),
            "unit": "GB/s", "ms_per_step": round(rec["ms"], 4), "engine": rec["engine"],
            "weight_layout": rec["layout"], "dense_equivalent_tflops": round(rec["tflops_dense_equivalent"], 2),
            "roofline": rec["roofline"], "clocks": rec["clocks"]}
    del codes, books
    torch.cuda.empty_cache()
    sub = copy.copy(args)
    sub.no_e2e = sub.no_cpu = True
    sec["cfg3"] = compact(run_cfg3(sub, world, rank, local))
    torch.cuda.empty_cache()
    sec["cfg4"] = compact(run_cfg4(sub, world, rank, local))
    torch.cuda.empty_cache()
    sec["nf4-gemv"] = compact(run_nf4(sub, world, rank, local))
    torch.cuda.empty_cache()
    for group in (8, 16, 32):
        for dist in ("gauss", "heavy"):
            sub.group, sub.dist = group, dist
            for which, res in run_codec_both(sub, world, rank, local).items():
                sec[f"{which}-g{group}-{dist}"] = compact(res)
            torch.cuda.empty_cache()
    return sec


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
                backend.matmul_dense_grouped(xs, weights, out=ys, parts=args.e2e_parts)
            steps = max(5, args.steps)
            t0 = time.perf_counter()
            for _ in range(steps):
                backend.matmul_dense_grouped(xs, weights, out=ys, parts=args.e2e_parts)
            elapsed = (time.perf_counter() - t0) / steps
    # the copy ceiling of this host link: one plain pinned copy each way, timed alone
    dev_x = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    dev_y = torch.empty(pin_y.shape, dtype=torch.float32, device=x.device)
    link = {}
    for name, dst, src in (("h2d", dev_x, pin_x), ("d2h", pin_y, dev_y)):
        dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            dst.copy_(src, non_blocking=True)
        z.record()
        torch.cuda.synchronize()
        link[name] = a.elapsed_time(z) / 5
    del dev_x, dev_y
    h2d = xs.nbytes              # X (the status word is cleared on the device)
    d2h = ys.nbytes + 4          # Y and the status word
    return {"value": round(experts * (CODE_BYTES + BOOK_BYTES) / elapsed / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(elapsed * 1e3, 3),
            "copy_gbs": round((h2d + d2h) / elapsed / 1e9, 2),
            "link": {"h2d_gbs": round(xs.nbytes / link["h2d"] / 1e6, 2),
                     "d2h_gbs": round(ys.nbytes / link["d2h"] / 1e6, 2),
                     "overlapped_bound_ms": round(max(link["h2d"], link["d2h"]), 3),
                     "serial_copies_ms": round(link["h2d"] + link["d2h"], 3)},
            "api": "VQDevice.matmul_dense_grouped on a ResidentStack (C ABI ack_vq2_dense_host: weights "
                   "resident; X in, the product and Y out pipelined over parts of the experts on three "
                   "streams; pinned host memory)"}


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


def make_codec_data(torch, vq, args, group, rank, device):
    """cfg 5 inputs: 2^30 FP32 values (args.dist: block-normalised Gaussian,
    or duplicate-heavy: 16 exact atoms, atom 0 at 85%), and the codebook
    fitted on the CPU from a 65,536-vector sample."""
    n = args.values
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
    return x, book


def run_codec_both(args, world, rank, local, which=("encode", "decode")) -> dict:
    """cfg 5: encode and decode of 2^30 FP32 values, one dataset (args.group,
    args.dist); returns {which: result line}."""
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    group, n = args.group, args.values
    x, book = make_codec_data(torch, vq, args, group, rank, device)
    codes, status = cuda.encode(x, book, group)
    cuda.check(status)
    out = torch.empty_like(x)
    results = {}
    for w in which:
        if w == "encode":
            fn = lambda: cuda.encode(x, book, group, out=codes, status=status)  # noqa: E731
        else:
            fn = lambda: cuda.decode(codes, book, n, group, out=out, status=status)  # noqa: E731
        ms, clocks = _timed(torch, fn, args.steps, args.warmup, world, device, local)
        cuda.check(status)
        code_bytes = codes.numel() * 4
        algorithmic = 4 * n + code_bytes + 64 * group
        achieved = algorithmic / (ms / 1e3) / 1e9
        # x from torch is 16-byte aligned: encode runs the tensor-core kernel
        kernel = "k_encode_tc" if w == "encode" else "k_decode"
        result = {
            "metric": f"vq4 {w} Gvalues/s (cfg5, 2^30 values, g{group}, {args.dist})",
            "value": round(world * n / (ms / 1e3) / 1e9, 3), "unit": "Gvalues/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": f"synthetic ({args.dist})",
            "config": {"workload": f"cfg5-{w}-g{group}-{args.dist}", "values_per_gpu": n, "group": group,
                       "l2": "inputs larger than L2", "parallelism": f"range-sharded x{world}, no collective"},
            "roofline": roofline("hbm", achieved, kernel, algorithmic, f"{kernel}_cfg5_g{group}_{args.dist}"),
            # encode: the book-staging kernel and the encode kernel per step
            "gpu_launches": args.steps * (2 if w == "encode" else 1), "clocks": clocks,
        }
        if rank == 0 and not args.no_cpu:
            sys.path.insert(0, str(ROOT / "oracle"))
            import vq_oracle_c as oc
            m = 1 << 24
            xs, cb, bk = x[:m].cpu().numpy(), codes[: m // group // 8].cpu().numpy().view(np.uint32), book.cpu().numpy()
            t0 = time.perf_counter()
            reps = 0
            while time.perf_counter() - t0 < args.cpu_budget:
                if w == "encode":
                    oc.encode(xs, bk, group)
                else:
                    oc.decode(cb, bk, m, group)
                reps += 1
            el = time.perf_counter() - t0
            result["cpu_baseline"] = {"value": round(reps * m / el / 1e9, 4), "unit": "Gvalues/s",
                                      "cores": oc.threads(), "kind": "port",
                                      "sample": f"{reps} x 2^24 values, {el:.1f} s"}
        results[w] = result
    del x, out, codes
    return results


def run_codec(args, world, rank, local, which):
    """cfg 5: encode or decode of 2^30 FP32 values (args.dist: gauss or heavy)."""
    return run_codec_both(args, world, rank, local, (which,))[which]


def make_cfg3(torch, cuda, vq, device):
    """cfg 3 operands: X 4096 x 4096 ~ N(0, 1) and W 14336 x 4096 ~
    N(0, 0.02^2), each encoded g32 with a book fitted on the CPU from a
    4,096-vector sample. Returns (xc, xb, wc, wb, m, n, k, group)."""
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
    return xc, xb, wc, wb, m, n, k, group


def run_cfg3(args, world, rank, local):
    """cfg 3: both operands coded, X 4096 x 4096 (g32, own book) times
    W 14336 x 4096 (g32) transposed; the 16x16 codebook inner-product table."""
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    xc, xb, wc, wb, m, n, k, group = make_cfg3(torch, cuda, vq, device)
    status = cuda.status_word(device)
    y = torch.empty((m, n), dtype=torch.float32, device=device)
    fn = lambda: cuda.coded(xc, xb, wc, wb, m, n, k, group, flags=2, out=y, status=status)  # noqa: E731
    ms, clocks = _timed(torch, fn, args.steps, args.warmup, world, device, local)
    cuda.check(status)
    flops = 2.0 * m * n * k
    lookups = m * n * (k // group)
    byts = xc.numel() * 4 + wc.numel() * 4 + 2 * 64 * group + 4 * m * n
    return {
        "metric": "vq4 both-coded GEMM effective TFLOP/s (cfg3, 4096x4096 . (14336x4096)^T, g32)",
        "value": round(world * flops / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg3-coded-gemm", "M": m, "N": n, "K": k, "group": group,
                   "lut_lookups_per_s": lookups / (ms / 1e3), "parallelism": f"replicated x{world}"},
        "roofline": roofline("hbm", byts / (ms / 1e3) / 1e9, "k_coded_lut", byts, "k_coded_lut_cfg3",
                             note="the table lookups on the shared-memory pipe bound this kernel, not HBM"),
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
        "roofline": roofline("hbm", byts / (ms_encode / 1e3) / 1e9, "k_adamw_encode", byts,
                             "k_adamw_encode_cfg4",
                             note="compute-bound (three certified 16-entry searches per value); coded bytes only"),
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


def run_profile_cases(args, world, rank, local):
    """Small cases of every measured kernel, each launched three times, for
    ncu captures of per-launch DRAM traffic (`--workload profile`): decode and
    encode of 2^28 values per group and distribution, the grouped product of
    96 experts at M = 1, 4, 16, 64, cfg3 at its full size, and the fused
    AdamW pass of 8 cfg4 experts. Prints one line per case; no timing."""
    import torch

    from alelyon_compute_kit import cuda, vq
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    status = cuda.status_word(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(1)
    sub = __import__("copy").copy(args)
    sub.values = 1 << 28
    for group in (8, 16, 32):
        for dist in ("gauss", "heavy"):
            sub.dist = dist
            x, book = make_codec_data(torch, vq, sub, group, rank, device)
            codes, _ = cuda.encode(x, book, group, status=status)
            out = torch.empty_like(x)
            for _ in range(3):
                cuda.encode(x, book, group, out=codes, status=status)
            for _ in range(3):
                cuda.decode(codes, book, x.numel(), group, out=out, status=status)
            torch.cuda.synchronize()
            print("profile case", f"cfg5-g{group}-{dist}", flush=True)
            del x, codes, out
    experts = 96
    codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (experts, CODE_BYTES // 4), generator=gen, device=device,
                          dtype=torch.int32)
    books = torch.randn((experts, 16, GROUP), generator=gen, device=device) * 0.25
    for m in (1, 4, 16, 64):
        x = torch.randn((experts, m, K_COLS), generator=gen, device=device)
        engine = cuda.dense_engine(m, K_COLS, GROUP)
        layout = "canonical" if (m == 1 or engine == "tensor") else "tile32"
        run_codes = cuda.repack_tile32(codes, N_ROWS, K_COLS, GROUP, status=status)[0] if layout == "tile32" else codes
        for _ in range(3):
            cuda.dense(x, run_codes, books, N_ROWS, GROUP, layout=layout, engine=engine, status=status)
        torch.cuda.synchronize()
        print("profile case", f"cfg2-m{m}", engine, layout, flush=True)
    del codes, books, x, run_codes
    m, n, k, g = 4096, 14336, 4096, 32
    xc = torch.randint(-2 ** 31, 2 ** 31 - 1, (m * k // g // 8,), generator=gen, device=device, dtype=torch.int32)
    wc = torch.randint(-2 ** 31, 2 ** 31 - 1, (n * k // g // 8,), generator=gen, device=device, dtype=torch.int32)
    xb, wb = torch.randn((16, g), device=device), torch.randn((16, g), device=device) * 0.02
    for _ in range(3):
        cuda.coded(xc, xb, wc, wb, m, n, k, g, flags=2, status=status)
    torch.cuda.synchronize()
    print("profile case cfg3", flush=True)
    del xc, wc
    e, count, g = 8, 4096 * 1024, 8
    words = cuda.words_for(count, g)
    codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (e, 4, words), generator=gen, device=device, dtype=torch.int32)
    books = torch.randn((e, 4, 16, g), generator=gen, device=device) * 0.01
    books[:, 2] = books[:, 2].abs()
    coefs = torch.from_numpy(np.tile(np.array([1e-3, 0.9, 0.999, 1e-8, 0.01, 0.19, 0.002], np.float32),
                                     (e, 1))).to(device)
    for _ in range(3):
        cuda.adamw_encode(codes, books, coefs, books[:, :3].contiguous(), count, g, batch=e, status=status)
    torch.cuda.synchronize()
    print("profile case cfg4", flush=True)
    return None


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
    ap.add_argument("--e2e-parts", type=int, default=0,
                    help="expert ranges of the pipelined host-memory product (0: the library's choice)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the other workloads that the default cfg2 run measures beside the headline")
    ap.add_argument("--group", type=int, default=16)
    ap.add_argument("--layout", choices=("auto", "tile32", "canonical"), default="auto",
                    help="auto: canonical for M = 1 (the byte-table kernel), tile32 otherwise")
    ap.add_argument("--engine", choices=("auto", "lut", "tensor"), default="auto",
                    help="dense product kernels: tensor cores (M >= 8 by default) or lookup tables")
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
    elif args.workload == "nf4":
        result = run_nf4(args, world, rank, local)
    elif args.workload == "cfg3":
        result = run_cfg3(args, world, rank, local)
    elif args.workload == "cfg4":
        result = run_cfg4(args, world, rank, local)
    elif args.workload == "profile":
        result = run_profile_cases(args, world, rank, local)
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
