"""Run and update the coded linear experts of an `ExpertBank` on a B200.

The public surface is the reference harness's (`src/alelyon_compute_kit/
harness.py`): `VulkanExpertHarness` (also `ExpertHarness`) with `open`,
`forward`, `train_step` and `train`, the `ExpertStep` record, `HarnessError`
and the command line. A step is the reference's MSE update of one expert
(`harness.py:162-242`):

    X, T  -> coded images (fit_codebook + encode)
    P     =  decode(X) . decode(W)            (the shader's packed product)
    R     =  P - decode(T);  loss = mean(R^2) (float64);  R *= 2 / size
    G     =  decode(X)^T . decode(code(R))    (the packed product)
    G     *= min(1, max_norm / (||G|| + 1e-6))   (||G|| in float64)
    W, M, V <- VQAdamW(code(G));  commit to the bank

It runs on one of two engines:

* the device engine (the default: no `backend` given). The step stays in
  HBM: X and T are copied in once, the bank's W, M, V shards go from pinned
  host memory straight to device tensors, every fit, encode, product,
  residual, norm and optimizer pass is a kernel of this library on the
  same stream, and only the new coded state and three scalars come back.
  Its fits are the CPU fit's books bit for bit (`fit="device"`) or run on
  the CPU from a device-gathered sample (`fit="host"`, the reference's
  placement). The float64 loss and norm are summed in a different order
  from numpy's, so they can differ from the host arithmetic in their last
  bits; everything else is identical;
* the host engine, for an injected `backend` with the reference's
  operator protocol (`encode`, `decode`, `matmul`, `adamw`): the reference's
  flow on host arrays.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import tempfile
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import ack, expert_bank, vq

ENTRIES = vq.ENTRIES


class HarnessError(ValueError):
    """The supplied model state, arrays or job boundary is not admissible."""


@dataclass(frozen=True)
class ExpertStep:
    """Evidence for one committed expert update."""

    layer: int
    expert: int
    optimizer_step: int
    revision: int
    loss: float
    gradient_norm_before_clip: float
    clipped: bool
    elapsed_seconds: float
    persistent_state_bytes: int
    input_layout: dict
    activation_layout: dict
    gradient_layout: dict

    def to_dict(self) -> dict:
        return dict(self.__dict__)


def _matrix(value, name: str) -> np.ndarray:
    """A nonempty, finite, rank-2 float32 array, C-contiguous."""
    a = np.asarray(value)
    if a.dtype != np.float32 or a.ndim != 2:
        raise HarnessError(f"{name} must be a rank-2 float32 array")
    if a.size == 0 or not np.isfinite(a).all():
        raise HarnessError(f"{name} must be nonempty and finite")
    return np.ascontiguousarray(a)


def _positive(value, name: str) -> float:
    if isinstance(value, (bool, np.bool_)):
        raise HarnessError(f"{name} must be finite and positive")
    try:
        result = float(value)
    except (TypeError, ValueError) as exc:
        raise HarnessError(f"{name} must be finite and positive") from exc
    if not math.isfinite(result) or result <= 0:
        raise HarnessError(f"{name} must be finite and positive")
    return result


def _calibration(values: np.ndarray, group: int) -> np.ndarray:
    """fit_codebook needs one complete vector: a smaller input is padded for
    the fit only (the encoder still trims the padded tail)."""
    if values.size >= group:
        return values
    return np.pad(values.reshape(-1), (0, group - values.size))


@dataclass(frozen=True)
class _Update:
    tensors: tuple            # W', M', V' as VQArrays
    loss: float
    norm: float
    scale: float
    persistent_bytes: int
    layouts: tuple            # X, T, G wire layouts


# ------------------------------------------------------------- host engine ----

class _HostEngine:
    """The reference's arithmetic through an injected operator backend."""

    def __init__(self, backend, fit: str):
        self.backend, self.fit = backend, fit

    def _image(self, values: np.ndarray, group: int) -> vq.VQArray:
        sample = _calibration(values, group)
        if self.fit == "device":
            book = self.backend.fit_codebook(sample, group=group)
        else:
            book = vq.fit_codebook(sample, group=group)
        return self.backend.encode(values, book, group=group)

    def forward(self, x: np.ndarray, weight: vq.VQArray) -> np.ndarray:
        return self.backend.matmul(self._image(x, weight.group), weight)

    def update(self, x, target, state, hyper) -> _Update:
        weight, momentum, variance = state.tensors[:3]
        g = weight.group
        x_img = self._image(x, g)
        t_img = self._image(target, g)
        residual = self.backend.matmul(x_img, weight) - self.backend.decode(t_img)
        loss = float(np.mean(np.square(residual, dtype=np.float64)))
        if not math.isfinite(loss):
            raise HarnessError("expert loss is nonfinite")
        residual *= np.float32(2.0 / residual.size)
        gradient = self.backend.matmul(x_img, self._image(residual, g), transpose_a=True)
        norm = float(np.linalg.norm(gradient.astype(np.float64)))
        if not math.isfinite(norm):
            raise HarnessError("expert gradient norm is nonfinite")
        scale = min(1.0, hyper["max_grad_norm"] / (norm + 1e-6))
        gradient *= np.float32(scale)
        g_img = self._image(gradient, g)
        try:
            opt = vq.VQAdamW(self.backend, weight, lr=hyper["lr"], betas=(hyper["beta1"], hyper["beta2"]),
                             eps=hyper["eps"], weight_decay=hyper["weight_decay"], fit=self.fit)
            opt.momentum, opt.variance, opt.steps = momentum, variance, state.optimizer_step
            report = opt.step(g_img)
        except (TypeError, ValueError, ack.AckError) as exc:
            raise HarnessError(f"expert optimizer refused the update: {exc}") from exc
        return _Update((opt.weight, opt.momentum, opt.variance), loss, norm, scale,
                       report["persistent_state_bytes"], (x_img.layout, t_img.layout, g_img.layout))


# ----------------------------------------------------------- device engine ----

class _DeviceEngine:
    """The whole step on one CUDA device, through `alelyon_compute_kit.cuda`."""

    SAMPLE_VECTORS = 4096
    ITERATIONS = 4

    def __init__(self, device: ack.Device, fit: str):
        import torch

        from . import cuda
        self.torch, self.cuda, self.fit = torch, cuda, fit
        want = bytes(device.info.device_uuid).hex()
        for i in range(torch.cuda.device_count()):
            seen = str(torch.cuda.get_device_properties(i).uuid).lower().replace("gpu-", "").replace("-", "")
            if seen == want:
                self.dev = torch.device("cuda", i)
                break
        else:
            raise HarnessError("the ack device is not a CUDA device that PyTorch sees")

    # -- pieces ----------------------------------------------------------------------

    def _to_device(self, a: np.ndarray):
        torch = self.torch
        pinned = torch.from_numpy(a).pin_memory()
        return pinned.to(self.dev, non_blocking=True)

    def _book(self, values, group: int, status, init=None):
        """fit_codebook of a device tensor: on the device, or on the CPU from
        the sample the fit would draw (positions as vq.fit_codebook's)."""
        torch, cuda = self.torch, self.cuda
        flat = values.reshape(-1)
        if flat.numel() < group:
            host = _calibration(flat.cpu().numpy(), group)
            return torch.from_numpy(vq.fit_codebook(host, group=group)).to(self.dev)
        if self.fit == "device":
            book, _ = cuda.fit_codebook(flat, group, sample_vectors=self.SAMPLE_VECTORS, status=status)
            return book
        complete = flat.numel() // group
        pos = np.linspace(0, complete - 1, min(complete, self.SAMPLE_VECTORS), dtype=np.int64)
        rows = flat[: complete * group].view(complete, group)[torch.from_numpy(pos).to(self.dev)]
        book = vq.fit_codebook(rows.cpu().numpy().reshape(-1), group=group, sample_vectors=self.SAMPLE_VECTORS)
        return torch.from_numpy(book).to(self.dev)

    def _coded(self, values, group: int, status):
        book = self._book(values, group, status)
        codes, _ = self.cuda.encode(values.reshape(-1), book, group, status=status)
        return codes, book

    def _adamw(self, codes, books, coefs, count: int, group: int, status):
        """The fused VQAdamW step on device state: (E=1, 4, words) codes and
        (1, 4, 16, g) books of W, M, V, G -> new (3, words) codes, (3, 16, g)
        books and the changed-value count."""
        torch, cuda = self.torch, self.cuda
        complete = count // group
        positions = np.linspace(0, complete - 1, min(complete, self.SAMPLE_VECTORS), dtype=np.int64)
        pos = torch.from_numpy(positions.astype(np.uint32).view(np.int32)).to(self.dev)
        samples, _ = cuda.adamw_sample(codes, books, coefs, pos, count, group, status=status)
        if self.fit == "device":
            new_books, _ = cuda.adamw_fit(codes, books, coefs, samples, count, group, iterations=self.ITERATIONS,
                                          status=status)
        else:
            host_samples = samples.cpu().numpy().reshape(3, -1, group)
            old_books = books.cpu().numpy().reshape(4, ENTRIES, group)
            usage = torch.empty(ENTRIES, dtype=torch.int32, device=self.dev)
            fitted = []
            for which in range(3):
                def whole_usage(book, which=which):
                    trial = torch.from_numpy(np.ascontiguousarray(book, np.float32)).to(self.dev)
                    cuda.adamw_usage(codes, books, coefs, trial, count, group, which, out=usage, status=status)
                    return np.nonzero(usage.cpu().numpy())[0].tolist()
                fitted.append(vq._fit(host_samples[which], complete, group, self.ITERATIONS, old_books[which],
                                      whole_usage))
            new_books = torch.from_numpy(np.stack(fitted).astype(np.float32)[None]).to(self.dev)
        out, changed, _ = cuda.adamw_encode(codes, books, coefs, new_books, count, group, status=status)
        return out[0], new_books[0], changed

    # -- engine surface ----------------------------------------------------------------

    def forward(self, x: np.ndarray, weight: vq.VQArray) -> np.ndarray:
        torch, cuda = self.torch, self.cuda
        g = weight.group
        status = cuda.status_word(self.dev)
        xd = self._to_device(x)
        xc, xb = self._coded(xd, g, status)
        wc = torch.from_numpy(weight.codes.view(np.int32).copy()).to(self.dev)
        wb = torch.from_numpy(weight.codebook.copy()).to(self.dev)
        m, k = x.shape
        y, _ = cuda.matmul_exact(xc, xb, wc, wb, m, weight.shape[1], k, g, status=status)
        self._check(status)
        return y.cpu().numpy()

    def _check(self, status):
        flags = int(status.item()) & 0xFFFFFFFF
        if flags:
            raise HarnessError(f"device arithmetic refused the step: status={flags}")

    def update(self, x, target, bank, layer, expert, state, hyper) -> _Update:
        torch, cuda = self.torch, self.cuda
        weight = state.tensors[0]
        g = weight.group
        (k, n), b = weight.shape, x.shape[0]
        status = cuda.status_word(self.dev)
        dstate = bank.read_expert_to_device(layer, expert, self.dev)     # W, M, V: pinned read + one copy each
        xd, td = self._to_device(x), self._to_device(target)
        xc, xb = self._coded(xd, g, status)
        tc, tb = self._coded(td, g, status)
        pred, _ = cuda.matmul_exact(xc, xb, dstate.codes[0], dstate.books[0], b, n, k, g, status=status)
        resid, sumsq, _ = cuda.residual(pred, tc, tb, g, float(np.float32(2.0 / pred.numel())), status=status)
        rc, rb = self._coded(resid, g, status)
        grad, _ = cuda.matmul_exact(xc, xb, rc, rb, k, n, b, g, flags=1, status=status)
        clipped, stats, _ = cuda.clip_norm(grad, hyper["max_grad_norm"], status=status)
        gc, gb = self._coded(clipped, g, status)
        try:
            coefs_np = vq._adamw_coefficients(state.tensors[:3] + (weight,), hyper["lr"], hyper["beta1"],
                                              hyper["beta2"], hyper["eps"], hyper["weight_decay"],
                                              state.optimizer_step + 1)
        except ValueError as exc:
            raise HarnessError(f"expert optimizer refused the update: {exc}") from exc
        codes = torch.stack([dstate.codes[0], dstate.codes[1], dstate.codes[2], gc])[None].contiguous()
        books = torch.stack([dstate.books[0], dstate.books[1], dstate.books[2], gb])[None].contiguous()
        coefs = torch.from_numpy(coefs_np[None]).to(self.dev)
        new_codes, new_books, _ = self._adamw(codes, books, coefs, k * n, g, status)
        # the only device-to-host traffic: the new state and the scalars
        host_codes = new_codes.cpu().numpy().view(np.uint32)
        host_books = new_books.cpu().numpy()
        loss = float(sumsq.item()) / pred.numel()
        norm, scale = (float(v) for v in stats.cpu().numpy())
        if not math.isfinite(loss):
            raise HarnessError("expert loss is nonfinite")
        if not math.isfinite(norm):
            raise HarnessError("expert gradient norm is nonfinite")
        self._check(status)
        tensors = tuple(vq.VQArray(weight.shape, g, host_codes[i], host_books[i]) for i in range(3))
        layouts = tuple(vq.storage_layout(shape, g) for shape in (x.shape, target.shape, weight.shape))
        return _Update(tensors, loss, norm, scale, sum(t.layout["serialized_bytes"] for t in tensors), layouts)


# ----------------------------------------------------------------- harness ----

class VulkanExpertHarness:
    """One durable linear expert through the native vq4 path.

    With no `backend`, the harness opens (or uses the given) `ack.Device`
    and runs the device engine; an injected `backend` runs the host engine.
    Importing this module opens nothing."""

    def __init__(self, bank: expert_bank.ExpertBank, *, backend=None, device=None, fit: str = "host"):
        """`fit` places the codebook fits: "host" (the CPU, as the reference)
        or "device" (the same books bit for bit, computed on the GPU)."""
        if not isinstance(bank, expert_bank.ExpertBank):
            raise HarnessError("bank must be an ExpertBank")
        if fit not in ("host", "device"):
            raise HarnessError(f"fit must be 'host' or 'device', not {fit!r}")
        if backend is not None and device is not None:
            raise HarnessError("supply backend or device, not both")
        self.bank, self.fit = bank, fit
        self._device, self._owned_device = device, False
        if backend is not None:
            if fit == "device" and not hasattr(backend, "fit_codebook"):
                raise HarnessError("fit='device' needs a backend that fits codebooks on the device")
            self.backend = backend
            self._engine = _HostEngine(backend, fit)
        else:
            if device is None:
                self._device, self._owned_device = ack.Device(), True
            self.backend = vq.VQDevice(self._device)
            self._engine = _DeviceEngine(self._device, fit)

    @classmethod
    def open(cls, root, *, device=None, backend=None, fit: str = "host") -> "VulkanExpertHarness":
        """Open an existing bank without creating or initialising payloads."""
        return cls(expert_bank.ExpertBank.open(root), backend=backend, device=device, fit=fit)

    def __enter__(self) -> "VulkanExpertHarness":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self) -> None:
        if self._owned_device and self._device is not None:
            self._device.close()
        self._device = None if self._owned_device else self._device

    def _state(self, layer: int, expert: int) -> expert_bank.ExpertState:
        try:
            state = self.bank.read_expert_state(layer, expert)
        except expert_bank.ExpertBankError as exc:
            raise HarnessError(str(exc)) from exc
        if len(state.tensors) < 3:
            raise HarnessError("expert state must contain weight, momentum and variance")
        w, m, v = state.tensors[:3]
        if not (w.shape == m.shape == v.shape and w.group == m.group == v.group):
            raise HarnessError("expert optimizer state geometry disagrees")
        return state

    def forward(self, inputs, *, layer: int = 0, expert: int = 0) -> np.ndarray:
        """`inputs @ weight` through the packed product (inputs coded first)."""
        x = _matrix(inputs, "inputs")
        weight = self._state(layer, expert).tensors[0]
        if x.shape[1] != weight.shape[0]:
            raise HarnessError(f"inputs have width {x.shape[1]}, expert expects {weight.shape[0]}")
        return self._engine.forward(x, weight)

    def train_step(self, inputs, targets, *, layer: int = 0, expert: int = 0, lr: float = 1e-3, beta1: float = 0.9,
                   beta2: float = 0.95, eps: float = 1e-8, weight_decay: float = 0.0,
                   max_grad_norm: float = 1.0) -> ExpertStep:
        """One MSE update, committed atomically to the bank."""
        x, target = _matrix(inputs, "inputs"), _matrix(targets, "targets")
        if x.shape[0] != target.shape[0]:
            raise HarnessError("inputs and targets must have the same row count")
        state = self._state(layer, expert)
        weight = state.tensors[0]
        if x.shape[1] != weight.shape[0] or target.shape[1] != weight.shape[1]:
            raise HarnessError("inputs/targets do not match expert matrix geometry")
        hyper = {"lr": lr, "beta1": beta1, "beta2": beta2, "eps": eps, "weight_decay": weight_decay,
                 "max_grad_norm": _positive(max_grad_norm, "max_grad_norm")}
        started = time.perf_counter()
        if isinstance(self._engine, _DeviceEngine):
            up = self._engine.update(x, target, self.bank, layer, expert, state, hyper)
        else:
            up = self._engine.update(x, target, state, hyper)
        try:
            receipt = self.bank.write_expert(layer, expert, up.tensors, updated_count=weight.layout["elements"],
                                             optimizer_step=state.optimizer_step + 1)
        except expert_bank.ExpertBankError as exc:
            raise HarnessError(f"expert update was not committed: {exc}") from exc
        elapsed = time.perf_counter() - started
        if not math.isfinite(elapsed) or elapsed <= 0:
            raise HarnessError("expert step elapsed time is invalid")
        return ExpertStep(layer=layer, expert=expert, optimizer_step=state.optimizer_step + 1,
                          revision=receipt["revision"], loss=up.loss, gradient_norm_before_clip=up.norm,
                          clipped=up.scale < 1.0, elapsed_seconds=elapsed, persistent_state_bytes=up.persistent_bytes,
                          input_layout=up.layouts[0], activation_layout=up.layouts[1], gradient_layout=up.layouts[2])

    def train(self, inputs, targets, *, steps: int = 1, **kwargs) -> tuple[ExpertStep, ...]:
        """Bounded sequential steps, committing after each."""
        if type(steps) is not int or not 1 <= steps <= 1_000_000:
            raise HarnessError("steps must be an integer in 1..1000000")
        return tuple(self.train_step(inputs, targets, **kwargs) for _ in range(steps))


ExpertHarness = VulkanExpertHarness


# -------------------------------------------------------------- command line ----

def _load_matrix(path: Path, name: str) -> np.ndarray:
    if path.is_symlink() or not path.is_file():
        raise HarnessError(f"{name} must be a regular file")
    try:
        value = np.load(path, allow_pickle=False)
    except (OSError, ValueError) as exc:
        raise HarnessError(f"{name} is not a readable NumPy array") from exc
    if not isinstance(value, np.ndarray):
        raise HarnessError(f"{name} must be a single .npy array, not an archive")
    return _matrix(value, name)


def _save_matrix(path: Path, value: np.ndarray, *, force: bool) -> None:
    """Write `value` as .npy atomically (temporary file, fsync, replace)."""
    if path.exists() and not force:
        raise HarnessError(f"refusing to overwrite existing output: {path}")
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", suffix=".tmp", dir=path.parent)
    try:
        with os.fdopen(fd, "wb") as stream:
            np.save(stream, value, allow_pickle=False)
            stream.flush()
            os.fsync(stream.fileno())
        os.replace(tmp, path)
    finally:
        Path(tmp).unlink(missing_ok=True)


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--bank", type=Path, required=True)
    parser.add_argument("--input", type=Path, required=True)
    parser.add_argument("--output", type=Path, required=True)
    parser.add_argument("--target", type=Path)
    parser.add_argument("--layer", type=int, default=0)
    parser.add_argument("--expert", type=int, default=0)
    parser.add_argument("--steps", type=int, default=1)
    parser.add_argument("--lr", type=float, default=1e-3)
    parser.add_argument("--max-grad-norm", type=float, default=1.0)
    parser.add_argument("--device", action="store_true", help="explicitly open the CUDA device")
    parser.add_argument("--fit", choices=("host", "device"), default="host",
                        help="where codebooks are fitted (the same books either way)")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args(argv)
    if not args.device:
        parser.error("--device is required; execution is never implicit")
    inputs = _load_matrix(args.input, "input")
    with VulkanExpertHarness.open(args.bank, fit=args.fit) as harness:
        if args.target is not None:
            targets = _load_matrix(args.target, "target")
            steps = harness.train(inputs, targets, steps=args.steps, layer=args.layer, expert=args.expert,
                                  lr=args.lr, max_grad_norm=args.max_grad_norm)
        result = harness.forward(inputs, layer=args.layer, expert=args.expert)
        _save_matrix(args.output, result, force=args.force)
        report = {"mode": "forward" if args.target is None else "train", "shape": list(result.shape),
                  "device": harness._device.capability_record(), "model_quality_validated": False}
        if args.target is not None:
            report["steps"] = [s.to_dict() for s in steps]
            del report["shape"]
    print(json.dumps(report, sort_keys=True, allow_nan=False))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
