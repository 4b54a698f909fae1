"""Coded expert banks on disk: the reference's `ack-expert-bank/v1` layout,
read and written by this library, with a path into device memory.

On-disk format (the interface shared with the reference's
`_kit/python/expert_bank.py`; a bank written by either opens in the other):

* `<root>/bank.json`: canonical JSON `{"schema": "ack-expert-bank/v1",
  "config": {"layers", "experts_per_layer", "matrix_shapes", "group"}}`.
  Canonical means sorted keys, no whitespace, UTF-8, no NaN or infinity,
  no duplicate keys; a file that does not round-trip is refused. Its
  SHA-256 is the bank's identity (`config_sha256`).
* `<root>/expert-<layer>-<expert>.json`: the committed generation of one
  expert, canonical JSON with exactly the keys `schema`, `config_sha256`,
  `layer`, `expert`, `generation` (32 hex digits), `revision` (1, 2, ...),
  `optimizer_step`, `parameter_update_applications`, `update_commits` and
  `shards` (one `{"bytes", "sha256"}` per configured matrix).
* `<root>/expert-<layer>-<expert>-g<generation>-t<index>.vq`: matrix `index`
  of that generation, the `VQArray` wire image.

A commit writes the new shards and a `pending-<generation>.json` with
exclusive creation and fsync, checks that neither the bank nor the expert's
pointer changed meanwhile, then atomically replaces the pointer; a refused
commit removes what it wrote. Readers see a pointer either whole or not at
all. One writer per bank, any number of readers.

Device I/O (`read_expert_to_device`): each shard file is read into pinned
host memory and copied once to the device, where the codes and the codebook
land in separate, 16-byte aligned tensors -- the operands of the CUDA path,
with no pageable staging and no re-packing on the host.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import re
import stat
import time
import uuid
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

import numpy as np

from .vq import ENTRIES, GROUPS, VQArray, storage_layout

SCHEMA = "ack-expert-bank/v1"
MAX_SHARD_BYTES = 128 * 1024 * 1024
MAX_METADATA_BYTES = 128 * 1024

_POINTER_NAME = re.compile(r"expert-([0-9]+)-([0-9]+)\.json\Z")
_SHA256 = re.compile(r"[0-9a-f]{64}\Z")
_GENERATION = re.compile(r"[0-9a-f]{32}\Z")
_INT_MAX = (1 << 63) - 1


class ExpertBankError(ValueError):
    """A bank, payload, declaration or boundary is not admissible."""


def _int_in(value, name: str, low: int = 0, high: int = _INT_MAX) -> int:
    if type(value) is not int or value < low or value > high:
        raise ExpertBankError(f"{name} must be an integer in {low}..{high}")
    return value


# ----------------------------------------------------------- canonical JSON ----

class CanonicalJson:
    """The bank's metadata encoding: one byte string per value."""

    @staticmethod
    def dump(value) -> bytes:
        return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode("utf-8")

    @classmethod
    def load(cls, data: bytes):
        def unique(pairs):
            keys = [k for k, _ in pairs]
            if len(set(keys)) != len(keys):
                raise ExpertBankError("duplicate metadata key")
            return dict(pairs)

        def finite_only(token):
            raise ExpertBankError("nonfinite metadata")

        try:
            value = json.loads(data, object_pairs_hook=unique, parse_constant=finite_only)
            again = cls.dump(value)
        except ExpertBankError:
            raise
        except (UnicodeError, json.JSONDecodeError, RecursionError, ValueError) as exc:
            raise ExpertBankError("invalid bank metadata") from exc
        if again != data:
            raise ExpertBankError("noncanonical bank metadata")
        return value

    @staticmethod
    def require(value, keys: set, what: str) -> dict:
        if not isinstance(value, dict) or set(value) != keys:
            raise ExpertBankError(f"invalid {what} fields")
        return value


def _sha256(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


# ------------------------------------------------------------------- files ----

class _Files:
    """Bounded reads of regular files, durable exclusive writes, and the
    pointer replacement (retried: on some platforms a reader holding the
    target open makes the replacement fail for a moment)."""

    REPLACE_TRIES = 50
    REPLACE_PAUSE_S = 0.02

    @staticmethod
    def read(path: Path, limit: int) -> bytes:
        info = path.lstat()
        if path.is_symlink() or not stat.S_ISREG(info.st_mode) or info.st_size > limit:
            raise ExpertBankError("file is not regular or exceeds byte limit")
        with path.open("rb") as stream:
            data = stream.read(limit + 1)
        if len(data) != info.st_size or len(data) > limit:
            raise ExpertBankError("file changed size or exceeds byte limit")
        return data

    @staticmethod
    def create(path: Path, data: bytes) -> None:
        with path.open("xb") as stream:
            stream.write(data)
            stream.flush()
            os.fsync(stream.fileno())

    @classmethod
    def publish(cls, pending: Path, target: Path) -> None:
        for attempt in range(cls.REPLACE_TRIES):
            try:
                os.replace(pending, target)
                return
            except PermissionError as exc:
                if attempt == cls.REPLACE_TRIES - 1:
                    raise ExpertBankError("pointer replacement refused; a reader may hold the pointer open") from exc
                time.sleep(cls.REPLACE_PAUSE_S)


# ------------------------------------------------------------------ config ----

@dataclass(frozen=True)
class BankConfig:
    """A bank's fixed geometry: layers x experts_per_layer experts, each a
    list of coded matrices of the given shapes and one vector group."""

    layers: int
    experts_per_layer: int
    matrix_shapes: tuple[tuple[int, int], ...]
    group: int = 16

    def __post_init__(self):
        _int_in(self.layers, "layers", 1, 1_000_000)
        _int_in(self.experts_per_layer, "experts_per_layer", 1, 1_000_000)
        if type(self.group) is not int or self.group not in GROUPS:
            raise ExpertBankError("group must be 8, 16 or 32")
        shapes = self.matrix_shapes
        if not isinstance(shapes, (tuple, list)) or not 1 <= len(shapes) <= 16:
            raise ExpertBankError("matrix_shapes must contain 1..16 matrices")
        checked = []
        for shape in shapes:
            if not isinstance(shape, (tuple, list)) or len(shape) != 2:
                raise ExpertBankError("each matrix must have two dimensions")
            dims = tuple(_int_in(d, "matrix dimension", 1) for d in shape)
            try:
                size = storage_layout(dims, self.group)["serialized_bytes"]
            except ValueError as exc:
                raise ExpertBankError(str(exc)) from exc
            if size > MAX_SHARD_BYTES:
                raise ExpertBankError("matrix exceeds shard byte limit")
            checked.append(dims)
        object.__setattr__(self, "matrix_shapes", tuple(checked))
        _int_in(self.potential_parameters, "potential_parameters")

    @property
    def parameters_per_expert(self) -> int:
        return sum(r * c for r, c in self.matrix_shapes)

    @property
    def potential_parameters(self) -> int:
        return self.layers * self.experts_per_layer * self.parameters_per_expert

    def shard_bytes(self, index: int) -> int:
        return storage_layout(self.matrix_shapes[index], self.group)["serialized_bytes"]

    def to_dict(self) -> dict:
        return {"layers": self.layers, "experts_per_layer": self.experts_per_layer,
                "matrix_shapes": [list(s) for s in self.matrix_shapes], "group": self.group}

    @classmethod
    def from_dict(cls, value) -> "BankConfig":
        v = CanonicalJson.require(value, {"layers", "experts_per_layer", "matrix_shapes", "group"}, "config")
        return cls(v["layers"], v["experts_per_layer"], v["matrix_shapes"], v["group"])


@dataclass(frozen=True)
class ExpertState:
    """One committed generation: its tensors and the optimizer bookkeeping."""

    tensors: tuple[VQArray, ...]
    optimizer_step: int
    revision: int
    parameter_update_applications: int


@dataclass(frozen=True)
class DeviceExpertState:
    """One committed generation held in device memory: per matrix, its codes
    (int32 bit patterns of the u32 words) and its (16, group) codebook."""

    codes: tuple
    books: tuple
    shapes: tuple[tuple[int, int], ...]
    group: int
    optimizer_step: int
    revision: int
    parameter_update_applications: int


@dataclass(frozen=True)
class _Pointer:
    """A validated `expert-<l>-<e>.json` record."""

    layer: int
    expert: int
    generation: str
    revision: int
    optimizer_step: int
    applications: int
    commits: int
    shards: tuple[tuple[int, str], ...]   # (bytes, sha256) per matrix

    KEYS = frozenset({"schema", "config_sha256", "layer", "expert", "generation", "revision", "shards",
                      "parameter_update_applications", "update_commits", "optimizer_step"})

    def to_json(self, config_sha256: str) -> bytes:
        return CanonicalJson.dump({
            "schema": SCHEMA, "config_sha256": config_sha256, "layer": self.layer, "expert": self.expert,
            "generation": self.generation, "revision": self.revision, "optimizer_step": self.optimizer_step,
            "parameter_update_applications": self.applications, "update_commits": self.commits,
            "shards": [{"bytes": b, "sha256": h} for b, h in self.shards]})

    @classmethod
    def from_json(cls, data: bytes, bank: "ExpertBank", layer: int, expert: int) -> "_Pointer":
        v = CanonicalJson.require(CanonicalJson.load(data), set(cls.KEYS), "expert")
        identity_ok = (v["schema"] == SCHEMA and v["config_sha256"] == bank._config_sha256
                       and type(v["layer"]) is int and v["layer"] == layer
                       and type(v["expert"]) is int and v["expert"] == expert
                       and isinstance(v["generation"], str) and _GENERATION.fullmatch(v["generation"]))
        if not identity_ok:
            raise ExpertBankError("expert identity mismatch")
        revision = _int_in(v["revision"], "revision", 1)
        step = _int_in(v["optimizer_step"], "optimizer_step", 0, 1 << 53)
        applications = _int_in(v["parameter_update_applications"], "parameter_update_applications")
        commits = _int_in(v["update_commits"], "update_commits", 0, revision)
        per_expert = bank.config.parameters_per_expert
        if (applications == 0) != (commits == 0) or applications < commits or applications > commits * per_expert:
            raise ExpertBankError("inconsistent update counters")
        shards = v["shards"]
        if not isinstance(shards, list) or len(shards) != len(bank.config.matrix_shapes):
            raise ExpertBankError("expert shard count mismatch")
        parsed = []
        for index, shard in enumerate(shards):
            CanonicalJson.require(shard, {"bytes", "sha256"}, "shard")
            size = _int_in(shard["bytes"], "shard bytes", 1, MAX_SHARD_BYTES)
            digest = shard["sha256"]
            if size != bank.config.shard_bytes(index) or not isinstance(digest, str) or not _SHA256.fullmatch(digest):
                raise ExpertBankError("shard identity or layout mismatch")
            parsed.append((size, digest))
        return cls(layer, expert, v["generation"], revision, step, applications, commits, tuple(parsed))


# -------------------------------------------------------------------- bank ----

class ExpertBank:
    """A fixed logical bank of coded experts; creating or opening a bank
    initializes no expert."""

    def __init__(self, root: Path, config: BankConfig, config_sha256: str):
        self.root, self.config, self._config_sha256 = root, config, config_sha256

    @classmethod
    def create(cls, root, config: BankConfig) -> "ExpertBank":
        if not isinstance(config, BankConfig):
            raise ExpertBankError("config must be BankConfig")
        path = Path(root)
        path.mkdir(parents=False, exist_ok=False)   # never an existing directory, not even an empty one
        if path.is_symlink():
            raise ExpertBankError("bank root must not be a symlink")
        path = path.resolve(strict=True)
        data = CanonicalJson.dump({"schema": SCHEMA, "config": config.to_dict()})
        _Files.create(path / "bank.json", data)
        return cls(path, config, _sha256(data))

    @classmethod
    def open(cls, root) -> "ExpertBank":
        path = Path(root)
        if path.is_symlink() or not path.is_dir():
            raise ExpertBankError("bank root must be a regular directory")
        path = path.resolve(strict=True)
        data = _Files.read(path / "bank.json", MAX_METADATA_BYTES)
        head = CanonicalJson.require(CanonicalJson.load(data), {"schema", "config"}, "bank")
        if head["schema"] != SCHEMA:
            raise ExpertBankError("unsupported bank schema")
        return cls(path, BankConfig.from_dict(head["config"]), _sha256(data))

    # -- names and records ---------------------------------------------------------

    def _verify_config(self) -> None:
        same = (not self.root.is_symlink() and self.root.is_dir() and
                _sha256(_Files.read(self.root / "bank.json", MAX_METADATA_BYTES)) == self._config_sha256)
        if not same:
            raise ExpertBankError("bank configuration changed")

    def _name(self, layer: int, expert: int) -> str:
        _int_in(layer, "layer", 0, self.config.layers - 1)
        _int_in(expert, "expert", 0, self.config.experts_per_layer - 1)
        return f"expert-{layer}-{expert}"

    def _shard(self, layer: int, expert: int, generation: str, index: int) -> Path:
        return self.root / f"{self._name(layer, expert)}-g{generation}-t{index}.vq"

    def _load_pointer(self, layer: int, expert: int) -> _Pointer | None:
        path = self.root / f"{self._name(layer, expert)}.json"
        try:
            data = _Files.read(path, MAX_METADATA_BYTES)
        except FileNotFoundError:
            return None
        return _Pointer.from_json(data, self, layer, expert)

    def _shard_images(self, ptr: _Pointer):
        """Yield (index, verified wire bytes) of a committed generation."""
        for index, (size, digest) in enumerate(ptr.shards):
            path = self._shard(ptr.layer, ptr.expert, ptr.generation, index)
            try:
                data = _Files.read(path, MAX_SHARD_BYTES)
            except FileNotFoundError as exc:
                raise ExpertBankError(f"missing shard {path.name} of a committed generation") from exc
            if len(data) != size or _sha256(data) != digest:
                raise ExpertBankError("shard checksum mismatch")
            yield index, data

    def _decode_shard(self, index: int, data: bytes) -> VQArray:
        try:
            array = VQArray.from_bytes(data, max_bytes=MAX_SHARD_BYTES)
        except ValueError as exc:
            raise ExpertBankError(f"invalid VQ shard: {exc}") from exc
        if array.shape != self.config.matrix_shapes[index] or array.group != self.config.group:
            raise ExpertBankError("decoded shard geometry mismatch")
        return array

    # -- reads -----------------------------------------------------------------------

    def read_expert(self, layer: int, expert: int) -> tuple[VQArray, ...]:
        return self.read_expert_state(layer, expert).tensors

    def read_expert_state(self, layer: int, expert: int) -> ExpertState:
        """Tensors and optimizer bookkeeping of one pointer snapshot."""
        self._verify_config()
        ptr = self._load_pointer(layer, expert)
        if ptr is None:
            raise ExpertBankError("expert is not materialized")
        tensors = tuple(self._decode_shard(i, data) for i, data in self._shard_images(ptr))
        return ExpertState(tensors, ptr.optimizer_step, ptr.revision, ptr.applications)

    def read_expert_to_device(self, layer: int, expert: int, device) -> DeviceExpertState:
        """One pointer snapshot straight into device memory: each shard file
        is read (and verified) into pinned host memory, its header checked,
        and its codebook and codes copied to the device with one asynchronous
        copy each on the current stream. Returns after the copies are
        enqueued (PyTorch's pinned-memory allocator keeps each staging buffer
        until its copy has completed)."""
        import torch
        self._verify_config()
        ptr = self._load_pointer(layer, expert)
        if ptr is None:
            raise ExpertBankError("expert is not materialized")
        dev = torch.device(device)
        codes, books = [], []
        for index, data in self._shard_images(ptr):
            array = self._decode_shard(index, data)        # header and geometry checks
            lay = array.layout
            pinned = torch.empty(len(data), dtype=torch.uint8, pin_memory=True)
            pinned.numpy()[:] = np.frombuffer(data, dtype=np.uint8)
            book_at = len(data) - lay["code_bytes"] - lay["codebook_bytes"]
            book = pinned[book_at:book_at + lay["codebook_bytes"]].view(torch.float32)
            word = pinned[book_at + lay["codebook_bytes"]:].view(torch.int32)
            d_book = torch.empty((ENTRIES, self.config.group), dtype=torch.float32, device=dev)
            d_codes = torch.empty(word.numel(), dtype=torch.int32, device=dev)
            d_book.view(-1).copy_(book, non_blocking=True)
            d_codes.copy_(word, non_blocking=True)
            codes.append(d_codes)
            books.append(d_book)
        return DeviceExpertState(tuple(codes), tuple(books), self.config.matrix_shapes, self.config.group,
                                 ptr.optimizer_step, ptr.revision, ptr.applications)

    # -- writes ----------------------------------------------------------------------

    def write_expert(self, layer: int, expert: int, tensors: Sequence[VQArray], *,
                     updated_count: int = 0, optimizer_step: int | None = None) -> dict:
        """Commit a new generation of one expert (see the module docstring)."""
        self._verify_config()
        base = self._name(layer, expert)
        _int_in(updated_count, "updated_count", 0, self.config.parameters_per_expert)
        if optimizer_step is not None:
            _int_in(optimizer_step, "optimizer_step", 0, 1 << 53)
        shapes = self.config.matrix_shapes
        if not isinstance(tensors, (tuple, list)) or len(tensors) != len(shapes):
            raise ExpertBankError("one VQArray per configured matrix is required")
        for array, shape in zip(tensors, shapes):
            if not isinstance(array, VQArray) or array.shape != shape or array.group != self.config.group:
                raise ExpertBankError("VQArray geometry mismatch")
            if array.layout["serialized_bytes"] > MAX_SHARD_BYTES:
                raise ExpertBankError("shard byte limit exceeded")
        before = self._load_pointer(layer, expert)
        step_before = before.optimizer_step if before else 0
        step = step_before if optimizer_step is None else optimizer_step
        if step < step_before:
            raise ExpertBankError("optimizer_step must not regress")
        if before is not None:
            for _ in self._shard_images(before):    # a corrupt committed generation is refused
                pass
        generation = uuid.uuid4().hex
        images = []
        for array in tensors:
            data = array.to_bytes()
            VQArray.from_bytes(data, max_bytes=MAX_SHARD_BYTES)   # the bytes about to be written parse back
            images.append(data)
        ptr = _Pointer(layer, expert, generation, before.revision + 1 if before else 1, step,
                       updated_count + (before.applications if before else 0),
                       int(updated_count > 0) + (before.commits if before else 0),
                       tuple((len(d), _sha256(d)) for d in images))
        _int_in(ptr.applications, "parameter_update_applications")
        pending = self.root / f"pending-{generation}.json"
        created: list[Path] = []
        try:
            for index, data in enumerate(images):
                path = self._shard(layer, expert, generation, index)
                _Files.create(path, data)
                created.append(path)
            _Files.create(pending, ptr.to_json(self._config_sha256))
            created.append(pending)
            self._verify_config()
            if self._load_pointer(layer, expert) != before:
                raise ExpertBankError("another writer changed this expert")
            _Files.publish(pending, self.root / f"{base}.json")
        except BaseException:
            for path in created:     # a refused commit leaves nothing behind
                path.unlink(missing_ok=True)
            raise
        return {"layer": layer, "expert": expert, "revision": ptr.revision, "optimizer_step": step,
                "materialized_parameters": self.config.parameters_per_expert, "updated_count": updated_count,
                "parameter_update_applications": ptr.applications,
                "generation_bytes": sum(size for size, _ in ptr.shards)}

    def initialize_expert(self, layer: int, expert: int, *, seed: int = 0, zero_optimizer_state: bool = False) -> dict:
        """Deterministic first generation of an expert. Matrix i draws from
        `default_rng(SeedSequence([seed, layer, expert, i]))`: its code words
        uniform u32 (unused high nibbles of the last word cleared), its
        codebook N(0, 1) / sqrt(rows). `zero_optimizer_state=True` (the
        VQAdamW harness contract) makes matrices 1 and 2, the momentum and
        the variance, zero codes with a zero codebook."""
        self._verify_config()
        self._name(layer, expert)
        _int_in(seed, "seed", 0, (1 << 64) - 1)
        if not isinstance(zero_optimizer_state, bool):
            raise ExpertBankError("zero_optimizer_state must be bool")
        if zero_optimizer_state and len(self.config.matrix_shapes) < 3:
            raise ExpertBankError("zero optimizer state needs three matrix roles")
        if self._load_pointer(layer, expert) is not None:
            raise ExpertBankError("expert is already materialized")
        g = self.config.group
        tensors = []
        for index, shape in enumerate(self.config.matrix_shapes):
            lay = storage_layout(shape, g)
            words = lay["code_bytes"] // 4
            if zero_optimizer_state and index in (1, 2):
                tensors.append(VQArray(shape, g, np.zeros(words, np.uint32), np.zeros((ENTRIES, g), np.float32)))
                continue
            rng = np.random.default_rng(np.random.SeedSequence([seed, layer, expert, index]))
            codes = rng.integers(0, 1 << 32, words, dtype=np.uint32)
            used = lay["vectors"] % 8
            if used:
                codes[-1] &= np.uint32((1 << (4 * used)) - 1)
            book = rng.standard_normal((ENTRIES, g), dtype=np.float32)
            book *= np.float32(1.0 / math.sqrt(shape[0]))
            tensors.append(VQArray(shape, g, codes, book))
        return self.write_expert(layer, expert, tensors)

    def stats(self) -> dict:
        """Validate every committed generation and count: experts, parameters,
        declared update applications, committed and on-disk bytes (logical
        file lengths, unreferenced shards of interrupted commits included).
        A coherent census needs a quiescent writer."""
        self._verify_config()
        materialized = applications = updated = committed = disk = 0
        for path in self.root.iterdir():
            info = path.lstat()
            if path.is_symlink() or not stat.S_ISREG(info.st_mode):
                raise ExpertBankError("unexpected nonregular bank entry")
            disk += info.st_size
            match = _POINTER_NAME.fullmatch(path.name)
            if not match:
                continue
            layer, expert = int(match[1]), int(match[2])
            if path.name != f"{self._name(layer, expert)}.json":
                raise ExpertBankError("noncanonical expert filename")
            ptr = self._load_pointer(layer, expert)
            if ptr is None:
                raise ExpertBankError("expert pointer disappeared")
            for _ in self._shard_images(ptr):
                pass
            materialized += 1
            applications += ptr.applications
            updated += int(ptr.commits > 0)
            committed += sum(size for size, _ in ptr.shards)
        return {"potential_experts": self.config.layers * self.config.experts_per_layer,
                "potential_parameters": self.config.potential_parameters,
                "materialized_experts": materialized,
                "materialized_parameters": materialized * self.config.parameters_per_expert,
                "updated_experts": updated, "parameter_update_applications": applications,
                "unique_updated_parameters": None, "committed_payload_bytes": committed, "disk_bytes": disk}


# --------------------------------------------------------------- scheduling ----

@dataclass(frozen=True)
class GainObservation:
    """One held-out measurement of an expert update."""

    loss_before: float
    loss_after: float
    elapsed_s: float
    samples: int
    updated_count: int

    @property
    def gain_per_second(self) -> float:
        if not self.updated_count:
            return 0.0
        return max(0.0, self.loss_before - self.loss_after) / self.elapsed_s


class GainScheduler:
    """Pick experts to update: a share `exploration_fraction` of every
    request (carried across requests as credit) goes round-robin over all
    experts; the rest goes to the best observed loss reduction per second,
    ties to the lower expert id; round-robin fills any remainder. A score is
    an observation, not a promise."""

    def __init__(self, total_experts: int, exploration_fraction: float = 0.2):
        self.total_experts = _int_in(total_experts, "total_experts", 1)
        f = exploration_fraction
        if isinstance(f, bool) or not isinstance(f, (int, float)) or not math.isfinite(f) or not 0 < f <= 1:
            raise ExpertBankError("exploration_fraction must be in (0, 1]")
        self.exploration_fraction = float(f)
        self.observations: dict[int, GainObservation] = {}
        self._cursor = 0
        self._credit = 0.0

    def observe(self, expert: int, loss_before: float, loss_after: float, elapsed_s: float, samples: int,
                updated_count: int, *, heldout: bool = True) -> None:
        _int_in(expert, "expert", 0, self.total_experts - 1)
        if heldout is not True:
            raise ExpertBankError("scheduler requires held-out loss observations")
        for name, value in (("loss_before", loss_before), ("loss_after", loss_after), ("elapsed_s", elapsed_s)):
            if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
                raise ExpertBankError(f"{name} must be finite")
        if elapsed_s <= 0:
            raise ExpertBankError("elapsed_s must be positive")
        _int_in(samples, "samples", 1)
        _int_in(updated_count, "updated_count")
        obs = GainObservation(float(loss_before), float(loss_after), float(elapsed_s), samples, updated_count)
        if not math.isfinite(obs.gain_per_second):
            raise ExpertBankError("gain per second is not finite")
        self.observations[expert] = obs

    def _next_unpicked(self, picked: list[int]) -> int:
        while self._cursor in picked:
            self._cursor = (self._cursor + 1) % self.total_experts
        chosen = self._cursor
        self._cursor = (self._cursor + 1) % self.total_experts
        return chosen

    def select(self, count: int) -> tuple[int, ...]:
        _int_in(count, "count", 1, min(self.total_experts, 4096))
        self._credit += count * self.exploration_fraction
        explore = min(count, int(self._credit + 1e-12))
        self._credit = max(0.0, self._credit - explore)
        picked: list[int] = []
        for _ in range(explore):
            picked.append(self._next_unpicked(picked))
        scored = sorted((-obs.gain_per_second, e) for e, obs in self.observations.items() if obs.gain_per_second > 0)
        for _, e in scored:
            if len(picked) == count:
                break
            if e not in picked:
                picked.append(e)
        while len(picked) < count:
            picked.append(self._next_unpicked(picked))
        return tuple(picked)
