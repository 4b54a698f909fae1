"""ctypes binding of the B200 C ABI (`libalelyon_compute_kit.so`).

Mirrors the reference's `ack` module (`src/alelyon_compute_kit/_kit/python/
ack.py`): the same `Device`, `Buffer`, error classes, `AckAbiInfo` /
`AckDeviceInfo` structures, `abi_info`, `capability_record` and library
lookup (`ACK_LIBRARY`, then the package's `_lib/`). `VQDevice` relies on the
same private members the reference's uses (`Device._lock`, `_lib.cdll`,
`_require_open`, `_handle`, `buffer`; `Buffer._handle`).

Two deliberate differences, both at the handshake (reference ack.py:862-905):
this library carries the core device entries and the vq4/v1 extension only,
so the handshake requires ABI 14, the 96-byte `AckAbiInfo` and the vq symbols,
and does NOT require the reference's twelve dense operator families, whose
schema words this library reports as 0 (absent). No stub of those families
is exported or bound here.

`Device()` opens a CUDA device (`ACK_DEVICE=gpu:<n>`, or the current CUDA
device). There is no CPU fallback: without the library or a B200, `Device()`
raises `AckUnavailable`.
"""
from __future__ import annotations

import ctypes
import operator
import os
import sys
import threading
import warnings
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent

ACK_OK = 0
ACK_ERR_NULL = -1
ACK_ERR_VULKAN = -2      # a driver (CUDA runtime) error
ACK_ERR_SHAPE = -3
ACK_ERR_SIZE = -4
ACK_ERR_LIVE_BUFFERS = -5
ACK_ERR_CLOSED = -6
ACK_ERR_FOREIGN = -7
ACK_ERR_FREED = -8
ACK_ERR_ABI = -9
ACK_ERR_POISONED = -10
ACK_ERR_UNSUPPORTED_OP = -11
ACK_ERR_TIMING = -12

ACK_ABI_VERSION = 14
ACK_DEVICE_INFO_VERSION = 1
ACK_VQ_SCHEMA = 1
ACK_VQ2_SCHEMA = 1

_MAX_NBYTES = min((1 << 64) - 1, sys.maxsize)
_POD_SIZES = {"b": (1,), "i": (1, 2, 4, 8), "u": (1, 2, 4, 8), "f": (2, 4, 8), "c": (8, 16)}


class AckAbiInfo(ctypes.Structure):
    """What `ack_abi_info` fills in (96 bytes, the reference layout)."""

    _fields_ = [
        ("size", ctypes.c_uint32), ("version", ctypes.c_uint32), ("operators", ctypes.c_uint64),
        ("shaders", ctypes.c_uint64), ("build", ctypes.c_uint64),
        ("op_schema_matmul_bf16", ctypes.c_uint32), ("op_schema_cast", ctypes.c_uint32),
        ("capability_streams", ctypes.c_uint32), ("capability_rng", ctypes.c_uint32),
        ("capability_optimizer", ctypes.c_uint32), ("capability_serialization", ctypes.c_uint32),
        ("op_schema_matmul_f32", ctypes.c_uint32), ("op_schema_pointwise", ctypes.c_uint32),
        ("op_schema_reduce", ctypes.c_uint32), ("op_schema_rowwise", ctypes.c_uint32),
        ("op_schema_loss", ctypes.c_uint32), ("op_schema_embedding", ctypes.c_uint32),
        ("op_schema_matmul_f16", ctypes.c_uint32), ("op_schema_index", ctypes.c_uint32),
        ("op_schema_convert", ctypes.c_uint32), ("op_schema_intwise", ctypes.c_uint32),
    ]


class AckDeviceInfo(ctypes.Structure):
    """What `ack_device_info` fills in (616 bytes, the reference layout)."""

    _fields_ = [
        ("size", ctypes.c_uint32), ("version", ctypes.c_uint32), ("api_version", ctypes.c_uint32),
        ("driver_version_raw", ctypes.c_uint32), ("driver_id", ctypes.c_uint32),
        ("vendor_id", ctypes.c_uint32), ("device_id", ctypes.c_uint32), ("device_type", ctypes.c_uint32),
        ("device_uuid", ctypes.c_uint8 * 16), ("driver_uuid", ctypes.c_uint8 * 16),
        ("features", ctypes.c_uint64), ("subgroup_size", ctypes.c_uint32),
        ("timestamp_valid_bits", ctypes.c_uint32), ("timestamp_period_ns", ctypes.c_float),
        ("max_push_constant_bytes", ctypes.c_uint32), ("device_local_bytes", ctypes.c_uint64),
        ("max_storage_buffer_bytes", ctypes.c_uint64), ("max_workgroup_invocations", ctypes.c_uint32),
        ("max_workgroup_count", ctypes.c_uint32 * 3), ("max_workgroup_size", ctypes.c_uint32 * 3),
        ("matmul_tile", ctypes.c_uint32), ("matmul_k_multiple", ctypes.c_uint32),
        ("matmul_layouts", ctypes.c_uint32), ("matmul_operand_dtype", ctypes.c_uint32),
        ("matmul_result_dtype", ctypes.c_uint32), ("cast_modes", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32), ("identity", ctypes.c_uint64),
        ("device_name", ctypes.c_char * 256), ("driver_name", ctypes.c_char * 64),
        ("driver_info", ctypes.c_char * 128),
    ]


class AckVqOperands(ctypes.Structure):
    """Operands of `ack_vq_launch`: device pointers with byte capacities."""

    _fields_ = [("size", ctypes.c_uint32), ("nslots", ctypes.c_uint32),
                ("bytes", ctypes.c_uint64 * 8), ("ptr", ctypes.c_void_p * 8)]


class AckError(RuntimeError):
    """A kit call returned an error code; the message is the kit's."""


class AckUnavailable(AckError):
    """No shared library, or no usable CUDA device."""


class AckShapeError(AckError):
    """A shape the kit refuses."""


class AckPoisoned(AckError):
    """The device's CUDA context failed; every later call on it refuses.
    Close it and start a new process."""


def _kit_error(what: str, rc: int, message: str) -> AckError:
    cls = AckPoisoned if rc == ACK_ERR_POISONED else AckError
    return cls(f"{what}: {message}")


def _checked_nbytes(nbytes) -> int:
    if isinstance(nbytes, (bool, np.bool_)):
        raise AckError("nbytes must be a positive integer, not a boolean")
    try:
        count = operator.index(nbytes)
    except TypeError as exc:
        raise AckError("nbytes must be a positive integer") from exc
    if not 0 < count <= _MAX_NBYTES:
        raise AckError(f"nbytes must be in 1..{_MAX_NBYTES}")
    return count


def _pod_dtype(dtype) -> np.dtype:
    try:
        result = np.dtype(dtype)
    except (TypeError, ValueError) as exc:
        raise AckError("unsupported buffer dtype") from exc
    if (result.hasobject or result.fields is not None or result.subdtype is not None
            or result.itemsize not in _POD_SIZES.get(result.kind, ())):
        raise AckError(f"unsupported buffer dtype {result} is refused; use a plain fixed-width numeric or bool dtype")
    return result


def _library_candidates() -> list[Path]:
    out: list[Path] = []
    if os.environ.get("ACK_LIBRARY"):
        out.append(Path(os.environ["ACK_LIBRARY"]))
    out.append(_HERE / "_lib" / "libalelyon_compute_kit.so")
    out.append(_HERE / "libalelyon_compute_kit.so")
    return out


def library_path() -> Path | None:
    for candidate in _library_candidates():
        if candidate.is_file():
            return candidate
    return None


def to_bf16(x) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even; NaNs stay quiet NaNs."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = bits + np.uint32(0x7FFF) + ((bits >> 16) & 1)
    is_nan = ((bits & 0x7F800000) == 0x7F800000) & ((bits & 0x007FFFFF) != 0)
    return np.where(is_nan, (bits >> 16) | 0x0040, rounded >> 16).astype(np.uint16)


def from_bf16(h) -> np.ndarray:
    """bf16 bit patterns -> float32, exactly."""
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class _Lib:
    def __init__(self, path: Path) -> None:
        self.path = path
        try:
            self.cdll = ctypes.CDLL(str(path))
        except OSError as exc:
            raise AckUnavailable(f"cannot load {path}: {exc}") from exc
        self.info: AckAbiInfo | None = None
        try:
            self._declare()
        except AttributeError as exc:
            raise AckUnavailable(f"library {path} lacks a core or vq symbol ({exc})") from exc

    def _declare(self) -> None:
        c = self.cdll
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        c.ack_abi_info.restype = ctypes.c_int32
        c.ack_abi_info.argtypes = [ctypes.POINTER(AckAbiInfo), sz]
        c.ack_device_info.restype = ctypes.c_int32
        c.ack_device_info.argtypes = [vp, ctypes.POINTER(AckDeviceInfo), sz]
        c.ack_open.restype = vp
        c.ack_open.argtypes = []
        c.ack_close.restype = ctypes.c_int32
        c.ack_close.argtypes = [vp]
        c.ack_device_name.restype = ctypes.c_int32
        c.ack_device_name.argtypes = [vp, ctypes.c_char_p, sz]
        c.ack_live_objects.restype = ctypes.c_int32
        c.ack_live_objects.argtypes = [vp, ctypes.POINTER(ctypes.c_int64)]
        c.ack_leaked_on_poison.restype = ctypes.c_int32
        c.ack_leaked_on_poison.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64)]
        c.ack_last_error.restype = ctypes.c_int32
        c.ack_last_error.argtypes = [ctypes.c_char_p, sz]
        c.ack_buffer_alloc.restype = vp
        c.ack_buffer_alloc.argtypes = [vp, ctypes.c_uint64]
        c.ack_buffer_free.restype = ctypes.c_int32
        c.ack_buffer_free.argtypes = [vp, vp]
        c.ack_upload.restype = ctypes.c_int32
        c.ack_upload.argtypes = [vp, vp, vp, sz]
        c.ack_download.restype = ctypes.c_int32
        c.ack_download.argtypes = [vp, vp, vp, sz]
        c.ack_vq_schema.restype = ctypes.c_uint32
        c.ack_vq_schema.argtypes = []
        c.ack_vq.restype = ctypes.c_int32
        c.ack_vq.argtypes = [vp] * 7 + [vp, sz]
        c.ack_vq2_schema.restype = ctypes.c_uint32
        c.ack_vq2_schema.argtypes = []
        c.ack_vq2.restype = ctypes.c_int32
        c.ack_vq2.argtypes = [vp, ctypes.POINTER(vp), sz, vp, sz]
        c.ack_vq_launch.restype = ctypes.c_int32
        c.ack_vq_launch.argtypes = [vp, sz, ctypes.POINTER(AckVqOperands), vp]
        c.ack_vq_plan_probe.restype = ctypes.c_int32
        c.ack_vq_plan_probe.argtypes = [vp, sz, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint32),
                                        ctypes.POINTER(ctypes.c_uint32)]
        c.ack_vq_plan_validate_buffers.restype = ctypes.c_int32
        c.ack_vq_plan_validate_buffers.argtypes = [vp, sz, ctypes.POINTER(ctypes.c_uint64),
                                                   ctypes.POINTER(ctypes.c_uint64), sz]
        c.ack_vq_plan_validate_dispatch.restype = ctypes.c_int32
        c.ack_vq_plan_validate_dispatch.argtypes = [vp, sz, ctypes.POINTER(ctypes.c_uint32)]
        c.ack_inject_fault.restype = ctypes.c_int32
        c.ack_inject_fault.argtypes = [vp, ctypes.c_int32, ctypes.c_int32]
        c.ack_kernel_manifest.restype = ctypes.c_int32
        c.ack_kernel_manifest.argtypes = [ctypes.c_char_p, sz, ctypes.POINTER(sz)]
        u32, dp = ctypes.c_uint32, ctypes.POINTER(ctypes.c_double)
        # the NF4 comparator (ffi.rs:7365 ack_nf4_decode, :8017 ack_gemv_nf4) and its device-pointer forms
        c.ack_nf4_decode.restype = ctypes.c_int32
        c.ack_nf4_decode.argtypes = [vp] * 9 + [u32] * 6 + [dp]
        c.ack_gemv_nf4.restype = ctypes.c_int32
        c.ack_gemv_nf4.argtypes = [vp] * 10 + [u32] * 9 + [dp]
        c.ack_nf4_decode_launch.restype = ctypes.c_int32
        c.ack_nf4_decode_launch.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64)] + [u32] * 6 + [vp]
        c.ack_gemv_nf4_launch.restype = ctypes.c_int32
        c.ack_gemv_nf4_launch.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64)] + [u32] * 9 + [vp]

    def last_error(self) -> str:
        buf = ctypes.create_string_buffer(1024)
        self.cdll.ack_last_error(buf, len(buf))
        return buf.value.decode("utf-8", errors="replace")

    def abi_info(self) -> AckAbiInfo:
        info = AckAbiInfo()
        rc = self.cdll.ack_abi_info(ctypes.byref(info), ctypes.sizeof(info))
        if rc != ACK_OK:
            raise AckUnavailable(f"ack_abi_info refused ({rc}): {self.last_error()}")
        return info

    def handshake(self) -> AckAbiInfo:
        """Refuse a library whose ABI version, struct size or vq schema is not
        the one this module is written for."""
        info = self.abi_info()
        if info.size != ctypes.sizeof(AckAbiInfo):
            raise AckUnavailable(f"library reports an AckAbiInfo of {info.size} bytes; this module's is "
                                 f"{ctypes.sizeof(AckAbiInfo)}")
        if info.version != ACK_ABI_VERSION:
            raise AckUnavailable(f"library ABI version {info.version} is not the {ACK_ABI_VERSION} this module "
                                 "is written for")
        if self.cdll.ack_vq_schema() != ACK_VQ_SCHEMA:
            raise AckUnavailable("incompatible vq4 extension schema")
        if self.cdll.ack_vq2_schema() != ACK_VQ2_SCHEMA:
            raise AckUnavailable("incompatible vq4 B200 extension schema")
        self.info = info
        return info


_LIB: _Lib | None = None
_LIB_LOCK = threading.Lock()


def _lib() -> _Lib:
    global _LIB
    with _LIB_LOCK:
        if _LIB is None:
            path = library_path()
            if path is None:
                raise AckUnavailable(
                    "libalelyon_compute_kit.so is not built; run `make -C alelyon-compute-kit_b200` "
                    "(or __graft_entry__.build()), or point ACK_LIBRARY at it")
            lib = _Lib(path)
            lib.handshake()
            _LIB = lib
        return _LIB


def abi_info() -> AckAbiInfo:
    """The loaded library's ABI description."""
    lib = _lib()
    return lib.info if lib.info is not None else lib.handshake()


def kernel_manifest() -> dict:
    """The library's kernel manifest: sha256 of each source it was built
    from, the kernels each defines, nvcc release and flags, arch."""
    import json
    lib = _lib()
    need = ctypes.c_size_t()
    lib.cdll.ack_kernel_manifest(None, 0, ctypes.byref(need))
    buf = ctypes.create_string_buffer(need.value)
    rc = lib.cdll.ack_kernel_manifest(buf, need.value, None)
    if rc != ACK_OK:
        raise AckError(f"ack_kernel_manifest refused ({rc}): {lib.last_error()}")
    return json.loads(buf.value.decode())


def dispatch_stats_available() -> bool:
    """This library has no `ack_dispatch_stats`; time with CUDA events instead."""
    return False


def _api_version_string(packed: int) -> str:
    return f"{(packed >> 22) & 0x7F}.{(packed >> 12) & 0x3FF}.{packed & 0xFFF}"


def capability_record(abi: AckAbiInfo, info: AckDeviceInfo) -> dict:
    """A JSON-serialisable record of what a run ran on (the reference's
    `capability_record`, ack.py:527-596, with the fields this library fills)."""
    return {
        "schema": 1,
        "abi": {
            "version": abi.version, "operators": abi.operators,
            "vq_schema": ACK_VQ_SCHEMA, "vq2_schema": ACK_VQ2_SCHEMA,
            "shaders": f"{abi.shaders:016x}", "build": f"{abi.build:016x}",
        },
        "device": {
            "name": info.device_name.decode("utf-8", errors="replace"),
            "vendor_id": info.vendor_id, "device_id": info.device_id, "device_type": info.device_type,
            "device_uuid": bytes(info.device_uuid).hex(),
            "driver_version_raw": info.driver_version_raw,
            "driver_name": info.driver_name.decode("utf-8", errors="replace"),
            "driver_info": info.driver_info.decode("utf-8", errors="replace"),
            "api_version": _api_version_string(info.api_version),
            "subgroup_size": info.subgroup_size,
            "device_local_bytes": info.device_local_bytes,
            "limits": {
                "max_storage_buffer_bytes": info.max_storage_buffer_bytes,
                "max_workgroup_invocations": info.max_workgroup_invocations,
                "max_workgroup_count": list(info.max_workgroup_count),
                "max_workgroup_size": list(info.max_workgroup_size),
            },
            "identity": f"{info.identity:016x}",
        },
    }


class Buffer:
    """A device buffer (cudaMalloc); explicit free() releases it."""

    def __init__(self, device: "Device", nbytes: int) -> None:
        self._device = device
        self._handle = None
        self._nbytes = _checked_nbytes(nbytes)
        with device._lock:
            device._require_open()
            handle = device._lib.cdll.ack_buffer_alloc(device._handle, self._nbytes)
            if not handle:
                raise AckError(f"buffer alloc: {device._lib.last_error()}")
            device._buffers.add(handle)
            self._handle = handle

    @property
    def nbytes(self) -> int:
        return self._nbytes

    def _require_live(self) -> None:
        if not self._handle:
            raise AckError("buffer has been freed")
        self._device._require_open()

    def upload_bytes(self, data) -> None:
        with self._device._lock:
            self._require_live()
            view = memoryview(data).cast("B")
            if not view.contiguous:
                raise AckError("upload needs a contiguous buffer")
            if view.nbytes != self.nbytes:
                raise AckError(f"upload of {view.nbytes} bytes into a {self.nbytes}-byte buffer")
            source = (ctypes.c_char * view.nbytes).from_buffer_copy(view)
            lib = self._device._lib
            rc = lib.cdll.ack_upload(self._device._handle, self._handle, ctypes.cast(source, ctypes.c_void_p),
                                     view.nbytes)
            if rc != ACK_OK:
                raise _kit_error("upload", rc, lib.last_error())

    def download_bytes(self) -> bytes:
        with self._device._lock:
            self._require_live()
            out = (ctypes.c_char * self.nbytes)()
            lib = self._device._lib
            rc = lib.cdll.ack_download(self._device._handle, self._handle, ctypes.cast(out, ctypes.c_void_p),
                                       self.nbytes)
            if rc != ACK_OK:
                raise _kit_error("download", rc, lib.last_error())
            return bytes(out)

    def upload(self, data) -> None:
        with self._device._lock:
            self._require_live()
            array = np.asarray(data)
            _pod_dtype(array.dtype)
            if array.nbytes != self.nbytes:
                raise AckError(f"upload of {array.nbytes} bytes into a {self.nbytes}-byte buffer")
            raw = np.ascontiguousarray(array)
            lib = self._device._lib
            rc = lib.cdll.ack_upload(self._device._handle, self._handle, raw.ctypes.data, raw.nbytes)
            if rc != ACK_OK:
                raise _kit_error("upload", rc, lib.last_error())

    def download(self, dtype, out: np.ndarray | None = None) -> np.ndarray:
        with self._device._lock:
            self._require_live()
            dtype = _pod_dtype(dtype)
            if self.nbytes % dtype.itemsize:
                raise AckError(f"buffer size {self.nbytes} is not divisible by dtype itemsize {dtype.itemsize}")
            if out is None:
                out = np.empty(self.nbytes // dtype.itemsize, dtype=dtype)
            elif out.dtype != dtype or out.nbytes != self.nbytes or not out.flags.c_contiguous:
                raise AckError("download target must be a contiguous array of the buffer's size and dtype")
            lib = self._device._lib
            rc = lib.cdll.ack_download(self._device._handle, self._handle, out.ctypes.data, out.nbytes)
            if rc != ACK_OK:
                raise _kit_error("download", rc, lib.last_error())
            return out

    def free(self) -> None:
        with self._device._lock:
            if self._handle:
                self._device._require_open()
                lib = self._device._lib
                rc = lib.cdll.ack_buffer_free(self._device._handle, self._handle)
                self._device._buffers.discard(self._handle)
                self._handle = None
                if rc != ACK_OK:
                    raise _kit_error("free", rc, lib.last_error())

    def __del__(self) -> None:  # best effort; explicit free() is the contract
        try:
            self.free()
        except AckError as exc:
            try:
                warnings.warn(f"ack.Buffer finaliser: {exc}", ResourceWarning, stacklevel=2)
            except Exception:
                pass
        except Exception:
            pass


class Device:
    """One CUDA device with its own stream. Free its buffers before close();
    calls through one Device are serialised."""

    def __init__(self) -> None:
        self._lock = threading.RLock()
        self._buffers: set[int] = set()
        self._handle = None
        self._lib = lib = _lib()
        self._handle = lib.cdll.ack_open()
        if not self._handle:
            raise AckUnavailable(f"ack_open: {lib.last_error()}")
        try:
            buf = ctypes.create_string_buffer(256)
            rc = lib.cdll.ack_device_name(self._handle, buf, len(buf))
            if rc != ACK_OK:
                raise AckError(f"device name: {lib.last_error()}")
            self.name = buf.value.decode("utf-8", errors="replace")
            info = AckDeviceInfo()
            rc = lib.cdll.ack_device_info(self._handle, ctypes.byref(info), ctypes.sizeof(info))
            if rc != ACK_OK:
                raise AckError(f"device info: {lib.last_error()}")
            if info.size != ctypes.sizeof(AckDeviceInfo) or info.version != ACK_DEVICE_INFO_VERSION:
                raise AckUnavailable(f"library reports an AckDeviceInfo of {info.size} bytes version {info.version}")
            self.info = info
            self.identity = info.identity
        except BaseException:
            self.close()
            raise
        # The operator entries enqueue work and return; no duration exists at
        # that moment, so this is NaN after a successful call (reference
        # ack.py:1095-1116). Time with CUDA events instead.
        self.last_ms: float | None = None

    def capability_record(self) -> dict:
        with self._lock:
            self._require_open()
            return capability_record(self._lib.info if self._lib.info is not None else self._lib.handshake(),
                                     self.info)

    def _require_open(self) -> None:
        if not self._handle:
            raise AckError("device is closed")

    def live_objects(self) -> int:
        with self._lock:
            self._require_open()
            out = ctypes.c_int64()
            rc = self._lib.cdll.ack_live_objects(self._handle, ctypes.byref(out))
            if rc != ACK_OK:
                raise _kit_error("live objects", rc, self._lib.last_error())
            return int(out.value)

    def leaked_on_poison(self) -> int:
        with self._lock:
            self._require_open()
            out = ctypes.c_uint64()
            rc = self._lib.cdll.ack_leaked_on_poison(self._handle, ctypes.byref(out))
            if rc != ACK_OK:
                raise _kit_error("leaked on poison", rc, self._lib.last_error())
            return int(out.value)

    def close(self) -> None:
        """Close only on ACK_OK; a refusal keeps the handle valid."""
        with self._lock:
            if self._handle:
                if self._buffers:
                    raise AckError("device has live buffers still allocated; free them before close")
                rc = self._lib.cdll.ack_close(self._handle)
                if rc == ACK_ERR_CLOSED:
                    self._handle = None
                    raise AckError(f"close: {self._lib.last_error()}")
                if rc != ACK_OK:
                    raise AckError(f"close: {self._lib.last_error()}")
                self._handle = None

    def __enter__(self) -> "Device":
        with self._lock:
            self._require_open()
            return self

    def __exit__(self, *exc) -> None:
        self.close()

    def buffer(self, nbytes: int) -> Buffer:
        return Buffer(self, nbytes)
