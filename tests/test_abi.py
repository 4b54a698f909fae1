"""Host-only C ABI checks: the library loads, exports every symbol the
header declares, keeps the reference's struct layouts, and refuses bad
calls by code and name before touching any handle (the reference's
`_kit/tests/vq4_abi.rs`). No device is opened."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from abi_util import block, last_error, lib
from alelyon_compute_kit import ack

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "alelyon_compute_kit.h"
FORGED = ctypes.c_void_p(2 ** 64 - 1)   # usize::MAX, never a live id


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ack_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry():
    path = ack.library_path()
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # nothing beyond the header is exported
    assert sorted(n for n in exported if n.startswith("ack_")) == names


def test_struct_layouts_are_the_references():
    assert ctypes.sizeof(ack.AckAbiInfo) == 96
    assert ctypes.sizeof(ack.AckDeviceInfo) == 616
    assert ack.AckDeviceInfo.identity.offset == 160
    assert ack.AckDeviceInfo.device_name.offset == 168
    info = ack.abi_info()
    assert info.size == 96 and info.version == ack.ACK_ABI_VERSION == 14
    assert info.operators == 0  # no dense operator family is claimed


def test_kernel_manifest_names_the_sources_the_library_was_built_from():
    """The CUDA counterpart of the reference's MANIFEST.json vq4 entry: every
    source's sha256 must be that of the file in this tree (a stale build
    fails here), and AckAbiInfo.shaders hashes the same text."""
    import hashlib
    m = ack.kernel_manifest()
    assert m["arch"] == "sm_100a" and m["format"] == "vq4/v1"
    assert "compute_100a" in m["flags"] and "release 12" in m["compiler"]
    pkg = ROOT / "alelyon-compute-kit_b200"
    for name, entry in m["sources"].items():
        path = next(p for p in [pkg / "csrc" / name, ROOT / "include" / name] if p.exists())
        assert entry["source_sha256"] == hashlib.sha256(path.read_bytes()).hexdigest(), name
    kernels = set().union(*(set(entry["kernels"]) for entry in m["sources"].values()))
    assert {"k_decode", "k_encode", "k_encode_tc", "k_dense_t32", "k_dense_pair", "k_coded_lut", "k_adamw_encode",
            "k_fit_assign", "k_encode_static"} <= kernels
    c = lib().cdll
    need = ctypes.c_size_t()
    assert c.ack_kernel_manifest(None, 0, ctypes.byref(need)) == ack.ACK_OK
    short = ctypes.create_string_buffer(8)
    assert c.ack_kernel_manifest(short, 8, None) == ack.ACK_ERR_SIZE
    assert c.ack_kernel_manifest(None, 0, None) == ack.ACK_ERR_NULL
    buf = ctypes.create_string_buffer(need.value)
    assert c.ack_kernel_manifest(buf, need.value, None) == ack.ACK_OK
    h = 0xcbf29ce484222325
    for byte in buf.value:
        h = ((h ^ byte) * 0x100000001b3) & (2 ** 64 - 1)
    assert ack.abi_info().shaders == h


def test_optional_extension_does_not_relabel_existing_abi_layout():  # vq4_abi.rs:30
    c = lib().cdll
    assert c.ack_vq_schema() == 1
    assert c.ack_vq2_schema() == 1


def call_vq(plan, length):
    c = lib().cdll
    return c.ack_vq(FORGED, FORGED, FORGED, FORGED, FORGED, FORGED, FORGED, plan, length)


def test_null_and_wrong_sized_blocks_refuse_before_any_handle_lookup():  # vq4_abi.rs:39
    assert call_vq(None, 32) == ack.ACK_ERR_NULL
    assert "null plan" in last_error()
    plan = block([0, 1, 1, 1, 8, 16, 0, 0])
    for length in (0, 1, 31, 33, 2 ** 63):
        assert call_vq(plan, length) == ack.ACK_ERR_SIZE
        assert "plan has" in last_error()


@pytest.mark.parametrize("words,code,name", [
    ([4, 1, 1, 1, 8, 16, 0, 0], ack.ACK_ERR_SHAPE, "vq-operation-out-of-range"),
    ([0, 1, 1, 1, 4, 16, 0, 0], ack.ACK_ERR_SHAPE, "vq-unsupported-group"),
    ([0, 1, 1, 1, 8, 15, 0, 0], ack.ACK_ERR_SHAPE, "vq-codebook-entries-not-16"),
    ([2, 1, 1, 1, 8, 16, 4, 0], ack.ACK_ERR_SHAPE, "vq-unsupported-flags"),
    ([0, 1, 1, 1, 8, 16, 0, 1], ack.ACK_ERR_SHAPE, "vq-nonzero-reserved-word"),
    ([0, 0, 1, 1, 8, 16, 0, 0], ack.ACK_ERR_SHAPE, "vq-invalid-geometry"),
    ([0, 2 ** 32 - 1, 1, 1, 8, 16, 0, 0], ack.ACK_ERR_SIZE, "vq-address-limit-exceeded"),
    ([3, 1 << 28, 1, 1, 8, 16, 0, 0], ack.ACK_ERR_SIZE, "vq-address-limit-exceeded"),
])
def test_malformed_schema_refuses_by_name_before_any_device_lookup(words, code, name):  # vq4_abi.rs:50
    plan = block(words)
    assert call_vq(plan, len(plan)) == code
    assert last_error().endswith(name), last_error()


def test_all_valid_operations_reach_closed_device_refusal_without_dereference():  # vq4_abi.rs:100
    for op in range(4):
        plan = block([op, 1, 1, 1, 8, 16, 0, 0])
        assert call_vq(plan, len(plan)) == ack.ACK_ERR_CLOSED
        assert "is not open" in last_error()


def test_excessive_scalar_matmul_work_refuses_before_device_lookup():  # vq4_abi.rs:112
    plan = block([2, 1024, 1024, 257, 8, 16, 0, 0])
    assert call_vq(plan, len(plan)) == ack.ACK_ERR_SIZE
    assert last_error().endswith("vq-matmul-work-limit")


def test_vq2_refuses_before_device_lookup_and_reaches_closed_device():
    c = lib().cdll
    slots = (ctypes.c_void_p * 8)(*([FORGED.value] * 8))
    plan = block([16, 1, 8, 8, 8, 16, 2, 0, 1, 0, 0, 0, 0, 0, 0, 0])
    assert c.ack_vq2(FORGED, slots, 8, None, 64) == ack.ACK_ERR_NULL
    assert c.ack_vq2(FORGED, slots, 8, plan, 32) == ack.ACK_ERR_SIZE
    assert c.ack_vq2(FORGED, slots, 7, plan, 64) == ack.ACK_ERR_SIZE
    assert c.ack_vq2(FORGED, slots, 8, plan, 64) == ack.ACK_ERR_CLOSED
    assert "is not open" in last_error()


def test_pipelined_host_product_refuses_before_device_lookup():
    """ack_vq2_dense_host: null pointers, a wrong plan size, a malformed or
    non-dense plan refuse before any handle is looked up; a forged device
    reaches the closed-device refusal."""
    c = lib().cdll
    fn = c.ack_vq2_dense_host
    fn.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
    x = (ctypes.c_float * 64)()
    y = (ctypes.c_float * 64)()
    st = ctypes.c_uint32()
    args = lambda plan, n: (FORGED, plan, n, FORGED, FORGED, ctypes.addressof(x), ctypes.addressof(y), 0,  # noqa: E731
                            ctypes.addressof(st))
    dense = block([16, 1, 8, 8, 8, 16, 2, 0, 1, 0, 0, 0, 0, 0, 0, 0])
    assert fn(FORGED, None, 64, FORGED, FORGED, ctypes.addressof(x), ctypes.addressof(y), 0,
              ctypes.addressof(st)) == ack.ACK_ERR_NULL
    assert fn(FORGED, dense, 64, FORGED, FORGED, None, ctypes.addressof(y), 0, ctypes.addressof(st)) == ack.ACK_ERR_NULL
    assert fn(*args(dense, 32)) == ack.ACK_ERR_SIZE
    assert fn(*args(block([16, 1, 8, 8, 12, 16, 2, 0, 1, 0, 0, 0, 0, 0, 0, 0]), 64)) == ack.ACK_ERR_SHAPE
    assert last_error().endswith("vq2-unsupported-group")
    assert fn(*args(block([21, 64, 1, 1, 8, 16, 0, 0, 1, 0, 0, 0, 0, 0, 0, 0]), 64)) == ack.ACK_ERR_UNSUPPORTED_OP
    assert fn(*args(dense, 64)) == ack.ACK_ERR_CLOSED


def _cuda_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_cuda_present(), reason="fake device pointers: run only where no GPU can be reached")
def test_device_pointer_entry_refuses_without_launching():
    """Every call below must be refused by admission; the pointers are fake,
    so the test runs only on a machine without a GPU."""
    c = lib().cdll
    ops = ack.AckVqOperands()
    ops.size = ctypes.sizeof(ops)
    ops.nslots = 6
    plan = block([1, 512, 1, 1, 8, 16, 0, 0])   # decode 512 values: 32 code bytes in, 2048 bytes out
    assert c.ack_vq_launch(plan, len(plan), None, None) == ack.ACK_ERR_NULL
    small = ack.AckVqOperands()
    small.size = 8
    assert c.ack_vq_launch(plan, len(plan), ctypes.byref(small), None) == ack.ACK_ERR_ABI
    # a null operand where the plan reads one
    assert c.ack_vq_launch(plan, len(plan), ctypes.byref(ops), None) == ack.ACK_ERR_SHAPE
    assert last_error().endswith("vq-null-allocation-identity")
    # capacities are checked against the plan
    for i in range(6):
        ops.ptr[i] = 4096 * (i + 1) * 1024
        ops.bytes[i] = 4096
    ops.bytes[4] = 2047
    assert c.ack_vq_launch(plan, len(plan), ctypes.byref(ops), None) == ack.ACK_ERR_SIZE
    assert last_error().endswith("vq-binding-4-too-small")
    # overlapping output and input ranges
    ops.bytes[4] = 4096
    ops.ptr[4] = ops.ptr[0] + 16
    assert c.ack_vq_launch(plan, len(plan), ctypes.byref(ops), None) == ack.ACK_ERR_SHAPE
    assert last_error().endswith("vq-output-aliases-input")
    ops.ptr[4] = 999 * 1024 * 1024
    ops.ptr[5] = ops.ptr[4]
    assert c.ack_vq_launch(plan, len(plan), ctypes.byref(ops), None) == ack.ACK_ERR_SHAPE
    assert last_error().endswith("vq-status-aliases-operand")
    ops.ptr[5] = 998 * 1024 * 1024 + 2
    assert c.ack_vq_launch(plan, len(plan), ctypes.byref(ops), None) == ack.ACK_ERR_SHAPE
    assert last_error().endswith("operand-misaligned")


def test_core_entries_refuse_forged_and_null_handles():
    c = lib().cdll
    assert c.ack_close(None) == ack.ACK_ERR_NULL
    assert c.ack_close(FORGED) == ack.ACK_ERR_CLOSED
    assert not c.ack_buffer_alloc(FORGED, 16)
    assert not c.ack_buffer_alloc(FORGED, 0) and last_error() == "zero-byte buffer"
    data = ctypes.create_string_buffer(16)
    assert c.ack_upload(FORGED, FORGED, None, 16) == ack.ACK_ERR_NULL
    assert c.ack_upload(FORGED, FORGED, data, 16) == ack.ACK_ERR_CLOSED
    assert c.ack_download(FORGED, FORGED, data, 16) == ack.ACK_ERR_CLOSED
    assert c.ack_buffer_free(FORGED, FORGED) == ack.ACK_ERR_CLOSED
    out = ctypes.c_int64()
    assert c.ack_live_objects(FORGED, ctypes.byref(out)) == ack.ACK_ERR_CLOSED
    info = ack.AckAbiInfo()
    assert c.ack_abi_info(ctypes.byref(info), 95) == ack.ACK_ERR_ABI
    dinfo = ack.AckDeviceInfo()
    assert c.ack_device_info(FORGED, ctypes.byref(dinfo), 615) == ack.ACK_ERR_ABI
    assert c.ack_device_info(FORGED, ctypes.byref(dinfo), ctypes.sizeof(dinfo)) == ack.ACK_ERR_CLOSED
    buf = ctypes.create_string_buffer(8)
    assert c.ack_last_error(buf, 8) == 0 and len(buf.value) <= 7


def test_fault_injection_is_closed_unless_enabled(monkeypatch):
    monkeypatch.delenv("ACK_FAULT_INJECTION", raising=False)
    assert lib().cdll.ack_inject_fault(FORGED, 0, 700) == ack.ACK_ERR_UNSUPPORTED_OP
    monkeypatch.setenv("ACK_FAULT_INJECTION", "1")
    assert lib().cdll.ack_inject_fault(FORGED, 0, 700) == ack.ACK_ERR_CLOSED
