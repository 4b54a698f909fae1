"""Device-runtime behaviour through the C ABI on a real device: handle
refusals, live-buffer close, and failure detection by host-injected faults
(no GPU fault is ever caused: the injected code replaces the result of a
real, successful wait or allocation)."""
import ctypes

import numpy as np
import pytest

from alelyon_compute_kit import ack, vq

pytestmark = pytest.mark.gpu


def test_foreign_freed_and_live_buffer_refusals():
    a, b = ack.Device(), ack.Device()
    try:
        lib = a._lib
        buf = a.buffer(64)
        data = np.zeros(16, np.float32)
        rc = lib.cdll.ack_upload(b._handle, buf._handle, data.ctypes.data, 64)
        assert rc == ack.ACK_ERR_FOREIGN and "belongs to device" in lib.last_error()
        rc = lib.cdll.ack_close(a._handle)
        assert rc == ack.ACK_ERR_LIVE_BUFFERS
        handle = buf._handle
        buf.free()
        rc = lib.cdll.ack_upload(a._handle, handle, data.ctypes.data, 64)
        assert rc == ack.ACK_ERR_FREED
        with pytest.raises(ack.AckError, match="upload of"):
            a.buffer(64).upload(np.zeros(3, np.float32))
    finally:
        for dev in (a, b):
            for h in list(dev._buffers):
                dev._lib.cdll.ack_buffer_free(dev._handle, h)
            dev._buffers.clear()
            dev.close()


def test_injected_wait_failure_poisons_the_device(monkeypatch):
    monkeypatch.setenv("ACK_FAULT_INJECTION", "1")
    dev = ack.Device()
    lib = dev._lib
    buf = dev.buffer(16)
    buf.upload(np.arange(4, dtype=np.float32))
    assert lib.cdll.ack_inject_fault(dev._handle, 0, 700) == ack.ACK_OK   # reported as cudaErrorIllegalAddress
    with pytest.raises(ack.AckPoisoned):
        buf.download(np.float32)
    # every later call refuses by name
    with pytest.raises(ack.AckError, match="poisoned"):
        dev.buffer(16)
    backend = vq.VQDevice(dev)
    with pytest.raises(ack.AckError):
        backend.decode(vq.VQArray((8,), 8, np.zeros(1, np.uint32), np.zeros((16, 8), np.float32)))
    with pytest.raises(ack.AckPoisoned):
        buf.free()
    assert dev.leaked_on_poison() == 1
    dev.close()


def test_injected_allocation_failure_is_reported_and_recovers(monkeypatch):
    monkeypatch.setenv("ACK_FAULT_INJECTION", "1")
    with ack.Device() as dev:
        assert dev._lib.cdll.ack_inject_fault(dev._handle, 1, 0) == ack.ACK_OK
        with pytest.raises(ack.AckError, match="cudaErrorMemoryAllocation"):
            dev.buffer(1024)
        buf = dev.buffer(1024)
        buf.free()


def test_device_choice_by_environment(monkeypatch):
    monkeypatch.setenv("ACK_DEVICE", "cpu")
    with pytest.raises(ack.AckUnavailable, match="no CPU device"):
        ack.Device()
    monkeypatch.setenv("ACK_DEVICE", "gpu:999")
    with pytest.raises(ack.AckUnavailable, match="only"):
        ack.Device()
    monkeypatch.setenv("ACK_DEVICE", "gpu:0")
    with ack.Device() as dev:
        assert "B200" in dev.name


@pytest.mark.parametrize("mode", [1, 2])
def test_injected_encode_stall_reports_and_the_context_stays_usable(monkeypatch, mode):
    """A bounded wait that nothing will satisfy runs out on the GPU: the
    host arms a stall test of the next tensor-core encode (1: its TMA
    producer issues no load; 2: its consumers take no accumulator, so loads
    and MMAs are in flight when the waits give up). The kernel sets the
    stalled bit, drains its own work and returns; the host reads the bit,
    and the next encode on the same device is bit-exact again."""
    import vq_oracle_c as oc
    monkeypatch.setenv("ACK_FAULT_INJECTION", "1")
    group, n = 16, 1 << 22
    rng = np.random.default_rng(40 + mode)
    values = rng.standard_normal(n).astype(np.float32)
    book = vq.fit_codebook(values, group=group)
    with ack.Device() as dev:
        backend = vq.VQDevice(dev)
        assert dev._lib.cdll.ack_inject_fault(dev._handle, 2, mode) == ack.ACK_OK
        with pytest.raises(ack.AckError, match="stalled"):
            backend.encode(values, book, group=group)
        again = backend.encode(values, book, group=group)
        np.testing.assert_array_equal(again.codes, oc.encode(values, book, group))
        assert dev.leaked_on_poison() == 0


def test_stall_injection_refuses_unknown_codes(monkeypatch):
    monkeypatch.setenv("ACK_FAULT_INJECTION", "1")
    with ack.Device() as dev:
        assert dev._lib.cdll.ack_inject_fault(dev._handle, 2, 3) == ack.ACK_ERR_SHAPE
        assert "stall" in dev._lib.last_error()
