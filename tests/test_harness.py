"""Harness and expert bank on the host, with an injected backend (the
reference's `tests/test_harness.py` and its bank contract)."""
import json

import numpy as np
import pytest

import vq_oracle as o
from alelyon_compute_kit import expert_bank, harness, vq


class FakeBackend:
    def encode(self, values, codebook, *, group):
        return vq.encode(values, codebook, group=group)

    def decode(self, value):
        return value.decode()

    def matmul(self, left, right, *, transpose_a=False, transpose_b=False):
        a, b = left.decode(), right.decode()
        return (a.T if transpose_a else a) @ (b.T if transpose_b else b)

    def adamw(self, weight, momentum, variance, gradient, *, lr, beta1, beta2, eps, weight_decay, step):
        coefs = o.adamw_coefficients(lr, beta1, beta2, eps, weight_decay, step)
        return o.adamw_shader(*(s.decode() for s in (weight, momentum, variance, gradient)), coefs)


def _bank(tmp_path):
    bank = expert_bank.ExpertBank.create(tmp_path / "bank", expert_bank.BankConfig(1, 1, ((4, 3), (4, 3), (4, 3)), 8))
    bank.initialize_expert(0, 0, seed=4, zero_optimizer_state=True)
    return bank


def test_forward_uses_packed_expert_and_rejects_wrong_width(tmp_path):
    bank = _bank(tmp_path)
    runner = harness.VulkanExpertHarness(bank, backend=FakeBackend())
    inputs = np.arange(8, dtype=np.float32).reshape(2, 4)
    expected = inputs @ bank.read_expert_state(0, 0).tensors[0].decode()
    np.testing.assert_allclose(runner.forward(inputs), expected, rtol=0, atol=0)
    with pytest.raises(harness.HarnessError, match="width"):
        runner.forward(np.zeros((2, 5), dtype=np.float32))


def test_device_fit_needs_a_backend_that_fits_on_the_device(tmp_path):
    bank = _bank(tmp_path)
    with pytest.raises(harness.HarnessError, match="fit='device'"):
        harness.VulkanExpertHarness(bank, backend=FakeBackend(), fit="device")
    with pytest.raises(harness.HarnessError, match="fit must be"):
        harness.VulkanExpertHarness(bank, backend=FakeBackend(), fit="gpu")


def test_train_step_commits_optimizer_state_and_rejects_nonfinite(tmp_path):
    bank = _bank(tmp_path)
    runner = harness.VulkanExpertHarness(bank, backend=FakeBackend())
    before = bank.read_expert_state(0, 0)
    step = runner.train_step(np.ones((2, 4), np.float32), np.zeros((2, 3), np.float32), max_grad_norm=0.01)
    after = bank.read_expert_state(0, 0)
    assert step.optimizer_step == 1 and step.revision == 2
    assert after.optimizer_step == 1 and after.parameter_update_applications == 12
    assert step.persistent_state_bytes > 0
    assert before.tensors[0].to_bytes() != after.tensors[0].to_bytes()
    with pytest.raises(harness.HarnessError, match="finite"):
        runner.forward(np.full((2, 4), np.nan, dtype=np.float32))
    assert json.dumps(step.to_dict())


def test_bank_round_trip_and_refusals(tmp_path):
    cfg = expert_bank.BankConfig(2, 3, ((16, 8), (16, 8), (16, 8)), 16)
    bank = expert_bank.ExpertBank.create(tmp_path / "b", cfg)
    with pytest.raises(FileExistsError):
        expert_bank.ExpertBank.create(tmp_path / "b", cfg)
    bank.initialize_expert(1, 2, seed=9, zero_optimizer_state=True)
    again = expert_bank.ExpertBank.open(tmp_path / "b")
    state = again.read_expert_state(1, 2)
    assert state.revision == 1 and state.optimizer_step == 0
    assert not state.tensors[1].codes.any() and not state.tensors[1].codebook.any()
    with pytest.raises(expert_bank.ExpertBankError, match="already materialized"):
        bank.initialize_expert(1, 2)
    with pytest.raises(expert_bank.ExpertBankError, match="not materialized"):
        bank.read_expert_state(0, 0)
    receipt = bank.write_expert(1, 2, state.tensors, updated_count=5, optimizer_step=3)
    assert receipt["revision"] == 2 and receipt["parameter_update_applications"] == 5
    with pytest.raises(expert_bank.ExpertBankError, match="regress"):
        bank.write_expert(1, 2, state.tensors, optimizer_step=1)
    stats = bank.stats()
    assert stats["materialized_experts"] == 1 and stats["updated_experts"] == 1
    # a corrupted shard is refused
    generation = json.loads((tmp_path / "b" / "expert-1-2.json").read_bytes())["generation"]
    shard = tmp_path / "b" / f"expert-1-2-g{generation}-t0.vq"
    data = bytearray(shard.read_bytes())
    data[-1] ^= 1
    shard.write_bytes(bytes(data))
    with pytest.raises(expert_bank.ExpertBankError):
        bank.read_expert_state(1, 2)


def test_bank_pointer_format_is_canonical_json(tmp_path):
    bank = _bank(tmp_path)
    pointer = (tmp_path / "bank" / "expert-0-0.json").read_bytes()
    value = json.loads(pointer)
    assert json.dumps(value, sort_keys=True, separators=(",", ":")).encode() == pointer
    assert value["schema"] == "ack-expert-bank/v1" and len(value["shards"]) == 3


def test_gain_scheduler_reserves_exploration():
    s = expert_bank.GainScheduler(4, exploration_fraction=0.5)
    s.observe(2, 1.0, 0.5, 1.0, 10, 3)
    s.observe(3, 1.0, 0.2, 1.0, 10, 3)
    assert s.select(2) == (0, 3)
    with pytest.raises(expert_bank.ExpertBankError):
        s.observe(1, float("nan"), 0.0, 1.0, 1, 1)


# ---- format compatibility with the reference's own bank (tests/golden/bank.npz) ----

def _reference_bank(tmp_path, golden):
    data = golden("bank")
    root = tmp_path / "refbank"
    root.mkdir()
    for key in data.files:
        if key.startswith("file:"):
            (root / key[5:]).write_bytes(data[key].tobytes())
    return root, data


def test_a_bank_the_reference_wrote_opens_and_reads_here(tmp_path, golden):
    root, data = _reference_bank(tmp_path, golden)
    bank = expert_bank.ExpertBank.open(root)
    assert bank.config == expert_bank.BankConfig(2, 3, ((16, 8), (8, 24), (16, 8)), 8)
    assert bank.stats() == json.loads(str(data["stats"]))
    state = bank.read_expert_state(0, 1)
    assert (state.revision, state.optimizer_step, state.parameter_update_applications) == (2, 2, 7)
    first = bank.read_expert_state(1, 2)
    assert (first.revision, first.optimizer_step, first.parameter_update_applications) == (1, 0, 0)
    for i, t in enumerate(first.tensors):
        assert t.to_bytes() == data[f"init:1-2-t{i}"].tobytes()
    # and this library commits a further generation the reference's layout accepts
    receipt = bank.write_expert(1, 2, first.tensors, updated_count=3, optimizer_step=1)
    assert receipt["revision"] == 2
    assert expert_bank.ExpertBank.open(root).read_expert_state(1, 2).parameter_update_applications == 3


def test_initialize_expert_writes_the_references_bytes(tmp_path, golden):
    data = golden("bank")
    bank = expert_bank.ExpertBank.create(tmp_path / "b", expert_bank.BankConfig(2, 3, ((16, 8), (8, 24), (16, 8)), 8))
    bank.initialize_expert(0, 1, seed=3, zero_optimizer_state=True)
    bank.initialize_expert(1, 2, seed=5)
    for le in ((0, 1), (1, 2)):
        for i, t in enumerate(bank.read_expert(*le)):
            assert t.to_bytes() == data[f"init:{le[0]}-{le[1]}-t{i}"].tobytes(), (le, i)
    ref_bank_json = data["file:bank.json"].tobytes()
    assert (tmp_path / "b" / "bank.json").read_bytes() == ref_bank_json


def test_bank_metadata_must_be_canonical(tmp_path, golden):
    root, _ = _reference_bank(tmp_path, golden)
    pointer = root / "expert-1-2.json"
    text = pointer.read_bytes()
    pointer.write_bytes(text.replace(b",", b", ", 1))
    with pytest.raises(expert_bank.ExpertBankError, match="noncanonical"):
        expert_bank.ExpertBank.open(root).read_expert(1, 2)
    pointer.write_bytes(text[:-1] + b',"revision":1}')
    with pytest.raises(expert_bank.ExpertBankError):
        expert_bank.ExpertBank.open(root).read_expert(1, 2)
