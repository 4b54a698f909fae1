"""Generate the golden vectors that pin the oracle to the reference.

Run this in a container where the reference checkout exists (it is not
present on GPU machines, which only read the committed `.npz` fixtures):

    python tests/golden/gen_golden.py /path/to/reference          # everything
    python tests/golden/gen_golden.py /path/to/reference bank     # bank.npz only

Every array below is produced by the reference's own CPU code
(`src/alelyon_compute_kit/_kit/python/vq.py`: `fit_codebook`, `encode`,
`VQArray.decode`, `VQArray.to_bytes`; `_kit/python/expert_bank.py`:
`ExpertBank`). Nothing here is restated; the
restatement under `oracle/` is checked against these files by
`tests/test_oracle_golden.py`. Inputs are seeded synthetic data.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_reference(root: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(Path(root) / "src"))
    from alelyon_compute_kit._kit.python import vq  # noqa: E402
    return vq


def digest(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def main(root: str) -> None:
    vq = load_reference(root)

    # -- the smoke workload: 256x256 N(0, 0.02^2), seed 7, group 16 --------
    w = (np.random.default_rng(7).standard_normal((256, 256)) * 0.02).astype(np.float32)
    book = vq.fit_codebook(w, group=16)
    image = vq.encode(w, book, group=16)
    x = np.random.default_rng(8).standard_normal((1, 256)).astype(np.float32)
    x_book = vq.fit_codebook(x, group=16)
    x_image = vq.encode(x, x_book, group=16)
    wire = np.frombuffer(image.to_bytes(), dtype=np.uint8)
    np.savez_compressed(HERE / "cfg1.npz", w_sha256=np.array(digest(w)), book=book, codes=image.codes, wire=wire,
                        decoded_sha256=np.array(digest(image.decode())),
                        x=x, x_book=x_book, x_codes=x_image.codes,
                        x_wire=np.frombuffer(x_image.to_bytes(), dtype=np.uint8))

    # -- encode/decode with tails, every group ---------------------------------
    cases = {}
    for group in (8, 16, 32):
        for n in (1, group, 8 * group, 8 * group + 1, 1000, 4097, 3 * group - 5):
            seed = 1000 + 97 * group + n
            values = np.random.default_rng(seed).standard_normal(n).astype(np.float32)
            fit_input = values if n >= group else np.pad(values, (0, group - n))
            book = vq.fit_codebook(fit_input, group=group)
            arr = vq.encode(values, book, group=group)
            key = f"g{group}_n{n}"
            cases[key + "_values"] = values
            cases[key + "_book"] = book
            cases[key + "_codes"] = arr.codes
            cases[key + "_decoded"] = arr.decode()
            cases[key + "_wire"] = np.frombuffer(arr.to_bytes(), dtype=np.uint8)
    np.savez_compressed(HERE / "encode_decode.npz", **cases)

    # -- ties: duplicate rows, exact atoms, zero book, midpoints ----------------
    ties = {}
    for group in (8, 16, 32):
        rng = np.random.default_rng(50 + group)
        book = rng.standard_normal((16, group)).astype(np.float32)
        book[7] = book[2]                 # a duplicate row can never be selected
        book[12] = book[2]
        atoms = book[rng.integers(0, 16, 300)]
        mids = ((book[3].astype(np.float64) + book[9].astype(np.float64)) / 2).astype(np.float32)
        mid_block = np.repeat(mids[None, :], 20, axis=0)
        values = np.concatenate([atoms.reshape(-1), mid_block.reshape(-1),
                                 np.zeros(5 * group, np.float32)])
        arr = vq.encode(values, book, group=group)
        ties[f"g{group}_values"] = values
        ties[f"g{group}_book"] = book
        ties[f"g{group}_codes"] = arr.codes
        zero_book = np.zeros((16, group), np.float32)
        zvals = rng.standard_normal(8 * group + 3).astype(np.float32)
        ties[f"g{group}_zero_values"] = zvals
        ties[f"g{group}_zero_codes"] = vq.encode(zvals, zero_book, group=group).codes
        # duplicate-heavy data (cfg 5b construction at a small size)
        hv_rng = np.random.default_rng(10)
        hv_atoms = hv_rng.standard_normal((16, group)).astype(np.float32)
        count = 2048
        rare = int(round(count * 0.15))
        idx = np.zeros(count, dtype=np.int64)
        idx[:rare] = 1 + (np.arange(rare) % 15)
        hv_rng.shuffle(idx)
        heavy = hv_atoms[idx].reshape(-1)
        heavy_book = vq.fit_codebook(heavy, group=group, sample_vectors=65536)
        ties[f"g{group}_heavy_values"] = heavy
        ties[f"g{group}_heavy_book"] = heavy_book
        ties[f"g{group}_heavy_codes"] = vq.encode(heavy, heavy_book, group=group).codes
    np.savez_compressed(HERE / "ties.npz", **ties)

    # -- fit_codebook: the reference test's occupancy patterns and warm start ---
    fits = {}
    atoms = np.random.default_rng(1).standard_normal((16, 16))
    occupancy = {
        "even": [64] * 16,
        "common_rare": [120] * 8 + [8] * 8,
        "geometric": [max(1, int(512 * 0.55 ** i)) for i in range(16)],
        "dominant": [900] + [4] * 15,
    }
    for name, counts in occupancy.items():
        sample = np.repeat(atoms, counts, axis=0).astype(np.float32)
        fits[f"occ_{name}_values"] = sample.reshape(-1)
        fits[f"occ_{name}_book"] = vq.fit_codebook(sample.reshape(-1), group=16)
    for group, rare_at in ((8, -1), (8, 1), (16, -1), (32, -1)):
        vectors = 65536 // group
        ga = np.random.default_rng(1).standard_normal((16, group)).astype(np.float32)
        index = np.insert(np.arange(vectors - 1) % 15, rare_at % vectors, 15)
        values = ga[index].reshape(-1)
        key = f"warm_g{group}_r{rare_at % vectors}"
        fits[key + "_values_sha256"] = np.array(digest(values))
        fits[key + "_index"] = index.astype(np.uint8)
        fits[key + "_atoms"] = ga
        fits[key + "_book"] = vq.fit_codebook(values, group=group, init=ga)
    gauss = (np.random.default_rng(11).standard_normal(200_000) * 0.02).astype(np.float32)
    for group in (8, 16, 32):
        cold = vq.fit_codebook(gauss, group=group)
        fits[f"gauss_g{group}_cold"] = cold
        fits[f"gauss_g{group}_warm"] = vq.fit_codebook(gauss * np.float32(1.01), group=group, init=cold)
        fits[f"gauss_g{group}_big"] = vq.fit_codebook(gauss, group=group, sample_vectors=65536,
                                                      iterations=2)
    fits["gauss_values_sha256"] = np.array(digest(gauss))
    np.savez_compressed(HERE / "fit.npz", **fits)

    # -- wire images of several ranks -------------------------------------------
    wires = {}
    for shape in ((3,), (5, 7), (2, 3, 11), (4, 4, 4, 4), (1, 1, 1, 1, 1, 9)):
        for group in (8, 16, 32):
            n = int(np.prod(shape))
            values = np.random.default_rng(n + group).standard_normal(shape).astype(np.float32)
            book = np.random.default_rng(group).standard_normal((16, group)).astype(np.float32)
            arr = vq.encode(values, book, group=group)
            key = "x".join(map(str, shape)) + f"_g{group}"
            wires[key + "_values"] = values.reshape(-1)
            wires[key + "_book"] = book
            wires[key + "_wire"] = np.frombuffer(arr.to_bytes(), dtype=np.uint8)
            wires[key + "_layout"] = np.array([arr.layout[k] for k in (
                "elements", "vectors", "code_bytes", "codebook_bytes", "metadata_bytes",
                "serialized_bytes", "payload_bytes")], dtype=np.int64)
    np.savez_compressed(HERE / "wire.npz", **wires)
    print("golden fixtures written to", HERE)


def load_reference_bank(root: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(Path(root) / "src"))
    from alelyon_compute_kit._kit.python import expert_bank  # noqa: E402
    return expert_bank


def bank(root: str) -> None:
    """bank.npz: every file of a small expert bank written by the reference's
    own `ExpertBank` (two initialized experts, one of them with a second,
    updated generation), its `stats()` and each expert's pointer fields; the
    tests open it with this library's bank and write the same experts anew."""
    import json
    import tempfile
    eb = load_reference_bank(root)
    vq = load_reference(root)
    files = {}
    with tempfile.TemporaryDirectory() as tmp:
        cfg = eb.BankConfig(2, 3, ((16, 8), (8, 24), (16, 8)), 8)
        b = eb.ExpertBank.create(Path(tmp) / "bank", cfg)
        b.initialize_expert(0, 1, seed=3, zero_optimizer_state=True)
        b.initialize_expert(1, 2, seed=5)
        state = b.read_expert_state(0, 1)
        w = state.tensors[0]
        moved = vq.VQArray(w.shape, w.group, w.codes[::-1].copy(), w.codebook * np.float32(0.5))
        b.write_expert(0, 1, (moved,) + state.tensors[1:], updated_count=7, optimizer_step=2)
        for path in sorted((Path(tmp) / "bank").iterdir()):
            files["file:" + path.name] = np.frombuffer(path.read_bytes(), dtype=np.uint8)
        files["stats"] = np.array(json.dumps(b.stats(), sort_keys=True))
        # what a fresh bank's initialize_expert writes for the same identities
        fresh = eb.ExpertBank.create(Path(tmp) / "fresh", cfg)
        fresh.initialize_expert(0, 1, seed=3, zero_optimizer_state=True)
        fresh.initialize_expert(1, 2, seed=5)
        for le in ((0, 1), (1, 2)):
            for i, t in enumerate(fresh.read_expert(*le)):
                files[f"init:{le[0]}-{le[1]}-t{i}"] = np.frombuffer(t.to_bytes(), dtype=np.uint8)
    np.savez_compressed(HERE / "bank.npz", **files)
    print("bank fixture written to", HERE / "bank.npz")


if __name__ == "__main__":
    if len(sys.argv) == 3 and sys.argv[2] == "bank":
        bank(sys.argv[1])
    elif len(sys.argv) == 2:
        main(sys.argv[1])
        bank(sys.argv[1])
    else:
        raise SystemExit("usage: gen_golden.py <reference checkout root> [bank]")
