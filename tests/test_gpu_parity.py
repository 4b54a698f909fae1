"""CUDA parity of the vq4 path through the C ABI (`ack.Device` / `VQDevice`)
against the CPU oracle. Bit-exact: decode, encode (the reference's float64
choice), the shader-order packed-pair matmul (op 2) and AdamW (op 3), the
fused VQAdamW step. Tolerance (normwise 1e-5 of sum_k |a_k b_k|): the
north-star products, whose summation order differs from any reference."""
import json

import numpy as np
import pytest

import shader_cases as sc
import vq4_ref
import vq_oracle as o
import vq_oracle_c as oc
from alelyon_compute_kit import ack, vq
from alelyon_compute_kit.vq import VQAdamW, VQArray

pytestmark = pytest.mark.gpu

TOL = 1e-5  # normwise relative tolerance of the FP32 products


@pytest.fixture(scope="module")
def device():
    dev = ack.Device()
    yield dev
    dev.close()


@pytest.fixture(scope="module")
def backend(device):
    return vq.VQDevice(device)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def rand_book(rng, group, scale=1.0):
    return (rng.standard_normal((16, group)) * scale).astype(np.float32)


def normwise(y, y64, a, b):
    return float(np.max(np.abs(y.astype(np.float64) - y64) / np.maximum(np.abs(a) @ np.abs(b), 1e-30)))


def test_device_identity(device):
    assert "B200" in device.name
    assert device.info.vendor_id == 0x10DE and device.info.subgroup_size == 32
    assert device.live_objects() == 1
    record = device.capability_record()
    json.dumps(record)
    assert record["abi"]["version"] == 14


@pytest.mark.parametrize("group", [8, 16, 32])
def test_decode_is_bit_exact(backend, group):
    rng = np.random.default_rng(group)
    for n in (1, 3, group, 8 * group, 8 * group + 1, 4097, 100_003):
        book = rand_book(rng, group)
        vectors = (n + group - 1) // group
        codes = o.pack(rng.integers(0, 16, vectors))
        arr = VQArray((n,), group, codes, book)
        np.testing.assert_array_equal(bits(backend.decode(arr)), bits(o.decode(codes, book, n, group)))


@pytest.mark.parametrize("group", [8, 16, 32])
def test_encode_matches_reference_golden_bytes(backend, golden, group):
    g = golden("encode_decode")
    for n in (1, group, 8 * group, 8 * group + 1, 1000, 4097, 3 * group - 5):
        key = f"g{group}_n{n}"
        arr = backend.encode(g[key + "_values"], g[key + "_book"], group=group)
        assert arr.to_bytes() == g[key + "_wire"].tobytes(), key
    t = golden("ties")
    for suffix in ("", "_zero", "_heavy"):
        values = t[f"g{group}{suffix}_values"]
        book = t[f"g{group}_book"] if suffix == "" else (
            np.zeros((16, group), np.float32) if suffix == "_zero" else t[f"g{group}_heavy_book"])
        got = backend.encode(values, book, group=group).codes
        np.testing.assert_array_equal(got, t[f"g{group}{suffix}_codes"], err_msg=suffix)


def test_cfg1_on_the_device(backend, golden):
    g = golden("cfg1")
    w = o.gaussian((256, 256), 0.02, 7)
    image = backend.encode(w, g["book"], group=16)
    assert image.to_bytes() == g["wire"].tobytes() and len(image.to_bytes()) == 3128
    np.testing.assert_array_equal(backend.decode(image), image.decode())
    x_image = VQArray.from_bytes(g["x_wire"].tobytes())
    y = backend.matmul(x_image, image)
    np.testing.assert_array_equal(bits(y), bits(o.matmul_shader(x_image.codes, x_image.codebook, image.codes,
                                                                 image.codebook, 1, 256, 256, 16, 0)))


@pytest.mark.parametrize("group", [8, 16, 32])
def test_encode_bit_exact_at_scale_with_near_ties_counted(backend, group):
    """2^20 values of each cfg-5 distribution against the C oracle (float64,
    the reference's encoder); disagreements with the FP32 shader encoder are
    counted and must all be float64 near ties."""
    for name, values, book, head in sc.fp32_encode_cases(group):
        got = backend.encode_large(values, book, group=group)
        want = oc.encode(values, book, group)
        np.testing.assert_array_equal(got, want, err_msg=name)
        fp32 = o.nearest_fp32_shader(values[:head], book, group)
        mism = np.nonzero(fp32 != o.unpack(want, head // group))[0]
        ties = set(o.near_ties(values[:head], book, group, rel=1e-4).tolist())
        assert set(mism.tolist()) <= ties, "an FP32-vs-FP64 disagreement that is not a near tie"


def test_encode_decode_round_trip_is_idempotent(backend):
    rng = np.random.default_rng(5)
    for group in (8, 16, 32):
        book = rand_book(rng, group)
        codes = o.pack(rng.integers(0, 16, 4096 // group * 8))
        n = codes.size * 8 * group
        values = backend.decode_large(codes, book, n, group=group)
        again = backend.encode_large(values, book, group=group)
        np.testing.assert_array_equal(again, codes)


@pytest.mark.parametrize("flags", [0, 1, 2, 3])
def test_packed_pair_matmul_is_the_shader_bit_for_bit(backend, flags):
    for (m, n, k, group, ac, ab, bc, bb) in sc.matmul_cases(flags):
        a = VQArray((k, m) if flags & 1 else (m, k), group, ac, ab)
        b = VQArray((n, k) if flags & 2 else (k, n), group, bc, bb)
        y = backend.matmul(a, b, transpose_a=bool(flags & 1), transpose_b=bool(flags & 2))
        want = o.matmul_shader(ac, ab, bc, bb, m, n, k, group, flags)
        np.testing.assert_array_equal(bits(y), bits(want), err_msg=str((m, n, k, group)))
        if vq4_ref.available():
            ref, status = vq4_ref.matmul(ac, ab, bc, bb, m, n, k, group, flags)
            assert status == 0
            np.testing.assert_array_equal(bits(y), bits(ref), err_msg=str((m, n, k, group)))


def test_schema1_bounds_are_the_references(backend):
    a = VQArray((1024, 257), 8, np.zeros((1024 * 257 // 8 + 7) // 8, np.uint32), np.zeros((16, 8), np.float32))
    b = VQArray((257, 1024), 8, np.zeros((1024 * 257 // 8 + 7) // 8, np.uint32), np.zeros((16, 8), np.float32))
    with pytest.raises(ValueError, match="vq-matmul-work-limit"):
        backend.matmul(a, b)


def test_adamw_op3_is_the_shader_bit_for_bit(backend):
    for (n, group, codes, books, step) in sc.adamw_cases():
        states = [VQArray((n,), group, c, b) for c, b in zip(codes, books)]
        got = backend.adamw(*states, step=step, **sc.ADAMW_HYPER)
        want = o.adamw_shader(*(s.decode() for s in states), sc.adamw_coefficients(step))
        for g_, w_ in zip(got, want):
            np.testing.assert_array_equal(bits(g_), bits(w_))
        if vq4_ref.available():
            ref, status = vq4_ref.adamw(codes, books, sc.adamw_coefficients(step), n, group)
            assert status == 0
            for g_, r_ in zip(got, ref):
                np.testing.assert_array_equal(bits(g_), bits(r_))


def test_status_bits_refuse_outputs(backend):
    for name, plan, bindings, out_values, status in sc.status_cases():
        with pytest.raises(ack.AckError, match=f"status={status}"):
            backend._run(plan, bindings, out_values * 4, np.float32)


@pytest.mark.parametrize("group", [8, 16, 32])
def test_dense_activation_product_within_tolerance(backend, group):
    rng = np.random.default_rng(100 + group)
    for (m, n, k, e, nt) in ((1, 1000, 32 * group, 3, True), (3, 517, 64 * group, 2, True),
                             (8, 300, 32 * group, 1, True), (16, 257, 32 * group, 2, True),
                             (5, 129, 3 * group + 4, 2, True), (4, 200, 8 * group, 2, False),
                             (2, 96, 40, 1, False)):
        ws = []
        for _ in range(e):
            shape = (n, k) if nt else (k, n)
            count = n * k
            ws.append(VQArray(shape, group, o.pack(rng.integers(0, 16, (count + group - 1) // group)),
                              rand_book(rng, group, 0.05)))
        x = rng.standard_normal((e, m, k)).astype(np.float32)
        y = backend.matmul_dense_grouped(x, ws, transpose_b=nt)
        for i in range(e):
            wd = ws[i].decode().astype(np.float64)
            wmat = wd.T if nt else wd
            y64 = x[i].astype(np.float64) @ wmat
            err = normwise(y[i], y64, x[i].astype(np.float64), wmat)
            assert err <= TOL, (m, n, k, nt, err)


def test_dense_matches_cfg2_shapes(backend):
    """One cfg2 matrix (11008 x 4096, g16) for M in {1, 4, 16, 64}."""
    rng = np.random.default_rng(7)
    n, k, group = 11008, 4096, 16
    book = rand_book(rng, group, 0.25)
    codes = o.pack(rng.integers(0, 16, n * k // group))
    w = VQArray((n, k), group, codes, book)
    for m in (1, 4, 16, 64):
        x = rng.standard_normal((m, k)).astype(np.float32)
        y = backend.matmul_dense(x, w)
        y64 = o.dense_nt_f64(x, codes, book, n, k, group)
        wd = o.decode(codes, book, n * k, group).reshape(n, k).astype(np.float64)
        assert normwise(y, y64, x.astype(np.float64), wd.T) <= TOL


@pytest.mark.parametrize("group", [8, 16, 32])
def test_resident_stack_is_the_uploaded_product_bit_for_bit(backend, group):
    """Weights made resident once (tile32 repack on the device, or the wire
    layout) give the same bits as the per-call product, call after call,
    into a caller's output array too; ragged N exercises the padded tile."""
    rng = np.random.default_rng(300 + group)
    e, n, k = 3, 517, 64 * group
    ws = [VQArray((n, k), group, o.pack(rng.integers(0, 16, n * k // group)), rand_book(rng, group, 0.05))
          for _ in range(e)]
    stack = vq.VQStack.from_arrays(ws)
    for m in (1, 3):
        x = rng.standard_normal((e, m, k)).astype(np.float32)
        want = backend.matmul_dense_grouped(x, stack)
        for layout in ("tile32", "canonical"):
            with backend.resident(stack, layout=layout) as weights:
                assert len(weights) == e
                out = np.empty((e, m, n), dtype=np.float32)
                for _ in range(2):
                    got = backend.matmul_dense_grouped(x, weights, out=out)
                    assert got is out
                    np.testing.assert_array_equal(bits(got), bits(want))
                np.testing.assert_array_equal(bits(backend.matmul_dense_grouped(x, weights)), bits(want))
    with pytest.raises(ValueError, match="tile32"):
        backend.resident(vq.VQStack.from_arrays(
            [VQArray((n, 40 * group), group, o.pack(rng.integers(0, 16, n * 40)), rand_book(rng, group))]))


@pytest.mark.parametrize("group", [8, 16, 32])
def test_coded_product_within_tolerance(backend, group):
    rng = np.random.default_rng(200 + group)
    for (m, n, k, flags) in ((70, 300, 16 * group, 2), (64, 256, 8 * group, 2), (5, 9, 3 * group, 2),
                             (33, 40, 8 * group + 3, 2), (20, 30, 40, 0), (20, 30, 40, 1), (20, 30, 40, 3)):
        ab, bb = rand_book(rng, group), rand_book(rng, group)
        ac = o.pack(rng.integers(0, 16, (m * k + group - 1) // group))
        bc = o.pack(rng.integers(0, 16, (k * n + group - 1) // group))
        a = VQArray((k, m) if flags & 1 else (m, k), group, ac, ab)
        b = VQArray((n, k) if flags & 2 else (k, n), group, bc, bb)
        y = backend.matmul_coded(a, b, transpose_a=bool(flags & 1), transpose_b=bool(flags & 2))
        da = a.decode().astype(np.float64)
        db = b.decode().astype(np.float64)
        A = da.T if flags & 1 else da
        B = db.T if flags & 2 else db
        assert normwise(y, A @ B, A, B) <= TOL, (m, n, k, flags)


class HostShaderBackend:
    """The reference's arithmetic on the host: the CPU encoder, the shader's
    op 2 and op 3 restated by the oracle."""

    def encode(self, values, codebook, *, group):
        return vq.encode(values, codebook, group=group)

    def decode(self, value):
        return value.decode()

    def matmul(self, a, b, *, transpose_a=False, transpose_b=False):
        m, k = a.shape[::-1] if transpose_a else a.shape
        _, n = b.shape[::-1] if transpose_b else b.shape
        flags = int(transpose_a) | (int(transpose_b) << 1)
        return o.matmul_shader(a.codes, a.codebook, b.codes, b.codebook, m, n, k, a.group, flags)

    def adamw(self, weight, momentum, variance, gradient, *, lr, beta1, beta2, eps, weight_decay, step):
        coefs = o.adamw_coefficients(lr, beta1, beta2, eps, weight_decay, step)
        return o.adamw_shader(*(s.decode() for s in (weight, momentum, variance, gradient)), coefs)


@pytest.mark.parametrize("shape,group", [((37, 29), 8), ((256, 256), 16), ((1024, 512), 32), ((4096, 1024), 8)])
def test_fused_vqadamw_step_matches_the_reference_flow(backend, shape, group):
    rng = np.random.default_rng(sum(shape) + group)
    w = o.gaussian(shape, 0.02, 7)
    weight = vq.encode(w, vq.fit_codebook(w, group=group), group=group)
    dev_opt = VQAdamW(backend, weight, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    host_opt = VQAdamW(HostShaderBackend(), weight, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    for _ in range(2):
        g = (rng.standard_normal(shape) * 1e-3).astype(np.float32)
        gimg = vq.encode(g, vq.fit_codebook(g, group=group), group=group)
        r_dev = dev_opt.step(gimg)
        r_host = host_opt.step(gimg)
        for a, b in ((dev_opt.weight, host_opt.weight), (dev_opt.momentum, host_opt.momentum),
                     (dev_opt.variance, host_opt.variance)):
            assert a.to_bytes() == b.to_bytes()
        assert r_dev["changed_weight_values"] == r_host["changed_weight_values"]
        assert r_dev["step"] == r_host["step"]


@pytest.mark.parametrize("shape,group,sample", [((37, 29), 8, 4096), ((256, 256), 16, 4096),
                                                ((1024, 512), 32, 4096), ((4096, 1024), 8, 4096),
                                                ((512, 384), 16, 1000)])
def test_device_fit_is_the_cpu_fit_bit_for_bit(backend, shape, group, sample):
    """fit="device" (op 24) against fit="host" (the CPU Lloyd iterations) on
    the same steps: step 1 starts the moments from all-zero books (every
    entry but one empty: reseeds), later steps warm-start; a sample smaller
    than the tensor exercises the whole-tensor kept-entry rule."""
    rng = np.random.default_rng(sum(shape) + group + sample)
    w = o.gaussian(shape, 0.02, 7)
    weight = vq.encode(w, vq.fit_codebook(w, group=group), group=group)
    opts = {fit: VQAdamW(backend, weight, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, fit=fit)
            for fit in ("host", "device")}
    for _ in range(3):
        g = (rng.standard_normal(shape) * 1e-3).astype(np.float32)
        gimg = vq.encode(g, vq.fit_codebook(g, group=group), group=group)
        reports = {}
        for fit, opt in opts.items():
            if sample != 4096:
                encoded, changed, _ = backend.adamw_fused(opt.weight, opt.momentum, opt.variance, gimg, lr=1e-3,
                                                          beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01,
                                                          step=opt.steps + 1, sample_vectors=sample, fit=fit)
                opt.weight, opt.momentum, opt.variance = encoded
                opt.steps += 1
                reports[fit] = changed
            else:
                reports[fit] = opt.step(gimg)["changed_weight_values"]
        h, d = opts["host"], opts["device"]
        for a, b in ((h.weight, d.weight), (h.momentum, d.momentum), (h.variance, d.variance)):
            np.testing.assert_array_equal(bits(a.codebook), bits(b.codebook))
            assert a.to_bytes() == b.to_bytes()
        assert reports["host"] == reports["device"]


@pytest.mark.parametrize("group", [8, 16, 32])
def test_device_fit_codebook_is_the_cpu_function_bit_for_bit(backend, group):
    """VQDevice.fit_codebook against vq.fit_codebook: cold and warm starts,
    Gaussian, duplicate-heavy (empty entries, reseeds), a ragged tail, a
    sample smaller than the tensor (the kept-entry rule), 0 to 6 iterations."""
    rng = np.random.default_rng(40 + group)
    atoms = rng.standard_normal((16, group)).astype(np.float32)
    cases = [
        (o.gaussian((300, 7 * group + 3), 1.0, 1), {}),
        (o.block_normalised(o.gaussian((4096, 2 * group), 0.5, 2), group), {"sample_vectors": 1000}),
        (atoms[np.insert(np.arange(5000) % 12, 4000, 14)].reshape(-1), {}),
        (atoms[np.insert(np.arange(9000) % 15, 3, 15)].reshape(-1), {"sample_vectors": 512}),
        (o.gaussian((64, group), 1.0, 3), {"iterations": 0}),
        (o.gaussian((2000, group), 1.0, 4), {"iterations": 6, "sample_vectors": 16}),
    ]
    for values, kw in cases:
        for init in (None, "warm"):
            start = None if init is None else vq.fit_codebook(values, group=group, iterations=1, sample_vectors=64)
            want = vq.fit_codebook(values, group=group, init=start, **kw)
            got = backend.fit_codebook(values, group=group, init=start, **kw)
            np.testing.assert_array_equal(bits(got), bits(want))


@pytest.mark.parametrize("group,rare_at", [(8, -1), (16, -1), (32, -1), (8, 1)])
def test_fused_zero_gradient_moves_no_weight(backend, group, rare_at):
    """The reference audit's acceptance test on the device path; with the
    rare entry outside the calibration sample (group 8, position 1) the
    whole-tensor usage check runs on the device."""
    vectors = 65536 // group
    atoms = np.random.default_rng(1).standard_normal((16, group)).astype(np.float32)
    index = np.insert(np.arange(vectors - 1) % 15, rare_at % vectors, 15)
    values = atoms[index].reshape(-1)
    weight = vq.encode(values, atoms, group=group)
    zero = VQArray(weight.shape, group, np.zeros_like(weight.codes), np.zeros((16, group), np.float32))
    for fit in ("host", "device"):
        opt = VQAdamW(backend, weight, lr=1e-3, weight_decay=0.0, fit=fit)
        before = opt.weight.decode().copy()
        report = opt.step(zero)
        assert report["changed_weight_values"] == 0 == int((before != opt.weight.decode()).sum())
        assert len(np.unique(opt.weight.codebook.round(6), axis=0)) == 16


@pytest.mark.parametrize("fit", ["host", "device"])
def test_harness_on_the_device_equals_the_host_arithmetic(tmp_path, device, fit):
    from alelyon_compute_kit import expert_bank, harness
    rng = np.random.default_rng(12)
    roots = []
    for name in ("dev", "host"):
        bank = expert_bank.ExpertBank.create(tmp_path / name, expert_bank.BankConfig(1, 2, ((64, 48),) * 3, 16))
        bank.initialize_expert(0, 1, seed=5, zero_optimizer_state=True)
        roots.append(bank)
    x = rng.standard_normal((8, 64)).astype(np.float32)
    t = rng.standard_normal((8, 48)).astype(np.float32)
    dev_h = harness.VulkanExpertHarness(roots[0], device=device, fit=fit)
    host_h = harness.VulkanExpertHarness(roots[1], backend=HostShaderBackend())
    # the device engine keeps the step in HBM; its float64 loss and norm are
    # sums in another order than numpy's (relative 1e-12), the committed
    # state is the host arithmetic's bit for bit; a clipped and an unclipped step
    for max_norm in (1e-3, 10.0):
        a = dev_h.train_step(x, t, expert=1, beta2=0.999, max_grad_norm=max_norm)
        b = host_h.train_step(x, t, expert=1, beta2=0.999, max_grad_norm=max_norm)
        assert abs(a.loss - b.loss) <= 1e-12 * abs(b.loss)
        assert abs(a.gradient_norm_before_clip - b.gradient_norm_before_clip) <= 1e-12 * b.gradient_norm_before_clip
        assert a.clipped == b.clipped and a.optimizer_step == b.optimizer_step and a.revision == b.revision
        assert a.input_layout == b.input_layout and a.gradient_layout == b.gradient_layout
        assert a.persistent_state_bytes == b.persistent_state_bytes
        for ta, tb in zip(roots[0].read_expert(0, 1), roots[1].read_expert(0, 1)):
            assert ta.to_bytes() == tb.to_bytes()
    np.testing.assert_array_equal(dev_h.forward(x, expert=1), host_h.forward(x, expert=1))


@pytest.mark.parametrize("group", [8, 16, 32])
def test_harness_residual_and_clip_ops(group):
    """Ops 26 and 27 against numpy: the residual and its scaling bit for bit,
    the float64 sums within 1e-12 relative, the clip's scale and output."""
    import torch

    from alelyon_compute_kit import cuda
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(60 + group)
    for count in (1, group + 3, 100_003, 1 << 22):
        book = rand_book(rng, group)
        codes = o.pack(rng.integers(0, 16, (count + group - 1) // group))
        pred = rng.standard_normal(count).astype(np.float32)
        scale = np.float32(2.0 / count)
        r, s, st = cuda.residual(torch.from_numpy(pred).to(dev), torch.from_numpy(codes.view(np.int32)).to(dev),
                                 torch.from_numpy(book).to(dev), group, float(scale))
        cuda.check(st)
        want = pred - o.decode(codes, book, count, group)
        np.testing.assert_array_equal(bits(r.cpu().numpy()), bits(want * scale))
        ref = float(np.sum(np.square(want, dtype=np.float64)))
        assert abs(float(s.item()) - ref) <= 1e-12 * ref
        for max_norm in (1e-3, 1e9):
            g = torch.from_numpy(want).to(dev)
            out, stats, st = cuda.clip_norm(g, max_norm)
            cuda.check(st)
            norm = float(np.linalg.norm(want.astype(np.float64)))
            got_norm, got_scale = (float(v) for v in stats.cpu().numpy())
            assert abs(got_norm - norm) <= 1e-12 * norm
            sc = min(1.0, max_norm / (got_norm + 1e-6))
            assert got_scale == sc
            np.testing.assert_array_equal(bits(out.cpu().numpy()), bits(want * np.float32(sc)))
