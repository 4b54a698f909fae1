"""The candidate mask of the certified nearest-entry search, built from signs.

The encoders (`k_encode_tc` in csrc/vq_codec.cu, `enc_vector` in
csrc/vq_device.cuh) take the entries e with f_e <= thr. Instead of sixteen
compares they compute d_e = fma(f_e, -1, thr) = RN(thr - f_e) and gather the
sign bits of d_e with funnel shifts (`__funnelshift_l(d, acc, 1)` =
(acc << 1) | (d >> 31)) in two chains of eight, then invert. This restates
that construction in numpy float32 (IEEE round-to-nearest, subnormals kept)
and checks it bit for bit against the compare mask on the inputs where it
could differ: ties (f_e == thr gives +0, a candidate), neighbours one ulp
apart, subnormal differences, signed zeros in f, large magnitudes and +inf.
The one zero difference that comes out -0 is (-0) - (+0); the encoders'
threshold is never -0 (thr = fma(2, eps, min f) with eps >= 2^-118 > 0, and
an exact zero fma result is +0 unless both addends are -0), so thr = -0 is
outside the construction's domain and is checked as such below. A
flush-to-zero difference would keep its sign (-0.0), so the mask does not
depend on the denormal mode either. A NaN f_e has an unspecified sign; the
encoders only use the mask when the minimum and the bound are finite, which
rules NaN entries out (x or the book nonfinite), so NaN is not part of it.
CPU only: no device code runs here."""
import numpy as np
import pytest

pytestmark = pytest.mark.filterwarnings("ignore::RuntimeWarning")


def _funnelshift_l(lo: int, hi: int) -> int:
    """__funnelshift_l(lo, hi, 1): the high word of (hi:lo) << 1."""
    return ((hi << 1) | (lo >> 31)) & 0xFFFFFFFF


def sign_mask(f: np.ndarray, thr: np.float32) -> int:
    """The device construction: pairs of entries, p from 3 down to 0, entries
    2p+1 then 2p into the low chain and 2p+9 then 2p+8 into the high one."""
    d = (np.float32(thr) - f.astype(np.float32)).astype(np.float32)  # RN(thr - f), exact in sign
    bits = d.view(np.uint32).astype(np.int64)
    lo = hi = 0
    for p in range(3, -1, -1):
        lo = _funnelshift_l(int(bits[2 * p + 1]), lo)
        lo = _funnelshift_l(int(bits[2 * p]), lo)
        hi = _funnelshift_l(int(bits[2 * p + 9]), hi)
        hi = _funnelshift_l(int(bits[2 * p + 8]), hi)
    return ~((hi << 8) | lo) & 0xFFFF


def compare_mask(f: np.ndarray, thr: np.float32) -> int:
    return sum(1 << e for e in range(16) if np.float32(f[e]) <= np.float32(thr))


def _cases(rng):
    tiny = np.float32(np.finfo(np.float32).smallest_subnormal)
    for _ in range(2000):
        scale = np.float32(10.0) ** rng.integers(-40, 38)
        f = (rng.standard_normal(16) * scale).astype(np.float32)
        thr = np.float32(np.min(f) + abs(rng.standard_normal()) * scale * 1e-3)
        yield f, thr
    for _ in range(500):
        thr = np.float32(rng.standard_normal() * 10.0 ** rng.integers(-38, 38))
        f = np.full(16, thr, np.float32)
        up, down = np.nextafter(thr, np.float32(np.inf)), np.nextafter(thr, np.float32(-np.inf))
        pick = rng.integers(0, 3, 16)
        f[pick == 1], f[pick == 2] = up, down
        yield f, thr
    for thr in (np.float32(0.0), tiny, -tiny, np.float32(3.0e38), np.float32(-3.0e38)):
        f = np.array([0.0, -0.0, tiny, -tiny, 2 * tiny, -2 * tiny, 1e-38, -1e-38,
                      3.0e38, -3.0e38, np.inf, 1.0, -1.0, 5e-45, -5e-45, 0.0], np.float32)
        yield f, thr


def test_sign_mask_equals_the_compare_mask():
    rng = np.random.default_rng(2024)
    checked = 0
    for f, thr in _cases(rng):
        assert sign_mask(f, thr) == compare_mask(f, thr), (f, thr)
        checked += 1
    assert checked > 2500


def test_the_threshold_is_never_negative_zero():
    """thr = fma(2, eps, fb) with eps > 0: an exact zero comes out +0, the
    only zero the sign construction relies on (numpy float32 stands in for
    the device's round-to-nearest fma, whose exact-zero sign rule is the
    same as addition's)."""
    for eps in (np.float32(2.0 ** -118), np.float32(1e-37), np.float32(0.5), np.float32(3.0)):
        fb = np.float32(-2.0) * eps
        thr = np.float32(2.0) * eps + fb
        assert thr == 0 and not np.signbit(thr)


def test_bit_e_is_entry_e():
    """Each entry lands on its own bit: one entry above the threshold at a time."""
    thr = np.float32(1.0)
    for e in range(16):
        f = np.zeros(16, np.float32)
        f[e] = np.float32(2.0)
        assert sign_mask(f, thr) == 0xFFFF & ~(1 << e)
