"""The filter search's per-pair error bound (metalfaiss_b200/csrc/mf_filter.cu),
checked on the CPU with numpy's IEEE fp16 rounding (round to nearest, ties to
even, as __floats2half2_rn rounds): for a query q, a list centroid c and rows
x of that list, the filter's approximate distance

    a = |q - c|^2 + |x - c|^2 - 2 <fp16(s_q (q - c)), fp16(s_l (x - c))> / (s_q s_l)

stays within e of the exact distance |q - x|^2, where s_q and s_l are the
kernel's powers of two and e its bound. The products are accumulated the worst
way the bound allows for the tensor cores: one addend at a time into an fp32
accumulator that truncates toward zero (each step loses less than one unit in
the 24th bit of the larger term; hardware that adds several terms at once
or rounds to nearest loses less). tests/test_gpu_mma_accum.py measures the
device's own accumulation. Cases: isotropic data, coordinates near fp16
rounding boundaries, one dominant coordinate (where Cauchy-Schwarz is tight),
tiny and huge magnitudes, and residuals with elements that underflow fp16."""
import math

import numpy as np
import pytest


def scale_exp(n: float) -> int:
    """12 - e for n = m 2^e, 0.5 <= m < 1 (0 for n == 0): n 2^(12-e) in [2^11, 2^12)."""
    if not n > 0:
        return 0
    _, e = math.frexp(n)
    return 12 - e


def list_scale(resid: np.ndarray):
    """R_l (rounded up as the bank kernel rounds it), s_l, the rows' rn and
    beta_l (R^2 beta < 2^15, the norm extension's power of two)."""
    rn = (resid.astype(np.float32) ** 2).sum(1, dtype=np.float32)
    R = float(np.sqrt(np.float32(rn.max()))) * (1.0 + 2.0 ** -10)
    e = max(-60, min(60, scale_exp(R)))
    er = math.frexp(R)[1] if R > 0 else 0
    eb = max(-120, min(120, 15 - 2 * er))
    return R, 2.0 ** e, rn, 2.0 ** eb


def pair_bound(q, c, R, XN, sl, d):
    """The kernel's e for this pair, in the same fp32 steps (including the
    term of the norm fold: (d + 3) 2^-22 R^2)."""
    qc = (q - c).astype(np.float32)
    dc = float((qc * qc).sum(dtype=np.float32))
    nrm = math.sqrt(dc) * (1.0 + 2.0 ** -17)
    sq = 2.0 ** scale_exp(nrm)
    qn = float((q.astype(np.float32) ** 2).sum(dtype=np.float32))
    e = (float.fromhex("0x1.09p-9") * nrm * R
         + 2.0 ** -22 * math.sqrt(d) * (nrm / sl + R / sq)
         + (d + 20) * 2.0 ** -23 * (qn + XN + dc + R * R)
         + (d + 3) * 2.0 ** -22 * R * R + 2.0 ** -100)
    return e, sq, dc


def to_f32_toward_zero(v: np.ndarray) -> np.ndarray:
    """fp64 values rounded to fp32 toward zero (as float64)."""
    f = v.astype(np.float32)
    over = np.abs(f.astype(np.float64)) > np.abs(v)
    f[over] = np.nextafter(f[over], np.float32(0))
    return f.astype(np.float64)


def truncating_dot(X: np.ndarray, q: np.ndarray) -> np.ndarray:
    """Row dot products of fp16 operands (as float64: the products are exact)
    accumulated one addend at a time in fp32 with truncation toward zero."""
    acc = np.zeros(X.shape[0], np.float64)
    for i in range(X.shape[1]):
        acc = to_f32_toward_zero(acc + X[:, i] * q[i])
    return acc


def test_truncating_accumulation_emulation():
    x = np.array([[2048.0] + [1.0] * 127])
    q = np.array([2048.0] + [0.4995] * 127)
    got = truncating_dot(x, q)[0]
    assert got == 2.0 ** 22  # every tail below one unit (0.5) is dropped
    assert abs(got - float(x[0] @ q)) <= 128 * 2.0 ** -22 * float(np.abs(x[0]) @ np.abs(q))


def check(q, c, X, rng_name=""):
    d = q.shape[0]
    resid = (X - c).astype(np.float32)
    R, sl, rn, beta = list_scale(resid)
    XN = float((X.astype(np.float32) ** 2).sum(1, dtype=np.float32).max())
    e, sq, dc = pair_bound(q, c, R, XN, sl, d)
    assert math.isfinite(e), "the bound must be finite for these magnitudes"
    qh = ((q - c).astype(np.float32) * np.float32(sq)).astype(np.float16).astype(np.float64)
    xh = (resid * np.float32(sl)).astype(np.float16).astype(np.float64)
    assert np.all(np.isfinite(qh)) and np.all(np.isfinite(xh)), "fp16 overflow"
    # the norm fold: each row extended by [hi, lo] of beta rn (fp16), the query
    # by [A_e, A_e] with A_e = -s_q s_l / (2 beta); the tensor cores then give
    # s_q s_l (dot - rn / 2), and a = dc - 2 acc / (s_q s_l)
    ae = -sq * sl / (2.0 * beta)
    assert 2.0 ** -24 <= abs(ae) <= 2.0 ** 15 and float(np.float16(ae)) == ae
    v = (rn.astype(np.float32) * np.float32(beta)).astype(np.float32)
    hi = v.astype(np.float16)
    lo = (v - hi.astype(np.float32)).astype(np.float16)
    xa = np.concatenate([xh, hi.astype(np.float64)[:, None], lo.astype(np.float64)[:, None]], 1)
    qa = np.concatenate([qh, [ae, ae]])
    acc = truncating_dot(xa, qa)
    a = dc - 2.0 * acc / (sq * sl)
    t = ((X.astype(np.float64) - q.astype(np.float64)) ** 2).sum(1)
    err = np.abs(a - t)
    assert err.max() <= e, f"{rng_name}: error {err.max():.4g} above the bound {e:.4g}"
    return err.max() / e


@pytest.mark.parametrize("d", [64, 96, 128])
def test_bound_isotropic(d):
    rng = np.random.Generator(np.random.PCG64(d))
    worst = 0.0
    for _ in range(20):
        c = (rng.standard_normal(d) * 2).astype(np.float32)
        X = (c + rng.standard_normal((500, d))).astype(np.float32)
        q = (c + rng.standard_normal(d) * rng.uniform(0.1, 6)).astype(np.float32)
        worst = max(worst, check(q, c, X, "isotropic"))
    assert worst < 1.0


def test_bound_rounding_boundaries():
    """Elements halfway between fp16 neighbours after scaling (the rounding's
    worst case), all of one sign so the errors add up."""
    rng = np.random.Generator(np.random.PCG64(7))
    d = 128
    for _ in range(20):
        c = np.zeros(d, np.float32)
        # values 1 + (2j + 1) 2^-11: halfway between fp16 neighbours in [1, 2)
        j = rng.integers(0, 1023, size=(300, d))
        X = (1.0 + (2 * j + 1) * 2.0 ** -11).astype(np.float32)
        q = (1.0 + (2 * rng.integers(0, 1023, size=d) + 1) * 2.0 ** -11).astype(np.float32)
        check(q, c, X, "boundaries")


def test_bound_dominant_coordinate():
    """One large coordinate carries the norm: Cauchy-Schwarz is nearly tight."""
    d = 128
    rng = np.random.Generator(np.random.PCG64(11))
    for _ in range(20):
        c = np.zeros(d, np.float32)
        X = (rng.standard_normal((200, d)) * 1e-3).astype(np.float32)
        X[:, 0] = rng.uniform(1.0, 2.0, size=200).astype(np.float32)
        q = (rng.standard_normal(d) * 1e-3).astype(np.float32)
        q[0] = np.float32(rng.uniform(1.0, 2.0))
        check(q, c, X, "dominant")


@pytest.mark.parametrize("scale", [1e-30, 1e-6, 1e6, 1e15])
def test_bound_magnitudes(scale):
    d = 96
    rng = np.random.Generator(np.random.PCG64(int(abs(math.log10(scale))) + 3))
    for _ in range(10):
        c = (rng.standard_normal(d) * 2 * scale).astype(np.float32)
        X = (c + rng.standard_normal((300, d)) * scale).astype(np.float32)
        q = (c + rng.standard_normal(d) * scale).astype(np.float32)
        check(q, c, X, f"scale {scale}")


def test_bound_underflowing_elements():
    """Residual elements 2^-40 below the list's largest norm: fp16 subnormals
    or zeros after scaling; the bound's underflow term covers them."""
    d = 64
    rng = np.random.Generator(np.random.PCG64(19))
    for _ in range(10):
        c = np.zeros(d, np.float32)
        X = (rng.standard_normal((200, d)) * 2.0 ** -40).astype(np.float32)
        X[:, :2] = rng.uniform(1.0, 2.0, size=(200, 2)).astype(np.float32)
        q = (rng.standard_normal(d) * 2.0 ** -40).astype(np.float32)
        q[:2] = rng.uniform(1.0, 2.0, size=2).astype(np.float32)
        check(q, c, X, "underflow")


def test_scale_brings_norm_into_range():
    for n in (1e-20, 0.3, 1.0, 1.5, 2047.9, 4096.0, 1e20):
        s = 2.0 ** scale_exp(n)
        assert 2.0 ** 11 <= n * s < 2.0 ** 12
