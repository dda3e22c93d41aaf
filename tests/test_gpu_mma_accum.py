"""Device evidence for the filter search's error bound: the fp32 accumulation
of fp16 products on the tensor cores, measured through mf_diag_f16_dot in
both instruction forms the filter search uses (tcgen05.mma kind::f16 with A in
tensor memory and B loaded by TMA, as the tensor-core filter pass issues it;
mma.sync m16n8k16, as the few-query filter pass issues it).

The bound in mf_filter.cu takes |acc - sum_i p_i| <= d 2^-22 sum_i |p_i| for
the accumulation of d exact products p_i = a_i b_i (a product of two fp16
values is exact in fp32): each addend truncated by less than one unit in the
24th significant bit of the largest term of its addition, whatever the number
of terms the hardware adds at once; round-to-nearest is tighter. Published
measurements of NVIDIA tensor cores describe multi-term additions that align
to the largest exponent and truncate (Fasi, Higham, Mikaitis, Pranesh,
"Numerical behavior of NVIDIA tensor cores", PeerJ Computer Science, 2021).

The operands are built to defeat the accumulator: a dominant product followed
(or preceded) by many products just under one or one half unit of the
accumulator, runs of equal magnitude and alternating sign, cancellation down
to tiny tails, wide exponent ranges, and plain Gaussian values. The exact sums
come from fp64 (exact for these products and lengths). Each case asserts the
worst |acc - exact| / sum|p_i| over its 16384 (or 128) dot products is within
the bound, and prints the worst ratio seen."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import _native as nat

pytestmark = pytest.mark.gpu

ROWS = {0: (128, 128), 1: (16, 8)}  # engine -> (rows of A, rows of B)


def _f16(x):
    return np.asarray(x, np.float64).astype(np.float16)


def _case(name, m, n, d, rng):
    """fp16 A (m, d), B (n, d) for an adversarial pattern."""
    A = np.zeros((m, d), np.float64)
    B = np.zeros((n, d), np.float64)
    if name == "dominant_first_tails_under_ulp":
        # accumulator at 2^22 after the first product (ulp 0.5); the tails
        # are just under one ulp (truncation drops them) or half an ulp
        # (round-to-nearest drops them)
        A[:, 0] = 2048.0
        B[:, 0] = 2048.0
        A[:, 1:] = 1.0
        tails = np.where(np.arange(n) % 2 == 0, 0.4995, 0.2498)
        B[:, 1:] = tails[:, None] * (1.0 - 2.0 ** -10 * rng.integers(0, 4, (n, d - 1)))
    elif name == "dominant_last_tails_under_ulp":
        A[:, -1] = 2048.0
        B[:, -1] = 2048.0
        A[:, :-1] = 1.0
        B[:, :-1] = 0.4995
    elif name == "dominant_mid_block_negative_tails":
        A[:, 5] = -2048.0
        B[:, 5] = 2047.0
        A[:, :5] = 1.0
        A[:, 6:] = 1.0
        B[:, :5] = -0.4995
        B[:, 6:] = -0.4995
    elif name == "alternating_equal_magnitude":
        sign = np.where(np.arange(d) % 2 == 0, 1.0, -1.0)
        A[:] = sign[None, :] * 1000.0
        B[:] = 1000.0 + rng.integers(-8, 9, (n, d))
    elif name == "cancellation_to_tails":
        half = d // 2
        big = rng.uniform(500, 2000, (m, half))
        A[:, :half] = big
        A[:, half:] = -big
        B[:] = 1.0
        B[:, -1] = 1.0 + 2.0 ** -10
    elif name == "wide_exponents":
        A[:] = np.exp2(rng.uniform(-12, 12, (m, d))) * rng.choice([-1.0, 1.0], (m, d))
        B[:] = np.exp2(rng.uniform(-12, 12, (n, d))) * rng.choice([-1.0, 1.0], (n, d))
    elif name == "gaussian":
        A[:] = rng.standard_normal((m, d)) * 1000.0
        B[:] = rng.standard_normal((n, d)) * 1000.0
    else:
        raise ValueError(name)
    return _f16(A), _f16(B)


CASES = ["dominant_first_tails_under_ulp", "dominant_last_tails_under_ulp",
         "dominant_mid_block_negative_tails", "alternating_equal_magnitude",
         "cancellation_to_tails", "wide_exponents", "gaussian"]


def _run(engine, A, B, d):
    dev = torch.device("cuda", 0)
    m, n = ROWS[engine]
    a = torch.from_numpy(A.view(np.uint16).astype(np.int16)).to(dev)
    b = torch.from_numpy(B.view(np.uint16).astype(np.int16)).to(dev)
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
    nat.call("mf_diag_f16_dot", 0, nat.stream_of(dev), engine, nat.ptr(a), nat.ptr(b), d,
             nat.ptr(out))
    torch.cuda.synchronize()
    assert nat.device_error(0) == 0, "a bounded device wait timed out"
    return out.cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("engine,d", [(0, 64), (0, 72), (0, 128), (1, 64), (1, 128)],
                         ids=["tcgen05-d64", "tcgen05-d72", "tcgen05-d128", "mma.sync-d64",
                              "mma.sync-d128"])
def test_fp16_accumulation_within_the_filter_bound(cuda_device, case, engine, d):
    m, n = ROWS[engine]
    rng = np.random.Generator(np.random.PCG64(1000 * CASES.index(case) + 10 * d + engine))
    A, B = _case(case, m, n, d, rng)
    a64, b64 = A.astype(np.float64), B.astype(np.float64)
    exact = a64 @ b64.T
    absum = np.abs(a64) @ np.abs(b64).T
    got = _run(engine, A, B, d)
    assert np.isfinite(got).all()
    live = absum > 0
    ratio = np.zeros_like(absum)
    ratio[live] = np.abs(got[live] - exact[live]) / absum[live]
    assert np.all(got[~live] == 0)
    worst = float(ratio.max())
    bound = d * 2.0 ** -22
    print(f"[accum] engine={'tcgen05' if engine == 0 else 'mma.sync'} d={d} case={case}: "
          f"worst |acc-exact|/sum|p| = {worst:.3e} = 2^{np.log2(worst) if worst else -np.inf:.2f}"
          f" (bound d*2^-22 = 2^{np.log2(bound):.2f})")
    assert worst <= bound, (case, worst, bound)


def test_probe_matches_plain_products(cuda_device):
    """The probe itself: small integers, where fp32 accumulation is exact."""
    rng = np.random.Generator(np.random.PCG64(3))
    for engine, d in ((0, 128), (0, 72), (1, 128)):
        m, n = ROWS[engine]
        A = _f16(rng.integers(-8, 9, (m, d)))
        B = _f16(rng.integers(-8, 9, (n, d)))
        got = _run(engine, A, B, d)
        np.testing.assert_array_equal(got, A.astype(np.float64) @ B.astype(np.float64).T)
