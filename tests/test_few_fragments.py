"""The operand layout of the fp16 few-query pass (few_scan_kernel in FLT form,
metalfaiss_b200/csrc/mf_few.cu), checked on the CPU.

The kernel feeds mma.sync.m16n8k16 (A: 16 queries x 16 elements, B: 16
elements x 8 rows) from a permuted K order. In K-steps 2p and 2p + 1, lane
(g, t) = (lane / 4, lane % 4) holds elements e0 .. e0 + 3 with
e0 = 32 p + 8 t + 4 (step & 1) of queries g, g + 8 and of row g, split as the
fragments' register pairs; elements at or past d are zeros. Here the
fragments are placed in the logical A and B tiles by PTX's documented
m16n8k16 layouts, and the sum over K-steps must equal the rows' dot products:
the permutation is a bijection of each step's 16 elements and the same on
both operands."""
import numpy as np
import pytest


def lane_elements(step: int, t: int) -> int:
    """First of the four elements lane (g, t) holds in K-step `step`."""
    return 32 * (step >> 1) + 8 * t + 4 * (step & 1)


def fragments(Q: np.ndarray, X: np.ndarray, step: int, d: int):
    """Per lane, the kernel's A registers (a0..a7) and B registers (b0..b3) of
    one K-step: A from queries g and g + 8, B from row g, for vectors of d
    elements (the arrays may be wider)."""
    A = np.zeros((32, 8))
    B = np.zeros((32, 4))
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        e0 = lane_elements(step, t)
        if e0 >= d:
            continue
        lo, hi = Q[g, e0:e0 + 4], Q[g + 8, e0:e0 + 4]
        # af[s][0] = (lo.x, lo.y), [1] = (hi.x, hi.y), [2] = (lo.z, lo.w), [3] = (hi.z, hi.w)
        A[lane] = [lo[0], lo[1], hi[0], hi[1], lo[2], lo[3], hi[2], hi[3]]
        # b0, b1 = the row's uint4 .x (elements e0, e0+1); b2, b3 = .y (e0+2, e0+3)
        B[lane] = X[g, e0:e0 + 4]
    return A, B


def logical_tiles(A: np.ndarray, B: np.ndarray):
    """PTX m16n8k16 (.f16 A/B): a_i sits at row g (i in 0,1,4,5) or g + 8
    (2,3,6,7), column 2t + (i & 1) + 8 (i >= 4); b_i at k = 2t + (i & 1) +
    8 (i >= 2), column n = g."""
    At = np.zeros((16, 16))
    Bt = np.zeros((16, 8))
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        for i in range(8):
            row = g + (8 if i in (2, 3, 6, 7) else 0)
            col = 2 * t + (i & 1) + (8 if i >= 4 else 0)
            At[row, col] = A[lane, i]
        for i in range(4):
            k = 2 * t + (i & 1) + (8 if i >= 2 else 0)
            Bt[k, g] = B[lane, i]
    return At, Bt


def test_each_step_covers_its_elements_once():
    for t_steps in range(4):  # pairs of K-steps for d up to 128
        got = sorted(lane_elements(s, t) + j
                     for s in (2 * t_steps, 2 * t_steps + 1) for t in range(4) for j in range(4))
        assert got == list(range(32 * t_steps, 32 * t_steps + 32))


@pytest.mark.parametrize("d", [64, 72, 80, 96, 128])
def test_permuted_steps_give_the_dot_products(d):
    rng = np.random.default_rng(d)
    Q = rng.integers(-8, 8, size=(16, d)).astype(np.float64)
    X = rng.integers(-8, 8, size=(8, d)).astype(np.float64)
    acc = np.zeros((16, 8))
    nsteps = 2 * ((d + 31) // 32)
    for step in range(nsteps):
        At, Bt = logical_tiles(*fragments(Q, X, step, d))
        acc += At @ Bt
    np.testing.assert_array_equal(acc, Q @ X.T)


@pytest.mark.parametrize("d", [72, 80])
def test_lanes_past_d_hold_zeros(d):
    """For d not a multiple of 32 the last pair of steps is partly empty, and
    no element at or past d is read."""
    Q = np.ones((16, 128))
    X = np.ones((8, 128))
    Q[:, d:] = np.nan
    X[:, d:] = np.nan
    for step in range(2 * ((d + 31) // 32)):
        A, B = fragments(Q, X, step, d)
        assert np.isfinite(A).all() and np.isfinite(B).all()
