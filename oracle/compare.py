"""Result comparison under the parity rule of this path (test infrastructure only).

Rule: labels equal the oracle's except at near-ties, where the two candidates'
exact (fp64) distances differ by <= 1e-5 relative; distances within 1e-4
relative of the oracle's (fp32). An absolute floor `atol` covers distances that
are ~0 after the fp32 norm-expansion cancellation (||q||^2 + ||x||^2 - 2 q.x),
which the reference computes the same way (python/metalfaiss/distances.py:170-173);
it widens the distance check only. The near-tie test is relative alone
(`tie_atol`, default 0), so the band stays at 1e-5 of the distance whatever
the norms of the data.
"""
from __future__ import annotations

import numpy as np

RTOL = 1e-4
TIE_RTOL = 1e-5


def l2_atol(xq, xb) -> float:
    """Cancellation floor for squared-L2 by norm expansion in fp32."""
    qn = float(np.max(np.sum(np.square(np.asarray(xq, np.float64)), axis=1))) if len(xq) else 0.0
    bn = float(np.max(np.sum(np.square(np.asarray(xb, np.float64)), axis=1))) if len(xb) else 0.0
    return 4e-6 * (qn + bn) + 1e-6


def check_knn(D, I, D_ref, I_ref, exact_of, *, rtol=RTOL, tie_rtol=TIE_RTOL, atol=1e-6,
              tie_atol=0.0):
    """Returns a list of human-readable violations (empty = parity holds).

    exact_of(q, labels) -> fp64 distances of `labels` (np.inf for -1) for query q.
    atol: absolute floor of the distance check; tie_atol: of the near-tie
    test (0: purely relative).
    """
    D = np.asarray(D, np.float64)
    D_ref = np.asarray(D_ref, np.float64)
    I = np.asarray(I, np.int64)
    I_ref = np.asarray(I_ref, np.int64)
    errs = []
    if D.shape != D_ref.shape or I.shape != I_ref.shape:
        return [f"shape {D.shape}/{I.shape} != reference {D_ref.shape}/{I_ref.shape}"]
    for q in range(D.shape[0]):
        # distances, rank by rank
        both_inf = np.isinf(D[q]) & np.isinf(D_ref[q])
        tol = rtol * np.abs(np.where(np.isinf(D_ref[q]), 0, D_ref[q])) + atol
        with np.errstate(invalid="ignore"):  # inf - inf where both are empty slots
            bad = ~both_inf & ~(np.abs(D[q] - D_ref[q]) <= tol)
        if bad.any():
            j = int(np.argmax(bad))
            errs.append(f"q{q} rank{j}: distance {D[q, j]!r} vs reference {D_ref[q, j]!r}")
            continue
        if np.any(np.diff(D[q][~np.isinf(D[q])]) < 0):
            errs.append(f"q{q}: distances not ascending")
            continue
        valid = I[q] >= 0
        if len(set(I[q][valid].tolist())) != int(valid.sum()):
            errs.append(f"q{q}: duplicate labels {I[q]}")
            continue
        if np.array_equal(I[q], I_ref[q]):
            continue
        diff = np.nonzero(I[q] != I_ref[q])[0]
        e_got = exact_of(q, I[q][diff])
        e_ref = exact_of(q, I_ref[q][diff])
        scale = np.maximum(np.abs(e_ref), np.abs(e_got))
        ok = np.abs(e_got - e_ref) <= tie_rtol * scale + tie_atol
        # -1 padding must agree exactly
        ok &= (I[q][diff] >= 0) == (I_ref[q][diff] >= 0)
        if not ok.all():
            j = int(diff[np.argmin(ok)])
            errs.append(
                f"q{q} rank{j}: label {I[q, j]} (exact {e_got[np.argmin(ok)]!r}) vs reference "
                f"{I_ref[q, j]} (exact {e_ref[np.argmin(ok)]!r}) is not a near-tie")
    return errs


def exact_lookup(xq, xb, metric, ids=None):
    """exact_of for check_knn when labels map to rows of xb through `ids`."""
    from .oracle import pairwise_exact

    xq = np.asarray(xq, np.float64)
    xb = np.asarray(xb, np.float64)
    pos_of = None
    if ids is not None:
        ids = np.asarray(ids, np.int64)
        pos_of = {int(v): i for i, v in enumerate(ids.tolist())}

    def exact_of(q, labels):
        out = np.full(len(labels), np.inf)
        for t, lab in enumerate(np.asarray(labels).tolist()):
            if lab < 0:
                continue
            p = lab if pos_of is None else pos_of[lab]
            out[t] = pairwise_exact(xq[q:q + 1], xb[p:p + 1], metric)[0, 0]
        return out

    return exact_of


def check_range(lims, D, L, lims_ref, D_ref, L_ref, exact_of, radius, *, rtol=RTOL, atol=1e-6,
                tie_rtol=TIE_RTOL):
    """Range results as per-query sets: a label may differ from the oracle's set
    only when its exact distance is within the near-tie band of the radius."""
    errs = []
    nq = len(lims) - 1
    for q in range(nq):
        a = dict(zip(L[lims[q]:lims[q + 1]].tolist(), D[lims[q]:lims[q + 1]].tolist()))
        b = dict(zip(L_ref[lims_ref[q]:lims_ref[q + 1]].tolist(),
                     D_ref[lims_ref[q]:lims_ref[q + 1]].tolist()))
        for lab in set(a) ^ set(b):
            e = exact_of(q, np.array([lab]))[0]
            if abs(e - radius) > tie_rtol * abs(radius) + atol:
                errs.append(f"q{q}: label {lab} (exact {e!r}) differs from the oracle, radius {radius}")
                break
        for lab in set(a) & set(b):
            if abs(a[lab] - b[lab]) > rtol * abs(b[lab]) + atol:
                errs.append(f"q{q}: label {lab} distance {a[lab]} vs {b[lab]}")
                break
    return errs
