"""CPU oracle for the metalfaiss_b200 search path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (and plain C under oracle/c/), the reference
MetalFaiss algorithm for flat kNN, IVFFlat search, k-means and range search,
each function citing the reference file:line it follows. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import it, and only as
the parity reference of the tests or the timed CPU baseline: the product path (metalfaiss_b200) never
imports, links or calls anything here.

Pinning: the reference is Python on Apple MLX and cannot run here (no MLX, no
Metal). tests/golden/make_golden.py imports the reference's own modules with a
numpy stand-in for mlx.core and runs the reference's Metal kernel sources
compiled as C++ (oracle/ref_msl), and commits the resulting input/output vectors
under tests/golden/. tests/test_oracle_golden.py checks this oracle against
them. MLX's own arithmetic (matmul order, argsort tie order) is not reproduced
by that stand-in, so parity is pinned to the reference's composition logic and
kernel sources, not to MLX's floating-point rounding.
"""
