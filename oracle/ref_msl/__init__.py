"""Builds the reference's Metal kernel sources as C++ for the CPU (oracle only).

The reference's list-scan kernels exist only as Metal Shading Language strings
inside python/metalfaiss/faissmlx/kernels/ivf_kernels.py. build_ref.py reads
those strings from the reference tree (never copied into this repository),
wraps them with msl_shim.h — a small C++ emulation of the MSL address-space
qualifiers, thread-position built-ins and threadgroup barriers — and compiles
them into oracle/_ref/libivf_kernels_ref.so. runner.py launches them with
Metal's dispatchThreads semantics (`grid` counts threads, the last
threadgroup may be partial). This executes the reference's own kernel code on
the CPU so the golden vectors of tests/golden/ come from it.
"""
