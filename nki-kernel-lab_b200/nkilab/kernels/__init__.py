"""Kernel-level entry points with the reference's kernel names, layouts and tile
constants (nkilab/kernels/*.py in Nags-gk/nki-kernel-lab).

In the reference these are ``@nki.jit`` kernels called as
``nki.simulate(kernel)(*arrays)``; here each is a plain function over device (or
host) arrays that runs the corresponding B200 CUDA kernel.
"""
