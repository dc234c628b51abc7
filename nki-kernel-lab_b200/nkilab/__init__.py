"""nkilab (B200): the nki-kernel-lab kernel set as sm_100a CUDA kernels.

Import layout mirrors the reference package: ``nkilab.ops`` (host wrappers),
``nkilab.kernels`` (kernel-level entry points), ``nkilab.model`` (decoder block).
Importing ``nkilab`` itself needs no GPU; ``nkilab.ops`` loads the CUDA library.
"""
__version__ = "0.1.0"
