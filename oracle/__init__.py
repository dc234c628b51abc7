"""Test infrastructure: the CPU oracle for the nkilab B200 kernels.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this
package; the product (nki-kernel-lab_b200/) never does. See nki_oracle.py.
"""
