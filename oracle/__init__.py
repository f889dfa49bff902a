"""CPU oracle for the catseye matmul hot path — test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package; the product (catseye_b200, libcatsgpu.so) never does.
"""
from .cpu import Oracle, Reference, build_oracle, ref_available  # noqa: F401
