"""TEST INFRASTRUCTURE ONLY: the CPU oracle for p0pc0rn's 4-bit matmul path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import this package. It is the
checker, never the thing measured or shipped: the product package (p0pc0rn_b200) does not import it.
The arithmetic lives in oracle.c (a C restatement of the reference's JS/WGSL, each function citing the
reference file:line it follows); this package wraps it with ctypes + numpy. Parity status: unpinned
against reference-produced outputs (the reference is JS + WebGPU and cannot run here); pinned against
the reference's own known-answer checks and hand-derived vectors in tests/test_oracle.py.
"""
