"""CPU oracle for nvattn — TEST INFRASTRUCTURE ONLY.

Restates the reference's algorithm for the attention path on the CPU so the
CUDA kernels can be checked against it. Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg may import it; the product path never does.
See reference_math.py for the restatement and its citations.
"""
