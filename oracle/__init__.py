"""CPU oracle for the quantized attention path — TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline / reference legs of `bench.py` may
import this package, and only as a checker. The product path (the CUDA library behind
`lingbot_b200`) never calls into it.
"""
