"""CPU oracle for the B200 speculative-decoding engine: TEST INFRASTRUCTURE ONLY.

Plain restatements (numpy, and C for the n-gram scan) of the reference's algorithm for the
hot path, each function citing the reference file:line it follows
(beriltatli/speculative-decoder). Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import anything here, and only as the checker or the timed CPU
baseline, never on the product path: the engine has no CPU fallback.

Pinning: tests/golden/ holds input/output vectors produced by running the reference itself
(tests/golden/make_golden.py, which imports the reference read-only in a separate process);
tests/test_oracle.py checks every function here against them.
"""
