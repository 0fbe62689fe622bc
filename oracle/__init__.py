"""CPU oracle of the inference-kernel path (TEST INFRASTRUCTURE, not product code).

A plain PyTorch/numpy restatement of what the reference's own PyTorch `Model`s and
harness oracles compute for the three operators.  Only tests, the smoke check and
the CPU-baseline leg of bench.py may import this package; the product package never
does and has no CPU path of its own.

Parity is pinned: tests/golden/make_golden.py imports the reference's functions
themselves, checks that this restatement reproduces them, and stores their outputs
as fixtures under tests/golden/ which tests/test_oracle_golden.py replays.
"""
