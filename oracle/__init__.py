"""TEST INFRASTRUCTURE — the CPU oracle of the region arithmetic.

Used only by tests/, __graft_entry__.smoke() (as the checker) and bench.py's
cpu_baseline leg (as the timed CPU baseline). The product path never imports
this package.

Parity status: the comparison policy (numeric_ref) and the launch grammar are
pinned against the reference's own known-answer tests (tests/golden/). The
floating-point region arithmetic restates MLX 0.32.2 / mlx-lm 0.31.3 as the
reference writes it down (autotuner/scaffold/lower.py) and is UNPINNED: MLX
is not installed here and the reference stores no golden outputs.
"""
