"""CPU oracle for wxx_b200 parity tests -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's (Mo-Ehab/wxx) WGSL kernels and model
forwards.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs use it, and only as the checker or the timed CPU implementation; the
product package (wxx_b200) never imports it.

Parity pinning: the reference itself cannot run in this environment (its wgpu
backend needs a graphics adapter), so the oracle is pinned against
(1) golden vectors produced by the reference's own pure-numpy test helpers
(tests/golden/make_golden.py extracts them from the reference test files),
(2) the reference tests' known-answer formulas, restated in tests/, and
(3) independent float64 implementations (numpy.fft, float64 matmul).
matmul, conv2d and the FFT have no known-answer test in the reference
(only gradient checks and shape checks); for those, parity is pinned to the
float64 mathematics rather than to reference outputs.
"""

from . import init, kernels, models

__all__ = ["init", "kernels", "models"]
