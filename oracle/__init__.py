"""CPU oracle for Sheaf's compiled fwd+VJP path. TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic that Sheaf's compiled
`value_and_grad` modules perform (the stdlib math in sheaf/lib/nn.shf, the
nanoGPT model in examples/nanogpt/model.shf, the VJP rules in
sheaf/src/autodiff/reverse.rs, the PRNG in sheaf/src/core/prng.rs and the
bf16 rounding in sheaf/src/core/dtype.rs). Every function cites the
reference file:line it follows.

It is the checker, never the thing measured or shipped: only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may
import it. The product path (``sheaf_b200``) never imports this package and
has no CPU fallback.

Pinning: the op rules are checked against the reference's own golden vectors
(sheaf/tests/vag_tests.yaml, interpreter_tests.yaml, the analytic layer-norm
test in interpreter_tests.rs:146-170) and the PRNG against the Random123
known-answer vectors in core/prng.rs:170-179 (tests/test_oracle_goldens.py).
Whole-model values at nanoGPT scale are not pinned by any reference test;
there the oracle is the composition of those pinned rules.
"""
