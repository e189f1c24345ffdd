"""CPU oracle for the Gemma-4-12B text-decoder hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the thing measured or shipped: only tests/,
`__graft_entry__.smoke()` and bench.py's CPU-baseline leg may import it.  It restates,
in numpy, the reference's input synthesis
(scripts/fixture_prng.py) and the per-kernel math of its expected-output generator
(scripts/generate_references.py).  It is pinned against the golden vectors produced by
running that generator (tests/golden/reference_fixtures.npz, tests/golden/make_golden.py).
"""
