"""CPU oracle of the batched multi-adapter LoRA path — TEST INFRASTRUCTURE ONLY.

A restatement, in numpy and plain Python, of the reference algorithm
(Knowledgator/PolyLoRA, src/polylora/): each function cites the reference
file:line it follows.  It is pinned against golden vectors produced by the
reference itself (tests/golden/make_golden.py imports the reference package
and runs it on seeded inputs; tests/test_oracle_golden.py checks this oracle
against those files).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this package, and only as the checker or the timed CPU baseline.  The
product package ``polylora_b200`` never imports it and has no CPU compute path.
"""
