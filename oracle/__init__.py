"""TEST INFRASTRUCTURE ONLY.

CPU restatement of the reference's optimizer step (vincentzed/cs336-a1-sol,
transformer_lm/sol_modules.py and transformer_lm/train_sol.py), used as the
checker for the B200 engine. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / --impl reference legs may import it. The engine
(cs336-a1-sol_b200/sol_b200) never imports or calls anything here.

Pinning: oracle/ref_step.py is pinned bit-for-bit against the reference itself
(imported in the build container) through the golden digests in tests/golden/
(made by tests/golden/make_golden.py). The Gram Newton-Schulz / Polar Express
path has no reference golden (the gram-newton-schulz package is not in the
reference tree): that part is "parity unpinned" against the package and is
checked against the fp64 restatement in oracle/gram_ns_ref.py and against SVD.
"""
