"""CPU oracle for the retrieve_b200 parity tests. TEST INFRASTRUCTURE ONLY.

A plain restatement (numpy, plus C in ``oracle/c``) of the reference's algorithms
for the scoring-and-selection path of rmnigm/retrieve, each function citing the
reference file:line it follows. It is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it. The
product (``retrieve_b200``) never does, and has no CPU path at all.

Parity pinning: the restatements are checked against golden vectors produced by
running the reference's own torch path in the build container
(``tests/golden/make_golden.py`` → ``tests/golden/*.npz``) and against the
known-answer facts of the reference's test suite (``tests/test_oracle_pins.py``).
"""
