"""CPU oracle for the ReCaVSR DiT hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's algorithms (each function cites the
reference file:line it follows). Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / ``--impl reference`` legs may import this
package, and only as the checker or the timed CPU baseline. The product
(``recavsr_b200``) never imports it and has no CPU fallback.

Parity pin: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors produced by the reference itself (``tests/golden/make_golden.py``
imports ``recavsr_infer`` with two import shims and records its outputs).
"""
