"""CPU oracle for the learner-update hot path. TEST INFRASTRUCTURE ONLY.

A numpy restatement of scaleresearch/tt-rl's learner arithmetic, each
function citing the reference file:line it follows. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it, and only as the checker or the timed CPU baseline -- never as
a code path of the product. The product (``tt-rl_b200/ttrl_b200``) has no
CPU fallback and never imports this package.

Parity pinning: the restatement is checked against golden vectors produced
by the reference's own code (``tests/golden/make_golden.py`` runs the
reference's autograd tape, ops, Adam and losses over a numpy stand-in for
``ttnn``, and its numpy deploy forward for the conv tower) in
``tests/test_oracle_golden.py``.
"""
