"""CPU oracle for the NSA GR selected-block path: TEST INFRASTRUCTURE ONLY.

This package restates, in numpy / torch-on-CPU, the reference algorithm of
Sispheqgj/cxlsparse for the hot path this repository accelerates. Each
function cites the reference file:line it follows (paths are relative to the
reference project root).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline /
reference arm may import it, and only as the checker or the timed CPU
baseline. The product package ``cxlsparse_b200`` never imports this package
and has no CPU fallback.

Parity pinning: the planner restatement is pinned against fixtures generated
by running the reference's own planner (``tests/golden/make_golden.py``) and
against the known-answer vectors written in the reference's tests.
"""
