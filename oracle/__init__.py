"""CPU oracle for the crumpet_b200 hot path -- TEST INFRASTRUCTURE ONLY.

A restatement of the reference algorithms in numpy, used as the checker by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py``.  Nothing in the ``crumpet_b200`` package imports this package;
the product path has no CPU fallback.

Parity pin: ``tests/golden/`` holds digests and arrays produced by the
reference's own pure-PyTorch functions (torch-ext/crumpet/reference.py) and,
for attention, by the reference Triton kernel (torch-ext/crumpet/
fused_attention.py:48-146) run under the Triton CPU interpreter; the script
that made them is ``tests/golden/make_golden.py``.  ``tests/test_oracle.py``
checks this oracle against those fixtures before any GPU result is compared
with it.
"""
