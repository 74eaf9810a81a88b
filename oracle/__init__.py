"""CPU parity oracle for the AEISU 2x inference path (TEST INFRASTRUCTURE ONLY).

This package restates, in plain numpy, the algorithm of the reference's portable
PyTorch path (aeisu/model.py, aeisu/reconstruction.py, aeisu/runtime.py) and of
its SPYR8 mixed FP8/FP16 artifact numerics.  It is the checker, never the product:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(``cpu_baseline`` / ``--impl reference``) may import it.  The product path in
``aeisu_b200`` never imports anything from here and fails loudly when its CUDA
library is missing.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference PyTorch model
itself (imported from a reference checkout) and commits its outputs as fixtures;
``tests/test_oracle_golden.py`` checks this restatement against every one of them
and against the known-answer tests of the reference's own test suite
(tests/test_reference.py:31-61, 109-117).
"""
