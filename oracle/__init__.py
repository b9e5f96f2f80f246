"""CPU oracle for the MergeNet DTEM spatial-routing hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, in plain numpy, the
reference algorithm the CUDA library reproduces.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may
import it, and only as the parity reference or as the timed CPU baseline; the product
path (``mergenet_b200``) never calls into it.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
(its own ``DTEMBlock._merge_train``, ``ThreTopK`` and carrier block) on seeded
inputs and stores the outputs as fixtures; ``tests/test_oracle_golden.py``
checks this oracle against them.
"""
