"""CPU restatement of the Orthrus dual-view hot path, used only as the checker.

This package is test infrastructure. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it; the product package ``orthrus_training_b200`` never
does, and its CUDA path fails loudly when the compiled library is missing instead of falling
back to anything here.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference implementation
(ekonst41/orthrus-training, pure Python) on seeded inputs and stores its outputs as fixtures,
and ``tests/test_oracle_golden.py`` checks this restatement against them.
"""

from oracle.orthrus_oracle import *  # noqa: F401,F403
