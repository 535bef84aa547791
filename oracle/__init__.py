"""Test oracle: a CPU restatement of diffrast's reference backend for the render path.

This package is test infrastructure. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` may import it, and there only as the checker or the timed CPU
baseline. The product (``diffrast_b200``) never imports it and has no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference package itself on seeded
scenes and stores its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this
restatement against those fixtures on every CPU test run.
"""

from oracle.restatement import *  # noqa: F401,F403
