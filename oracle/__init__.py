"""CPU oracle for the OLMoE sparse-MoE hot path (test infrastructure only).

This package is the checker, never the product: only ``tests/``, the
``smoke()`` self-check in ``__graft_entry__`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The shipped path
(``trifuse_b200``) never imports anything from here and fails loudly when its
CUDA library is missing.

Parity status: the operator bodies are pinned against golden vectors produced
by the reference's own torch CPU operators (``native_affine_ops.py``) composed
exactly as the reference's OLMoE export adapter composes them; see
``tests/golden/make_golden.py``.  MLX itself (the reference's numerical
backend) is not available on this machine, so results at the MLX boundary are
pinned only through those torch bodies.
"""
from .olmoe import *  # noqa: F401,F403
