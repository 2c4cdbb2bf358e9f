"""CPU oracle for the INT8 group-128 MoE matmul path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg use it, and only as the checker (or as the timed CPU
baseline), never as a fallback for the CUDA path.

Parity status: pinned. ``tests/golden/make_golden.py`` runs the reference's
own code (``qwen35_deploy.convert.quantize``, ``routing.plan_routes``,
``gpu_routes.plan`` and the Triton kernels under ``TRITON_INTERPRET=1``) on
seeded inputs and stores the outputs as fixtures; ``tests/test_oracle_golden.py``
checks every oracle function against them.
"""
from .oracle import *  # noqa: F401,F403
