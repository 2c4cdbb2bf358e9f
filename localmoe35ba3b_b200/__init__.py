"""B200-native (sm_100a) INT8 group-128 MoE matmul path.

Drop-in replacements for the reference runtime's operator API
(``qwen35_deploy.operators.int8`` / ``w8a8`` / ``routing`` and
``qwen35_deploy.runtime.gpu_routes`` / ``prefill``), backed by hand-written
CUDA in ``liblocalmoe_b200.so`` (C ABI: ``include/localmoe_b200.h``).
"""
from . import _native  # noqa: F401

__all__ = ['operators', 'runtime']
