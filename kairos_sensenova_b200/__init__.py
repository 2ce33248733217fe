"""B200-native (sm_100a) implementation of the Kairos hybrid-attention hot path.

Public operators keep the reference's PyTorch signatures:

* :func:`chunk_gated_delta_rule`  -- ``fla/ops/gated_delta_rule/chunk.py:216``
"""
from .gated_delta_rule import chunk_gated_delta_rule  # noqa: F401

__all__ = ['chunk_gated_delta_rule']
