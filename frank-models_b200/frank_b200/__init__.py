"""frank_b200: B200-native (sm_100a) MoE FFN hot path of frank-models.

Public surface
  B200Module            reference-shaped module: mul_mat_id / moe_ffn_block / swiglu
  MoEFFNBlock           weights packed once, reusable workspace (serving/bench path)
  ops.*                 typed torch wrappers over the C ABI (include/frank_moe.h)
"""

from . import _lib, ops  # noqa: F401
from .module import B200Module  # noqa: F401
from .ops import MoEFFNBlock, PackedExperts  # noqa: F401

__all__ = ["B200Module", "MoEFFNBlock", "PackedExperts", "ops"]
