"""The gated delta rule on B200 (sm_100a): the drop-in, its autograd op and the reference's utilities
(the reference's src/macai/gated_delta/__init__.py exports the same four names)."""
from .op import GatedDeltaRule, chunk_gated_delta_rule, l2norm, recurrent_reference

__all__ = ["GatedDeltaRule", "chunk_gated_delta_rule", "l2norm", "recurrent_reference"]
