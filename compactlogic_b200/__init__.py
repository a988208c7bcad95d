"""compactlogic_b200 — the CompactLogic logic-layer hot path on hand-written sm_100a kernels.

Drop-in for the reference package: ``from compactlogic_b200 import *`` provides the same
LogicLayer / ConvLayer / GroupSum / hooks API (compactlogic/__init__.py:1).
"""
from .compactlogic import *  # noqa: F401,F403
from .compactlogic import __all__ as _api
from .packed import PackedLogicNet, packed_from_state_dict  # noqa: F401

__all__ = list(_api) + ["PackedLogicNet", "packed_from_state_dict"]
