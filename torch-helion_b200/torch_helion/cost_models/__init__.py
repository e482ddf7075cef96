"""Cost models: the B200 roofline estimator used by the planner."""

from .b200 import B200Spec, CostBreakdown, CostModelError, kernel_cost, search_tiles

__all__ = ["B200Spec", "CostBreakdown", "CostModelError", "kernel_cost", "search_tiles"]
