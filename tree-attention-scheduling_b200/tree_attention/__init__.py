"""B200-native tree-shared decode attention (drop-in for the reference ``tree_attention``)."""
from .tree import KVTree
from .schedule import CostModel, Plan, schedule

__all__ = ["KVTree", "CostModel", "Plan", "schedule"]
