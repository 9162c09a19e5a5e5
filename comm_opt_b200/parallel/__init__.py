"""Communication substrate: symmetric heap, tensor-parallel communicator, variant table."""
from .communicator import TPCommError, TPCommTimeout, TPCommunicator
from .config import CommConfig
from .health import RankFailure, RankMonitor
from .symm import HeapLayout, SymmetricHeap, plan_layout
from .variant_table import VARIANT_NAMES, VARIANTS, Choice, VariantTable

__all__ = ["TPCommunicator", "CommConfig", "RankMonitor", "RankFailure", "TPCommError", "TPCommTimeout", "SymmetricHeap", "HeapLayout", "plan_layout",
           "VariantTable", "Choice", "VARIANTS", "VARIANT_NAMES"]
