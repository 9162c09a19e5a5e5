"""comm_opt_b200: Blackwell-native decode-time tensor-parallel communication.

    from comm_opt_b200 import fused_allreduce_add_rmsnorm, layer_boundary
    out, residual = fused_allreduce_add_rmsnorm(x, residual, gamma, eps)
"""
from .api import fused_allreduce_add_rmsnorm, layer_boundary, release

__all__ = ["fused_allreduce_add_rmsnorm", "layer_boundary", "release"]
