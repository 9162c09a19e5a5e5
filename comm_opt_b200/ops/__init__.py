"""Ops: fp32 oracles (reference.py) and the native decode kernels (kernels.py)."""
