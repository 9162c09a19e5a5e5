"""Llama-shaped tensor-parallel decode runner and its projection layers."""
