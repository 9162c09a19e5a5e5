"""Utilities: results directories and environment snapshots, timing statistics, GPU clocks."""
