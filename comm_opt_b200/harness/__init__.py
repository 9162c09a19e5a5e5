"""Measurement harness: sweeps, microbenchmarks, profiling drivers, analyzers, results directories."""
