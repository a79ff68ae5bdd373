"""Benchmarks: kernel microbenchmarks, the all-reduce sweep and the reference's tables."""
