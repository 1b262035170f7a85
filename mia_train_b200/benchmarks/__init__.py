"""Benchmark workloads beyond the default `bench.py` configuration."""
