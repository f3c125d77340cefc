"""Benchmark workloads beyond the headline training benchmark (``bench.py``)."""
