"""Measurement helpers shared by bench.py and the sweep runner."""
