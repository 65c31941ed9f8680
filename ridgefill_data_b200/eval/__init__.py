"""Evaluation harness pieces: synthetic data, cost model, metrics."""
