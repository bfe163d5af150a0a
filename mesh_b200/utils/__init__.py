"""Utilities: per-op microbenchmarks, decode-step profiling driver, logging and timing helpers."""
