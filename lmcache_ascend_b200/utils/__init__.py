"""Shared utilities: logging, hashing, cache keys, NVTX, metrics, timing."""
