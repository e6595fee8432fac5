"""Multiprocess mode: one cache-server process holds the CPU tier and moves KV
for serving workers that hand it their paged caches by IPC handle."""
