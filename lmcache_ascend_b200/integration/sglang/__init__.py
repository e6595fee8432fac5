"""integration/sglang"""
