"""integration/vllm"""
