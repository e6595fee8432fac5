"""integration"""
