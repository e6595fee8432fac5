"""v1/blend"""
