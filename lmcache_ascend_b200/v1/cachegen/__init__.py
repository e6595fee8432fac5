"""v1/cachegen"""
