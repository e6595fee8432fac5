"""v1/storage_backend/pd"""
