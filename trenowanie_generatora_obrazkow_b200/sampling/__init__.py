"""sampling"""
