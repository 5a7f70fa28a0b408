"""everserve_b200.utils"""
