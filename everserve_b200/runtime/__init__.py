"""everserve_b200.runtime"""
