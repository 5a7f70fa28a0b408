"""everserve_b200.parallel"""
