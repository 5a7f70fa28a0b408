"""everserve_b200.plugin"""
