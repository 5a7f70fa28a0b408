"""everserve_b200.reference"""
