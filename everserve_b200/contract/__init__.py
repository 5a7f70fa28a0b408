"""everserve_b200.contract"""
