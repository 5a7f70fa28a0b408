"""everserve_b200.proto"""
