"""everserve_b200.state"""
