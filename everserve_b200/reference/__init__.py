"""The CPU reference tier: placement-independent arithmetic, the SHRINK outcome, and an exact
in-process store. Not on any GPU serving path; it is the specification the GPU path is checked
against and the tier the SHRINK outcome runs on.

Reference parity: core/everserve/reference/__init__.py:3-33.
"""
