"""fgw_b200: B200-native (sm_100a) paged multi-head-attention forward with FGW's operators/mha API.

The compute path is ``libfgw_mha.so`` (hand-written CUDA behind the C ABI in include/fgw_mha.h),
loaded through ``fgw_b200._native``; ``fgw_b200.operators.mha.current`` is the drop-in Python API.
"""
__version__ = "0.1.0"
