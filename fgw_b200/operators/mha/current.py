"""Current paged MHA entry points (FGW operators/mha/current.py:7 re-exports v7 the same way).

Callers of ``operators.mha.current`` switch their import to ``fgw_b200.operators.mha.current``;
the call signature, tensor contract, metadata attributes and ValueError conditions are unchanged.
"""
from fgw_b200.operators.mha.kernels.mha_paged_fwd_sm100 import build_kernel, mha_paged_decode, route

__all__ = ["build_kernel", "mha_paged_decode", "route"]
