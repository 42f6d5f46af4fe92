"""ferry_b200 -- B200-native implementation of FERRY's per-MoE-layer hot path.

The package mirrors the reference's Python API (ferry.metadata, ferry.policy,
ferry.quota, ferry.layout, ferry.transport, ferry.runtime and the native
module ferry_expert_ops) over libferryb.so, a C-ABI library of hand-written
sm_100a kernels (include/ferryb.h).
"""
__version__ = '0.1.0'
