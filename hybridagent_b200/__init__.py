"""B200 (sm_100a) ZeRO-1 AdamW step, a drop-in for HybridAgent's hybrid_rl.optimizer.ZeroOneAdamW.

The compute path is ``lib/libhybridagent_b200.so`` (hand-written CUDA + NCCL behind the C ABI
of ``include/hybridagent_b200.h``); this package is its Python host side.
"""
from .optimizer import ZeroOneAdamW

__all__ = ["ZeroOneAdamW"]
