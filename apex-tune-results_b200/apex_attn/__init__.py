"""apex_attn — B200-native (sm_100a) fused causal attention forward.

Drop-in for the operator of mls-bench_fused_attention/fused_attention.py:155-193.
"""
from .ops import (custom_attention_forward, device_status, selftest_wait_timeout,
                  supports_head_dim)
from . import _lib
from . import torch_op  # registers torch.ops.apex_attn.fwd

__all__ = ["custom_attention_forward", "device_status", "selftest_wait_timeout",
           "supports_head_dim", "library_path", "version"]


def library_path() -> str:
    return _lib.LIB_PATH


def version() -> int:
    return int(_lib.load().apex_attn_version())
