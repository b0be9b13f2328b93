"""apex_attn — B200-native (sm_100a) fused causal attention, forward and backward.

Drop-in for the operator of mls-bench_fused_attention/fused_attention.py:155-193; the
backward and the autograd-enabled ``torch.ops.apex_attn.fwd`` serve training callers such
as the reference's nanochat model.
"""
from .ops import (custom_attention_backward, custom_attention_forward,
                  custom_attention_varlen_backward, custom_attention_varlen_forward, device_status,
                  forward_kernel_for, selftest_wait_timeout, set_forward_kernel, supports_head_dim)
from . import _lib
from . import torch_op  # registers torch.ops.apex_attn.fwd / .bwd
from .torch_op import attention

__all__ = ["attention", "custom_attention_forward", "custom_attention_backward",
           "custom_attention_varlen_forward", "custom_attention_varlen_backward", "device_status",
           "forward_kernel_for", "selftest_wait_timeout", "set_forward_kernel", "supports_head_dim", "library_path", "version"]


def library_path() -> str:
    return _lib.LIB_PATH


def version() -> int:
    return int(_lib.load().apex_attn_version())
