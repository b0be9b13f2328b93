"""The forward as a torch.library custom op, ``torch.ops.apex_attn.fwd``.

The reference's only model-level caller of attention, nanochat, wraps its Blackwell kernel
the same way: a ``torch.library`` custom op returning (out, lse) so that torch.compile
traces through it without a graph break (nanochat_autoresearch/solutions/train.py:493-538).
This op calls the same C ABI as ``custom_attention_forward``; its fake implementation
gives torch.compile the output shapes and dtypes without running the kernel.

    o, lse = torch.ops.apex_attn.fwd(q, k, v, causal, sm_scale, window_left)

q: [B, H, N, D]; k, v: [B, H_kv, N, D] (H_kv divides H); sm_scale <= 0 means 1/sqrt(D);
window_left < 0 means no window. Returns o (q's dtype, contiguous) and lse (fp32 [B, H, N]).
"""
from __future__ import annotations

import math

import torch

from .ops import custom_attention_forward


@torch.library.custom_op("apex_attn::fwd", mutates_args=())
def fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, sm_scale: float,
        window_left: int) -> tuple[torch.Tensor, torch.Tensor]:
    scale = sm_scale if sm_scale > 0 else 1.0 / math.sqrt(q.shape[-1])
    return custom_attention_forward(q, k, v, causal=causal, sm_scale=scale, return_lse=True,
                                    window_left=window_left if window_left >= 0 else None)


@fwd.register_fake
def _(q, k, v, causal, sm_scale, window_left):
    b, h, n, _ = q.shape
    o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    lse = torch.empty((b, h, n), dtype=torch.float32, device=q.device)
    return o, lse
