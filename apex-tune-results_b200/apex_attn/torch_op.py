"""The forward and backward as torch.library custom ops, ``torch.ops.apex_attn.fwd`` / ``.bwd``.

The reference's only model-level caller of attention, nanochat, wraps its Blackwell kernel
the same way: a ``torch.library`` custom op returning (out, lse) so that torch.compile
traces through it without a graph break (nanochat_autoresearch/solutions/train.py:493-538).
This op calls the same C ABI as ``custom_attention_forward``; its fake implementation
gives torch.compile the output shapes and dtypes without running the kernel.

    o, lse = torch.ops.apex_attn.fwd(q, k, v, causal, sm_scale, window_left)

q: [B, H, N, D]; k, v: [B, H_kv, N, D] (H_kv divides H); sm_scale <= 0 means 1/sqrt(D);
window_left < 0 means no window. Returns o (q's dtype, contiguous) and lse (fp32 [B, H, N]).

``fwd`` is differentiable: its registered autograd formula saves q, k, v, o and lse and
calls ``torch.ops.apex_attn.bwd(q, k, v, o, dout, lse, causal, sm_scale, window_left)``,
the sm_100a backward, mirroring nanochat's fa4_causal / fa4_bwd pair
(nanochat_autoresearch/solutions/train.py:493-531). ``attention(q, k, v, ...)`` returns
just o from the differentiable op.
"""
from __future__ import annotations

import math

import torch

from .ops import custom_attention_backward, custom_attention_forward


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


@torch.library.custom_op("apex_attn::bwd", mutates_args=())
def bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, dout: torch.Tensor,
        lse: torch.Tensor, causal: bool, sm_scale: float,
        window_left: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    scale = sm_scale if sm_scale > 0 else 1.0 / math.sqrt(q.shape[-1])
    return custom_attention_backward(q, k, v, o, lse, dout, causal=causal, sm_scale=scale,
                                     window_left=window_left if window_left >= 0 else None)


@bwd.register_fake
def _(q, k, v, o, dout, lse, causal, sm_scale, window_left):
    return (torch.empty(q.shape, dtype=q.dtype, device=q.device),
            torch.empty(k.shape, dtype=k.dtype, device=k.device),
            torch.empty(v.shape, dtype=v.dtype, device=v.device))


def _setup_context(ctx, inputs, output):
    q, k, v, causal, sm_scale, window_left = inputs
    o, lse = output
    ctx.save_for_backward(q, k, v, o, lse)
    ctx.causal, ctx.sm_scale, ctx.window_left = causal, sm_scale, window_left


def _backward(ctx, dout, dlse):
    # The logsumexp output is a by-product for the backward; it takes no gradient.
    q, k, v, o, lse = ctx.saved_tensors
    dq, dk, dv = torch.ops.apex_attn.bwd(q, k, v, o, dout.contiguous(), lse, ctx.causal,
                                         ctx.sm_scale, ctx.window_left)
    return dq, dk, dv, None, None, None


fwd.register_autograd(_backward, setup_context=_setup_context)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
              sm_scale: float | None = None, window_left: int | None = None) -> torch.Tensor:
    """Differentiable attention output (see the module docstring)."""
    o, _ = torch.ops.apex_attn.fwd(q, k, v, causal, -1.0 if sm_scale is None else float(sm_scale),
                                   -1 if window_left is None else int(window_left))
    return o
