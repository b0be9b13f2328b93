"""Plain PyTorch fp32 attention on the GPU: the full-size numerics reference for the
floating-point kernel (the CPU oracle is too slow at BASELINE sizes). It is pinned
against the CPU oracle in tests/test_attn_gpu.py before it is trusted."""
from __future__ import annotations

import math

import torch


@torch.no_grad()
def attention_fp32(q, k, v, causal=True, sm_scale=None, row_chunk=1024, head_chunk=16,
                   with_lse=True):
    """fp32 softmax(QK^T * scale + mask) V on q's device; returns (o fp32, lse fp32)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        B, H, N, D = q.shape
        if sm_scale is None:
            sm_scale = 1.0 / math.sqrt(D)
        qf = q.reshape(B * H, N, D)
        kf = k.reshape(B * H, N, D)
        vf = v.reshape(B * H, N, D)
        o = torch.empty((B * H, N, D), dtype=torch.float32, device=q.device)
        lse = torch.empty((B * H, N), dtype=torch.float32, device=q.device) if with_lse else None
        for h0 in range(0, B * H, head_chunk):
            h1 = min(B * H, h0 + head_chunk)
            kh = kf[h0:h1].float()
            vh = vf[h0:h1].float()
            for r0 in range(0, N, row_chunk):
                r1 = min(N, r0 + row_chunk)
                kmax = r1 if causal else N
                s = torch.matmul(qf[h0:h1, r0:r1].float(), kh[:, :kmax].transpose(1, 2)) * sm_scale
                if causal:
                    rows = torch.arange(r0, r1, device=q.device)[:, None]
                    cols = torch.arange(kmax, device=q.device)[None, :]
                    s.masked_fill_(cols > rows, float("-inf"))
                l = torch.logsumexp(s, dim=-1, keepdim=True)
                o[h0:h1, r0:r1] = torch.matmul(torch.exp(s - l), vh[:, :kmax])
                if with_lse:
                    lse[h0:h1, r0:r1] = l[..., 0]
                del s
        return o.reshape(B, H, N, D), (lse.reshape(B, H, N) if with_lse else None)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
