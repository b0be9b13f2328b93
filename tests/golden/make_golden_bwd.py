"""Generates the backward golden vectors tests/golden/bwd_*.npz.

Run in the build container, where the read-only reference checkout exists:

    python tests/golden/make_golden_bwd.py /path/to/Apex-Tune-results

The gradients come from torch autograd (float64, CPU) through the MLS-Bench harness oracle
``reference_attention`` (mls-bench_fused_attention/harness/pristine_custom_triton_bench.py,
identical to submission.py:223-232) for the causal and full cases. Grouped-query and
sliding-window cases, which that oracle cannot express, go through the same
``F.scaled_dot_product_attention`` call with ``enable_gqa=True`` or an explicit boolean
mask of the window flash_attn_func(window_size=(w, 0)) applies
(nanochat_autoresearch/solutions/train.py:719).

Each file stores q, k, v, dout (bf16 bit patterns), the float64-derived dq, dk, dv as
float32, and meta = [B, H, H_kv, N, D, causal, window_left (-1 = none)].
Nothing on the GPU box reads the reference checkout: tests only read the .npz files.
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, H, H_kv, N, D, causal, window_left)
CASES = [
    ("bwd_b1h2n256d64_causal", 1, 2, 2, 256, 64, True, -1),
    ("bwd_b1h1n200d128_causal", 1, 1, 1, 200, 128, True, -1),
    ("bwd_b2h1n160d64_full", 2, 1, 1, 160, 64, False, -1),
    ("bwd_b1h4kv2n192d64_gqa", 1, 4, 2, 192, 64, True, -1),
    ("bwd_b1h1n256d128_win40", 1, 1, 1, 256, 128, True, 40),
]


def _load_harness(ref_root: str):
    path = os.path.join(ref_root, "mls-bench_fused_attention", "harness",
                        "pristine_custom_triton_bench.py")
    spec = importlib.util.spec_from_file_location("ref_harness", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    harness = _load_harness(ref_root)
    for name, B, H, HKV, N, D, causal, win in CASES:
        g = torch.Generator().manual_seed(7)
        q = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, HKV, N, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, HKV, N, D, generator=g).to(torch.bfloat16)
        do = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16)
        q64, k64, v64 = (t.double().requires_grad_(True) for t in (q, k, v))
        scale = 1.0 / math.sqrt(D)
        if HKV == H and win < 0:
            o = harness.reference_attention(q64, k64, v64, causal=causal, sm_scale=scale)
        elif win < 0:
            o = F.scaled_dot_product_attention(q64, k64, v64, is_causal=causal, scale=scale,
                                               enable_gqa=True)
        else:
            i = torch.arange(N)[:, None]
            j = torch.arange(N)[None, :]
            visible = (j <= i) & (j >= i - win)
            o = F.scaled_dot_product_attention(q64, k64, v64, attn_mask=visible, scale=scale,
                                               enable_gqa=HKV != H)
        o.backward(do.double())
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            q=_bits(q), k=_bits(k), v=_bits(v), dout=_bits(do),
            dq=q64.grad.float().numpy(), dk=k64.grad.float().numpy(), dv=v64.grad.float().numpy(),
            meta=np.array([B, H, HKV, N, D, int(causal), win], dtype=np.int64))
        print(f"{name}: |dq|max={q64.grad.abs().max():.3f} |dk|max={k64.grad.abs().max():.3f} "
              f"|dv|max={v64.grad.abs().max():.3f}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("APEX_REFERENCE_ROOT", ""))
