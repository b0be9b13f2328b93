"""Reads the golden fixtures written by tests/golden/make_golden.py."""
from __future__ import annotations

import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def load_case(path: str) -> dict:
    z = np.load(path, allow_pickle=False)
    dtype = str(z["dtype"])
    out = {"name": os.path.basename(path)[:-4], "dtype": dtype}
    for key in ("q", "k", "v"):
        a = z[key]
        if dtype == "bfloat16":
            a = bf16_bits_to_f32(a)
        out[key] = a.astype(np.float32)
    B, H, N, D, causal = (int(x) for x in z["meta"])
    out.update(B=B, H=H, N=N, D=D, causal=bool(causal), o_sdpa=z["o_sdpa"], lse_sdpa=z["lse_sdpa"],
               o_kernel=z["o_kernel"] if "o_kernel" in z.files else None)
    return out


def cases() -> list[str]:
    """Forward fixtures (tests/golden/make_golden.py)."""
    return sorted(p for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(p).startswith("bwd_"))


def bwd_cases() -> list[str]:
    """Backward fixtures (tests/golden/make_golden_bwd.py)."""
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "bwd_*.npz")))


def load_bwd_case(path: str) -> dict:
    z = np.load(path, allow_pickle=False)
    out = {"name": os.path.basename(path)[:-4]}
    for key in ("q", "k", "v", "dout"):
        out[key] = bf16_bits_to_f32(z[key]).astype(np.float32)
    for key in ("dq", "dk", "dv"):
        out[key] = z[key]
    B, H, HKV, N, D, causal, win = (int(x) for x in z["meta"])
    out.update(B=B, H=H, HKV=HKV, N=N, D=D, causal=bool(causal), window=None if win < 0 else win)
    return out
