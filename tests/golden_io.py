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
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
