"""Generates the golden attention vectors in tests/golden/ from the reference's own code.

Run in the build container, where the read-only reference checkout exists:

    python tests/golden/make_golden.py /path/to/Apex-Tune-results

For every case it stores the seeded inputs and
  * ``o_sdpa`` / ``lse_sdpa`` — the MLS-Bench harness oracle ``reference_attention``
    (mls-bench_fused_attention/harness/pristine_custom_triton_bench.py, identical to
    submission.py:223-232) run on CPU in fp32; lse from torch.logsumexp of the same
    masked, scaled scores;
  * ``o_kernel`` — the reference Triton kernel ``_attn_fwd_plain``
    (mls-bench_fused_attention/fused_attention.py:8-87) executed by the Triton CPU
    interpreter (TRITON_INTERPRET=1) with fp32 tensors, where it can run. Its module
    imports ``triton.tools.experimental_descriptor`` (fused_attention.py:5), which this
    Triton no longer ships, so a stub module is installed first; the TMA kernel that
    needs it (``_attn_fwd_tma``) is not executed. For head dims the reference routes to
    the TMA kernel (d=128) the plain kernel is launched directly with the d=64 tile
    settings of ``_CONFIGS`` (fused_attention.py:148-152).

bf16 cases store inputs as bf16 bit patterns (uint16) to keep the fixtures small.
Nothing on the GPU box reads the reference checkout: tests only read the .npz files.
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, H, N, D, causal, dtype, q_scale, run_kernel)
CASES = [
    ("c1_b1h2n256d64_fp32", 1, 2, 256, 64, True, "float32", 1.0, True),
    ("b1h2n320d128_bf16", 1, 2, 320, 128, True, "bfloat16", 1.0, True),
    ("b1h1n192d256_bf16", 1, 1, 192, 256, True, "bfloat16", 1.0, True),
    ("b2h1n200d64_noncausal_bf16", 2, 1, 200, 64, False, "bfloat16", 1.0, True),
    ("b1h2n256d128_bigq_bf16", 1, 2, 256, 128, True, "bfloat16", 8.0, False),
    ("b1h1n100d64_fp16", 1, 1, 100, 64, True, "float16", 1.0, True),
]


def _load(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _inputs(B, H, N, D, dtype, q_scale, seed=42):
    g = torch.Generator().manual_seed(seed)
    shape = (B, H, N, D)
    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[dtype]
    q = (torch.randn(shape, generator=g) * q_scale).to(tdt)
    k = torch.randn(shape, generator=g).to(tdt)
    v = torch.randn(shape, generator=g).to(tdt)
    return q, k, v


def _store(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.contiguous().numpy()
    return t.numpy()


def main(ref_root: str) -> None:
    fa_dir = os.path.join(ref_root, "mls-bench_fused_attention")
    harness = _load(os.path.join(fa_dir, "harness", "pristine_custom_triton_bench.py"), "ref_harness")
    stub = types.ModuleType("triton.tools.experimental_descriptor")
    stub.create_2d_tma_descriptor = lambda *a, **k: None
    sys.modules["triton.tools.experimental_descriptor"] = stub
    fa = _load(os.path.join(fa_dir, "fused_attention.py"), "ref_fused_attention")

    for name, B, H, N, D, causal, dtype, q_scale, run_kernel in CASES:
        q, k, v = _inputs(B, H, N, D, dtype, q_scale)
        q32, k32, v32 = q.float(), k.float(), v.float()
        scale = 1.0 / math.sqrt(D)
        o_sdpa = harness.reference_attention(q32, k32, v32, causal=causal, sm_scale=scale)
        s = (q32 @ k32.transpose(-1, -2)) * scale
        if causal:
            s = s.masked_fill(torch.ones(N, N, dtype=torch.bool).triu(1), float("-inf"))
        lse = torch.logsumexp(s, dim=-1)
        out = dict(q=_store(q), k=_store(k), v=_store(v), o_sdpa=o_sdpa.numpy(), lse_sdpa=lse.numpy(),
                   meta=np.array([B, H, N, D, int(causal)], dtype=np.int64),
                   dtype=np.array(dtype), q_scale=np.array(q_scale))
        if run_kernel:
            o = torch.empty_like(q32)
            cfg = fa._CONFIGS[64]
            grid = (math.ceil(N / cfg["BLOCK_M"]), B * H)
            fa._attn_fwd_plain[grid](
                q32, k32, v32, o, scale * 1.4426950408889634,
                q32.stride(1), q32.stride(2), q32.stride(3),
                k32.stride(1), k32.stride(2), k32.stride(3),
                v32.stride(1), v32.stride(2), v32.stride(3),
                o.stride(1), o.stride(2), o.stride(3),
                N, BLOCK_M=cfg["BLOCK_M"], BLOCK_N=cfg["BLOCK_N"], BLOCK_DMODEL=D,
                IS_CAUSAL=causal, LPT=bool(cfg["lpt"] and causal),
                num_warps=cfg["num_warps"], num_stages=cfg["num_stages"])
            out["o_kernel"] = o.numpy()
            print(f"{name}: |kernel - sdpa|max = {(o - o_sdpa).abs().max().item():.3e}")
        else:
            print(f"{name}: sdpa only")
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("APEX_REFERENCE_ROOT", ""))
