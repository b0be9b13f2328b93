"""A runner with the command line and output lines of the MLS-Bench fused-attention
harness (mls-bench_fused_attention/submission.py:264-341), driving this package's
``custom_attention_forward``.

    python -m apex_attn.mls_harness --batch 4 --seqlen 4096 --nheads 32 --headdim 64 --causal

It is a full-file submission in the sense of the MLS-Bench runner: that runner executes a
kernel file directly when it defines ``def main():`` and takes ``--batch``
(mls-bench_fused_attention/bench.py:87-88), and parses the ``TRAIN_METRICS:`` /
``TEST_METRICS:`` lines printed here with the regexes at bench.py:60-73.

What it does, as the harness does:
* seeds torch (CPU and CUDA) with ``--seed`` and draws q, k, v with ``randn`` on the GPU
  (submission.py:278-287);
* checks the output against torch SDPA on the same GPU with the 1e-2 max-abs gate
  (submission.py:298-317);
* times this kernel and SDPA with CUDA events (25 warm-up, 100 timed calls, median;
  submission.py:243-261);
* reports TFLOP/s with 4*B*N^2*H*d FLOPs, halved for causal (submission.py:235-240), and
  ``speedup_vs_sdpa``.

Its command line, its metric lines and its timing loop restate submission.py:243-341 on
purpose: they are the protocol the runner's parser reads, so they must match it. The
kernel it drives is this package's own.
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import torch
import torch.nn.functional as F

if __package__:
    from .ops import custom_attention_forward
else:  # run as a script (python apex_attn/mls_harness.py ...), as the MLS-Bench runner does
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from apex_attn.ops import custom_attention_forward

CORRECTNESS_THRESHOLD = 1e-2


def sdpa_attention(q, k, v, causal=True, sm_scale=None):
    """torch SDPA on the GPU: the harness's comparison kernel."""
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    return F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=sm_scale)


def attention_flops(batch, nheads, seqlen, headdim, causal):
    f = 4 * batch * seqlen * seqlen * nheads * headdim
    return f // 2 if causal else f


def median_latency_ms(fn, q, k, v, causal, sm_scale, warmup=25, rep=100):
    for _ in range(warmup):
        fn(q, k, v, causal=causal, sm_scale=sm_scale)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(rep)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(rep)]
    for i in range(rep):
        starts[i].record()
        fn(q, k, v, causal=causal, sm_scale=sm_scale)
        ends[i].record()
    torch.cuda.synchronize()
    times = sorted(s.elapsed_time(e) for s, e in zip(starts, ends))
    return times[len(times) // 2]


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description="B200 fused attention, MLS-Bench harness interface")
    ap.add_argument("--batch", type=int, required=True)
    ap.add_argument("--seqlen", type=int, required=True)
    ap.add_argument("--nheads", type=int, required=True)
    ap.add_argument("--headdim", type=int, required=True)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--dtype", default="float16", choices=["float16", "bfloat16"])
    ap.add_argument("--warmup", type=int, default=25)
    ap.add_argument("--rep", type=int, default=100)
    ap.add_argument("--output-dir", type=str, default=".")
    ap.add_argument("--seed", type=int, default=42)
    return ap.parse_args(argv)


def failure_line(max_diff=1.0):
    return (f"TEST_METRICS: speedup_vs_sdpa=0.0 tflops=0.0 latency_ms=999999.0 "
            f"sdpa_latency_ms=0.0 max_diff={max_diff:.6e} correct=0")


def success_lines(latency_ms, sdpa_latency_ms, flops, max_diff):
    tflops = flops / (latency_ms * 1e-3) / 1e12
    sdpa_tflops = flops / (sdpa_latency_ms * 1e-3) / 1e12
    speedup = sdpa_latency_ms / latency_ms
    return [
        f"TRAIN_METRICS: latency_ms={latency_ms:.3f} tflops={tflops:.1f} "
        f"sdpa_latency_ms={sdpa_latency_ms:.3f} sdpa_tflops={sdpa_tflops:.1f} "
        f"speedup_vs_sdpa={speedup:.3f}",
        f"TEST_METRICS: speedup_vs_sdpa={speedup:.4f} tflops={tflops:.4f} "
        f"latency_ms={latency_ms:.4f} sdpa_latency_ms={sdpa_latency_ms:.4f} "
        f"max_diff={max_diff:.6e} correct=1",
    ]


def run(argv=None):
    args = parse_args(argv)
    torch.manual_seed(args.seed)
    torch.cuda.manual_seed_all(args.seed)
    dtype = torch.float16 if args.dtype == "float16" else torch.bfloat16
    q = torch.randn(args.batch, args.nheads, args.seqlen, args.headdim, dtype=dtype, device="cuda")
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    sm_scale = 1.0 / math.sqrt(args.headdim)
    flops = attention_flops(args.batch, args.nheads, args.seqlen, args.headdim, args.causal)
    print(f"Config: batch={args.batch} seqlen={args.seqlen} nheads={args.nheads} "
          f"headdim={args.headdim} causal={args.causal} dtype={args.dtype}")
    print(f"FLOPs: {flops / 1e12:.3f} TFLOPs per forward pass")

    ref = sdpa_attention(q, k, v, causal=args.causal, sm_scale=sm_scale)
    try:
        out = custom_attention_forward(q, k, v, causal=args.causal, sm_scale=sm_scale)
    except Exception as e:  # the harness reports a failed kernel, it does not crash
        print(f"ERROR: custom kernel failed: {e}")
        print(failure_line())
        return 1
    max_diff = (out.float() - ref.float()).abs().max().item()
    mean_diff = (out.float() - ref.float()).abs().mean().item()
    print(f"TRAIN_METRICS: max_diff={max_diff:.6e} mean_diff={mean_diff:.6e}")
    if max_diff > CORRECTNESS_THRESHOLD:
        print(f"FAIL: max_diff {max_diff:.6e} > threshold {CORRECTNESS_THRESHOLD}")
        print(failure_line(max_diff))
        return 1
    latency = median_latency_ms(custom_attention_forward, q, k, v, args.causal, sm_scale,
                                args.warmup, args.rep)
    sdpa_latency = median_latency_ms(sdpa_attention, q, k, v, args.causal, sm_scale,
                                     args.warmup, args.rep)
    for line in success_lines(latency, sdpa_latency, flops, max_diff):
        print(line)
    return 0


def main():
    return run()


if __name__ == "__main__":
    raise SystemExit(main())
