"""The MLS-Bench drop-in files: the splice-mode kernel file and the full-file runner
(apex_attn/mls_harness.py), checked against the interface of the MLS-Bench runner
(mls-bench_fused_attention/bench.py): how it recognises a full-file submission (:87-88)
and the output lines it parses (:60-73)."""
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "apex-tune-results_b200")
RUNNER = os.path.join(PKG, "apex_attn", "mls_harness.py")

# The runner's parse patterns (mls-bench_fused_attention/bench.py:60-73).
TRAIN_RE = re.compile(r"TRAIN_METRICS: max_diff=([\d.eE+-]+) mean_diff=([\d.eE+-]+)")
TEST_RE = re.compile(r"TEST_METRICS: speedup_vs_sdpa=([\d.]+) tflops=([\d.]+) "
                     r"latency_ms=([\d.]+) sdpa_latency_ms=([\d.]+) "
                     r"max_diff=([\d.eE+-]+) correct=(\d+)")


def test_runner_is_recognised_as_full_submission():
    text = open(RUNNER).read()
    assert "def main():" in text and "--batch" in text


def test_metric_lines_match_the_runner_patterns():
    from apex_attn import mls_harness as m
    lines = m.success_lines(0.25, 0.4, m.attention_flops(4, 32, 4096, 64, True), 1.95e-3)
    g = TEST_RE.search("\n".join(lines))
    assert g and int(g.group(6)) == 1
    assert abs(float(g.group(2)) - m.attention_flops(4, 32, 4096, 64, True) / 0.25e-3 / 1e12) < 1e-3
    assert abs(float(g.group(1)) - 0.4 / 0.25) < 1e-4
    fail = TEST_RE.search(m.failure_line(0.5))
    assert fail and int(fail.group(6)) == 0


def test_cli_and_flop_convention():
    from apex_attn import mls_harness as m
    a = m.parse_args(["--batch", "2", "--seqlen", "8192", "--nheads", "16", "--headdim", "128", "--causal"])
    assert (a.batch, a.seqlen, a.nheads, a.headdim, a.causal, a.dtype, a.seed) == (2, 8192, 16, 128, True, "float16", 42)
    assert m.attention_flops(2, 16, 8192, 128, True) == 4 * 2 * 8192 ** 2 * 16 * 128 // 2


def test_splice_kernel_file_exports_operator():
    ns = {}
    sys.path.insert(0, PKG)
    exec(open(os.path.join(PKG, "mls_kernel.py")).read(), ns)
    from apex_attn import custom_attention_forward
    assert ns["custom_attention_forward"] is custom_attention_forward


@pytest.mark.gpu
@pytest.mark.parametrize("D,dtype", [(64, "float16"), (128, "bfloat16"), (256, "float16")])
def test_runner_end_to_end_on_gpu(D, dtype):
    import torch
    if not torch.cuda.is_available() or torch.cuda.get_device_capability() != (10, 0):
        pytest.skip("needs a B200 (sm_100)")
    cmd = [sys.executable, RUNNER, "--batch", "1", "--seqlen", "1000", "--nheads", "4", "--headdim", str(D),
           "--causal", "--dtype", dtype, "--warmup", "2", "--rep", "5"]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    text = out.stdout + out.stderr
    g = TEST_RE.search(text)
    assert out.returncode == 0 and g, text[-2000:]
    assert int(g.group(6)) == 1 and float(g.group(5)) <= 1e-2 and float(g.group(2)) > 0
    assert TRAIN_RE.search(text)
