"""The allocation-free entry point apex_attn_fwd_noalloc, through the C ABI.

Some callers of this library cannot call cudaMalloc: for example a serving runtime or
memory pool that owns the device budget, or a plugin whose host forbids allocations
outside its own allocator. apex_attn_fwd_noalloc serves them by keeping the kernel's
scratch (the device status word and the scheduler's work-item counter) in a fixed static
device array instead of a cudaMalloc'd buffer. The caller (here: the test, through torch)
still allocates the inputs and outputs.

Both entry points run the same kernel with the same schedule on the same inputs, so their
outputs must be bit-identical; a difference would mean the static scratch changed the
scheduling or the results.

This file is named so that pytest collects it last: if it fails, a run that stops at
the first failure has already run every other test. It must pass both alone in a fresh
process and after the other tests.
"""
import ctypes
import os
import subprocess
import sys

import pytest
import torch

from apex_attn import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _strides(t):
    b, h, n, d = t.shape
    return [h * n * d, n * d, d]


def _call(fn, q, k, v, causal=True):
    """Calls one of the two C entry points on caller-allocated buffers."""
    B, H, N, D = q.shape
    o = torch.empty_like(q)
    lse = torch.empty((B, H, N), dtype=torch.float32, device=q.device)
    st = (ctypes.c_longlong * 12)(*(_strides(q) * 4))
    dt = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_FP16
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, H, N, D, dt,
            1 if causal else 0, float(D) ** -0.5, st, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK, _lib.strerror(rc)
    return o, lse


def _require_b200():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability() != (10, 0):
        pytest.skip("needs a B200 (sm_100)")


def _noalloc_status(lib):
    flags = ctypes.c_int(-1)
    rc = lib.apex_attn_noalloc_status(torch.cuda.current_device(), ctypes.byref(flags))
    return rc, flags.value


@pytest.mark.gpu
def test_noalloc_matches_fwd_on_two_calls_in_a_row():
    _require_b200()
    from oracle.attention_oracle import make_inputs
    lib = _lib.load()
    cases = [(2, 3, 777, 128, True, "bfloat16", 1), (1, 4, 1000, 64, False, "float16", 2)]
    for B, H, N, D, causal, dtype, seed in cases:  # two noalloc calls, back to back
        q, k, v = (t.cuda() for t in make_inputs(B, H, N, D, seed=seed, dtype=dtype))
        o_na, l_na = _call(lib.apex_attn_fwd_noalloc, q, k, v, causal)
        o_ref, l_ref = _call(lib.apex_attn_fwd, q, k, v, causal)
        torch.cuda.synchronize()
        assert torch.isfinite(o_na.float()).all()
        assert torch.equal(o_na, o_ref), (o_na.float() - o_ref.float()).abs().max().item()
        assert torch.equal(l_na, l_ref), (l_na - l_ref).abs().max().item()
    assert _noalloc_status(lib) == (_lib.OK, 0)
    assert _lib.load().apex_attn_device_status(torch.cuda.current_device(), ctypes.byref(ctypes.c_int())) == _lib.OK


_FRESH = r"""
import ctypes, sys
sys.path[:0] = [{root!r}, {pkg!r}, {tests!r}]
import torch
from apex_attn import _lib
import gpu_ref
from oracle.attention_oracle import make_inputs
from test_zz_no_alloc import _call, _noalloc_status
lib = _lib.load()
q, k, v = (t.cuda() for t in make_inputs(2, 2, 600, 128, seed=5))
outs = [_call(lib.apex_attn_fwd_noalloc, q, k, v, True) for _ in range(2)]
torch.cuda.synchronize()
ro, rl = gpu_ref.attention_fp32(q, k, v, causal=True)
for o, l in outs:
    assert (o.float() - ro).abs().max().item() <= 1e-2
    assert (l - rl).abs().max().item() <= 2e-3
assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
assert _noalloc_status(lib) == (_lib.OK, 0)
print("fresh-noalloc-ok")
"""


@pytest.mark.gpu
def test_noalloc_alone_in_a_fresh_process():
    """A process whose only library calls are allocation-free ones: the static scratch must
    work without the allocating path's per-device set-up having run first."""
    _require_b200()
    code = _FRESH.format(root=ROOT, pkg=os.path.join(ROOT, "apex-tune-results_b200"),
                         tests=os.path.join(ROOT, "tests"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0 and "fresh-noalloc-ok" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


def test_noalloc_rejects_bad_and_oversized_requests():
    """Validation happens before any CUDA call, so this needs no GPU."""
    lib = _lib.load()
    fake = 0x10000
    st = (ctypes.c_longlong * 12)(*([64 * 256, 256 * 64, 64] * 4))
    args = lambda B, H, N, D: (fake, fake, fake, fake, None, B, H, N, D, 0, 1, 0.125, st, None)
    assert lib.apex_attn_fwd_noalloc(*args(1 << 20, 1 << 11, 256, 64)) == _lib.ERR_TOO_LARGE
    assert lib.apex_attn_fwd_noalloc(*args(1, 1, 256, 96)) == _lib.ERR_UNSUPPORTED_HEAD_DIM
    assert lib.apex_attn_fwd_noalloc(*args(0, 1, 256, 64)) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_noalloc_status(0, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_noalloc_status(-1, ctypes.byref(ctypes.c_int())) == _lib.ERR_NO_DEVICE
    assert "exceed" in _lib.strerror(_lib.ERR_TOO_LARGE)
