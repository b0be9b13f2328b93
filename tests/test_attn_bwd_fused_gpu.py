"""The fused one-pass backward (APEX_ATTN_BWD_FUSED, ``deterministic=False``). Needs a B200.

The fused mode runs the dK/dV pass with a fifth GEMM per step, dQ(query tile) = dS K, and
adds each step's dQ tile into an fp32 accumulator with global reductions before a cast
writes dq. So:

* dk and dv come from the same instructions in the same order as in the deterministic
  mode: they must be equal bit for bit;
* dq sums the same fp32 tile products in another order and is rounded once to 16 bits
  at the end: it must meet the oracle tolerance of the deterministic mode
  (|g - ref| <= 1e-2 + 2^-7 |ref| against the float64 gradient) and stay within
  2^-7 |dq| + 2e-3 of the deterministic dq (a few 16-bit rounding steps).
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _b200():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if torch.cuda.get_device_capability() != (10, 0):
        pytest.skip("needs sm_100")
    import apex_attn
    assert os.path.exists(apex_attn.library_path())
    yield
    assert apex_attn.device_status() == 0


from oracle.attention_oracle import attention_bwd_np, attention_np  # noqa: E402
from test_attn_bwd_gpu import (ATOL, ATOL_E2E, CASES, _torch_fp32_grads, assert_grads,  # noqa: E402
                               inputs)

DQ_RTOL = 2.0 ** -7
DQ_ATOL = 2e-3


def both_modes(q, k, v, o, lse, do, **kw):
    from apex_attn import custom_attention_backward
    det = custom_attention_backward(q, k, v, o, lse, do, deterministic=True, **kw)
    fus = custom_attention_backward(q, k, v, o, lse, do, deterministic=False, **kw)
    torch.cuda.synchronize()
    return det, fus


def assert_fused_matches_deterministic(det, fus, label=""):
    dq_d, dk_d, dv_d = det
    dq_f, dk_f, dv_f = fus
    assert torch.equal(dk_f, dk_d), f"{label} dk differs between modes"
    assert torch.equal(dv_f, dv_d), f"{label} dv differs between modes"
    assert torch.isfinite(dq_f.float()).all(), f"{label} dq not finite"
    diff = (dq_f.float() - dq_d.float()).abs()
    bound = DQ_ATOL + DQ_RTOL * dq_d.float().abs()
    worst = (diff / bound).max().item()
    assert worst <= 1.0, f"{label} dq: max|fused - deterministic| {diff.max().item():.3e}, err/bound {worst:.2f}"


@pytest.mark.parametrize("B,H,HKV,N,D,causal,win,dtype", CASES)
def test_fused_bwd_vs_oracle(B, H, HKV, N, D, causal, win, dtype):
    q, k, v, do = inputs(B, H, HKV, N, D, dtype, seed=N + D)
    o, lse = attention_np(*(t.float().numpy() for t in (q, k, v)), causal=causal, window_left=win)
    o = torch.from_numpy(o).to(q.dtype).cuda()
    lse = torch.from_numpy(lse).cuda()
    det, fus = both_modes(q.cuda(), k.cuda(), v.cuda(), o, lse, do.cuda(), causal=causal, window_left=win)
    ref = attention_bwd_np(*(t.float().numpy() for t in (q, k, v, do)), causal=causal, window_left=win)
    label = f"B{B} H{H}/{HKV} N{N} D{D} causal={causal} win={win} {dtype}"
    assert_grads(fus, ref, label + " fused", atol=ATOL)
    assert_fused_matches_deterministic(det, fus, label)


@pytest.mark.parametrize("D,causal,HKV,win", [(128, True, 4, None), (64, True, 4, None),
                                             (128, False, 2, None), (64, True, 2, 1000)])
def test_fused_bwd_n4096_vs_torch_fp32(D, causal, HKV, win):
    from apex_attn import custom_attention_backward, custom_attention_forward
    q, k, v, do = (t.cuda() for t in inputs(1, 4, HKV, 4096, D, seed=31))
    o, lse = custom_attention_forward(q, k, v, causal=causal, return_lse=True, window_left=win)
    got = custom_attention_backward(q, k, v, o, lse, do, causal=causal, window_left=win, deterministic=False)
    torch.cuda.synchronize()
    ref = _torch_fp32_grads(q, k, v, do, causal=causal, window_left=win)
    assert_grads(got, [r.cpu().numpy() for r in ref], f"fused N4096 D{D} causal={causal}", atol=ATOL_E2E)


@pytest.mark.parametrize("D", [64, 128])
def test_fused_bwd_full_size_c2_c3(D):
    """BASELINE's C2 (d=64: B4 H16 N4096) and C3 (d=128: B4 H32 N8192) shapes, end to end:
    dk, dv bit-equal to the deterministic mode, dq within a few roundings of it."""
    from apex_attn import custom_attention_forward
    B, H, N = (4, 16, 4096) if D == 64 else (4, 32, 8192)
    g = torch.Generator(device="cuda").manual_seed(42)
    q, k, v, do = (torch.randn(B, H, N, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(4))
    o, lse = custom_attention_forward(q, k, v, return_lse=True)
    det, fus = both_modes(q, k, v, o, lse, do)
    assert_fused_matches_deterministic(det, fus, f"full size D{D}")


@pytest.mark.parametrize("causal", [True, False])
def test_fused_bwd_varlen_matches_deterministic(causal):
    """Packed batch: for full attention the last key block of a sequence also holds the next
    sequence's keys, which the fused pass must keep out of dq."""
    from apex_attn import custom_attention_varlen_backward, custom_attention_varlen_forward
    lens = [700, 1, 129, 1000, 256]
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    total = int(cu[-1]) + 40  # rows after the last sequence belong to none
    g = torch.Generator(device="cuda").manual_seed(7)
    for D, HKV in ((64, 2), (128, 4)):
        q, do = (torch.randn(total, 4, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(2))
        k, v = (torch.randn(total, HKV, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(2))
        o, lse = custom_attention_varlen_forward(q, k, v, cu, max(lens), causal=causal, return_lse=True)
        det = custom_attention_varlen_backward(q, k, v, o, lse, do, cu, max(lens), causal=causal)
        fus = custom_attention_varlen_backward(q, k, v, o, lse, do, cu, max(lens), causal=causal,
                                               deterministic=False)
        torch.cuda.synchronize()
        assert_fused_matches_deterministic(det, fus, f"varlen D{D} causal={causal}")
        assert (fus[0][int(cu[-1]):] == 0).all()  # rows outside every sequence are not written


def test_fused_bwd_repeats_within_tolerance_and_leaves_status_clean():
    """Two fused calls on the same inputs: dk, dv identical, dq equal up to reduction order."""
    from apex_attn import custom_attention_backward, custom_attention_forward, device_status
    q, k, v, do = (t.cuda() for t in inputs(2, 4, 2, 3000, 128, seed=8))
    o, lse = custom_attention_forward(q, k, v, return_lse=True)
    a = custom_attention_backward(q, k, v, o, lse, do, deterministic=False)
    b = custom_attention_backward(q, k, v, o, lse, do, deterministic=False)
    torch.cuda.synchronize()
    assert_fused_matches_deterministic(a, b, "repeat")
    assert device_status() == 0


def test_fused_bwd_workspace_and_mode_validation():
    import ctypes

    from apex_attn import _lib
    lib = _lib.load()
    base = lib.apex_attn_bwd_workspace_bytes(2, 4, 1000)
    assert lib.apex_attn_bwd_workspace_bytes_mode(2, 4, 1000, 128, 0) == base
    fused = lib.apex_attn_bwd_workspace_bytes_mode(2, 4, 1000, 128, 1)
    assert fused >= base + 2 * 4 * 1000 * 128 * 4
    q, k, v, do = (t.cuda() for t in inputs(1, 2, 2, 256, 64, seed=2))
    from apex_attn import custom_attention_forward
    o, lse = custom_attention_forward(q, k, v, return_lse=True)
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    strides = []
    for t in (q, k, v, o, do, dq, dk, dv):
        strides += [t.stride(0), t.stride(1), t.stride(2)]
    args = _lib.BwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), dout=do.data_ptr(),
                        lse=lse.data_ptr(), dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), batch=1,
                        heads_q=2, heads_kv=2, seqlen=256, head_dim=64, dtype=_lib.DTYPE_BF16, causal=1,
                        window_left=-1, sm_scale=0.125, strides=(ctypes.c_longlong * 24)(*strides))
    small = lib.apex_attn_bwd_workspace_bytes(1, 2, 256)
    ws = torch.empty(lib.apex_attn_bwd_workspace_bytes_mode(1, 2, 256, 64, 1), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # the deterministic workspace is too small for the fused mode
    assert lib.apex_attn_bwd_mode(ctypes.byref(args), 1, ws.data_ptr(), small, stream) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_mode(ctypes.byref(args), 2, ws.data_ptr(), ws.numel(), stream) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_mode(ctypes.byref(args), 1, ws.data_ptr(), ws.numel(), stream) == _lib.OK
    torch.cuda.synchronize()
