"""Packed variable-length forward (apex_attn_fwd_varlen) against the oracle. Needs a B200.

Tolerances as for the batched forward: o max-abs <= 1e-2 against the fp32 oracle on the
same 16-bit inputs, lse max-abs <= 2e-3; rows outside every sequence stay untouched (zero).
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

O_TOL = 1e-2
LSE_TOL = 2e-3


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


from oracle.attention_oracle import attention_varlen_np  # noqa: E402

TDT = {"bfloat16": torch.bfloat16, "float16": torch.float16}


def packed_inputs(lens, H, HKV, D, dtype="bfloat16", seed=0, extra_rows=0):
    g = torch.Generator().manual_seed(seed)
    total = sum(lens) + extra_rows
    t = TDT[dtype]
    q = torch.randn(total, H, D, generator=g).to(t)
    k = torch.randn(total, HKV, D, generator=g).to(t)
    v = torch.randn(total, HKV, D, generator=g).to(t)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return q, k, v, cu


def run_and_check(lens, H, HKV, D, causal=True, window=None, dtype="bfloat16", seed=0, extra_rows=0):
    from apex_attn import custom_attention_varlen_forward
    q, k, v, cu = packed_inputs(lens, H, HKV, D, dtype, seed, extra_rows)
    cu_t = torch.from_numpy(cu).cuda()
    o, lse = custom_attention_varlen_forward(q.cuda(), k.cuda(), v.cuda(), cu_t, max(lens), causal=causal,
                                             return_lse=True, window_left=window)
    torch.cuda.synchronize()
    ro, rl = attention_varlen_np(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu,
                                 causal=causal, window_left=window)
    o = o.float().cpu().numpy()
    lse = lse.cpu().numpy()
    assert np.isfinite(o).all()
    err = np.abs(o - ro).max()
    lerr = np.abs(lse - rl).max()
    assert err <= O_TOL, f"lens={lens} D={D} causal={causal} win={window}: max|o - oracle| = {err:.3e}"
    assert lerr <= LSE_TOL, f"max|lse - oracle| = {lerr:.3e}"
    return o


CASES = [
    # lens, H, HKV, D, causal, window, dtype
    ([300, 1, 128, 129, 700], 2, 2, 128, True, None, "bfloat16"),
    ([300, 1, 128, 129, 700], 2, 2, 128, False, None, "bfloat16"),
    ([64, 0, 500, 17], 4, 1, 64, True, None, "bfloat16"),       # an empty sequence, GQA 4:1
    ([1000, 255, 256, 257], 2, 2, 64, False, None, "bfloat16"),
    ([200, 333, 5], 2, 2, 256, True, None, "bfloat16"),
    ([640, 130, 900], 4, 2, 128, True, 100, "bfloat16"),       # window + GQA
    ([384, 96, 512], 2, 2, 64, True, None, "float16"),
    ([1], 1, 1, 128, True, None, "bfloat16"),
]


@pytest.mark.parametrize("lens,H,HKV,D,causal,win,dtype", CASES)
def test_varlen_vs_oracle(lens, H, HKV, D, causal, win, dtype):
    run_and_check(lens, H, HKV, D, causal=causal, window=win, dtype=dtype, seed=sum(lens) + D)


def test_rows_outside_sequences_untouched():
    o = run_and_check([100, 200], 2, 2, 64, extra_rows=77, seed=3)
    assert not o[300:].any()


@pytest.mark.parametrize("D", [64, 128, 256])
def test_equal_lengths_match_batched_forward_bitwise(D):
    """A packed batch of equal-length sequences is the batched problem in [B, N, H, D]
    storage: the results are the same bits when the same kernel computes both (packed
    batches always run on the two-sub-tile kernel, so the batched call is pinned to it)."""
    import apex_attn
    from apex_attn import custom_attention_forward, custom_attention_varlen_forward
    B, N, H = 3, 700, 4
    g = torch.Generator(device="cuda").manual_seed(D)
    q, k, v = (torch.randn(B, N, H, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    apex_attn.set_forward_kernel("two_subtile")
    try:
        ob, lb = custom_attention_forward(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                          causal=True, return_lse=True)
    finally:
        apex_attn.set_forward_kernel("auto")
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device="cuda")
    ov, lv = custom_attention_varlen_forward(q.reshape(B * N, H, D), k.reshape(B * N, H, D),
                                             v.reshape(B * N, H, D), cu, N, causal=True, return_lse=True)
    torch.cuda.synchronize()
    assert torch.equal(ov.reshape(B, N, H, D), ob.transpose(1, 2))
    assert torch.equal(lv.reshape(H, B, N).permute(1, 0, 2), lb)


def test_malformed_offsets_stay_in_bounds():
    """Offsets past `total`, decreasing offsets and a max_seqlen below the longest sequence
    are clamped on the device: no fault, status 0, and no row past `total` written (checked
    through the C ABI on an output buffer with guard rows after the `total` rows)."""
    import ctypes
    from apex_attn import _lib, device_status
    total, H, D = 500, 2, 64
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(total, H, D, generator=g, device="cuda").to(torch.bfloat16)
    o = torch.full((total + 64, H, D), 7.0, dtype=torch.bfloat16, device="cuda")
    cu = torch.tensor([0, 300, 200, 900], dtype=torch.int32, device="cuda")
    st = [H * D, D] * 4
    args = _lib.VarlenArgs(q=q.data_ptr(), k=q.data_ptr(), v=q.data_ptr(), o=o.data_ptr(), lse=None,
                           cu_seqlens=cu.data_ptr(), batch=3, heads_q=H, heads_kv=H, total=total,
                           max_seqlen=256, head_dim=D, dtype=_lib.DTYPE_BF16, causal=1, window_left=-1,
                           sm_scale=0.125, strides=(ctypes.c_longlong * 8)(*st))
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.load().apex_attn_fwd_varlen(ctypes.byref(args), stream) == 0
    torch.cuda.synchronize()
    assert device_status() == 0
    assert torch.isfinite(o.float()).all()
    assert (o[total:] == 7.0).all()
    assert not (o[:256] == 7.0).all()  # the first sequence (cut to 256 rows) was written


# ---------------------------------------------------------------- backward --
from oracle.attention_oracle import attention_varlen_bwd_np, grad_close  # noqa: E402

BWD_CASES = [
    # lens, H, HKV, D, causal, window, dtype
    ([300, 1, 128, 129, 700], 2, 2, 128, True, None, "bfloat16"),
    ([300, 1, 128, 129, 700], 2, 2, 128, False, None, "bfloat16"),
    ([64, 0, 500, 17], 4, 1, 64, True, None, "bfloat16"),
    ([1000, 255, 256, 257], 2, 2, 64, False, None, "bfloat16"),
    ([640, 130, 900], 4, 2, 128, True, 100, "bfloat16"),
    ([384, 96, 512], 2, 2, 64, True, None, "float16"),
]


@pytest.mark.parametrize("lens,H,HKV,D,causal,win,dtype", BWD_CASES)
def test_varlen_backward_vs_oracle(lens, H, HKV, D, causal, win, dtype):
    """Backward given the oracle's o and lse; tolerance of the batched backward parity
    (1e-2 + 2^-7 |ref|)."""
    from apex_attn import custom_attention_varlen_backward
    from oracle.attention_oracle import attention_varlen_np
    q, k, v, cu = packed_inputs(lens, H, HKV, D, dtype, seed=sum(lens) + 7 * D)
    g = torch.Generator().manual_seed(1)
    do = torch.randn(q.shape, generator=g).to(q.dtype)
    f32 = [t.float().numpy() for t in (q, k, v, do)]
    o, lse = attention_varlen_np(*f32[:3], cu, causal=causal, window_left=win)
    got = custom_attention_varlen_backward(
        q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(o).to(q.dtype).cuda(), torch.from_numpy(lse).cuda(),
        do.cuda(), torch.from_numpy(cu).cuda(), max(lens), causal=causal, window_left=win)
    torch.cuda.synchronize()
    ref = attention_varlen_bwd_np(*f32, cu, causal=causal, window_left=win)
    for name, a, r in zip(("dq", "dk", "dv"), got, ref):
        ok, ratio = grad_close(a.float().cpu().numpy(), r)
        assert ok, f"lens={lens} D={D} causal={causal} win={win} {name}: err/bound {ratio:.2f}"


@pytest.mark.parametrize("D", [64, 128])
def test_varlen_backward_equal_lengths_match_batched_bitwise(D):
    from apex_attn import (custom_attention_backward, custom_attention_forward,
                           custom_attention_varlen_backward, custom_attention_varlen_forward)
    B, N, H = 3, 700, 4
    g = torch.Generator(device="cuda").manual_seed(D + 1)
    q, k, v, do = (torch.randn(B, N, H, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(4))
    t = lambda x: x.transpose(1, 2)
    import apex_attn
    apex_attn.set_forward_kernel("two_subtile")  # the packed forward's kernel: same o and lse bits
    try:
        ob, lb = custom_attention_forward(t(q), t(k), t(v), causal=True, return_lse=True)
    finally:
        apex_attn.set_forward_kernel("auto")
    gb = custom_attention_backward(t(q), t(k), t(v), ob, lb, t(do), causal=True)
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device="cuda")
    p = lambda x: x.reshape(B * N, H, D)
    ov, lv = custom_attention_varlen_forward(p(q), p(k), p(v), cu, N, causal=True, return_lse=True)
    gv = custom_attention_varlen_backward(p(q), p(k), p(v), ov, lv, p(do), cu, N, causal=True)
    torch.cuda.synchronize()
    for a, b in zip(gv, gb):
        assert torch.equal(a.reshape(B, N, H, D), b.transpose(1, 2))


def test_varlen_backward_malformed_offsets_stay_in_bounds():
    from apex_attn import custom_attention_varlen_backward, device_status
    total, H, D = 500, 2, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn(total, H, D, generator=g, device="cuda").to(torch.bfloat16)
    lse = torch.zeros(H, total, device="cuda")
    cu = torch.tensor([0, 300, 200, 900], dtype=torch.int32, device="cuda")
    dq, dk, dv = custom_attention_varlen_backward(q, q, q, q, lse, q, cu, 256, causal=False)
    torch.cuda.synchronize()
    assert device_status() == 0
    for t in (dq, dk, dv):
        assert torch.isfinite(t.float()).all()


def test_varlen_cuda_graph_capture_and_replay():
    from apex_attn import custom_attention_varlen_backward, custom_attention_varlen_forward
    q, k, v, cu = packed_inputs([300, 1, 700], 2, 1, 64, seed=4)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    do = torch.randn(q.shape, device="cuda").to(q.dtype)
    cu = torch.from_numpy(cu).cuda()

    def step():
        o, lse = custom_attention_varlen_forward(q, k, v, cu, 700, return_lse=True)
        return (o,) + tuple(custom_attention_varlen_backward(q, k, v, o, lse, do, cu, 700))

    eager = step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            outs = step()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(outs, eager):
        assert torch.equal(a, b)
