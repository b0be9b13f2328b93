"""Seeded random sweep of the forward and backward against the CPU oracle. Needs a B200.

The hand-picked cases in the other files cover each feature. This file draws combinations
of them that nobody picked: head dim, sequence length (ragged, down to 1), batch and
heads, grouped-query ratio, causal or full, sliding window, bf16 or fp16, and contiguous
[B, H, N, D] or a strided [B, N, H, D] view. The draws are fixed by the seed, so a failure
reproduces; each case id names its configuration.

Tolerances are the ones the rest of the suite uses:
- forward: o max-abs <= 1e-2 against the fp32 oracle on the same 16-bit inputs
  (+ 2^-8 |ref| when a window of fewer than 16 keys makes |o| large), lse <= 2e-3;
- backward, given the oracle's o and lse: |g - ref| <= 1e-2 + 2^-7 |ref| for dq, dk, dv
  against the float64 oracle gradient.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

O_TOL = 1e-2
LSE_TOL = 2e-3
G_ATOL = 1e-2
G_RTOL = 2.0 ** -7
TDT = {"bfloat16": torch.bfloat16, "float16": torch.float16}


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


from oracle.attention_oracle import attention_bwd_np, attention_np, grad_close  # noqa: E402


def draw_configs(n, seed, head_dims, max_n, max_heads):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        D = int(rng.choice(head_dims))
        N = int(rng.choice([1, 2, 127, 128, 129, 255, 256, 300, 511, 640, 777, 1000, max_n]))
        N = min(N, max_n)
        B = int(rng.integers(1, 3))
        Hkv = int(rng.integers(1, 3))
        H = Hkv * int(rng.choice([1, 1, 2, 3]))
        H = min(H, max_heads)
        H -= H % Hkv
        causal = bool(rng.random() < 0.7)
        window = None
        if causal and rng.random() < 0.35:
            window = int(rng.choice([0, 3, 64, 127, 128, 200, 1000]))
        dtype = "bfloat16" if rng.random() < 0.7 else "float16"
        bnhd = bool(rng.random() < 0.3)
        out.append(dict(B=B, H=H, Hkv=Hkv, N=N, D=D, causal=causal, window=window, dtype=dtype,
                        bnhd=bnhd, seed=int(rng.integers(1 << 30))))
    return out


def case_id(c):
    w = "" if c["window"] is None else f"-w{c['window']}"
    return (f"b{c['B']}h{c['H']}kv{c['Hkv']}n{c['N']}d{c['D']}-{'c' if c['causal'] else 'f'}{w}-"
            f"{'bf16' if c['dtype'] == 'bfloat16' else 'fp16'}{'-bnhd' if c['bnhd'] else ''}")


def make(c, with_do=False):
    """CPU 16-bit tensors q [B, H, N, D], k and v [B, Hkv, N, D] (and do), plus the views
    the kernel gets: the same data either contiguous or as a strided [B, N, H, D] buffer
    seen through transpose(1, 2)."""
    g = torch.Generator().manual_seed(c["seed"])
    t = TDT[c["dtype"]]
    B, H, Hkv, N, D = c["B"], c["H"], c["Hkv"], c["N"], c["D"]
    q = torch.randn(B, H, N, D, generator=g).to(t)
    k = torch.randn(B, Hkv, N, D, generator=g).to(t)
    v = torch.randn(B, Hkv, N, D, generator=g).to(t)
    do = torch.randn(B, H, N, D, generator=g).to(t) if with_do else None

    def dev(x):
        if x is None:
            return None
        if c["bnhd"]:
            return x.transpose(1, 2).contiguous().cuda().transpose(1, 2)  # [B, N, H, D] storage
        return x.cuda()

    return (q, k, v, do), tuple(dev(x) for x in (q, k, v, do))


FWD = draw_configs(100, seed=2024, head_dims=[64, 128, 256], max_n=1200, max_heads=6)


@pytest.mark.parametrize("c", FWD, ids=[case_id(c) for c in FWD])
def test_forward_random_config(c):
    from apex_attn import custom_attention_forward
    (q, k, v, _), (qd, kd, vd, _) = make(c)
    o, lse = custom_attention_forward(qd, kd, vd, causal=c["causal"], return_lse=True,
                                      window_left=c["window"])
    torch.cuda.synchronize()
    ro, rl = attention_np(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=c["causal"],
                          window_left=c["window"])
    o = o.float().cpu().numpy()
    assert np.isfinite(o).all()
    rel = 2.0 ** -8 if c["window"] is not None and c["window"] < 16 else 0.0
    diff = np.abs(o - ro)
    assert (diff - (O_TOL + rel * np.abs(ro))).max() <= 0, f"max|o - oracle| = {diff.max():.3e}"
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL


BWD = draw_configs(40, seed=7, head_dims=[64, 128], max_n=700, max_heads=4)


@pytest.mark.parametrize("c", BWD, ids=[case_id(c) for c in BWD])
def test_backward_random_config(c):
    from apex_attn import custom_attention_backward
    (q, k, v, do), (qd, kd, vd, dod) = make(c, with_do=True)
    f32 = [t.float().numpy() for t in (q, k, v, do)]
    ro, rl = attention_np(*f32[:3], causal=c["causal"], window_left=c["window"])
    o = torch.from_numpy(ro).to(q.dtype)
    if c["bnhd"]:
        o = o.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    else:
        o = o.cuda()
    got = custom_attention_backward(qd, kd, vd, o, torch.from_numpy(rl).cuda(), dod, causal=c["causal"],
                                    window_left=c["window"])
    torch.cuda.synchronize()
    ref = attention_bwd_np(*f32, causal=c["causal"], window_left=c["window"])
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        g = g.float().cpu().numpy()
        assert g.shape == r.shape, (name, g.shape, r.shape)
        assert np.isfinite(g).all(), f"{name} not finite"
        ok, ratio = grad_close(g, r, atol=G_ATOL, rtol=G_RTOL)
        assert ok, f"{name}: max|err| {np.abs(g - r).max():.3e}, worst err/bound {ratio:.2f}"
