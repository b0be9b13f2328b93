"""CPU oracle for the fused causal attention forward. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg may import
this module, and only as the checker or the timed CPU baseline. The product path
(apex_attn) never calls it and has no CPU fallback.

What it restates
----------------
* ``attention_np`` — the reference's math path in plain numpy: the harness oracle
  ``reference_attention`` (mls-bench_fused_attention/submission.py:223-232) is
  ``F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=sm_scale)``, i.e.
  ``softmax(Q K^T * scale + causal_mask) V`` with ``scale = 1/sqrt(d)`` by default
  (submission.py:225-226). The reference kernels compute the same quantity
  (fused_attention.py:61-87: sum_j exp2(qk*scale*log2e) v_j / sum_j exp2(...)).
  It also returns the natural-log logsumexp of each masked, scaled score row, which the
  reference does not produce (the B200 kernel optionally does).
* ``reference_attention_cpu`` — the harness oracle itself restated for CPU tensors:
  the same ``F.scaled_dot_product_attention`` call (submission.py:227-232; its
  ``sdp_kernel`` context only selects CUDA backends, so it is dropped on CPU).
  This is what the CPU baseline times.
* ``attention_bwd_np`` — the gradients dQ, dK, dV of the same quantity for an upstream
  gradient dO: the backward that nanochat's Blackwell attention op calls
  (``_flash_attn_bwd(q, k, v, out, grad_output, lse, causal=True, window_size_left=...)``,
  nanochat_autoresearch/solutions/train.py:491,508-519). It is the textbook derivative of
  softmax(S) V, written out (P = softmax(S), dV = P^T dO, dP = dO V^T,
  dS = P * (dP - rowsum(dO * O)), dQ = scale dS K, dK = scale dS^T Q; grouped-query heads
  sum into their shared K/V head).
* ``attention_varlen_np`` — ``attention_np`` per sequence of a packed variable-length
  batch (flash-attn's varlen layout: rows cu_seqlens[b] .. cu_seqlens[b+1] - 1).
* ``compute_flops`` — submission.py:235-240 (4*B*N^2*H*d, halved when causal).
* ``make_inputs`` — the harness's seeded ``randn`` inputs (submission.py:278-287), drawn
  on the CPU generator in fp32 and rounded to the kernel dtype, so CPU and GPU see the
  same values.

Pinning: tests/golden/ holds vectors produced by the reference's own code in the build
container (the harness ``reference_attention`` and the reference Triton kernel
``_attn_fwd_plain`` run under the Triton CPU interpreter); tests/test_oracle.py checks
this module against them. See tests/golden/make_golden.py. The backward is pinned to
torch autograd through the same harness oracle (``bwd_*.npz``, written by
tests/golden/make_golden_bwd.py).
"""
from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634


def compute_flops(batch: int, nheads: int, seqlen: int, headdim: int, causal: bool) -> int:
    """FLOPs of one forward (submission.py:235-240)."""
    flops = 4 * batch * seqlen * seqlen * nheads * headdim
    if causal:
        flops //= 2
    return flops


def attention_np(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = True,
                 sm_scale: float | None = None, chunk: int = 512, dtype=np.float32,
                 heads: list[int] | None = None, window_left: int | None = None):
    """softmax(Q K^T * scale + mask) V and its row logsumexp, chunked over query rows.

    q: [B, H, N, D]; k, v: [B, H_kv, N, D] with H_kv dividing H (query head h reads K/V head
    h // (H // H_kv): grouped-query attention; H_kv = H is the reference's case).
    window_left (causal only): row i sees keys i - window_left .. i.
    heads: optional list of flattened (b*H + h) indices to compute (others left zero).
    Returns (o [B,H,N,D] float32, lse [B,H,N] float32).
    """
    B, H, N, D = q.shape
    group = H // k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    o = np.zeros((B, H, N, D), dtype=np.float32)
    lse = np.zeros((B, H, N), dtype=np.float32)
    sel = range(B * H) if heads is None else heads
    for bh in sel:
        b, h = divmod(int(bh), H)
        qh = q[b, h].astype(dtype, copy=False)
        kh = k[b, h // group].astype(dtype, copy=False)
        vh = v[b, h // group].astype(dtype, copy=False)
        for r0 in range(0, N, chunk):
            r1 = min(N, r0 + chunk)
            kmax = r1 if causal else N
            s = (qh[r0:r1] @ kh[:kmax].T) * dtype(sm_scale)
            if causal:
                rows = np.arange(r0, r1)[:, None]
                cols = np.arange(kmax)[None, :]
                hidden = cols > rows
                if window_left is not None:
                    hidden |= cols < rows - window_left
                s = np.where(hidden, -np.inf, s)
            m = s.max(axis=1, keepdims=True)
            e = np.exp(s - m)
            l = e.sum(axis=1, keepdims=True)
            o[b, h, r0:r1] = (e @ vh[:kmax]) / l
            lse[b, h, r0:r1] = (m + np.log(l))[:, 0]
    return o, lse


def attention_varlen_np(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens, causal: bool = True,
                        sm_scale: float | None = None, window_left: int | None = None):
    """attention_np over a packed batch: q [total, H, D], k, v [total, H_kv, D]; sequence b is
    rows cu_seqlens[b] .. cu_seqlens[b+1] - 1 and attends only within itself.
    Returns (o [total, H, D] float32, zero outside every sequence; lse [H, total] float32)."""
    total, H, D = q.shape
    o = np.zeros((total, H, D), dtype=np.float32)
    lse = np.zeros((H, total), dtype=np.float32)
    cu = [int(x) for x in cu_seqlens]
    for b in range(len(cu) - 1):
        a, e = cu[b], cu[b + 1]
        if e <= a:
            continue
        seq = lambda t: np.ascontiguousarray(t[a:e].transpose(1, 0, 2))[None]
        ob, lb = attention_np(seq(q), seq(k), seq(v), causal=causal, sm_scale=sm_scale,
                              window_left=window_left)
        o[a:e] = ob[0].transpose(1, 0, 2)
        lse[:, a:e] = lb[0]
    return o, lse


def attention_bwd_np(q: np.ndarray, k: np.ndarray, v: np.ndarray, do: np.ndarray,
                     causal: bool = True, sm_scale: float | None = None,
                     window_left: int | None = None, dtype=np.float64, heads: list[int] | None = None):
    """Gradients of softmax(Q K^T * scale + mask) V with respect to q, k and v.

    q, do: [B, H, N, D]; k, v: [B, H_kv, N, D] (grouped-query heads as in attention_np).
    The forward's O and logsumexp are recomputed here in `dtype` (float64 by default), so
    the result is the exact gradient of the masked attention, not of a rounded O.
    heads: optional flattened (b*H + h) query-head indices to include (others contribute
    nothing; their dq rows stay zero).
    Returns (dq [B,H,N,D], dk [B,H_kv,N,D], dv [B,H_kv,N,D]) as float32.
    """
    B, H, N, D = q.shape
    hkv = k.shape[1]
    group = H // hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    dq = np.zeros((B, H, N, D), dtype=np.float64)
    dk = np.zeros((B, hkv, N, D), dtype=np.float64)
    dv = np.zeros((B, hkv, N, D), dtype=np.float64)
    rows = np.arange(N)[:, None]
    cols = np.arange(N)[None, :]
    hidden = np.zeros((N, N), dtype=bool)
    if causal:
        hidden = cols > rows
        if window_left is not None:
            hidden |= cols < rows - window_left
    sel = range(B * H) if heads is None else heads
    for bh in sel:
        b, h = divmod(int(bh), H)
        g = h // group
        qh = q[b, h].astype(dtype)
        kh = k[b, g].astype(dtype)
        vh = v[b, g].astype(dtype)
        doh = do[b, h].astype(dtype)
        s = np.where(hidden, -np.inf, (qh @ kh.T) * sm_scale)
        m = s.max(axis=1, keepdims=True)
        e = np.exp(s - m)
        p = e / e.sum(axis=1, keepdims=True)
        o = p @ vh
        dp = doh @ vh.T
        delta = (doh * o).sum(axis=1, keepdims=True)  # = rowsum(P * dP)
        ds = p * (dp - delta)
        dq[b, h] = (ds @ kh) * sm_scale
        dk[b, g] += (ds.T @ qh) * sm_scale
        dv[b, g] += p.T @ doh
    return dq.astype(np.float32), dk.astype(np.float32), dv.astype(np.float32)


def attention_varlen_bwd_np(q, k, v, do, cu_seqlens, causal: bool = True, sm_scale: float | None = None,
                            window_left: int | None = None):
    """attention_bwd_np per sequence of a packed batch (layout of attention_varlen_np).
    Returns (dq [total, H, D], dk, dv [total, H_kv, D]) float32, zero outside every sequence."""
    dq = np.zeros(q.shape, dtype=np.float32)
    dk = np.zeros(k.shape, dtype=np.float32)
    dv = np.zeros(k.shape, dtype=np.float32)
    cu = [int(x) for x in cu_seqlens]
    for b in range(len(cu) - 1):
        a, e = cu[b], cu[b + 1]
        if e <= a:
            continue
        seq = lambda t: np.ascontiguousarray(t[a:e].transpose(1, 0, 2))[None]
        gq, gk, gv = attention_bwd_np(seq(q), seq(k), seq(v), seq(do), causal=causal, sm_scale=sm_scale,
                                      window_left=window_left)
        dq[a:e] = gq[0].transpose(1, 0, 2)
        dk[a:e] = gk[0].transpose(1, 0, 2)
        dv[a:e] = gv[0].transpose(1, 0, 2)
    return dq, dk, dv


def grad_close(actual: np.ndarray, expected: np.ndarray, atol: float = 1e-2,
               rtol: float = 2.0 ** -7) -> tuple[bool, float]:
    """Tolerance of the 16-bit backward: |a - e| <= atol + rtol |e| elementwise.

    The kernel rounds P and dS to 16 bits for the tensor cores and the gradients to the
    output dtype; the bf16 rounding of a gradient of magnitude ~4 alone is 2^-7. Returns
    (ok, worst ratio of |a - e| to the bound).
    """
    bound = atol + rtol * np.abs(expected)
    ratio = float((np.abs(actual.astype(np.float64) - expected) / bound).max()) if expected.size else 0.0
    return ratio <= 1.0, ratio


def reference_attention_cpu(q, k, v, causal: bool = True, sm_scale: float | None = None):
    """The harness oracle (submission.py:223-232) on CPU torch tensors."""
    import torch.nn.functional as F

    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    return F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=sm_scale)


def make_inputs(batch: int, nheads: int, seqlen: int, headdim: int, seed: int = 42,
                dtype: str = "bfloat16", scale_q: float = 1.0):
    """Seeded N(0,1) q, k, v as CPU torch tensors of `dtype` (generated in fp32).

    Mirrors submission.py:278-287 (torch.manual_seed(seed); randn for q, k, v) but on the
    CPU generator so that the CPU oracle and the GPU kernel see identical values.
    """
    import torch

    g = torch.Generator().manual_seed(seed)
    shape = (batch, nheads, seqlen, headdim)
    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[dtype]
    q = (torch.randn(shape, generator=g) * scale_q).to(tdt)
    k = torch.randn(shape, generator=g).to(tdt)
    v = torch.randn(shape, generator=g).to(tdt)
    return q, k, v


def to_np32(t) -> np.ndarray:
    """CPU torch tensor (any float dtype) -> float32 numpy array."""
    import torch

    return t.detach().to("cpu", torch.float32).numpy()
