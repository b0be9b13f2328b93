"""The operator surface of mls-bench_fused_attention, backed by the sm_100a kernel.

``custom_attention_forward(q, k, v, causal=True, sm_scale=None)`` has the signature,
defaults, output and error behaviour of the reference operator
(mls-bench_fused_attention/fused_attention.py:155-193; spec comment submission.py:20-26):

* q, k, v: ``[batch, nheads, seqlen, headdim]`` CUDA tensors, fp16 or bf16;
* ``sm_scale`` defaults to ``1/sqrt(headdim)`` (fused_attention.py:158-159);
* an unsupported ``headdim`` raises ``KeyError(headdim)``, as ``_CONFIGS[headdim]`` does
  (fused_attention.py:162);
* the result is a new contiguous tensor of q's shape and dtype, produced asynchronously
  on the current CUDA stream (fused_attention.py:161).

Extensions beyond the reference:
* ``return_lse=True`` also returns the fp32 natural-log logsumexp ``[batch, nheads, seqlen]``;
* grouped-query attention: k and v may have fewer heads than q (a divisor of q's);
* ``window_left=w`` (causal only): row i attends to keys i - w .. i (a sliding window, as in
  flash_attn_func(window_size=(w, 0)) at nanochat_autoresearch/solutions/train.py:719). Inputs whose layout the TMA tensor maps accept
directly (unit head-dim stride, other strides multiples of 8 elements) are not copied;
others are made contiguous first, like the reference's ``.contiguous()`` (:157).
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16}


def supports_head_dim(headdim: int) -> bool:
    return bool(_lib.load().apex_attn_supports_head_dim(int(headdim)))


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    if t.stride(-1) != 1 or t.data_ptr() % 16 != 0:
        return t.contiguous()
    for size, stride in zip(t.shape[:3], t.stride()[:3]):
        if size > 1 and stride % 8 != 0:
            return t.contiguous()
    return t


def _strides(t: torch.Tensor) -> list[int]:
    """(batch, head, seq) element strides; size-1 dims get their contiguous stride."""
    b, h, n, d = t.shape
    contiguous = (h * n * d, n * d, d)
    return [s if size > 1 else c for size, s, c in zip((b, h, n), t.stride()[:3], contiguous)]


def custom_attention_forward(q, k, v, causal=True, sm_scale=None, return_lse=False, window_left=None):
    """Causal (or full) attention forward on B200; see the module docstring."""
    if q.dim() != 4 or k.dim() != 4 or k.shape != v.shape:
        raise ValueError(f"q, k, v must be [B, H, N, D] with k and v alike, got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    batch, nheads, seqlen, headdim = q.shape
    kv_heads = k.shape[1]
    if (k.shape[0], k.shape[2], k.shape[3]) != (batch, seqlen, headdim) or nheads % kv_heads != 0:
        raise ValueError(f"k and v must be [B, H_kv, N, D] with H_kv dividing q's heads, got q "
                         f"{tuple(q.shape)}, k {tuple(k.shape)}")
    if not supports_head_dim(headdim):
        raise KeyError(headdim)
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q, k, v must all be float16 or bfloat16, got {q.dtype}, {k.dtype}, {v.dtype}")
    if not (q.is_cuda and k.is_cuda and v.is_cuda) or not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be CUDA tensors on one device")
    if window_left is not None and (window_left < 0 or not causal):
        raise ValueError("window_left must be >= 0 and needs causal=True")
    q, k, v = _tma_ready(q), _tma_ready(k), _tma_ready(v)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(headdim)
    o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    lse = torch.empty((batch, nheads, seqlen), dtype=torch.float32, device=q.device) if return_lse else None
    if q.numel() == 0:
        return (o, lse) if return_lse else o
    strides = _strides(q) + _strides(k) + _strides(v) + _strides(o)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    lib = _lib.load()
    if kv_heads == nheads and window_left is None:
        # The reference-shaped entry point (fused_attention.py:155-193).
        rc = lib.apex_attn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
            lse.data_ptr() if lse is not None else None,
            batch, nheads, seqlen, headdim, _DTYPES[q.dtype], 1 if causal else 0, float(sm_scale),
            (ctypes.c_longlong * 12)(*strides), stream)
    else:
        args = _lib.FwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(),
                            lse=lse.data_ptr() if lse is not None else None, batch=batch,
                            heads_q=nheads, heads_kv=kv_heads, seqlen=seqlen, head_dim=headdim,
                            dtype=_DTYPES[q.dtype], causal=1 if causal else 0,
                            window_left=-1 if window_left is None else int(window_left),
                            sm_scale=float(sm_scale), strides=(ctypes.c_longlong * 12)(*strides))
        rc = lib.apex_attn_fwd_ex(ctypes.byref(args), stream)
    _lib.check(rc, "custom_attention_forward")
    return (o, lse) if return_lse else o


def custom_attention_varlen_forward(q, k, v, cu_seqlens, max_seqlen, causal=True, sm_scale=None,
                                    return_lse=False, window_left=None):
    """Attention over a packed batch of variable-length sequences (flash-attn's varlen
    layout): q [total, H, D], k and v [total, H_kv, D]; sequence b is rows
    cu_seqlens[b] .. cu_seqlens[b+1] - 1 (int32 CUDA tensor of batch + 1 offsets, cu[0] = 0,
    nondecreasing, cu[-1] = total); max_seqlen is the longest sequence. Each sequence
    attends only within itself (causal / window relative to its first row). Returns o
    [total, H, D] (rows outside every sequence are left as zeros) and, with return_lse,
    the fp32 logsumexp [H, total]. Head dims 64, 128, 256; bf16 or fp16; GQA as for the
    batched operator.
    """
    if q.dim() != 3 or k.dim() != 3 or k.shape != v.shape:
        raise ValueError(f"q, k, v must be [total, H, D] with k and v alike, got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    total, nheads, headdim = q.shape
    kv_heads = k.shape[1]
    if (k.shape[0], k.shape[2]) != (total, headdim) or nheads % kv_heads != 0:
        raise ValueError("k and v must be [total, H_kv, D] with H_kv dividing q's heads")
    if not supports_head_dim(headdim):
        raise KeyError(headdim)
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q, k, v must all be float16 or bfloat16, got {q.dtype}, {k.dtype}, {v.dtype}")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be a 1-D int32 tensor of batch + 1 offsets")
    if not all(t.is_cuda and t.device == q.device for t in (q, k, v, cu_seqlens)):
        raise ValueError("q, k, v, cu_seqlens must be CUDA tensors on one device")
    if window_left is not None and (window_left < 0 or not causal):
        raise ValueError("window_left must be >= 0 and needs causal=True")
    if int(max_seqlen) <= 0:
        raise ValueError("max_seqlen must be positive")

    def ready(t):
        if t.stride(-1) != 1 or t.data_ptr() % 16 != 0 or any(s % 8 for s in t.stride()[:2]):
            return t.contiguous()
        return t
    q, k, v = ready(q), ready(k), ready(v)
    cu_seqlens = cu_seqlens.contiguous()
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(headdim)
    o = torch.zeros(q.shape, dtype=q.dtype, device=q.device)
    lse = torch.zeros((nheads, total), dtype=torch.float32, device=q.device) if return_lse else None
    if total == 0:
        return (o, lse) if return_lse else o
    strides = [q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
               o.stride(0), o.stride(1)]
    args = _lib.VarlenArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(),
                           lse=lse.data_ptr() if lse is not None else None,
                           cu_seqlens=cu_seqlens.data_ptr(), batch=cu_seqlens.numel() - 1,
                           heads_q=nheads, heads_kv=kv_heads, total=total, max_seqlen=int(max_seqlen),
                           head_dim=headdim, dtype=_DTYPES[q.dtype], causal=1 if causal else 0,
                           window_left=-1 if window_left is None else int(window_left),
                           sm_scale=float(sm_scale), strides=(ctypes.c_longlong * 8)(*strides))
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _lib.check(_lib.load().apex_attn_fwd_varlen(ctypes.byref(args), stream), "custom_attention_varlen_forward")
    return (o, lse) if return_lse else o


_BWD_MODES = {True: 0, False: 1}  # APEX_ATTN_BWD_DETERMINISTIC, APEX_ATTN_BWD_FUSED


def custom_attention_backward(q, k, v, o, lse, dout, causal=True, sm_scale=None, window_left=None,
                              deterministic=True):
    """Gradients (dq, dk, dv) of custom_attention_forward for the upstream gradient `dout`.

    The backward nanochat's attention op calls (``_flash_attn_bwd(q, k, v, out,
    grad_output, lse, causal=True, window_size_left=w)``,
    nanochat_autoresearch/solutions/train.py:491,508-519): `o` and `lse` are the forward's
    output and fp32 logsumexp (``custom_attention_forward(..., return_lse=True)``); the
    other arguments mean what they mean for the forward. Head dims 64 and 128 (others
    raise KeyError). dq has q's shape, dk and dv k's (grouped-query heads summed); all in
    q's dtype. Runs asynchronously on the current CUDA stream.

    deterministic=True (default): two passes, bitwise reproducible. False: the fused
    one-pass algorithm, faster, whose dq is accumulated in fp32 with global reductions and
    so varies in its last bits from run to run (dk, dv do not); it needs a workspace of
    4 * B * H * N * D more bytes.
    """
    if q.dim() != 4 or k.shape != v.shape or o.shape != q.shape or dout.shape != q.shape:
        raise ValueError(f"expected q, o, dout [B, H, N, D] and k, v [B, H_kv, N, D], got q "
                         f"{tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}, o "
                         f"{tuple(o.shape)}, dout {tuple(dout.shape)}")
    batch, nheads, seqlen, headdim = q.shape
    kv_heads = k.shape[1]
    if (k.shape[0], k.shape[2], k.shape[3]) != (batch, seqlen, headdim) or nheads % kv_heads != 0:
        raise ValueError(f"k and v must be [B, H_kv, N, D] with H_kv dividing q's heads, got q "
                         f"{tuple(q.shape)}, k {tuple(k.shape)}")
    if headdim not in (64, 128):
        raise KeyError(headdim)
    if q.dtype not in _DTYPES or any(t.dtype != q.dtype for t in (k, v, o, dout)):
        raise TypeError("q, k, v, o, dout must share one dtype, float16 or bfloat16")
    if lse.shape != (batch, nheads, seqlen) or lse.dtype != torch.float32:
        raise ValueError(f"lse must be float32 [B, H, N], got {lse.dtype} {tuple(lse.shape)}")
    tensors = (q, k, v, o, dout, lse)
    if not all(t.is_cuda and t.device == q.device for t in tensors):
        raise ValueError("all tensors must be CUDA tensors on one device")
    if window_left is not None and (window_left < 0 or not causal):
        raise ValueError("window_left must be >= 0 and needs causal=True")
    q, k, v, o, dout = (_tma_ready(t) for t in (q, k, v, o, dout))
    lse = lse.contiguous()
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(headdim)
    dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    dk = torch.empty(k.shape, dtype=q.dtype, device=q.device)
    dv = torch.empty(k.shape, dtype=q.dtype, device=q.device)
    if q.numel() == 0:
        return dq, dk.zero_(), dv.zero_()
    lib = _lib.load()
    mode = _BWD_MODES[bool(deterministic)]
    ws_bytes = int(lib.apex_attn_bwd_workspace_bytes_mode(batch, nheads, seqlen, headdim, mode))
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    strides = []
    for t in (q, k, v, o, dout, dq, dk, dv):
        strides += _strides(t)
    args = _lib.BwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(),
                        dout=dout.data_ptr(), lse=lse.data_ptr(), dq=dq.data_ptr(),
                        dk=dk.data_ptr(), dv=dv.data_ptr(), batch=batch, heads_q=nheads,
                        heads_kv=kv_heads, seqlen=seqlen, head_dim=headdim,
                        dtype=_DTYPES[q.dtype], causal=1 if causal else 0,
                        window_left=-1 if window_left is None else int(window_left),
                        sm_scale=float(sm_scale), strides=(ctypes.c_longlong * 24)(*strides))
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = lib.apex_attn_bwd_mode(ctypes.byref(args), mode, workspace.data_ptr(), ws_bytes, stream)
    _lib.check(rc, "custom_attention_backward")
    return dq, dk, dv


def custom_attention_varlen_backward(q, k, v, o, lse, dout, cu_seqlens, max_seqlen, causal=True,
                                     sm_scale=None, window_left=None, deterministic=True):
    """Gradients (dq, dk, dv) of custom_attention_varlen_forward: packed q, o, dout
    [total, H, D], k, v [total, H_kv, D], lse fp32 [H, total] from the forward, cu_seqlens and
    max_seqlen as for the forward. Head dims 64 and 128. Rows outside every sequence come
    back as zeros. Asynchronous on the current stream; `deterministic` as for
    custom_attention_backward.
    """
    if q.dim() != 3 or k.shape != v.shape or o.shape != q.shape or dout.shape != q.shape:
        raise ValueError("expected q, o, dout [total, H, D] and k, v [total, H_kv, D]")
    total, nheads, headdim = q.shape
    kv_heads = k.shape[1]
    if (k.shape[0], k.shape[2]) != (total, headdim) or nheads % kv_heads != 0:
        raise ValueError("k and v must be [total, H_kv, D] with H_kv dividing q's heads")
    if headdim not in (64, 128):
        raise KeyError(headdim)
    if q.dtype not in _DTYPES or any(t.dtype != q.dtype for t in (k, v, o, dout)):
        raise TypeError("q, k, v, o, dout must share one dtype, float16 or bfloat16")
    if lse.shape != (nheads, total) or lse.dtype != torch.float32:
        raise ValueError(f"lse must be float32 [H, total], got {lse.dtype} {tuple(lse.shape)}")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be a 1-D int32 tensor of batch + 1 offsets")
    if not all(t.is_cuda and t.device == q.device for t in (q, k, v, o, dout, lse, cu_seqlens)):
        raise ValueError("all tensors must be CUDA tensors on one device")
    if window_left is not None and (window_left < 0 or not causal):
        raise ValueError("window_left must be >= 0 and needs causal=True")

    def ready(t):
        if t.stride(-1) != 1 or t.data_ptr() % 16 != 0 or any(s % 8 for s in t.stride()[:2]):
            return t.contiguous()
        return t
    q, k, v, o, dout = (ready(t) for t in (q, k, v, o, dout))
    lse, cu_seqlens = lse.contiguous(), cu_seqlens.contiguous()
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(headdim)
    dq = torch.zeros(q.shape, dtype=q.dtype, device=q.device)
    dk = torch.zeros(k.shape, dtype=q.dtype, device=q.device)
    dv = torch.zeros(k.shape, dtype=q.dtype, device=q.device)
    if total == 0:
        return dq, dk, dv
    batch = cu_seqlens.numel() - 1
    lib = _lib.load()
    mode = _BWD_MODES[bool(deterministic)]
    ws_bytes = int(lib.apex_attn_bwd_workspace_bytes_mode(batch, nheads, int(max_seqlen), headdim, mode))
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    strides = []
    for t in (q, k, v, o, dout, dq, dk, dv):
        strides += [t.stride(0), t.stride(1)]
    args = _lib.BwdVarlenArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(),
                              dout=dout.data_ptr(), lse=lse.data_ptr(), dq=dq.data_ptr(),
                              dk=dk.data_ptr(), dv=dv.data_ptr(), cu_seqlens=cu_seqlens.data_ptr(),
                              batch=batch, heads_q=nheads, heads_kv=kv_heads, total=total,
                              max_seqlen=int(max_seqlen), head_dim=headdim, dtype=_DTYPES[q.dtype],
                              causal=1 if causal else 0,
                              window_left=-1 if window_left is None else int(window_left),
                              sm_scale=float(sm_scale), strides=(ctypes.c_longlong * 16)(*strides))
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = lib.apex_attn_bwd_varlen_mode(ctypes.byref(args), mode, workspace.data_ptr(), ws_bytes, stream)
    _lib.check(rc, "custom_attention_varlen_backward")
    return dq, dk, dv


_FWD_KERNELS = {"auto": 0, "two_subtile": 1, "tile": 2}


def set_forward_kernel(kind: str = "auto") -> None:
    """Selects the forward kernel for later calls in this process: "auto" (default: for
    batched calls at head dim 128 without a window, the tile kernel when the call has
    fewer than 3 x (SM count) 256-row query items, or N <= 2048 and fewer than 8 x (SM
    count); the two-sub-tile kernel otherwise), "two_subtile" (that kernel everywhere) or
    "tile" (the tile kernel wherever it applies). Both give results within the operator's
    tolerance; this exists to measure them side by side."""
    if kind not in _FWD_KERNELS:
        raise ValueError(f"kind must be one of {sorted(_FWD_KERNELS)}, got {kind!r}")
    _lib.check(_lib.load().apex_attn_set_forward_kernel(_FWD_KERNELS[kind]), "set_forward_kernel")


def forward_kernel_for(batch: int, heads: int, seq_len: int, head_dim: int, *, num_sms: int,
                       window: int | None = None, packed: bool = False) -> str:
    """Names the forward kernel ("tile" or "two_subtile") that a call of these dimensions
    runs under the current selection on a device with `num_sms` SMs. For a packed batch,
    `batch` is the sequence count and `seq_len` the longest sequence. Launches nothing."""
    rc = _lib.load().apex_attn_forward_kernel_for(batch, heads, seq_len, head_dim,
                                                   -1 if window is None else window,
                                                   1 if packed else 0, num_sms)
    if rc < 0:
        _lib.check(rc, "forward_kernel_for")
    return "tile" if rc == 2 else "two_subtile"


def device_status(device: int | None = None) -> int:
    """Synchronises `device`, returns and clears its status bits (0 = no kernel fault)."""
    if device is None:
        device = torch.cuda.current_device()
    flags = ctypes.c_int(0)
    rc = _lib.load().apex_attn_device_status(int(device), ctypes.byref(flags))
    if rc not in (_lib.OK, _lib.ERR_DEVICE_TIMEOUT):
        _lib.check(rc, "apex_attn_device_status")
    return int(flags.value)


def selftest_wait_timeout(timeout_us: int = 1000) -> None:
    """Launches the bounded-wait self-test kernel on the current stream."""
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.load().apex_attn_selftest_wait_timeout(int(timeout_us), stream),
               "apex_attn_selftest_wait_timeout")
