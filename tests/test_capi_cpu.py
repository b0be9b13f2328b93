"""C-ABI checks that need no GPU: the library loads, exports exactly what
include/apex_attn.h declares, and rejects bad arguments with the documented codes
before touching CUDA."""
import ctypes
import os
import re

import pytest

from apex_attn import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "apex_attn.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(apex_attn_\w+)\s*\(", text, re.M)))


def header_codes():
    text = open(HEADER).read()
    return {name: int(val) for name, val in re.findall(r"#define (APEX_ATTN_(?:OK|ERR_\w+))\s+(-?\d+)", text)}


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_library_exports_every_header_symbol(lib):
    syms = header_symbols()
    assert "apex_attn_fwd" in syms and len(syms) >= 6
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SYMBOLS), "ctypes table out of sync with the header"


def test_status_codes_match_header():
    codes = header_codes()
    for name, val in codes.items():
        py = getattr(_lib, name.replace("APEX_ATTN_", ""))
        assert py == val, name


def test_strerror_covers_every_code(lib):
    for name, val in header_codes().items():
        msg = _lib.strerror(val)
        assert msg and msg != "unknown status", name
    assert _lib.strerror(12345) == "unknown status"


def test_version_and_head_dims(lib):
    assert lib.apex_attn_version() >= 100
    for d in (64, 128, 256):
        assert lib.apex_attn_supports_head_dim(d) == 1
    for d in (0, 32, 96, 512):
        assert lib.apex_attn_supports_head_dim(d) == 0


FAKE = 0x10000  # 16-byte aligned, never dereferenced: validation fails first


def call(lib, q=FAKE, k=FAKE, v=FAKE, o=FAKE, lse=None, B=1, H=2, N=256, D=64, dtype=0,
         causal=1, scale=0.125, strides=None):
    if strides is None:
        strides = [H * N * D, N * D, D] * 4
    arr = (ctypes.c_longlong * 12)(*strides) if strides is not False else None
    return lib.apex_attn_fwd(q, k, v, o, lse, B, H, N, D, dtype, causal, scale, arr, None)


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(o=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(strides=False), _lib.ERR_INVALID_ARGUMENT),
    (dict(B=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(N=-5), _lib.ERR_INVALID_ARGUMENT),
    (dict(D=96), _lib.ERR_UNSUPPORTED_HEAD_DIM),
    (dict(D=32), _lib.ERR_UNSUPPORTED_HEAD_DIM),
    (dict(dtype=2), _lib.ERR_UNSUPPORTED_DTYPE),
    (dict(scale=0.0), _lib.ERR_BAD_SCALE),
    (dict(scale=-1.0), _lib.ERR_BAD_SCALE),
    (dict(scale=float("nan")), _lib.ERR_BAD_SCALE),
    (dict(scale=float("inf")), _lib.ERR_BAD_SCALE),
    (dict(strides=[2 * 256 * 64, 256 * 64, 60] * 4), _lib.ERR_BAD_LAYOUT),
    (dict(strides=[2 * 256 * 64, 256 * 64, 32] * 4), _lib.ERR_BAD_LAYOUT),
    (dict(strides=[2 * 256 * 64, -256 * 64, 64] * 4), _lib.ERR_BAD_LAYOUT),
    (dict(q=FAKE + 8), _lib.ERR_BAD_LAYOUT),
    (dict(lse=FAKE + 2), _lib.ERR_BAD_LAYOUT),
    (dict(B=1 << 20, H=1 << 11), _lib.ERR_TOO_LARGE),
])
def test_argument_validation(lib, kw, code):
    assert call(lib, **kw) == code


def test_valid_arguments_without_device_report_no_device(lib):
    # Host memory (or no GPU at all) is rejected after validation, never dereferenced.
    import torch
    if torch.cuda.is_available():
        pytest.skip("checks the no-device path")
    assert call(lib) == _lib.ERR_NO_DEVICE


def _ex_args(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, o=FAKE, lse=None, batch=1, heads_q=4, heads_kv=2, seqlen=256,
             head_dim=64, dtype=0, causal=1, window_left=-1, sm_scale=0.125)
    a.update(kw)
    st = (ctypes.c_longlong * 12)(*([4 * 256 * 64, 256 * 64, 64] * 4))
    return _lib.FwdArgs(strides=st, **a)


def test_ex_struct_layout_matches_c_abi():
    # x86-64 / aarch64 layout of apex_attn_fwd_args: 5 pointers, 8 ints, 1 float, padding
    # to 8 bytes, then 12 long longs.
    assert ctypes.sizeof(_lib.FwdArgs) == 176
    assert _lib.FwdArgs.strides.offset == 80 and _lib.FwdArgs.sm_scale.offset == 72


@pytest.mark.parametrize("kw,code", [
    (dict(heads_kv=3), _lib.ERR_INVALID_ARGUMENT),            # 4 % 3 != 0
    (dict(heads_kv=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(window_left=-2), _lib.ERR_INVALID_ARGUMENT),
    (dict(window_left=16, causal=0), _lib.ERR_INVALID_ARGUMENT),  # windows are causal-only
    (dict(head_dim=96), _lib.ERR_UNSUPPORTED_HEAD_DIM),
    (dict(q=None), _lib.ERR_INVALID_ARGUMENT),
])
def test_ex_argument_validation(lib, kw, code):
    a = _ex_args(**kw)
    assert lib.apex_attn_fwd_ex(ctypes.byref(a), None) == code


def test_ex_null_args(lib):
    assert lib.apex_attn_fwd_ex(None, None) == _lib.ERR_INVALID_ARGUMENT


# ---------------------------------------------------------------- backward --
def _bwd_args(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, o=FAKE, dout=FAKE, lse=FAKE, dq=FAKE, dk=FAKE, dv=FAKE,
             batch=1, heads_q=4, heads_kv=2, seqlen=256, head_dim=64, dtype=0, causal=1,
             window_left=-1, sm_scale=0.125)
    strides = kw.pop("strides", [4 * 256 * 64, 256 * 64, 64] * 8)
    a.update(kw)
    return _lib.BwdArgs(strides=(ctypes.c_longlong * 24)(*strides), **a)


def _c_layout(struct: str, fields: list[str]) -> list[int]:
    """sizeof and offsetof of `struct` as the C compiler lays it out from the header."""
    import subprocess
    import tempfile
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"apex_attn.h\"\nint main(void){"
    src += f'printf("%zu", sizeof({struct}));'
    for f in fields:
        src += f'printf(" %zu", offsetof({struct}, {f}));'
    src += "return 0;}\n"
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "l.c"), os.path.join(d, "l")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        return [int(x) for x in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]


@pytest.mark.parametrize("cls,struct", [(_lib.FwdArgs, "apex_attn_fwd_args"),
                                        (_lib.BwdArgs, "apex_attn_bwd_args"),
                                        (_lib.VarlenArgs, "apex_attn_varlen_args"),
                                        (_lib.BwdVarlenArgs, "apex_attn_bwd_varlen_args")])
def test_ctypes_structs_match_c_compiler_layout(cls, struct):
    import shutil
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    names = [f[0] for f in cls._fields_]
    expect = _c_layout(struct, names)
    assert [ctypes.sizeof(cls)] + [getattr(cls, n).offset for n in names] == expect


def test_bwd_workspace_bytes(lib):
    assert lib.apex_attn_bwd_workspace_bytes(2, 3, 130) == 2 * 2 * 3 * 256 * 4
    assert lib.apex_attn_bwd_workspace_bytes(1, 1, 128) == 2 * 128 * 4
    assert lib.apex_attn_bwd_workspace_bytes(0, 3, 130) == 0
    assert lib.apex_attn_bwd_workspace_bytes(1, 1, -1) == 0


@pytest.mark.parametrize("kw,code", [
    (dict(dout=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(lse=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(dq=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(heads_kv=3), _lib.ERR_INVALID_ARGUMENT),
    (dict(window_left=8, causal=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(seqlen=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(head_dim=256), _lib.ERR_UNSUPPORTED_HEAD_DIM),
    (dict(head_dim=96), _lib.ERR_UNSUPPORTED_HEAD_DIM),
    (dict(dtype=5), _lib.ERR_UNSUPPORTED_DTYPE),
    (dict(sm_scale=0.0), _lib.ERR_BAD_SCALE),
    (dict(strides=[4 * 256 * 64, 256 * 64, 64] * 7 + [4 * 256 * 64, 256 * 64, 36]), _lib.ERR_BAD_LAYOUT),
    (dict(strides=[4 * 256 * 64, 256 * 64, 32] * 8), _lib.ERR_BAD_LAYOUT),
    (dict(dv=FAKE + 8), _lib.ERR_BAD_LAYOUT),
    (dict(lse=FAKE + 2), _lib.ERR_BAD_LAYOUT),
])
def test_bwd_argument_validation(lib, kw, code):
    a = _bwd_args(**kw)
    assert lib.apex_attn_bwd(ctypes.byref(a), FAKE, 1 << 20, None) == code


def test_bwd_workspace_checks(lib):
    a = _bwd_args()
    need = lib.apex_attn_bwd_workspace_bytes(1, 4, 256)
    assert lib.apex_attn_bwd(ctypes.byref(a), None, need, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd(ctypes.byref(a), FAKE, need - 4, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd(ctypes.byref(a), FAKE + 4, need, None) == _lib.ERR_BAD_LAYOUT
    assert lib.apex_attn_bwd(None, FAKE, need, None) == _lib.ERR_INVALID_ARGUMENT


# ----------------------------------------------------------------- varlen ----
def _varlen_args(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, o=FAKE, lse=None, cu_seqlens=FAKE, batch=3, heads_q=4,
             heads_kv=2, total=1000, max_seqlen=500, head_dim=128, dtype=0, causal=1,
             window_left=-1, sm_scale=0.088)
    strides = kw.pop("strides", [4 * 128, 128, 2 * 128, 128, 2 * 128, 128, 4 * 128, 128])
    a.update(kw)
    return _lib.VarlenArgs(strides=(ctypes.c_longlong * 8)(*strides), **a)


@pytest.mark.parametrize("kw,code", [
    (dict(cu_seqlens=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(q=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(batch=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(total=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(max_seqlen=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(heads_kv=3), _lib.ERR_INVALID_ARGUMENT),
    (dict(window_left=5, causal=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(head_dim=96), _lib.ERR_UNSUPPORTED_HEAD_DIM),
    (dict(dtype=9), _lib.ERR_UNSUPPORTED_DTYPE),
    (dict(sm_scale=-1.0), _lib.ERR_BAD_SCALE),
    (dict(strides=[4 * 128, 100, 256, 128, 256, 128, 512, 128]), _lib.ERR_BAD_LAYOUT),  # not x8
    (dict(strides=[4 * 128, 64, 256, 128, 256, 128, 512, 128]), _lib.ERR_BAD_LAYOUT),   # head rows overlap
    (dict(cu_seqlens=FAKE + 2), _lib.ERR_BAD_LAYOUT),
    (dict(o=FAKE + 8), _lib.ERR_BAD_LAYOUT),
    (dict(batch=1 << 28, max_seqlen=1 << 20), _lib.ERR_TOO_LARGE),
])
def test_varlen_argument_validation(lib, kw, code):
    a = _varlen_args(**kw)
    assert lib.apex_attn_fwd_varlen(ctypes.byref(a), None) == code


def test_varlen_null_args(lib):
    assert lib.apex_attn_fwd_varlen(None, None) == _lib.ERR_INVALID_ARGUMENT


def _bwd_varlen_args(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, o=FAKE, dout=FAKE, lse=FAKE, dq=FAKE, dk=FAKE, dv=FAKE,
             cu_seqlens=FAKE, batch=3, heads_q=4, heads_kv=2, total=1000, max_seqlen=500,
             head_dim=128, dtype=0, causal=1, window_left=-1, sm_scale=0.088)
    strides = kw.pop("strides", [512, 128, 256, 128, 256, 128, 512, 128, 512, 128, 512, 128, 256, 128, 256, 128])
    a.update(kw)
    return _lib.BwdVarlenArgs(strides=(ctypes.c_longlong * 16)(*strides), **a)


@pytest.mark.parametrize("kw,code", [
    (dict(cu_seqlens=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(dout=None), _lib.ERR_INVALID_ARGUMENT),
    (dict(total=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(heads_kv=3), _lib.ERR_INVALID_ARGUMENT),
    (dict(head_dim=256), _lib.ERR_UNSUPPORTED_HEAD_DIM),
    (dict(sm_scale=0.0), _lib.ERR_BAD_SCALE),
    (dict(strides=[512, 120] + [256, 128] * 7), _lib.ERR_BAD_LAYOUT),
    (dict(cu_seqlens=FAKE + 2), _lib.ERR_BAD_LAYOUT),
    (dict(dk=FAKE + 8), _lib.ERR_BAD_LAYOUT),
])
def test_bwd_varlen_argument_validation(lib, kw, code):
    a = _bwd_varlen_args(**kw)
    assert lib.apex_attn_bwd_varlen(ctypes.byref(a), FAKE, 1 << 24, None) == code


def test_bwd_varlen_workspace_checks(lib):
    a = _bwd_varlen_args()
    need = lib.apex_attn_bwd_workspace_bytes(3, 4, 500)
    assert lib.apex_attn_bwd_varlen(ctypes.byref(a), FAKE, need - 16, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_varlen(None, FAKE, need, None) == _lib.ERR_INVALID_ARGUMENT


# ----------------------------------------------------- backward modes --------
def test_bwd_workspace_bytes_by_mode(lib):
    """Mode 0 (deterministic) needs what apex_attn_bwd needs; mode 1 (fused) adds a
    256-byte-aligned fp32 dQ accumulator of batch * heads * seqlen * head_dim values."""
    for b, h, n, d in ((2, 3, 130, 64), (1, 1, 128, 128), (4, 32, 8192, 128)):
        base = lib.apex_attn_bwd_workspace_bytes(b, h, n)
        assert lib.apex_attn_bwd_workspace_bytes_mode(b, h, n, d, 0) == base
        assert lib.apex_attn_bwd_workspace_bytes_mode(b, h, n, d, 1) == (base + 255) // 256 * 256 + b * h * n * d * 4
    assert lib.apex_attn_bwd_workspace_bytes_mode(0, 3, 130, 64, 1) == 0
    assert lib.apex_attn_bwd_workspace_bytes_mode(1, 1, 128, 0, 1) == 0


def test_bwd_mode_validation(lib):
    a = _bwd_args()
    det = lib.apex_attn_bwd_workspace_bytes_mode(1, 4, 256, 64, 0)
    fused = lib.apex_attn_bwd_workspace_bytes_mode(1, 4, 256, 64, 1)
    for bad in (-1, 2, 7):
        assert lib.apex_attn_bwd_mode(ctypes.byref(a), bad, FAKE, fused, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_mode(ctypes.byref(a), 1, FAKE, det, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_mode(ctypes.byref(a), 1, FAKE, fused - 4, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_mode(None, 1, FAKE, fused, None) == _lib.ERR_INVALID_ARGUMENT
    # valid arguments reach the device lookup, which fails on host (fake) pointers
    assert lib.apex_attn_bwd_mode(ctypes.byref(a), 1, FAKE, fused, None) == _lib.ERR_NO_DEVICE
    v = _bwd_varlen_args()
    vf = lib.apex_attn_bwd_workspace_bytes_mode(3, 4, 500, 128, 1)
    assert lib.apex_attn_bwd_varlen_mode(ctypes.byref(v), 3, FAKE, vf, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_varlen_mode(ctypes.byref(v), 1, FAKE, vf - 16, None) == _lib.ERR_INVALID_ARGUMENT
    # the accumulator holds heads x total rows, which batch x max_seqlen must cover
    big = _bwd_varlen_args(total=1501)
    assert lib.apex_attn_bwd_varlen_mode(ctypes.byref(big), 1, FAKE, 1 << 30, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.apex_attn_bwd_varlen_mode(ctypes.byref(v), 1, FAKE, vf, None) == _lib.ERR_NO_DEVICE


def test_num_sms_hint_without_device(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("checks the no-device path")
    assert lib.apex_attn_num_sms_hint(0) == _lib.ERR_NO_DEVICE
    assert lib.apex_attn_num_sms_hint(-1) == _lib.ERR_NO_DEVICE


@pytest.mark.parametrize("B,H,N,D,window,packed,want", [
    # d=128, N >= 4096: the tile kernel below 3 x 148 = 444 256-row items
    (1, 13, 8192, 128, -1, 0, 2),    # 416 items
    (1, 14, 8192, 128, -1, 0, 1),    # 448
    (3, 8, 4096, 128, -1, 0, 2),     # 384
    (2, 16, 4096, 128, -1, 0, 1),    # 512
    (4, 32, 8192, 128, -1, 0, 1),    # C3: 4096
    # d=128, N <= 2048: below 8 x 148 = 1184 items
    (147, 1, 2048, 128, -1, 0, 2),   # 1176
    (148, 1, 2048, 128, -1, 0, 1),   # 1184
    (8, 32, 1024, 128, -1, 0, 2),    # 1024
    (16, 32, 1024, 128, -1, 0, 1),   # 2048
    (8, 32, 512, 128, -1, 0, 2),     # 512 (N=512 rounds up to 2 items per head)
    # the two-sub-tile kernel for d=64 and d=256, windows and packed batches
    (1, 8, 2048, 64, -1, 0, 1),
    (1, 1, 256, 256, -1, 0, 1),
    (1, 8, 2048, 128, 256, 0, 1),
    (1, 8, 2048, 128, -1, 1, 1),
])
def test_forward_kernel_selection(lib, B, H, N, D, window, packed, want):
    assert lib.apex_attn_forward_kernel_for(B, H, N, D, window, packed, 148) == want


def test_forward_kernel_selection_follows_pinning_and_validates(lib):
    import apex_attn
    try:
        apex_attn.set_forward_kernel("two_subtile")
        assert apex_attn.forward_kernel_for(1, 8, 2048, 128, num_sms=148) == "two_subtile"
        apex_attn.set_forward_kernel("tile")
        assert apex_attn.forward_kernel_for(4, 32, 8192, 128, num_sms=148) == "tile"
        assert apex_attn.forward_kernel_for(4, 32, 8192, 64, num_sms=148) == "tile"
        assert apex_attn.forward_kernel_for(1, 8, 2048, 256, num_sms=148) == "two_subtile"
        assert apex_attn.forward_kernel_for(1, 8, 2048, 128, num_sms=148, window=64) == "two_subtile"
        assert apex_attn.forward_kernel_for(1, 8, 2048, 128, num_sms=148, packed=True) == "two_subtile"
    finally:
        apex_attn.set_forward_kernel("auto")
    assert apex_attn.forward_kernel_for(1, 8, 2048, 128, num_sms=148) == "tile"
    for args in [(0, 1, 64, 128, -1, 0, 148), (1, 0, 64, 128, -1, 0, 148), (1, 1, 0, 128, -1, 0, 148),
                 (1, 1, 64, 96, -1, 0, 148), (1, 1, 64, 128, -2, 0, 148), (1, 1, 64, 128, -1, 0, 0)]:
        assert lib.apex_attn_forward_kernel_for(*args) == _lib.ERR_INVALID_ARGUMENT, args
    with pytest.raises(RuntimeError):
        apex_attn.forward_kernel_for(1, 1, 64, 96, num_sms=148)
