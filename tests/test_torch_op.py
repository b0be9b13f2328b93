"""torch.ops.apex_attn.fwd: the custom-op form of the forward (as nanochat wraps its
Blackwell attention, nanochat_autoresearch/solutions/train.py:493-538)."""
import pytest
import torch

import apex_attn  # noqa: F401  registers the op
from oracle.attention_oracle import make_inputs


def test_op_is_registered_with_fake_impl():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        q = torch.empty(2, 8, 100, 64, dtype=torch.bfloat16, device="cuda" if torch.cuda.is_available() else "cpu")
        k = torch.empty(2, 2, 100, 64, dtype=torch.bfloat16, device=q.device)
        o, lse = torch.ops.apex_attn.fwd(q, k, k, True, -1.0, -1)
        assert o.shape == q.shape and o.dtype == q.dtype
        assert lse.shape == (2, 8, 100) and lse.dtype == torch.float32


def test_op_schema():
    schema = str(torch.ops.apex_attn.fwd.default._schema)
    assert "apex_attn::fwd" in schema and "-> (Tensor, Tensor)" in schema


@pytest.mark.gpu
def test_op_eager_and_compiled_match_operator():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability() != (10, 0):
        pytest.skip("needs a B200 (sm_100)")
    from apex_attn import custom_attention_forward
    q, k, v = (t.cuda() for t in make_inputs(1, 4, 777, 128, seed=31))
    o_ref, l_ref = custom_attention_forward(q, k, v, return_lse=True)
    o, l = torch.ops.apex_attn.fwd(q, k, v, True, -1.0, -1)

    def f(q, k, v):
        o, lse = torch.ops.apex_attn.fwd(q, k, v, True, -1.0, -1)
        return o.float() * 2.0, lse

    # dynamo traces the op without a graph break (fullgraph); the eager backend runs the
    # traced graph as is, so nothing but this kernel and torch eager ops executes.
    oc, lc = torch.compile(f, backend="eager", fullgraph=True)(q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(l, l_ref)
    assert torch.equal(oc, o_ref.float() * 2.0) and torch.equal(lc, l_ref)


def test_bwd_op_fake_impl_and_schema():
    from torch._subclasses.fake_tensor import FakeTensorMode
    schema = str(torch.ops.apex_attn.bwd.default._schema)
    assert "apex_attn::bwd" in schema and "-> (Tensor, Tensor, Tensor)" in schema
    with FakeTensorMode():
        q = torch.empty(2, 8, 100, 128, dtype=torch.bfloat16)
        k = torch.empty(2, 2, 100, 128, dtype=torch.bfloat16)
        lse = torch.empty(2, 8, 100, dtype=torch.float32)
        dq, dk, dv = torch.ops.apex_attn.bwd(q, k, k, q, q, lse, True, -1.0, 64)
        assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == k.shape
        assert dq.dtype == dk.dtype == dv.dtype == torch.bfloat16


def test_fwd_op_backward_traces_to_bwd_op():
    """The registered autograd formula routes the gradient through apex_attn::bwd (checked on
    fake tensors: no kernel runs)."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    seen = []
    from torch.utils._python_dispatch import TorchDispatchMode

    class Record(TorchDispatchMode):
        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            seen.append(str(func))
            return func(*args, **(kwargs or {}))

    with FakeTensorMode():
        q = torch.empty(1, 4, 64, 64, dtype=torch.bfloat16, requires_grad=True)
        k = torch.empty(1, 2, 64, 64, dtype=torch.bfloat16, requires_grad=True)
        v = torch.empty(1, 2, 64, 64, dtype=torch.bfloat16, requires_grad=True)
        with Record():
            o, _ = torch.ops.apex_attn.fwd(q, k, v, True, -1.0, -1)
            o.backward(torch.ones_like(o))
        assert q.grad.shape == q.shape and k.grad.shape == k.shape and v.grad.shape == v.shape
    assert any("apex_attn.bwd" in s for s in seen), seen


@pytest.mark.gpu
def test_bwd_op_compiled_matches_eager():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability() != (10, 0):
        pytest.skip("needs a B200 (sm_100)")
    q, k, v = (t.cuda().requires_grad_(True) for t in make_inputs(1, 4, 300, 64, seed=32))
    do = make_inputs(1, 4, 300, 64, seed=33)[0].cuda()

    def f(q, k, v):
        o, _ = torch.ops.apex_attn.fwd(q, k, v, True, -1.0, -1)
        return o

    o = f(q, k, v)
    g_eager = torch.autograd.grad(o, (q, k, v), do)
    oc = torch.compile(f, backend="eager", fullgraph=True)(q, k, v)
    g_comp = torch.autograd.grad(oc, (q, k, v), do)
    torch.cuda.synchronize()
    for a, b in zip(g_eager, g_comp):
        assert torch.equal(a, b)
