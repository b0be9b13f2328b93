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
