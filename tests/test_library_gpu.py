"""The scan as torch operators (torch.ops.subq_audio.scan_fwd / scan_bwd):
their fake kernels agree with the real ones (shapes, dtypes, strides, the
handover size), they return what the direct C-ABI calls return, and a
surgered layer traces through torch.compile with fullgraph=True (no graph
break at the scan). torch.compile is a tracing check here, never the path
the kernels run on.
"""
import pytest
import torch

from subq_audio import library, ops  # noqa: F401  (library registers the operators)
from subq_audio.autograd import SubQLinearAttention

pytestmark = pytest.mark.gpu


def _inputs(B=2, H=4, Hkv=4, N=700, dtype=torch.bfloat16, decay=False, mask=True, seed=3):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, 64, generator=g).to(dtype).cuda()
    k = torch.randn(B, Hkv, N, 64, generator=g).to(dtype).cuda()
    v = torch.randn(B, Hkv, N, 64, generator=g).to(dtype).cuda()
    do = torch.randn(B, H, N, 64, generator=g).to(dtype).cuda()
    lg = (-torch.nn.functional.softplus(-(torch.randn(B, H, N, generator=g) + 3.0))).cuda() if decay else None
    m = None
    if mask:
        lens = torch.randint(N // 2, N + 1, (B,), generator=g)
        m = (torch.arange(N)[None, :] < lens[:, None]).to(torch.uint8).cuda()
    return q, k, v, do, lg, m


@pytest.mark.parametrize("decay,Hkv,reverse", [(False, 4, False), (True, 4, False), (False, 2, False),
                                               (False, 4, True)])
def test_operators_equal_direct_calls(decay, Hkv, reverse):
    q, k, v, do, lg, m = _inputs(Hkv=Hkv, decay=decay)
    o, S, z, handover = torch.ops.subq_audio.scan_fwd(q, k, v, lg, m, None, None, reverse, True)
    seg = ops.SegmentStates()
    o_ref, (S_ref, z_ref) = ops.scan_forward(q, k, v, log_gamma=lg, mask=m, return_state=True, reverse=reverse,
                                             segments=seg)
    assert torch.equal(o, o_ref) and torch.equal(S, S_ref) and torch.equal(z, z_ref)
    assert handover.numel() == seg.buf.numel()
    g = torch.ops.subq_audio.scan_bwd(q, k, v, do, lg, m, None, None, o, handover, reverse, decay)
    g_ref = ops.scan_backward(q, k, v, do, log_gamma=lg, mask=m, need_dlog_gamma=decay, reverse=reverse,
                              segments=seg)
    for a, b in zip(g, g_ref):
        if b is not None:
            assert torch.equal(a, b)


@pytest.mark.parametrize("decay", [False, True])
def test_opcheck_schema_and_fake_kernels(decay):
    q, k, v, do, lg, m = _inputs(N=300, decay=decay)
    S0 = torch.randn(2, 4, 64, 64, device="cuda") * 0.5
    z0 = torch.rand(2, 4, 64, device="cuda")
    fwd_args = (q, k, v, lg, m, S0, z0, False, True)
    torch.library.opcheck(torch.ops.subq_audio.scan_fwd.default, fwd_args,
                          test_utils=("test_schema", "test_faketensor"))
    o, _, _, handover = torch.ops.subq_audio.scan_fwd(*fwd_args)
    bwd_args = (q, k, v, do, lg, m, S0, z0, o, handover, False, decay)
    torch.library.opcheck(torch.ops.subq_audio.scan_bwd.default, bwd_args,
                          test_utils=("test_schema", "test_faketensor"))


def test_fake_output_strides_follow_q():
    """A [B, H, N, d] view of a [B, N, H, d] projection output: the fake and
    the real outputs both come in that memory order."""
    x = torch.randn(2, 500, 4, 64, device="cuda", dtype=torch.bfloat16)
    q = k = v = x.transpose(1, 2)
    real = torch.ops.subq_audio.scan_fwd(q, k, v, None, None, None, None, False, False)[0]
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode(allow_non_fake_inputs=True) as mode:
        fq = mode.from_tensor(q)
        fake = torch.ops.subq_audio.scan_fwd(fq, fq, fq, None, None, None, None, False, False)[0]
    assert fake.shape == real.shape and fake.stride() == real.stride()


@pytest.mark.parametrize("causal", [True, False])
def test_layer_traces_with_fullgraph(causal):
    torch.manual_seed(0)
    layer = SubQLinearAttention(256, num_heads=4, num_key_value_heads=2, is_causal=causal).cuda().to(torch.bfloat16)
    x = torch.randn(2, 384, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    ref = layer(x)[0]
    ref.float().square().mean().backward()
    ref_grads = [p.grad.clone() for p in layer.parameters()] + [x.grad.clone()]
    for p in layer.parameters():
        p.grad = None
    x.grad = None
    compiled = torch.compile(layer, fullgraph=True, backend="aot_eager")
    out = compiled(x)[0]
    out.float().square().mean().backward()
    torch.testing.assert_close(out, ref)
    for a, b in zip([p.grad for p in layer.parameters()] + [x.grad], ref_grads):
        torch.testing.assert_close(a, b)


@pytest.mark.parametrize("with_weight", [True, False])
def test_head_rmsnorm_operators_opcheck(with_weight):
    """The epilogue operators' schemas and fake kernels: output shapes, dtypes
    and strides ([B, N, H, D] memory for y, x's order for dx) as the real ones."""
    x = torch.randn(2, 300, 4, 64, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    dy = torch.randn(2, 300, 4, 64, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    w = (torch.rand(64, device="cuda") + 0.5) if with_weight else None
    torch.library.opcheck(torch.ops.subq_audio.head_rmsnorm_fwd.default, (x, w, 1e-5),
                          test_utils=("test_schema", "test_faketensor"))
    torch.library.opcheck(torch.ops.subq_audio.head_rmsnorm_bwd.default, (dy, x, w, 1e-5),
                          test_utils=("test_schema", "test_faketensor"))
