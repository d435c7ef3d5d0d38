"""The module's prologue and epilogue around the scan.

Epilogue: the per-head RMSNorm kernels (csrc/head_norm.cu,
subq_head_rmsnorm_fwd / _bwd) against torch's float32 RMSNorm and its
autograd: the reference's SubQLinearAttention epilogue, nn.RMSNorm(head_dim,
eps=1e-5) then the transpose copy to [B, L, H*D] (reference
python/subq_audio/autograd.py:706-710, 763-769). Tolerances: 1e-5 of max |ref|
for float32, 1e-2 for 16-bit outputs (one rounding of the output); dweight in
float32 at 1e-4 (sums over up to 10^5 rows in another order).

Prologue: q, k, v and the gate from one GEMM over the concatenated weights
against the four nn.Linear calls of the reference (autograd.py:735-751):
outputs and every gradient, with bias, GQA and without gating.
"""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from subq_audio import _capi, ops
from subq_audio.autograd import SubQLinearAttention

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _x(B, H, N, D, dtype, layout, seed):
    g = torch.Generator().manual_seed(seed)
    if layout == "bnhd":  # a projection-shaped [B, N, H, D] buffer viewed as [B, H, N, D]
        x = (torch.randn(B, N, H, D, generator=g) * 3.0).to(dtype).cuda().transpose(1, 2)
    else:
        x = (torch.randn(B, H, N, D, generator=g) * 3.0).to(dtype).cuda()
    w = (torch.rand(D, generator=g) + 0.5).cuda()
    return x, w


def _torch_ref(x, w, eps, dy=None):
    xf = x.detach().float().requires_grad_(True)
    wf = w.detach().float().requires_grad_(True) if w is not None else None
    y = F.rms_norm(xf, (x.shape[-1],), wf, eps)
    if dy is None:
        return y
    y.backward(dy.float())
    return y, xf.grad, (wf.grad if wf is not None else None)


CASES = [
    # B, H, N, D, dtype, layout
    (2, 4, 300, 64, torch.bfloat16, "bnhd"),
    (1, 3, 77, 64, torch.float16, "bhnd"),
    (2, 2, 129, 32, torch.float32, "bnhd"),
    (1, 1, 5, 8, torch.float32, "bhnd"),
    (1, 2, 33, 16, torch.bfloat16, "bhnd"),
    (3, 2, 50, 128, torch.bfloat16, "bnhd"),
    (1, 2, 41, 256, torch.float32, "bnhd"),
    (4, 12, 1024, 64, torch.bfloat16, "bnhd"),
]


@pytest.mark.parametrize("case", CASES, ids=[f"r{i}" for i in range(len(CASES))])
def test_forward_and_backward_match_torch(case):
    B, H, N, D, dtype, layout = case
    x, w = _x(B, H, N, D, dtype, layout, seed=N + D)
    y = ops.head_rmsnorm(x, w, 1e-5)
    # the output's memory is [B, N, H, D]: the module's transpose back is a view
    assert y.transpose(1, 2).is_contiguous()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    ref = _torch_ref(x, w, 1e-5)
    assert rel(y, ref) < tol
    g = torch.Generator().manual_seed(7)
    dy = torch.randn(B, N, H, D, generator=g).to(dtype).cuda().transpose(1, 2)
    _, rdx, rdw = _torch_ref(x, w, 1e-5, dy)
    dx, dw = ops.head_rmsnorm_backward(dy, x, w, 1e-5)
    assert rel(dx, rdx) < (1e-5 if dtype == torch.float32 else 1e-2)
    assert rel(dw, rdw) < 1e-4
    # dweight is reproducible bit for bit
    dx2, dw2 = ops.head_rmsnorm_backward(dy, x, w, 1e-5)
    assert torch.equal(dw, dw2) and torch.equal(dx, dx2)


def test_no_weight_is_the_reference_fallback():
    """Without nn.RMSNorm the reference normalises by out * rsqrt(mean(out^2) + 1e-5)."""
    x, _ = _x(2, 3, 100, 64, torch.float32, "bhnd", seed=3)
    y = ops.head_rmsnorm(x, None, 1e-5)
    torch.testing.assert_close(y, x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5), rtol=1e-5, atol=1e-6)
    dy = torch.randn_like(x)
    dx, dw = ops.head_rmsnorm_backward(dy, x, None, 1e-5)
    _, rdx, _ = _torch_ref(x, None, 1e-5, dy)
    assert dw is None and rel(dx, rdx) < 1e-5


def test_zero_rows_and_unaligned_rows():
    x, w = _x(1, 2, 1, 64, torch.float32, "bhnd", seed=5)
    x = x.clone()
    x[0, 0].zero_()  # a zero row: y = 0, dx = 0 (rsqrt(eps) finite)
    y = ops.head_rmsnorm(x, w)
    assert torch.equal(y[0, 0], torch.zeros_like(y[0, 0])) and torch.isfinite(y).all()
    # a view whose rows are not 16-byte aligned is copied before the kernels
    base = torch.randn(1, 2, 10, 65, device="cuda")[..., 1:]
    y2 = ops.head_rmsnorm(base, w)
    assert rel(y2, _torch_ref(base, w, 1e-5)) < 1e-5
    # empty: dweight is zero
    e = torch.empty(2, 3, 0, 64, device="cuda")
    dx, dw = ops.head_rmsnorm_backward(e, e, w)
    assert dx.shape == e.shape and torch.equal(dw, torch.zeros(64, device="cuda"))


def test_c_abi_rejects_unsupported_and_misaligned():
    x = torch.randn(1, 1, 4, 48, device="cuda")
    a = _capi.RmsArgs()
    a.batch, a.heads, a.seq_len, a.head_dim, a.dtype, a.eps = 1, 1, 4, 48, _capi.SUBQ_FP32, 1e-5
    a.x = ops._t4(x)
    a.y = ops._t4(x)
    with pytest.raises(_capi.SubqError) as ei:
        _capi.head_rmsnorm_fwd(a)
    assert ei.value.code == _capi.SUBQ_ERR_UNSUPPORTED
    z = torch.randn(1, 1, 4, 66, device="cuda")[..., 1:65]  # rows start 4 bytes past a boundary
    a.head_dim = 64
    a.x = ops._t4(z)
    a.y = ops._t4(z)
    with pytest.raises(ValueError, match="16-byte"):
        _capi.head_rmsnorm_fwd(a)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_module_epilogue_equals_torch_epilogue(dtype, monkeypatch):
    """SubQLinearAttention with the kernels' epilogue against the same module
    with torch's RMSNorm and transpose copy: output and every gradient."""
    torch.manual_seed(2)
    mod = SubQLinearAttention(256, num_heads=4, use_data_dependent_gating=True).cuda()
    with torch.no_grad():
        mod.head_norm.weight.uniform_(0.5, 1.5)
    x = torch.randn(2, 700, 256, device="cuda", requires_grad=True)

    def run():
        for p in mod.parameters():
            p.grad = None
        x.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16):
            y, _ = mod(x)
        y.float().square().mean().backward()
        return y.detach().float(), [p.grad.clone() for p in mod.parameters()] + [x.grad.clone()]

    y_k, g_k = run()
    monkeypatch.setattr(ops, "head_rmsnorm_supported", lambda t: False)
    y_t, g_t = run()
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    assert rel(y_k, y_t) < tol
    for a, b in zip(g_k, g_t):
        assert rel(a, b) < tol


@pytest.mark.parametrize("bias,kv_heads,gating,dtype", [(False, 4, True, torch.bfloat16),
                                                        (True, 2, True, torch.float32),
                                                        (True, 4, False, torch.bfloat16),
                                                        (False, 1, True, torch.float32)])
def test_fused_projections_equal_separate_linears(bias, kv_heads, gating, dtype, monkeypatch):
    torch.manual_seed(4)
    mod = SubQLinearAttention(256, num_heads=4, num_key_value_heads=kv_heads, bias=bias,
                              use_data_dependent_gating=gating).cuda()
    x = torch.randn(2, 500, 256, device="cuda", requires_grad=True)
    assert mod._fused_projections(x) is not None

    def run():
        for p in mod.parameters():
            p.grad = None
        x.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16):
            y, _ = mod(x)
        y.float().square().mean().backward()
        return y.detach().float(), {n: p.grad.clone() for n, p in mod.named_parameters()}, x.grad.clone()

    y_f, g_f, dx_f = run()
    monkeypatch.setattr(SubQLinearAttention, "_fused_projections", lambda self, h: None)
    y_s, g_s, dx_s = run()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert rel(y_f, y_s) < tol
    assert rel(dx_f, dx_s) < tol
    assert g_f.keys() == g_s.keys()
    for n in g_f:
        assert rel(g_f[n], g_s[n]) < tol, n
