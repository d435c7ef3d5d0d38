"""Autograd surface on the GPU: SubQAttentionFunction, chunkwise_flash_linear_attention,
SubQLinearAttention and surgery, against the reference's own outputs (fixtures
made by running the reference's python/subq_audio/autograd.py in float64) and
the oracle.

Reference tests these follow: tests/test_autograd.py (analytic grads vs loop,
gradchecks), tests/test_surgery_and_caching.py (chunked vs sequential,
padding invariance, cached generation).
"""
import os

import numpy as np
import pytest
import torch

import golden_inputs as gi
import oracle
from subq_audio import autograd as ag
from subq_audio import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a = a.detach().double().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _case(name):
    spec = gi.AUTOGRAD_CASES[name]
    q, k, v, dO, w, mask = gi.autograd_inputs(spec)
    t = lambda x: torch.tensor(x, dtype=torch.float64, device=DEV)  # noqa: E731
    wt = t(gi.NO_DECAY_W if w is None else w)
    mt = None if mask is None else torch.tensor(mask, device=DEV)
    return spec, t(q), t(k), t(v), t(dO), wt, mt, w is not None


# log(gamma) crosses the C ABI as float32, so the float64 kernels agree with
# the reference's float64 autograd to ~1e-7 relative, not to 1e-12.
TOL64 = 2e-6


@pytest.mark.parametrize("name", list(gi.AUTOGRAD_CASES))
def test_function_matches_reference_autograd(golden_dir, name):
    g = np.load(os.path.join(golden_dir, "autograd_cases.npz"))
    spec, q, k, v, dO, w, mask, has_decay = _case(name)
    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)
    w.requires_grad_(has_decay)
    out = ag.SubQAttentionFunction.apply(q, k, v, w, 64, mask)
    assert rel(out, g[f"{name}/o_fn"]) < TOL64
    out.backward(dO)
    for key, got in (("dq", q.grad), ("dk", k.grad), ("dv", v.grad)):
        assert rel(got, g[f"{name}/{key}"]) < TOL64, key
    if has_decay:
        assert rel(w.grad, g[f"{name}/dw"]) < 1e-4  # d log(gamma) leaves the kernel in float32


@pytest.mark.parametrize("name", ["mh_head", "mask_len", "causal3d_nodecay"])
def test_chunkwise_state_matches_reference(golden_dir, name):
    g = np.load(os.path.join(golden_dir, "autograd_cases.npz"))
    spec, q, k, v, _, w, mask, _ = _case(name)
    out, S = ag.chunkwise_flash_linear_attention(q, k, v, w, attention_mask=mask)
    assert rel(out, g[f"{name}/o"]) < TOL64
    refS = g[f"{name}/S"]
    assert rel(S.reshape(refS.shape), refS) < TOL64
    refZ = g[f"{name}/Z"]
    assert rel(S.Z.reshape(refZ.shape), refZ) < TOL64


def test_streaming_past_state_matches_reference(golden_dir):
    g = np.load(os.path.join(golden_dir, "streaming_case.npz"))
    q, k, v = (torch.tensor(x, device=DEV) for x in gi.stream_inputs())
    L = gi.STREAM_SPLIT
    full, _ = ag.chunkwise_flash_linear_attention(q, k, v, gi.NO_DECAY_W)
    assert rel(full, g["full"]) < TOL64
    parts, state = [], None
    for s in range(0, q.shape[2], L):
        o, state = ag.chunkwise_flash_linear_attention(q[:, :, s:s + L], k[:, :, s:s + L], v[:, :, s:s + L],
                                                       gi.NO_DECAY_W, past_state=state)
        parts.append(o)
    assert rel(torch.cat(parts, dim=2), g["streamed"]) < TOL64
    assert rel(state, g["S"]) < 1e-5  # the carried state is float32


def test_gradcheck_float64_qkv():
    torch.manual_seed(0)
    B, H, T, D = 1, 2, 37, 8
    q, k, v = (torch.randn(B, H, T, D, dtype=torch.float64, device=DEV, requires_grad=True) for _ in range(3))
    mask = torch.ones(B, T, dtype=torch.bool, device=DEV)
    mask[:, 30:] = False

    def fn(q_, k_, v_):
        return ag.SubQAttentionFunction.apply(q_, k_, v_, None, 64, mask)

    assert torch.autograd.gradcheck(fn, (q, k, v), eps=1e-6, atol=1e-6, rtol=1e-5)


def test_bidirectional_matches_oracle():
    torch.manual_seed(1)
    B, H, T, D = 2, 2, 90, 16
    q, k, v, dO = (torch.randn(B, H, T, D, dtype=torch.float64) for _ in range(4))
    w = torch.full((H,), 2.0, dtype=torch.float64)
    qg, kg, vg = (x.to(DEV).requires_grad_(True) for x in (q, k, v))
    out = ag.SubQAttentionFunction.apply(qg, kg, vg, w.to(DEV), 64, None, False)
    out.backward(dO.to(DEV))
    # oracle: forward scan + reversed scan - the doubly counted diagonal v
    f = lambda x: np.flip(x.numpy(), axis=2).copy()  # noqa: E731
    o1, _ = oracle.attention(q.numpy(), k.numpy(), v.numpy(), decay_w=w.numpy())
    o2, _ = oracle.attention(f(q), f(k), f(v), decay_w=w.numpy())
    ref = o1 + np.flip(o2, axis=2) - v.numpy()
    assert rel(out, ref) < TOL64
    d1 = oracle.attention_backward(q.numpy(), k.numpy(), v.numpy(), dO.numpy(), decay_w=w.numpy())
    d2 = oracle.attention_backward(f(q), f(k), f(v), f(dO), decay_w=w.numpy())
    assert rel(qg.grad, d1[0] + np.flip(d2[0], axis=2)) < TOL64
    assert rel(kg.grad, d1[1] + np.flip(d2[1], axis=2)) < TOL64
    assert rel(vg.grad, d1[2] + np.flip(d2[2], axis=2) - dO.numpy()) < TOL64


def test_bf16_masked_function_uses_tensor_cores_and_matches_oracle():
    """The C2 shape family (d=64, bf16, key-padding mask, gamma=1) at a size the
    oracle finishes quickly; <= 2e-2 on O and on every gradient."""
    g = torch.Generator().manual_seed(7)
    B, H, T, D = 2, 3, 1000, 64
    q, k, v, dO = (torch.randn(B, H, T, D, generator=g).to(torch.bfloat16) for _ in range(4))
    lens = torch.tensor([1000, 613])
    mask = torch.arange(T)[None, :] < lens[:, None]
    qg, kg, vg = (x.to(DEV).requires_grad_(True) for x in (q, k, v))
    out = ag.SubQAttentionFunction.apply(qg, kg, vg, None, 64, mask.to(DEV))
    assert ops.last_path() == "tensorcore"
    out.backward(dO.to(DEV))
    assert ops.last_path() == "tensorcore"
    n = lambda x: x.double().numpy()  # noqa: E731
    ref = oracle.attention(n(q), n(k), n(v), decay_w=None, attention_mask=mask.numpy())[0]
    dq, dk, dv, _ = oracle.attention_backward(n(q), n(k), n(v), n(dO), decay_w=None, attention_mask=mask.numpy())
    assert rel(out, ref) < 2e-2
    assert rel(qg.grad, dq) < 2e-2
    assert rel(kg.grad, dk) < 2e-2
    assert rel(vg.grad, dv) < 2e-2


def test_long_stream_fp16_matches_single_pass():
    """Config-3 shape: B=1, H=4, d=64, N=131072 in fp16, fed as 32 calls of 4096
    tokens carrying float32 S and z; the concatenation is compared with one
    float64 pass of the oracle over the whole sequence (<= 2e-2)."""
    g = torch.Generator().manual_seed(3)
    B, H, N, D, L = 1, 4, 131072, 64, 4096
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(torch.float16) for _ in range(3))
    qd, kd, vd = (x.to(DEV) for x in (q, k, v))
    outs, state = [], None
    for s in range(0, N, L):
        o, state = ag.chunkwise_flash_linear_attention(qd[:, :, s:s + L], kd[:, :, s:s + L], vd[:, :, s:s + L],
                                                       None, past_state=state)
        outs.append(o)
    out = torch.cat(outs, dim=2)
    assert ops.last_path() == "tensorcore"
    n = lambda x: x.double().numpy()  # noqa: E731
    ref, (S, z) = oracle.attention(n(q), n(k), n(v), decay_w=None)
    assert rel(out, ref) < 2e-2
    assert rel(state, S) < 1e-3
    assert rel(state.Z.reshape(z.shape), z) < 1e-3


def _module_reference(mod, x, mask=None):
    """The module's forward recomputed in float64 with the oracle scan."""
    B, L, _ = x.shape
    Hh, Dh = mod.num_heads, mod.head_dim
    xd = x.detach().double().cpu()
    lin = lambda m, t: t @ m.weight.detach().double().cpu().T + (0 if m.bias is None else m.bias.detach().double().cpu())  # noqa: E731,E501
    Q = lin(mod.q_proj, xd).view(B, L, Hh, Dh).transpose(1, 2)
    K = lin(mod.k_proj, xd).view(B, L, Hh, Dh).transpose(1, 2)
    V = lin(mod.v_proj, xd).view(B, L, Hh, Dh).transpose(1, 2)
    w = mod.raw_decay.detach().double().cpu().view(1, Hh, 1) + lin(mod.gate_proj, xd).transpose(1, 2)
    o, _ = oracle.attention(Q.numpy(), K.numpy(), V.numpy(), decay_w=w.numpy(),
                            attention_mask=None if mask is None else mask.cpu().numpy())
    o = torch.tensor(o)
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + 1e-5) * mod.head_norm.weight.detach().double().cpu()
    o = o.transpose(1, 2).reshape(B, L, Hh * Dh)
    return lin(mod.out_proj, o)


def test_linear_attention_module_matches_oracle():
    torch.manual_seed(2)
    mod = ag.SubQLinearAttention(hidden_size=64, num_heads=4).to(DEV)
    x = torch.randn(2, 75, 64, device=DEV)
    y, _ = mod(x)
    assert rel(y, _module_reference(mod, x).numpy()) < 1e-4
    y.pow(2).mean().backward()
    for name, p in mod.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name
    assert mod.raw_decay.grad.abs().sum() > 0


def test_module_cached_generation_matches_full_pass():
    """Prefill then token-by-token decode with use_cache equals one pass
    (reference tests/test_surgery_and_caching.py:168-214)."""
    torch.manual_seed(4)
    mod = ag.SubQLinearAttention(hidden_size=32, num_heads=2).to(DEV)
    x = torch.randn(1, 24, 32, device=DEV)
    full, _ = mod(x)
    y, st = mod(x[:, :16], use_cache=True)
    parts = [y]
    for t in range(16, 24):
        y, st = mod(x[:, t:t + 1], past_state=st, use_cache=True)
        parts.append(y)
    assert rel(torch.cat(parts, dim=1), full.detach().cpu().double().numpy()) < 1e-4


def test_module_padding_invariance():
    """Right padding under a mask leaves the live outputs unchanged
    (reference tests/test_surgery_and_caching.py:352-413)."""
    torch.manual_seed(5)
    mod = ag.SubQLinearAttention(hidden_size=32, num_heads=2).to(DEV)
    x = torch.randn(1, 20, 32, device=DEV)
    y, _ = mod(x)
    xp = torch.cat([x, torch.randn(1, 12, 32, device=DEV)], dim=1)
    mask = torch.zeros(1, 32, dtype=torch.bool, device=DEV)
    mask[:, :20] = True
    yp, _ = mod(xp, attention_mask=mask)
    assert rel(yp[:, :20], y.detach().cpu().double().numpy()) < 1e-4


class _ToyAttention(torch.nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.num_heads = h
        self.q_proj, self.k_proj, self.v_proj, self.out_proj = (torch.nn.Linear(d, d) for _ in range(4))

    def forward(self, x, attention_mask=None):
        return self.out_proj(self.v_proj(x)), None


class _ToyBlock(torch.nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.self_attn = _ToyAttention(d, h)
        self.mlp = torch.nn.Linear(d, d)

    def forward(self, x):
        a = self.self_attn(x)[0]
        return x + a + self.mlp(x)


def test_surgery_replaces_attention_and_trains():
    torch.manual_seed(6)
    model = torch.nn.Sequential(_ToyBlock(64, 4), _ToyBlock(64, 4)).to(DEV)
    from subq_audio.surgery import SubQBypassAttention, bypass_transformer_with_subq

    model, replaced = bypass_transformer_with_subq(model)
    assert len(replaced) == 2 and all(isinstance(b.self_attn, SubQBypassAttention) for b in model)
    x = torch.randn(2, 50, 64, device=DEV)
    loss = model(x).pow(2).mean()
    loss.backward()
    assert torch.isfinite(loss)
    assert model[0].self_attn.core.q_proj.weight.grad is not None
