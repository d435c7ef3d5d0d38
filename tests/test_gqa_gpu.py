"""Grouped K/V (GQA / MQA) in the kernels: K and V with kv_heads < heads,
query head h reading K/V head h // (heads // kv_heads), the backward summing
dK, dV over each group. Checked against the float64 oracle on K and V
repeated per query head (the reference's repeat_interleave,
python/subq_audio/autograd.py:746-748) with the oracle's dK, dV summed per
group, on the tensor-core and exact paths.
"""
import pytest
import torch

import oracle
from subq_audio import ops

from test_scan_gpu import oracle_inputs, rel_err, to_dev

pytestmark = pytest.mark.gpu


def _case(B, H, Hkv, N, dtype, seed, decay, mask, state):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, 64, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, 64, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, 64, generator=g).to(dtype)
    do = torch.randn(B, H, N, 64, generator=g).to(dtype)
    lg = (-torch.nn.functional.softplus(-(torch.randn(B, H, N, generator=g) + 3.0))) if decay else None
    m = None
    if mask:
        lens = torch.randint(N // 2, N + 1, (B,), generator=g)
        m = torch.arange(N)[None, :] < lens[:, None]
    st = (torch.randn(B, H, 64, 64, generator=g) * 0.5, torch.rand(B, H, 64, generator=g)) if state else None
    return q, k, v, do, lg, m, st


CASES = [
    # B, H, Hkv, N, dtype, decay, mask, state, path
    (2, 8, 2, 700, torch.bfloat16, False, True, False, "tensorcore"),
    (1, 4, 1, 1000, torch.bfloat16, True, False, True, "tensorcore"),   # multi-query
    (2, 6, 3, 300, torch.float16, False, False, True, "tensorcore"),
    (2, 4, 2, 200, torch.float32, True, True, True, "exact"),
]


@pytest.mark.parametrize("case", CASES, ids=[f"g{i}" for i in range(len(CASES))])
def test_grouped_kv_matches_oracle_on_repeated_heads(case):
    B, H, Hkv, N, dtype, decay, mask, state, path = case
    G = H // Hkv
    q, k, v, do, lg, m, st = _case(B, H, Hkv, N, dtype, 7 + N, decay, mask, state)
    kr, vr = k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)
    qn, kn, vn, don, lgn, mn, S0, z0 = oracle_inputs(q, kr, vr, do, lg, m, st, B, H, N)
    ref_o, ref_S, _, _ = oracle.forward(qn, kn, vn, log_gamma=lgn, mask=mn, normalize=True, scale=0.125, S0=S0,
                                        z0=z0)
    rq, rk, rv, rdlg = oracle.backward(qn, kn, vn, don, log_gamma=lgn, mask=mn, normalize=True, scale=0.125,
                                       S0=S0, z0=z0)
    rk = rk.reshape(B, Hkv, G, N, 64).sum(axis=2)
    rv = rv.reshape(B, Hkv, G, N, 64).sum(axis=2)
    o, (S, _) = ops.scan_forward(to_dev(q), to_dev(k), to_dev(v), log_gamma=to_dev(lg), mask=to_dev(m),
                                 state=to_dev(st), return_state=True, path=path)
    dq, dk, dv, dlg = ops.scan_backward(to_dev(q), to_dev(k), to_dev(v), to_dev(do), log_gamma=to_dev(lg),
                                        mask=to_dev(m), state=to_dev(st), need_dlog_gamma=decay, path=path)
    torch.cuda.synchronize()
    assert ops.last_path() == path
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert tuple(dk.shape) == (B, Hkv, N, 64) and tuple(dv.shape) == (B, Hkv, N, 64)
    assert rel_err(o, ref_o) < tol
    assert rel_err(S, ref_S) < max(tol, 1e-5)
    assert rel_err(dq, rq) < tol, "dq"
    assert rel_err(dk, rk) < tol, "dk"
    assert rel_err(dv, rv) < tol, "dv"
    if decay:
        assert rel_err(dlg, rdlg) < max(tol, 2e-4), "dlog_gamma"


def test_gqa_module_equals_repeated_heads():
    """SubQLinearAttention with num_key_value_heads < num_heads: outputs and
    parameter gradients through the grouped kernels equal those of the same
    computation with K and V repeated per query head."""
    from subq_audio.autograd import SubQLinearAttention, chunkwise_flash_linear_attention

    torch.manual_seed(3)
    mod = SubQLinearAttention(512, num_heads=8, num_key_value_heads=2).cuda()  # head_dim 64
    x = torch.randn(2, 600, 512, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y, _ = mod(x)
    assert ops.last_path() == "tensorcore"
    y.float().square().mean().backward()
    grads = {n: p.grad.detach().clone() for n, p in mod.named_parameters()}
    mod.zero_grad()

    def repeated(hidden):  # the reference's formulation: K, V repeated before the scan
        B, L, _ = hidden.shape
        Q = mod.q_proj(hidden).view(B, L, 8, 64).transpose(1, 2)
        K = mod.k_proj(hidden).view(B, L, 2, 64).transpose(1, 2).repeat_interleave(4, dim=1)
        V = mod.v_proj(hidden).view(B, L, 2, 64).transpose(1, 2).repeat_interleave(4, dim=1)
        w = mod.raw_decay.view(1, 8, 1) + mod.gate_proj(hidden).transpose(1, 2)
        out, _ = chunkwise_flash_linear_attention(Q, K, V, w)
        out = mod.head_norm(out).transpose(1, 2).reshape(B, L, 512)
        return mod.out_proj(out)

    with torch.autocast("cuda", dtype=torch.bfloat16):
        y2 = repeated(x)
    y2.float().square().mean().backward()
    assert rel_err(y, y2.detach().double().cpu().numpy()) < 1e-2
    for n, p in mod.named_parameters():
        assert rel_err(grads[n], p.grad.double().cpu().numpy()) < 3e-2, n
