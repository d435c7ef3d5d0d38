"""Reverse-time scans (the second direction of the bidirectional scan) on the
kernels, against the float64 oracle run on time-flipped inputs with its
outputs and gradients flipped back - the reference's own construction
(python/subq_audio/autograd.py:407-433 and :612-640 flip q, k, v, dO, the
mask and a per-token decay, scan causally and flip the results).
"""
import math

import pytest
import torch

import oracle
from subq_audio import ops

from test_scan_gpu import oracle_inputs, rel_err, to_dev

pytestmark = pytest.mark.gpu

CASES = [
    # B, H, Hkv, N, dtype, decay, mask, state, path
    (2, 2, 2, 1000, torch.bfloat16, None, True, False, "tensorcore"),
    (1, 1, 1, 3000, torch.bfloat16, "token", False, True, "tensorcore"),  # segments over a cluster
    (2, 4, 2, 700, torch.bfloat16, "token", True, False, "tensorcore"),   # grouped K/V
    (2, 2, 2, 777, torch.float16, None, True, True, "tensorcore"),
    (1, 2, 2, 1100, torch.bfloat16, "strong", True, False, "tensorcore"),  # exact fallback per sequence
    (2, 3, 3, 200, torch.float32, "token", True, True, "exact"),
    (1, 2, 1, 130, torch.float64, "head", False, False, "exact"),
]


@pytest.mark.parametrize("case", CASES, ids=[f"r{i}" for i in range(len(CASES))])
def test_reverse_scan_matches_oracle_on_flipped_inputs(case):
    B, H, Hkv, N, dtype, decay, mask, state, path = case
    G = H // Hkv
    g = torch.Generator().manual_seed(N + H)
    q = torch.randn(B, H, N, 64, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, 64, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, 64, generator=g).to(dtype)
    do = torch.randn(B, H, N, 64, generator=g).to(dtype)
    lg = None
    if decay in ("token", "strong"):
        lg = -torch.nn.functional.softplus(-(torch.randn(B, H, N, generator=g) + 3.0))
        if decay == "strong":
            lg[0, :, 300:800] = math.log(0.1)
    elif decay == "head":
        lg = -torch.nn.functional.softplus(-torch.linspace(1.0, 4.0, H))
    m = None
    if mask:
        lens = torch.randint(N // 2, N + 1, (B,), generator=g)
        m = torch.arange(N)[None, :] < lens[:, None]
    st = (torch.randn(B, H, 64, 64, generator=g) * 0.5, torch.rand(B, H, 64, generator=g)) if state else None

    # the oracle: a causal scan of the time-flipped sequence (K, V repeated per query head)
    tf = lambda x: torch.flip(x, dims=[2])  # noqa: E731  [B, H, N, *]
    kr, vr = k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)
    lg_f = torch.flip(lg, dims=[2]) if (lg is not None and lg.dim() == 3) else lg
    m_f = torch.flip(m, dims=[1]) if m is not None else None
    qn, kn, vn, don, lgn, mn, S0, z0 = oracle_inputs(tf(q), tf(kr), tf(vr), tf(do), lg_f, m_f, st, B, H, N)
    ref_o, ref_S, ref_z, _ = oracle.forward(qn, kn, vn, log_gamma=lgn, mask=mn, normalize=True, scale=0.125, S0=S0,
                                            z0=z0)
    rq, rk, rv, rdlg = oracle.backward(qn, kn, vn, don, log_gamma=lgn, mask=mn, normalize=True, scale=0.125, S0=S0,
                                       z0=z0)
    fl = lambda a: a[..., ::-1, :] if a.ndim == 4 else a[..., ::-1]  # noqa: E731  flip time back
    ref_o, rq, rdlg = fl(ref_o), fl(rq), fl(rdlg)
    rk = fl(rk).reshape(B, Hkv, G, N, 64).sum(axis=2)
    rv = fl(rv).reshape(B, Hkv, G, N, 64).sum(axis=2)

    o, (S, z) = ops.scan_forward(to_dev(q), to_dev(k), to_dev(v), log_gamma=to_dev(lg), mask=to_dev(m),
                                 state=to_dev(st), return_state=True, path=path, reverse=True)
    dq, dk, dv, dlg = ops.scan_backward(to_dev(q), to_dev(k), to_dev(v), to_dev(do), log_gamma=to_dev(lg),
                                        mask=to_dev(m), state=to_dev(st), need_dlog_gamma=lg is not None,
                                        path=path, reverse=True)
    torch.cuda.synchronize()
    assert ops.last_path() == path
    tol = {torch.float32: 1e-4, torch.float64: 1e-10}.get(dtype, 2e-2)
    assert rel_err(o, ref_o) < tol, "o"
    assert rel_err(S, ref_S) < max(tol, 1e-5), "S"
    assert rel_err(z, ref_z) < max(tol, 1e-5), "z"
    assert rel_err(dq, rq) < tol, "dq"
    assert rel_err(dk, rk) < tol, "dk"
    assert rel_err(dv, rv) < tol, "dv"
    if lg is not None:
        assert rel_err(dlg, rdlg) < max(tol, 2e-4), "dlog_gamma"


def test_bidirectional_function_uses_no_flipped_copies():
    """SubQAttentionFunction with is_causal=False (bf16, decay, mask) runs both
    directions on the tensor-core kernels and matches the float64 oracle's
    two-direction combination."""
    from subq_audio.autograd import SubQAttentionFunction

    B, H, N = 2, 4, 900
    g = torch.Generator().manual_seed(5)
    q, k, v, do = (torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16) for _ in range(4))
    w = torch.randn(B, H, N, generator=g) + 3.0
    lens = torch.randint(N // 2, N + 1, (B,), generator=g)
    am = (torch.arange(N)[None, :] < lens[:, None]).long()
    qd, kd, vd = (x.cuda().requires_grad_() for x in (q, k, v))
    wd = w.cuda().requires_grad_()
    out = SubQAttentionFunction.apply(qd, kd, vd, wd, 64, am.cuda(), False)
    out.backward(do.cuda())
    assert ops.last_path() == "tensorcore"
    # oracle: forward direction + flipped-time direction - the masked diagonal v
    lg = -torch.nn.functional.softplus(-w)
    mf = am.bool()
    qn, kn, vn, don, lgn, mn, _, _ = oracle_inputs(q, k, v, do, lg, mf, None, B, H, N)
    o1 = oracle.forward(qn, kn, vn, log_gamma=lgn, mask=mn, normalize=True, scale=0.125)[0]
    tf = lambda x: torch.flip(x, dims=[2])  # noqa: E731
    qn2, kn2, vn2, _, lgn2, mn2, _, _ = oracle_inputs(tf(q), tf(k), tf(v), tf(do), torch.flip(lg, dims=[2]),
                                                      torch.flip(mf, dims=[1]), None, B, H, N)
    o2 = oracle.forward(qn2, kn2, vn2, log_gamma=lgn2, mask=mn2, normalize=True, scale=0.125)[0][..., ::-1, :]
    m4 = mn[..., None]
    ref = (o1 + o2 - vn * m4) * m4
    assert rel_err(out, ref) < 2e-2
    assert all(torch.isfinite(t.grad).all() for t in (qd, kd, vd, wd))
