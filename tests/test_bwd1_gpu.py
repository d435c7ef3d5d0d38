"""The one-pass backward (the forward hands over its per-chunk states,
per-token normalisers and output; the backward's work is split evenly over
the SMs) against the float64 oracle, through the C ABI.

Metric: max |x - ref| / max |ref| over the tensor; tolerance 2e-2 for the
16-bit inputs (the oracle runs on the rounded inputs in float64).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from subq_audio import _capi, ops

from test_scan_gpu import make_case, oracle_inputs, rel_err, to_dev

pytestmark = pytest.mark.gpu

CASES = [
    # B, H, Hkv, N, dtype, mask, state, normalize, reverse
    (1, 2, 2, 100, torch.bfloat16, False, False, True, False),
    (1, 2, 2, 129, torch.bfloat16, True, False, True, False),
    (2, 2, 2, 1000, torch.bfloat16, True, True, True, False),
    (2, 1, 1, 777, torch.float16, True, True, True, False),
    (1, 3, 3, 300, torch.bfloat16, False, True, False, False),  # engine form (no normaliser)
    (8, 8, 8, 512, torch.bfloat16, True, False, True, False),
    (2, 3, 3, 1000, torch.bfloat16, True, True, True, True),     # reverse time
    (4, 4, 2, 2048, torch.bfloat16, True, False, True, False),   # grouped K/V
    (3, 5, 5, 4100, torch.bfloat16, True, False, True, False),   # pieces across many CTAs
    (1, 1, 1, 20000, torch.bfloat16, False, False, True, False), # one sequence over every SM
]


def _run(q, k, v, do, m, st, normalize, reverse):
    args = [to_dev(x) for x in (q, k, v, do)]
    seg = ops.SegmentStates()
    o, _ = ops.scan_forward(*args[:3], mask=to_dev(m), normalize=normalize, state=to_dev(st), reverse=reverse,
                            segments=seg, path="tensorcore")
    assert seg.buf is not None and seg.out is o
    dq, dk, dv, _ = ops.scan_backward(*args, mask=to_dev(m), normalize=normalize, state=to_dev(st), reverse=reverse,
                                      segments=seg, path="tensorcore")
    launches = ops.last_launches()
    torch.cuda.synchronize()
    assert _capi.device_status() == _capi.SUBQ_OK
    return o, dq, dk, dv, launches


@pytest.mark.parametrize("case", CASES, ids=[f"b1_{i}" for i in range(len(CASES))])
def test_one_pass_backward_matches_oracle(case):
    B, H, Hkv, N, dtype, mask, state, normalize, reverse = case
    G = H // Hkv
    g = torch.Generator().manual_seed(7 + N + H)
    q = torch.randn(B, H, N, 64, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, 64, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, 64, generator=g).to(dtype)
    do = torch.randn(B, H, N, 64, generator=g).to(dtype)
    m = None
    if mask:
        lens = torch.randint(max(1, N // 2), N + 1, (B,), generator=g)
        lens[-1] = max(1, N // 3)
        m = torch.arange(N)[None, :] < lens[:, None]
    st = (torch.randn(B, H, 64, 64, generator=g) * 0.5, torch.rand(B, H, 64, generator=g) if normalize else None) \
        if state else None
    o, dq, dk, dv, launches = _run(q, k, v, do, m, st, normalize, reverse)
    assert launches == 2 + (2 if G > 1 else 0), "the one-pass backward (suffix sums + scan) ran"

    # the oracle: causal scan with K, V repeated per query head; reverse time on flipped copies
    tf = (lambda x: torch.flip(x, dims=[2])) if reverse else (lambda x: x)  # noqa: E731
    kr, vr = k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)
    m_f = (torch.flip(m, dims=[1]) if reverse else m) if m is not None else None
    qn, kn, vn, don, _, mn, S0, z0 = oracle_inputs(tf(q), tf(kr), tf(vr), tf(do), None, m_f, st, B, H, N)
    scale = 1.0 / math.sqrt(64) if normalize else 1.0
    ref_o = oracle.forward(qn, kn, vn, mask=mn, normalize=normalize, scale=scale, S0=S0, z0=z0)[0]
    rq, rk, rv, _ = oracle.backward(qn, kn, vn, don, mask=mn, normalize=normalize, scale=scale, S0=S0, z0=z0)
    back = (lambda a: a[:, :, ::-1]) if reverse else (lambda a: a)  # noqa: E731
    ref_o, rq, rk, rv = back(ref_o), back(rq), back(rk), back(rv)
    if G > 1:
        rk = rk.reshape(B, Hkv, G, N, 64).sum(axis=2)
        rv = rv.reshape(B, Hkv, G, N, 64).sum(axis=2)
    assert rel_err(o, ref_o) < 2e-2, "o"
    assert rel_err(dq, rq) < 2e-2, "dq"
    assert rel_err(dk, rk) < 2e-2, "dk"
    assert rel_err(dv, rv) < 2e-2, "dv"
    if m is not None:  # gradients of padded tokens are exactly zero
        dead = ~m.cuda()
        for t in (dq, dk if G == 1 else None, dv if G == 1 else None):
            if t is not None:
                assert (t.float().abs().sum(-1)[dead[:, None, :].expand(B, t.shape[1], N)] == 0).all()


def test_one_pass_single_token_gradients_vanish():
    """N = 1: the normalised output of a single token is its value, so dq and
    dk are zero (the reference's float64 gradients are ~1e-17); the one-pass
    backward returns bf16 rounding noise there, far below dv."""
    q, k, v, do = (torch.randn(2, 3, 1, 64, dtype=torch.bfloat16) for _ in range(4))
    o, dq, dk, dv, launches = _run(q, k, v, do, None, None, True, False)
    assert launches == 2
    torch.testing.assert_close(o.float().cpu(), v.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dv.float().cpu(), do.float(), rtol=2e-2, atol=2e-2)
    assert dq.float().abs().max() < 1e-2 * do.float().abs().max()
    assert dk.float().abs().max() < 1e-2 * do.float().abs().max()


def test_one_pass_equals_recomputing_backward():
    """Same inputs through the one-pass backward and through the backward
    that recomputes the forward (no handover): the two agree to bf16 rounding."""
    B, H, N = 2, 4, 3000
    q, k, v, do, _, m, st = make_case(B, H, N, 64, 64, torch.bfloat16, seed=5, mask=True, state=True)
    args = [to_dev(x) for x in (q, k, v, do)]
    seg = ops.SegmentStates()
    ops.scan_forward(*args[:3], mask=to_dev(m), state=to_dev(st), segments=seg)
    one = ops.scan_backward(*args, mask=to_dev(m), state=to_dev(st), segments=seg)
    assert ops.last_launches() == 2
    rec = ops.scan_backward(*args, mask=to_dev(m), state=to_dev(st))
    assert ops.last_launches() == 1
    torch.cuda.synchronize()
    for a, b in zip(one[:3], rec[:3]):
        assert rel_err(a, b.double().cpu().numpy()) < 1e-2


def test_handover_from_another_call_is_reported():
    """A backward given the handover of a forward of another shape writes no
    gradient and reports SUBQ_ERR_STATE through the device status word."""
    B, H = 1, 2
    a = [torch.randn(B, H, 256, 64, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    seg = ops.SegmentStates()
    ops.scan_forward(*a, segments=seg)
    b = [torch.randn(B, H, 384, 64, device="cuda", dtype=torch.bfloat16) for _ in range(5)]
    torch.cuda.synchronize()
    assert _capi.device_status() == _capi.SUBQ_OK
    ops.scan_backward(*b[:4], segments=seg, forward_out=b[4])
    assert ops.last_launches() == 2
    assert _capi.device_status() == _capi.SUBQ_ERR_STATE
    assert _capi.device_status() == _capi.SUBQ_OK  # read and cleared


_FULL = {}


def _full_size_case():
    """The headline workload with the benchmark's own inputs: B=8, H=8, N=8192,
    d=64 bf16, key-padding lengths U[N/2, N] (inputs seed 1234, lengths seed
    4321, as bench.py rank 0 draws them), and the float64 oracle's forward and
    backward on them (computed once for the tests below)."""
    if not _FULL:
        B, H, N, D = 8, 8, 8192, 64
        g = torch.Generator(device="cpu").manual_seed(1234)
        q, k, v, do = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16) for _ in range(4))
        lens = torch.randint(N // 2, N + 1, (B,), generator=torch.Generator(device="cpu").manual_seed(4321))
        m = torch.arange(N)[None, :] < lens[:, None]
        f = lambda t: t.double().numpy()  # noqa: E731
        mn = np.broadcast_to(m.double().numpy()[:, None, :], (B, H, N))
        ref_o = oracle.forward(f(q), f(k), f(v), mask=mn, normalize=True, scale=1 / math.sqrt(D))[0]
        rq, rk, rv, _ = oracle.backward(f(q), f(k), f(v), f(do), mask=mn, normalize=True, scale=1 / math.sqrt(D))
        _FULL.update(inputs=(q, k, v, do, m), ref=(ref_o, rq, rk, rv))
    return _FULL["inputs"], _FULL["ref"]


def test_full_size_headline_workload_matches_oracle():
    """Forward + one-pass backward at the headline size, as the benchmark's
    step runs them (the forward hands its chunk states to the backward)."""
    (q, k, v, do, m), (ref_o, rq, rk, rv) = _full_size_case()
    o, dq, dk, dv, launches = _run(q, k, v, do, m, None, True, False)
    assert launches == 2
    for name, got, ref in (("o", o, ref_o), ("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert rel_err(got, ref) < 2e-2, name


def test_full_size_through_reference_function():
    """The same inputs through SubQAttentionFunction (the reference's autograd
    entry point, autograd.py:547-660): its forward on the tensor cores and its
    backward, which saves only q, k, v, w and recomputes the forward states."""
    from subq_audio.autograd import SubQAttentionFunction

    (q, k, v, do, m), (ref_o, rq, rk, rv) = _full_size_case()
    qd, kd, vd = (x.cuda().requires_grad_(True) for x in (q, k, v))
    o = SubQAttentionFunction.apply(qd, kd, vd, None, 64, m.cuda(), True)
    o.backward(do.cuda())
    torch.cuda.synchronize()
    assert _capi.device_status() == _capi.SUBQ_OK
    assert ops.last_path() == "tensorcore"
    for name, got, ref in (("o", o.detach(), ref_o), ("dq", qd.grad, rq), ("dk", kd.grad, rk), ("dv", vd.grad, rv)):
        assert rel_err(got, ref) < 2e-2, name
