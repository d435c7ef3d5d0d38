"""subq_bwd_noalloc (the backward with the library's static scratch), called
through the C ABI and compared with subq_bwd on the same inputs.

The file name sorts last, so in a full run it executes after every other
test; it also passes alone in a fresh process.
"""
import math

import pytest
import torch

from subq_audio import _capi, ops

pytestmark = pytest.mark.gpu


def _case(B, H, N, d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, N, d, generator=g).to(dtype).cuda() for _ in range(4))
    lens = torch.randint(N // 2, N + 1, (B,), generator=g)
    mask = (torch.arange(N)[None, :] < lens[:, None]).cuda()
    return q, k, v, do, mask


def _noalloc_args(q, k, v, do, mask, log_gamma=None, seg=None, keep=None):
    B, H, N, d = q.shape
    keep = [] if keep is None else keep
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    a = _capi.BwdArgs()
    a.desc = ops._desc(q, v, log_gamma, mask, True, None, 1e-5, False, "auto", keep)
    dlg = None
    if log_gamma is not None:
        dlg = torch.empty(B, H, N, dtype=torch.float32, device=q.device)
        a.dlog_gamma = dlg.data_ptr()
    a.q, a.k, a.v, a.dout = ops._t4(q), ops._t4(k), ops._t4(v), ops._t4(do)
    a.dq, a.dk, a.dv = ops._t4(dq), ops._t4(dk), ops._t4(dv)
    if seg is not None:  # the forward's handover and output: the one-pass backward
        a.segment_states = seg.buf.data_ptr()
        a.out = ops._t4(seg.out)
    a.stream = torch.cuda.current_stream().cuda_stream
    a.workspace, a.workspace_bytes = None, 0
    return a, (dq, dk, dv) if log_gamma is None else (dq, dk, dv, dlg)


def _noalloc_backward(q, k, v, do, mask, log_gamma=None, seg=None):
    """One subq_bwd_noalloc call: the caller provides inputs and outputs only
    (with a per-token decay also the d log(gamma) output, returned last)."""
    a, outs = _noalloc_args(q, k, v, do, mask, log_gamma, seg)
    _capi.bwd_noalloc(a)
    return outs


@pytest.mark.parametrize("dtype,d", [(torch.bfloat16, 64), (torch.float32, 16)])
def test_noalloc_backward_equals_subq_bwd_twice(dtype, d):
    q, k, v, do, mask = _case(2, 4, 1000, d, dtype, seed=11 + d)
    ref = ops.scan_backward(q, k, v, do, mask=mask)[:3]
    path = ops.last_path()
    for _ in range(2):  # the static scratch is reused by back-to-back calls
        got = _noalloc_backward(q, k, v, do, mask)
        torch.cuda.synchronize()
        assert ops.last_path() == path
        for x, y in zip(got, ref):
            assert torch.equal(x, y)


def test_noalloc_backward_with_decay_equals_subq_bwd_twice():
    """Per-token decay on the tensor-core path keeps its per-sequence fallback
    flags in the same static scratch (cleared by each call); one sequence
    decays strongly enough to take the exact fallback."""
    q, k, v, do, mask = _case(2, 3, 1200, 64, torch.bfloat16, seed=29)
    g = torch.Generator().manual_seed(30)
    lg = -torch.nn.functional.softplus(-(torch.randn(2, 3, 1200, generator=g) + 3.0))
    lg[1, 0, 200:700] = math.log(0.1)
    lg = lg.cuda()
    ref = ops.scan_backward(q, k, v, do, mask=mask, log_gamma=lg, need_dlog_gamma=True)
    assert ops.last_path() == "tensorcore"
    for _ in range(2):
        got = _noalloc_backward(q, k, v, do, mask, log_gamma=lg)
        torch.cuda.synchronize()
        assert ops.last_path() == "tensorcore"
        for x, y in zip(got, ref):
            assert torch.equal(x, y)


def test_noalloc_backward_rejects_calls_above_its_scratch():
    # 1,048,577 token-heads on the tensor-core path: one above the 8 MiB scratch
    N = (8 << 20) // 8 + 1
    q = torch.zeros(1, 1, N, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_capi.SubqError) as err:
        _noalloc_backward(q, q, q, q, None)
    assert err.value.code == _capi.SUBQ_ERR_WORKSPACE
    assert "8 MiB" in str(err.value)
    # exactly at capacity the call runs
    n_ok = (8 << 20) // 8 // 1024
    q2, k2, v2, do2, _ = _case(1, 1024, n_ok, 64, torch.bfloat16, seed=5)
    got = _noalloc_backward(q2, k2, v2, do2, None)
    ref = ops.scan_backward(q2, k2, v2, do2)[:3]
    for x, y in zip(got, ref):
        assert torch.equal(x, y)
    assert math.isfinite(got[0].float().abs().max().item())


def test_noalloc_backward_grouped_kv_equals_subq_bwd_twice():
    """Grouped K/V: the static scratch also holds dK, dV per query head until
    the group sums read them back (a second kernel reading the scratch)."""
    g = torch.Generator().manual_seed(41)
    B, H, Hkv, N = 2, 4, 2, 900
    q, do = (torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).cuda() for _ in range(2))
    k, v = (torch.randn(B, Hkv, N, 64, generator=g).to(torch.bfloat16).cuda() for _ in range(2))
    mask = (torch.arange(N)[None, :] < torch.tensor([N, 600])[:, None]).cuda()
    ref = ops.scan_backward(q, k, v, do, mask=mask)[:3]
    assert ops.last_path() == "tensorcore"
    for _ in range(2):
        got = _noalloc_backward(q, k, v, do, mask)
        torch.cuda.synchronize()
        for x, y in zip(got, ref):
            assert torch.equal(x, y)
    # one token above what fits: the grouped buffers make each token-head 264 bytes
    n_big = 64
    while True:
        qb = torch.zeros(1, H, n_big, 64, dtype=torch.bfloat16, device="cuda")
        kb = torch.zeros(1, Hkv, n_big, 64, dtype=torch.bfloat16, device="cuda")
        a, _ = _noalloc_args(qb, kb, kb, qb, None)
        if _capi.bwd_workspace_bytes(a) > (8 << 20):
            break
        n_big *= 2
    with pytest.raises(_capi.SubqError) as err:
        _capi.bwd_noalloc(a)
    assert err.value.code == _capi.SUBQ_ERR_WORKSPACE


def test_noalloc_one_pass_backward_equals_subq_bwd_twice():
    """With the forward's handover and output the backward runs in one pass;
    its scratch (the adjoint sums of the CTAs' first pieces) is then a fixed
    size, whatever the sequence length."""
    q, k, v, do, mask = _case(3, 4, 5000, 64, torch.bfloat16, seed=53)
    seg = ops.SegmentStates()
    ops.scan_forward(q, k, v, mask=mask, segments=seg)
    ref = ops.scan_backward(q, k, v, do, mask=mask, segments=seg)[:3]
    assert ops.last_launches() == 2  # the one-pass backward
    for _ in range(2):
        got = _noalloc_backward(q, k, v, do, mask, seg=seg)
        torch.cuda.synchronize()
        assert ops.last_launches() == 2
        for x, y in zip(got, ref):
            assert torch.equal(x, y)
