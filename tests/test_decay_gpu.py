"""Per-token decay on the tensor-core path (bf16), through the C ABI, against
the float64 oracle.

The kernels factor the intra-chunk decay through each chunk's midpoint and
hand sequences whose decay leaves that factorisation's range to the exact
kernel; both halves are covered here (mild decay stays on the tensor cores,
strong decay falls back per sequence), with masks, carried state, the
segment split of long sequences over a cluster, and every decay mode.
Tolerance: 2e-2 of max |ref| (bf16 inputs; the oracle runs on the
bf16-rounded inputs in float64).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from subq_audio import ops

from test_scan_gpu import make_case, oracle_inputs, rel_err, to_dev

pytestmark = pytest.mark.gpu


def token_log_gamma(B, H, N, seed, center=3.0, spread=1.0):
    g = torch.Generator().manual_seed(seed)
    return -torch.nn.functional.softplus(-(torch.randn(B, H, N, generator=g) * spread + center))


FWD_CASES = [
    # B, H, N, decay, mask, state, normalize
    (1, 1, 1, "token", False, False, True),
    (1, 1, 100, "token", False, False, True),
    (1, 2, 128, "token", True, False, True),
    (2, 2, 1000, "token", True, True, True),
    (1, 1, 3000, "token", False, True, True),   # long single sequence: segments over a cluster
    (2, 1, 2600, "token", True, True, True),
    (1, 3, 300, "token", False, True, False),   # unnormalised form
    (2, 3, 700, "head", True, False, True),
    (1, 2, 900, "scalar", False, True, True),
    (8, 8, 512, "token", True, False, True),
]


@pytest.mark.parametrize("case", FWD_CASES, ids=[f"f{i}" for i in range(len(FWD_CASES))])
def test_decayed_tensorcore_forward_matches_oracle(case):
    B, H, N, decay, mask, state, normalize = case
    q, k, v, do, lg, m, st = make_case(B, H, N, 64, 64, torch.bfloat16, seed=303 + N + H, decay=decay,
                                       mask=mask, state=state, normalize=normalize)
    qn, kn, vn, _, lgn, mn, S0, z0 = oracle_inputs(q, k, v, do, lg, m, st, B, H, N)
    scale = 0.125 if normalize else 1.0
    ref_o, ref_S, ref_z, _ = oracle.forward(qn, kn, vn, log_gamma=lgn, mask=mn, normalize=normalize,
                                            scale=scale, S0=S0, z0=z0)
    o, (S, z) = ops.scan_forward(to_dev(q), to_dev(k), to_dev(v), log_gamma=to_dev(lg), mask=to_dev(m),
                                 normalize=normalize, state=to_dev(st), return_state=True, path="tensorcore")
    torch.cuda.synchronize()
    assert ops.last_path() == "tensorcore"
    assert rel_err(o, ref_o) < 2e-2
    assert rel_err(S, ref_S) < 2e-2
    if normalize:
        assert rel_err(z, ref_z) < 2e-2


def test_decay_outside_the_factorised_range_falls_back_per_sequence():
    """Sequence 0 decays mildly, sequence 1 strongly (gamma ~ 0.1 on a stretch:
    far outside the midpoint factorisation), sequence 2 has one reset token
    (gamma ~ 1e-30) per chunk; all three in one call."""
    B, H, N = 3, 2, 1100
    q, k, v, do, _, m, st = make_case(B, H, N, 64, 64, torch.bfloat16, seed=5, mask=True, state=True)
    lg = token_log_gamma(B, H, N, seed=6)
    lg[1, :, 200:900] = math.log(0.1)
    lg[2, :, 64::128] = -69.0
    qn, kn, vn, _, lgn, mn, S0, z0 = oracle_inputs(q, k, v, do, lg, m, st, B, H, N)
    ref_o, ref_S, ref_z, _ = oracle.forward(qn, kn, vn, log_gamma=lgn, mask=mn, normalize=True, scale=0.125,
                                            S0=S0, z0=z0)
    o, (S, z) = ops.scan_forward(to_dev(q), to_dev(k), to_dev(v), log_gamma=to_dev(lg), mask=to_dev(m),
                                 state=to_dev(st), return_state=True, path="tensorcore")
    torch.cuda.synchronize()
    for b in range(B):
        assert rel_err(o[b], ref_o[b]) < 2e-2, b
        assert rel_err(S[b], ref_S[b]) < 2e-2, b
        assert rel_err(z[b], ref_z[b]) < 2e-2, b


def test_decayed_streaming_equals_single_pass():
    """Carried (S, z) across calls of unequal length reproduces one pass."""
    B, H, N = 1, 2, 1500
    q, k, v, _, _, _, _ = make_case(B, H, N, 64, 64, torch.bfloat16, seed=9)
    lg = token_log_gamma(B, H, N, seed=10).cuda()
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    full, (S_full, z_full) = ops.scan_forward(q, k, v, log_gamma=lg, return_state=True)
    outs, st = [], None
    for a, b in ((0, 333), (333, 900), (900, 1500)):
        o, st = ops.scan_forward(q[:, :, a:b], k[:, :, a:b], v[:, :, a:b], log_gamma=lg[:, :, a:b].contiguous(),
                                 state=st, return_state=True)
        outs.append(o)
    torch.cuda.synchronize()
    assert ops.last_path() == "tensorcore"
    ref = full.double().cpu().numpy()
    assert rel_err(torch.cat(outs, dim=2), ref) < 2e-2
    # the chunk grid differs between the two runs: bf16 operand rounding only
    assert rel_err(st[0], S_full.double().cpu().numpy()) < 2e-2
    assert rel_err(st[1], z_full.double().cpu().numpy()) < 2e-2


def test_decayed_forward_matches_exact_path():
    """The tensor-core and exact kernels agree on the decayed scan at a size
    the oracle would take long on (B=2, H=4, N=8192)."""
    B, H, N = 2, 4, 8192
    q, k, v, _, _, m, _ = make_case(B, H, N, 64, 64, torch.bfloat16, seed=12, mask=True)
    lg = token_log_gamma(B, H, N, seed=13).cuda()
    q, k, v, m = q.cuda(), k.cuda(), v.cuda(), m.cuda()
    o_tc, (S_tc, _) = ops.scan_forward(q, k, v, log_gamma=lg, mask=m, return_state=True, path="tensorcore")
    o_ex, (S_ex, _) = ops.scan_forward(q, k, v, log_gamma=lg, mask=m, return_state=True, path="exact")
    torch.cuda.synchronize()
    assert rel_err(o_tc, o_ex.double().cpu().numpy()) < 2e-2
    assert rel_err(S_tc, S_ex.double().cpu().numpy()) < 2e-2


BWD_CASES = [
    # B, H, N, decay, mask, state, normalize
    (1, 1, 100, "token", False, False, True),
    (1, 2, 128, "token", True, False, True),
    (2, 2, 1000, "token", True, True, True),
    (1, 1, 3000, "token", False, True, True),   # segments over a cluster: suffix and d log(gamma) carries
    (2, 1, 2600, "token", True, True, True),
    (1, 3, 300, "token", False, True, False),
    (2, 3, 700, "head", True, False, True),
    (1, 2, 900, "scalar", False, True, True),
    (8, 8, 512, "token", True, False, True),
]


@pytest.mark.parametrize("case", BWD_CASES, ids=[f"b{i}" for i in range(len(BWD_CASES))])
def test_decayed_tensorcore_backward_matches_oracle(case):
    B, H, N, decay, mask, state, normalize = case
    q, k, v, do, lg, m, st = make_case(B, H, N, 64, 64, torch.bfloat16, seed=404 + N + H, decay=decay,
                                       mask=mask, state=state, normalize=normalize)
    if decay == "token":  # a per-token spread wide enough that d log(gamma) varies along the sequence
        lg = token_log_gamma(B, H, N, seed=405 + N, center=2.5, spread=1.5)
    qn, kn, vn, don, lgn, mn, S0, z0 = oracle_inputs(q, k, v, do, lg, m, st, B, H, N)
    scale = 0.125 if normalize else 1.0
    rq, rk, rv, rdlg = oracle.backward(qn, kn, vn, don, log_gamma=lgn, mask=mn, normalize=normalize, scale=scale,
                                       S0=S0, z0=z0)
    dq, dk, dv, dlg = ops.scan_backward(to_dev(q), to_dev(k), to_dev(v), to_dev(do), log_gamma=to_dev(lg),
                                        mask=to_dev(m), normalize=normalize, state=to_dev(st),
                                        need_dlog_gamma=True, path="tensorcore")
    torch.cuda.synchronize()
    assert ops.last_path() == "tensorcore"
    assert rel_err(dq, rq) < 2e-2, "dq"
    assert rel_err(dk, rk) < 2e-2, "dk"
    assert rel_err(dv, rv) < 2e-2, "dv"
    assert rel_err(dlg, rdlg) < 2e-2, "dlog_gamma"
    # without the d log(gamma) output the gradients are the same
    dq2, dk2, dv2, _ = ops.scan_backward(to_dev(q), to_dev(k), to_dev(v), to_dev(do), log_gamma=to_dev(lg),
                                         mask=to_dev(m), normalize=normalize, state=to_dev(st), path="tensorcore")
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)


def test_decayed_backward_outside_the_range_falls_back_per_sequence():
    B, H, N = 3, 2, 1100
    q, k, v, do, _, m, st = make_case(B, H, N, 64, 64, torch.bfloat16, seed=15, mask=True, state=True)
    lg = token_log_gamma(B, H, N, seed=16)
    lg[1, :, 200:900] = math.log(0.1)
    lg[2, :, 64::128] = -69.0
    qn, kn, vn, don, lgn, mn, S0, z0 = oracle_inputs(q, k, v, do, lg, m, st, B, H, N)
    rq, rk, rv, rdlg = oracle.backward(qn, kn, vn, don, log_gamma=lgn, mask=mn, normalize=True, scale=0.125,
                                       S0=S0, z0=z0)
    dq, dk, dv, dlg = ops.scan_backward(to_dev(q), to_dev(k), to_dev(v), to_dev(do), log_gamma=to_dev(lg),
                                        mask=to_dev(m), state=to_dev(st), need_dlog_gamma=True, path="tensorcore")
    torch.cuda.synchronize()
    for b in range(B):
        assert rel_err(dq[b], rq[b]) < 2e-2, ("dq", b)
        assert rel_err(dk[b], rk[b]) < 2e-2, ("dk", b)
        assert rel_err(dv[b], rv[b]) < 2e-2, ("dv", b)
        assert rel_err(dlg[b], rdlg[b]) < 2e-2, ("dlg", b)


def test_decayed_backward_matches_exact_path_at_length():
    """B=2, H=4, N=8192 with a key-padding mask: tensor-core and exact kernels
    agree on dq, dk, dv and d log(gamma)."""
    B, H, N = 2, 4, 8192
    q, k, v, do, _, m, _ = make_case(B, H, N, 64, 64, torch.bfloat16, seed=22, mask=True)
    lg = token_log_gamma(B, H, N, seed=23).cuda()
    args = [t.cuda() for t in (q, k, v, do)]
    got = ops.scan_backward(*args, log_gamma=lg, mask=m.cuda(), need_dlog_gamma=True, path="tensorcore")
    ref = ops.scan_backward(*args, log_gamma=lg, mask=m.cuda(), need_dlog_gamma=True, path="exact")
    torch.cuda.synchronize()
    for name, x, y in zip(("dq", "dk", "dv", "dlg"), got, ref):
        assert rel_err(x, y.double().cpu().numpy()) < 2e-2, name


def test_gated_module_runs_on_tensor_cores_and_matches_exact():
    """SubQLinearAttention with data-dependent gating (per-token decay) in
    bf16: forward and parameter gradients through the tensor-core kernels
    agree with the same module on the exact kernels (float32 copies)."""
    from subq_audio.autograd import SubQLinearAttention
    torch.manual_seed(0)
    mod = SubQLinearAttention(256, num_heads=4).cuda()
    x = torch.randn(2, 1500, 256, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y, _ = mod(x)
    assert ops.last_path() == "tensorcore"
    y.float().square().mean().backward()
    g_tc = {n: p.grad.detach().clone() for n, p in mod.named_parameters()}
    mod.zero_grad()
    y32, _ = mod(x)  # float32 inputs: the CUDA-core kernels (chunked forward, exact backward)
    y32.square().mean().backward()
    assert ops.last_path() in ("exact", "chunked")
    assert rel_err(y, y32.detach().double().cpu().numpy()) < 3e-2
    for n, p in mod.named_parameters():
        assert rel_err(g_tc[n], p.grad.double().cpu().numpy()) < 5e-2, n
