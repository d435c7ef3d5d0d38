"""The chunk-parallel float32 forward (csrc/scan_chunk.cu) through the C ABI:
against the float64 oracle (tolerance 1e-4 of max |ref| for float32 inputs,
2e-2 for 16-bit inputs of shapes the tensor cores do not take), against the
token-recurrent exact kernel on the same inputs, and in the automatic path's
choice (float32 calls of 64 tokens or more). Cases cover every decay mode,
key-padding masks, carried state in and out, both output forms, GQA, odd
and wide head sizes, a gamma of 0, strong per-token decay, a streamed
sequence against one pass, and the engine's full-size workload (B=1, N=1024,
D=256 float32).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from subq_audio import ops

from test_scan_gpu import make_case, oracle_inputs, rel_err, to_dev

pytestmark = pytest.mark.gpu

CASES = [
    # B, H, N, d, e, dtype, decay, mask, state, normalize
    (1, 1, 64, 64, 64, torch.float32, "none", False, False, True),
    (1, 1, 1, 8, 8, torch.float32, "scalar", False, True, True),     # one token, one partial chunk
    (2, 3, 300, 16, 16, torch.float32, "scalar", False, False, False),
    (2, 2, 200, 32, 48, torch.float32, "token", True, True, True),
    (1, 2, 257, 128, 128, torch.float32, "head", True, True, False),
    (2, 2, 130, 5, 7, torch.float32, "token", True, True, True),     # d, e not multiples of 4
    (1, 1, 640, 256, 256, torch.float32, "scalar", False, True, False),
    (1, 2, 190, 200, 3, torch.float32, "none", True, False, True),
    (2, 2, 333, 32, 32, torch.bfloat16, "token", True, True, True),
    (1, 2, 150, 96, 80, torch.float16, "head", False, True, False),
    # enough sequences x columns for the sequential chunk walk (the rows above take
    # the chunk-parallel form: scores, state, prefix, outputs)
    (4, 8, 200, 64, 64, torch.float32, "token", True, True, True),
    (2, 20, 130, 32, 48, torch.float32, "scalar", False, True, False),
]


def _run(case, path):
    B, H, N, d, e, dtype, decay, mask, state, normalize = case
    q, k, v, do, lg, m, st = make_case(B, H, N, d, e, dtype, seed=41 + N + d, decay=decay, mask=mask,
                                       state=state, normalize=normalize)
    o, (S, z) = ops.scan_forward(to_dev(q), to_dev(k), to_dev(v), log_gamma=to_dev(lg), mask=to_dev(m),
                                 normalize=normalize, state=to_dev(st), return_state=True, path=path)
    torch.cuda.synchronize()
    return (q, k, v, do, lg, m, st), o, S, z


@pytest.mark.parametrize("case", CASES, ids=[f"k{i}" for i in range(len(CASES))])
def test_chunked_forward_matches_oracle(case):
    B, H, N, d, e, dtype, decay, mask, state, normalize = case
    (q, k, v, do, lg, m, st), o, S, z = _run(case, "chunked")
    assert ops.last_path() == "chunked"
    qn, kn, vn, _, lgn, mn, S0, z0 = oracle_inputs(q, k, v, do, lg, m, st, B, H, N)
    scale = 1.0 / math.sqrt(d) if normalize else 1.0
    ref_o, ref_S, ref_z, _ = oracle.forward(qn, kn, vn, log_gamma=lgn, mask=mn, normalize=normalize,
                                            scale=scale, S0=S0, z0=z0)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert rel_err(o, ref_o) < tol
    assert rel_err(S, ref_S) < max(tol, 1e-5)
    if normalize:
        assert rel_err(z, ref_z) < max(tol, 1e-5)


@pytest.mark.parametrize("case", CASES[:6], ids=[f"k{i}" for i in range(6)])
def test_chunked_forward_matches_exact_kernel(case):
    _, o_c, S_c, z_c = _run(case, "chunked")
    _, o_x, S_x, z_x = _run(case, "exact")
    torch.testing.assert_close(o_c, o_x, rtol=1e-4, atol=1e-4 * o_x.abs().max().item())
    torch.testing.assert_close(S_c, S_x, rtol=1e-4, atol=1e-4 * S_x.abs().max().item())
    if z_x is not None:
        torch.testing.assert_close(z_c, z_x, rtol=1e-5, atol=1e-5 * z_x.abs().max().item())


def test_both_forms_launch_counts():
    from subq_audio import _capi

    q = torch.randn(1, 2, 300, 32, device="cuda")
    ops.scan_forward(q, q, q, path="chunked")
    assert _capi.last_launches() == 4  # scores, state, prefix, outputs
    q = torch.randn(4, 8, 300, 64, device="cuda")
    ops.scan_forward(q, q, q, path="chunked")
    assert _capi.last_launches() == 2  # scores, sequential walk


def test_automatic_path_choice():
    q = torch.randn(1, 2, 64, 32, device="cuda")
    ops.scan_forward(q, q, q)
    assert ops.last_path() == "chunked"
    ops.scan_forward(q[:, :, :63], q[:, :, :63], q[:, :, :63])
    assert ops.last_path() == "exact"
    ops.scan_forward(q, q, q, reverse=True)  # reverse time keeps the recurrent kernel
    assert ops.last_path() == "exact"
    ops.scan_forward(q, q, q, log_gamma=math.log(1.01))  # a growing state too
    assert ops.last_path() == "exact"
    ops.scan_forward(q.double(), q.double(), q.double())
    assert ops.last_path() == "exact"
    qb = torch.randn(1, 2, 128, 64, device="cuda", dtype=torch.bfloat16)
    ops.scan_forward(qb, qb, qb)
    assert ops.last_path() == "tensorcore"


def test_grouped_kv_matches_repeated_heads():
    g = torch.Generator().manual_seed(5)
    B, H, Hkv, N, d = 2, 6, 2, 400, 48
    q = torch.randn(B, H, N, d, generator=g).cuda()
    k = torch.randn(B, Hkv, N, d, generator=g).cuda()
    v = torch.randn(B, Hkv, N, d, generator=g).cuda()
    lg = (-torch.nn.functional.softplus(-(torch.randn(B, H, N, generator=g) + 3.0))).cuda()
    o, (S, z) = ops.scan_forward(q, k, v, log_gamma=lg, return_state=True, path="chunked")
    kr, vr = k.repeat_interleave(3, dim=1), v.repeat_interleave(3, dim=1)
    o2, (S2, z2) = ops.scan_forward(q, kr, vr, log_gamma=lg, return_state=True, path="chunked")
    assert torch.equal(o, o2) and torch.equal(S, S2) and torch.equal(z, z2)


def test_zero_gamma_and_strong_decay():
    """gamma = 0 keeps only the current token (no NaN from the decay sums);
    per-token decay down to exp(-40) matches the recurrent kernel."""
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(1, 2, 300, 16, generator=g).cuda() for _ in range(3))
    o, _ = ops.scan_forward(q, k, v, log_gamma=float("-inf"), normalize=False, scale=1.0, path="chunked")
    phi = lambda x: torch.where(x > 0, x + 1, torch.exp(x))  # noqa: E731
    ref = (phi(q) * phi(k)).sum(-1, keepdim=True) * v
    torch.testing.assert_close(o, ref, rtol=1e-5, atol=1e-5)
    lg = -torch.rand(1, 2, 300, generator=g).cuda() * 40.0
    o_c, _ = ops.scan_forward(q, k, v, log_gamma=lg, path="chunked")
    o_x, _ = ops.scan_forward(q, k, v, log_gamma=lg, path="exact")
    assert rel_err(o_c, o_x.double().cpu().numpy()) < 1e-5


def test_streamed_sequence_equals_one_pass():
    g = torch.Generator().manual_seed(13)
    q, k, v = (torch.randn(2, 2, 1000, 32, generator=g).cuda() for _ in range(3))
    lg = math.log(0.98)
    full, (S_full, z_full) = ops.scan_forward(q, k, v, log_gamma=lg, return_state=True)
    assert ops.last_path() == "chunked"
    st, outs = None, []
    for s0 in range(0, 1000, 250):  # 250 = 3 whole chunks and a partial one
        sl = slice(s0, s0 + 250)
        o, st = ops.scan_forward(q[:, :, sl], k[:, :, sl], v[:, :, sl], log_gamma=lg, state=st,
                                 return_state=True)
        outs.append(o)
    torch.testing.assert_close(torch.cat(outs, dim=2), full, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(st[0], S_full, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(st[1], z_full, rtol=1e-5, atol=1e-4)


def test_engine_workload_matches_oracle_and_exact_path():
    """The engine's full-size single-head float32 forward (B=1, N=1024,
    D=256, U[0,1) inputs, gamma 0.99): the chunked kernels against the
    oracle (1e-4) and the recurrent kernel."""
    rng = np.random.default_rng(0)
    q, k, v = (rng.random((1, 1024, 256), dtype=np.float32) for _ in range(3))
    ref = oracle.engine_forward(q, k, v, 0.99)
    qd, kd, vd = (torch.from_numpy(x).cuda()[:, None] for x in (q, k, v))
    kw = dict(log_gamma=math.log(0.99), normalize=False, scale=1.0, flush_subnormal=True)
    o_c, _ = ops.scan_forward(qd, kd, vd, path="chunked", **kw)
    o_x, _ = ops.scan_forward(qd, kd, vd, path="exact", **kw)
    assert rel_err(o_c[:, 0], ref) < 1e-4
    assert rel_err(o_c, o_x.double().cpu().numpy()) < 1e-5


def test_engine_normalised_carry_equals_one_call():
    """The host engine's normalised form carries S and z in place between
    calls (the normaliser read by every column CTA and rewritten)."""
    from subq_audio import SubQEngine

    rng = np.random.default_rng(21)
    q, k, v = (rng.standard_normal((2, 512, 96)).astype(np.float32) * 0.5 for _ in range(3))
    eng = SubQEngine(64 * 1024 * 1024)
    full = eng.forward(q, k, v, 0.97, normalize=True)
    parts = [eng.forward(q[:, s:s + 128], k[:, s:s + 128], v[:, s:s + 128], 0.97, carry_state=s > 0,
                         normalize=True) for s in range(0, 512, 128)]
    np.testing.assert_allclose(np.concatenate(parts, axis=1), full, rtol=1e-4, atol=1e-5)
