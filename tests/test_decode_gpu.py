"""Streaming decode (ops.DecodeStep): one call per new token over preallocated
buffers with the float32 state carried on the device and updated in place,
against one pass over the whole sequence (reference: cached generation,
tests/test_surgery_and_caching.py:168-214, and the carried-state streaming
of python/subq_audio/autograd.py:343-352).
"""
import math

import pytest
import torch

from subq_audio import ops

from test_scan_gpu import rel_err

pytestmark = pytest.mark.gpu


def _seq(B, H, N, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, N, 64, generator=g).to(dtype).cuda() for _ in range(3))
    lg = (-torch.nn.functional.softplus(-(torch.randn(B, H, N, generator=g) + 3.0))).cuda()
    return q, k, v, lg


@pytest.mark.parametrize("dtype,decay", [(torch.bfloat16, "token"), (torch.float32, "head"),
                                         (torch.float16, None), (torch.bfloat16, None)])
def test_decode_steps_equal_one_pass(dtype, decay):
    B, H, N, N0 = 2, 3, 300, 200
    q, k, v, lg = _seq(B, H, N, dtype, seed=3)
    lg_head = torch.tensor([math.log(0.97), math.log(0.9), math.log(0.995)], device="cuda")
    lg_all = lg if decay == "token" else lg_head if decay == "head" else None
    full, (S_full, z_full) = ops.scan_forward(q, k, v, log_gamma=lg_all, return_state=True)
    # prefill, then single-token steps through preallocated buffers
    pre_lg = lg[:, :, :N0].contiguous() if decay == "token" else lg_all
    o0, (S, z) = ops.scan_forward(q[:, :, :N0], k[:, :, :N0], v[:, :, :N0], log_gamma=pre_lg, return_state=True)
    qb, kb, vb, ob = (torch.empty(B, H, 1, 64, dtype=dtype, device="cuda") for _ in range(4))
    lgb = torch.empty(B, H, 1, device="cuda") if decay == "token" else lg_all
    step = ops.DecodeStep(qb, kb, vb, ob, S, z, log_gamma=lgb)
    outs = [o0]
    for t in range(N0, N):
        qb.copy_(q[:, :, t:t + 1]), kb.copy_(k[:, :, t:t + 1]), vb.copy_(v[:, :, t:t + 1])
        if decay == "token":
            lgb.copy_(lg[:, :, t:t + 1])
        step.step()
        outs.append(ob.clone())
    torch.cuda.synchronize()
    assert ops.last_path() == "exact"  # single-token steps take the token-recurrent kernel
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert rel_err(torch.cat(outs, dim=2), full.double().cpu().numpy()) < tol
    assert rel_err(S, S_full.double().cpu().numpy()) < max(tol, 1e-3)
    assert rel_err(z, z_full.double().cpu().numpy()) < max(tol, 1e-3)


def test_decode_step_replays_in_a_cuda_graph():
    """The step allocates nothing and does not synchronise: captured once in a
    CUDA graph, replays with refilled buffers reproduce the eager steps."""
    B, H, N = 4, 12, 64
    q, k, v, lg = _seq(B, H, N, torch.bfloat16, seed=8)
    S = torch.zeros(B, H, 64, 64, device="cuda")
    z = torch.zeros(B, H, 64, device="cuda")
    S2, z2 = S.clone(), z.clone()
    qb, kb, vb, ob = (torch.empty(B, H, 1, 64, dtype=torch.bfloat16, device="cuda") for _ in range(4))
    lgb = torch.empty(B, H, 1, device="cuda")
    eager = ops.DecodeStep(qb, kb, vb, ob, S, z, log_gamma=lgb)
    graphed = ops.DecodeStep(qb, kb, vb, ob, S2, z2, log_gamma=lgb)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        S2_0, z2_0 = S2.clone(), z2.clone()
        graphed.step()  # warm-up outside the capture (the kernel's attributes are set once)
        S2.copy_(S2_0), z2.copy_(z2_0)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        graphed.step()
    ref, got = [], []
    for t in range(N):
        for dst, src in ((qb, q), (kb, k), (vb, v), (lgb, lg)):
            dst.copy_(src[:, :, t:t + 1])
        eager.step()
        ref.append(ob.clone())
        g.replay()
        got.append(ob.clone())
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(ref, 2), torch.cat(got, 2))
    assert torch.equal(S, S2) and torch.equal(z, z2)


def test_stream_of_tensor_core_calls_replays_in_a_cuda_graph():
    """The C3 serving form: a stream of 4096-token calls (tensor-core scans,
    cluster launches) sharing one in-place state, captured once as a CUDA graph
    (state reset included); replays equal the eager calls bit for bit."""
    B, H, N, L = 1, 4, 4 * 4096, 4096
    q, k, v, _ = _seq(B, H, N, torch.float16, seed=12)
    o_eager, o_graph = torch.empty_like(q), torch.empty_like(q)
    S, z = torch.zeros(B, H, 64, 64, device="cuda"), torch.zeros(B, H, 64, device="cuda")

    def calls(o):
        return [ops.DecodeStep(q[:, :, s:s + L], k[:, :, s:s + L], v[:, :, s:s + L], o[:, :, s:s + L], S, z)
                for s in range(0, N, L)]

    def run(steps):
        S.zero_(), z.zero_()
        for c in steps:
            c.step()

    eager, graphed = calls(o_eager), calls(o_graph)
    run(eager)
    torch.cuda.synchronize()
    assert ops.last_path() == "tensorcore"
    S_eager, z_eager = S.clone(), z.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run(graphed)  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run(graphed)
    o_graph.zero_()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(o_graph, o_eager)
    assert torch.equal(S, S_eager) and torch.equal(z, z_eager)
    full = ops.scan_forward(q, k, v)[0]
    assert rel_err(o_graph, full.double().cpu().numpy()) < 2e-2


def test_decode_step_rejects_buffers_it_would_copy():
    B, H = 1, 2
    qb, kb, vb, ob = (torch.empty(B, H, 1, 64, dtype=torch.bfloat16, device="cuda") for _ in range(4))
    S, z = torch.zeros(B, H, 64, 64, device="cuda"), torch.zeros(B, H, 64, device="cuda")
    with pytest.raises(ValueError):
        ops.DecodeStep(qb, kb, vb, ob, S.to(torch.float64), z)
    with pytest.raises(ValueError):  # a float64 log_gamma would be converted, not read in place
        ops.DecodeStep(qb, kb, vb, ob, S, z, log_gamma=torch.zeros(B, H, 1, dtype=torch.float64, device="cuda"))
