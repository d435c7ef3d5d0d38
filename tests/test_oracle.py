"""Pins the float64 oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by the reference itself (its C++ engine built from
source and its torch autograd path); see tests/golden/make_golden.py.
"""
import os

import numpy as np
import pytest

import golden_inputs as gi
import oracle


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_feature_map_known_answers(golden_dir):
    kat = _load(golden_dir, "feature_map_kat.npz")
    for x, ref in zip(kat["x"], kat["phi"]):
        assert abs(oracle.phi(x) - ref) < 1e-12
    # Known answers quoted by the reference's C++ unit test (1e-4 tolerance there).
    for x, ref in [(-1.0, 0.367879), (2.0, 3.0), (0.0, 1.0), (-2.0, 0.135335)]:
        assert abs(oracle.phi(x) - ref) < 1e-6
    assert oracle.phi_prime(3.0) == 1.0
    assert abs(oracle.phi_prime(-1.0) - np.exp(-1.0)) < 1e-15


@pytest.mark.parametrize("B,T,D,gamma", gi.ENGINE_CASES)
def test_oracle_matches_reference_engine(golden_dir, B, T, D, gamma):
    g = _load(golden_dir, "engine_cases.npz")
    tag = f"B{B}_T{T}_D{D}_g{gamma}"
    q, k, v, dO = gi.engine_inputs(B, T, D)
    o = oracle.engine_forward(q, k, v, gamma)
    scale = np.abs(g[f"{tag}/o"]).max()
    assert np.abs(o - g[f"{tag}/o"]).max() <= 1e-5 * scale
    dq, dk, dv, dg = oracle.engine_backward(dO, q, k, v, gamma)
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        ref = g[f"{tag}/{name}"]
        assert np.abs(got - ref).max() <= 1e-5 * max(np.abs(ref).max(), 1e-30), name
    ref_dg = float(g[f"{tag}/dgamma"])
    # d_gamma sums d*d*T float32 products in the reference: float32 summation error
    assert abs(dg - ref_dg) <= 2e-4 * max(abs(ref_dg), 1.0)


def test_oracle_matches_reference_engine_config1(golden_dir):
    g = _load(golden_dir, "config1_engine.npz")
    q, k, v = gi.config1_inputs()
    for gamma in (0.99, 1.0):
        ref = g[f"o_g{gamma}"]
        o = oracle.engine_forward(q, k, v, gamma)
        # the reference runs in float32 with -ffast-math; max relative error vs max |ref|
        assert np.abs(o - ref).max() / np.abs(ref).max() < 1e-5


@pytest.mark.parametrize("name", list(gi.AUTOGRAD_CASES))
def test_oracle_matches_reference_autograd(golden_dir, name):
    g = _load(golden_dir, "autograd_cases.npz")
    spec = gi.AUTOGRAD_CASES[name]
    q, k, v, dO, w, mask = gi.autograd_inputs(spec)
    w_arg = gi.NO_DECAY_W if w is None else w
    o, (S, z) = oracle.attention(q, k, v, decay_w=w_arg, attention_mask=mask)
    tol = 1e-9
    for key, got in (("o", o), ("o_fn", o)):
        ref = g[f"{name}/{key}"]
        assert np.abs(got - ref).max() <= tol * max(1.0, np.abs(ref).max()), key
    refS = g[f"{name}/S"]
    S_cmp = S if spec["H"] is not None else S[:, :1]
    assert np.abs(S_cmp.reshape(refS.shape) - refS).max() <= tol * max(1.0, np.abs(refS).max())
    refZ = g[f"{name}/Z"]
    assert np.abs(z.reshape(refZ.shape) - refZ).max() <= tol * max(1.0, np.abs(refZ).max())
    dq, dk, dv, dw = oracle.attention_backward(q, k, v, dO, decay_w=w_arg, attention_mask=mask)
    for key, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        ref = g[f"{name}/{key}"]
        assert np.abs(got - ref).max() <= 1e-8 * max(1.0, np.abs(ref).max()), key
    if w is not None:
        ref = g[f"{name}/dw"]
        assert np.abs(np.asarray(dw) - ref).max() <= 1e-8 * max(1.0, np.abs(ref).max())


def test_oracle_streaming_matches_single_pass(golden_dir):
    g = _load(golden_dir, "streaming_case.npz")
    q, k, v = gi.stream_inputs()
    L = gi.STREAM_SPLIT
    full, (S, z) = oracle.attention(q, k, v, decay_w=gi.NO_DECAY_W)
    assert np.abs(full - g["full"]).max() < 1e-10
    parts, state = [], None
    for s in range(0, q.shape[2], L):
        o, state = oracle.attention(q[:, :, s:s + L], k[:, :, s:s + L], v[:, :, s:s + L],
                                    decay_w=gi.NO_DECAY_W, past_state=state)
        parts.append(o)
    streamed = np.concatenate(parts, axis=2)
    assert np.abs(streamed - g["streamed"]).max() < 1e-10
    assert np.abs(state[0] - g["S"]).max() < 1e-8 * np.abs(g["S"]).max()
