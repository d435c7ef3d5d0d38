"""The native engine (subq_audio._C.SubQEngine) against the reference engine's
own outputs (golden fixtures) and its API contract (reference tests
test_cpp_python_parity.py, test_fuzz.py, test_package.py)."""
import json
import os
import struct

import numpy as np
import pytest

import golden_inputs as gi
from subq_audio import AudioTransformerEngine, SubQEngine, get_device_info

pytestmark = pytest.mark.gpu


def _g(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


@pytest.mark.parametrize("B,T,D,gamma", gi.ENGINE_CASES)
def test_engine_forward_matches_reference_engine(golden_dir, B, T, D, gamma):
    g = _g(golden_dir, "engine_cases.npz")
    tag = f"B{B}_T{T}_D{D}_g{gamma}"
    q, k, v, dO = gi.engine_inputs(B, T, D)
    eng = SubQEngine(128 * 1024 * 1024)
    o = eng.forward(q, k, v, decay_factor=gamma)
    ref = g[f"{tag}/o"]
    assert np.abs(o - ref).max() / np.abs(ref).max() < 1e-4
    np.testing.assert_allclose(o, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("B,T,D,gamma", gi.ENGINE_CASES)
def test_engine_backward_matches_reference_engine(golden_dir, B, T, D, gamma):
    g = _g(golden_dir, "engine_cases.npz")
    tag = f"B{B}_T{T}_D{D}_g{gamma}"
    q, k, v, dO = gi.engine_inputs(B, T, D)
    eng = SubQEngine(128 * 1024 * 1024)
    dq, dk, dv, dg = eng.backward(dO, q, k, v, decay_factor=gamma)
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        ref = g[f"{tag}/{name}"]
        assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-4, name
    ref_dg = float(g[f"{tag}/dgamma"])
    assert abs(dg - ref_dg) <= 5e-3 * max(1.0, abs(ref_dg))


def test_engine_config1_matches_reference(golden_dir):
    """B=1, N=1024, D=256 float32 U[0,1): max relative error <= 1e-4."""
    g = _g(golden_dir, "config1_engine.npz")
    q, k, v = gi.config1_inputs()
    eng = SubQEngine(256 * 1024 * 1024)
    for gamma in (0.99, 1.0):
        o = eng.forward(q, k, v, decay_factor=gamma)
        ref = g[f"o_g{gamma}"]
        assert np.abs(o - ref).max() / np.abs(ref).max() <= 1e-4


def test_small_values_are_not_flushed():
    rng = np.random.default_rng(7)
    q, k, v = [(rng.standard_normal((1, 4, 4)) * 0.5).astype(np.float32) for _ in range(3)]
    v = v * 1e-18
    import oracle

    ref = oracle.engine_forward(q, k, v, 0.9)
    assert 1e-30 < np.abs(ref).max() < 1e-15
    o = SubQEngine(16 * 1024 * 1024).forward(q, k, v, decay_factor=0.9)
    np.testing.assert_allclose(o, ref, rtol=1e-2, atol=0.0)


def test_host_chunking_carries_state(golden_dir):
    """A tiny arena forces several host chunks per call; the state carries across them."""
    q, k, v, _ = gi.engine_inputs(2, 130, 16)
    big = SubQEngine(64 * 1024 * 1024).forward(q, k, v, decay_factor=0.95)
    small = SubQEngine(2 * 16 * 16 * 4 + 4 * 2 * 16 * 4 * 40).forward(q, k, v, decay_factor=0.95)
    np.testing.assert_allclose(small, big, rtol=1e-5, atol=1e-5)


def test_carry_state_across_calls_matches_one_call():
    rng = np.random.default_rng(11)
    q, k, v = [rng.standard_normal((1, 256, 32)).astype(np.float32) * 0.5 for _ in range(3)]
    eng = SubQEngine(32 * 1024 * 1024)
    full = eng.forward(q, k, v, decay_factor=0.98)
    parts = [eng.forward(q[:, s:s + 64], k[:, s:s + 64], v[:, s:s + 64], decay_factor=0.98,
                         carry_state=(s > 0)) for s in range(0, 256, 64)]
    np.testing.assert_allclose(np.concatenate(parts, axis=1), full, rtol=1e-5, atol=1e-4)
    eng.reset_state()
    again = eng.forward(q[:, :64], k[:, :64], v[:, :64], decay_factor=0.98, carry_state=True)
    np.testing.assert_allclose(again, full[:, :64], rtol=1e-6, atol=1e-6)


def test_garbage_shapes_and_strided_inputs():
    eng = SubQEngine(10 * 1024 * 1024)
    with pytest.raises(RuntimeError):
        eng.forward(np.array(0.0, dtype=np.float32), np.array(0.0, dtype=np.float32),
                    np.array(0.0, dtype=np.float32))
    z = np.zeros((10, 10), dtype=np.float32)
    with pytest.raises(RuntimeError):
        eng.forward(z, z, z)
    big = [np.random.randn(2, 100, 64).astype(np.float32) for _ in range(3)]
    out = eng.forward(*(b[:, ::2, :] for b in big))
    assert out.shape == (2, 50, 64)


def test_nan_inf_ingestion():
    eng = SubQEngine(10 * 1024 * 1024)
    Q = np.full((1, 128, 64), np.nan, dtype=np.float32)
    K = np.full((1, 128, 64), np.inf, dtype=np.float32)
    V = np.full((1, 128, 64), -np.inf, dtype=np.float32)
    assert np.isnan(eng.forward(Q, K, V)).any()


def test_safetensors_overflow_header_is_rejected(tmp_path):
    bad = tmp_path / "overflow.safetensors"
    header = json.dumps({"__metadata__": {"format": "pt"},
                         "bad_tensor": {"dtype": "F32", "shape": [1024, 1024],
                                        "data_offsets": [0, (2 ** 64) - 1]}}).encode()
    bad.write_bytes(struct.pack("<Q", len(header)) + header)
    eng = SubQEngine(10 * 1024 * 1024)
    with pytest.raises(RuntimeError) as exc:
        eng.load(str(bad))
    assert "Failed to load safetensors file" in str(exc.value)


def test_safetensors_valid_file_loads(tmp_path):
    data = np.arange(12, dtype=np.float32)
    header = json.dumps({"w": {"dtype": "F32", "shape": [3, 4], "data_offsets": [0, 48]}}).encode()
    f = tmp_path / "ok.safetensors"
    f.write_bytes(struct.pack("<Q", len(header)) + header + data.tobytes())
    SubQEngine(10 * 1024 * 1024).load(str(f))


def test_device_info_and_wrapper():
    info = get_device_info()
    assert info["backend"] == "CUDA" and info["architecture"].startswith("SM ")
    assert isinstance(info["bfloat16_supported"], bool) and info["memory_size"] > 0
    w = AudioTransformerEngine(vram_capacity=64 * 1024 * 1024)
    assert w.device_info == info


def test_wrapper_dispatch_torch_cuda_float32_matches_numpy():
    import torch

    rng = np.random.default_rng(2)
    q, k, v = [rng.standard_normal((2, 70, 16)).astype(np.float32) * 0.5 for _ in range(3)]
    w = AudioTransformerEngine(vram_capacity=64 * 1024 * 1024)
    o_np = w.forward(q, k, v, decay_factor=0.9)
    o_t = w.forward(*(torch.from_numpy(x).cuda() for x in (q, k, v)), decay_factor=0.9)
    np.testing.assert_allclose(o_t.cpu().numpy(), o_np, rtol=1e-5, atol=1e-5)
    dO = rng.standard_normal((2, 70, 16)).astype(np.float32)
    g_np = w.backward(dO, q, k, v, decay_factor=0.9)
    g_t = w.backward(*(torch.from_numpy(x).cuda() for x in (dO, q, k, v)), decay_factor=0.9)
    for a, b in zip(g_np[:3], g_t[:3]):
        np.testing.assert_allclose(b.cpu().numpy(), a, rtol=1e-4, atol=1e-4)
    assert abs(g_np[3] - g_t[3]) <= 1e-3 * max(1.0, abs(g_np[3]))
