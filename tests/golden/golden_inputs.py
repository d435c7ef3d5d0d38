"""Seeded inputs of the golden fixtures (shared by the generator and the tests).

All inputs are synthetic: the reference's own parity tests draw N(0,1)*0.5
inputs (reference tests/test_cpp_python_parity.py:27-29) and its README
example draws U[0,1) inputs for B=1, N=1024, D=256; the same distributions
and shapes are reproduced here from numpy seeds.
"""
from __future__ import annotations

import zlib

import numpy as np

# (batch, seq_len, d_model, gamma): the reference's parity cases.
ENGINE_CASES = [
    (1, 7, 4, 0.5),
    (2, 64, 8, 0.9),
    (1, 65, 8, 0.99),
    (2, 130, 16, 0.95),
    (1, 130, 32, 0.8),
]

# The reference always passes a decay parameter; w = 30 gives
# log(gamma) = -softplus(-30) = -9.4e-14, i.e. gamma == 1 to double precision.
NO_DECAY_W = 30.0

AUTOGRAD_CASES = {
    "causal3d_nodecay": dict(B=2, H=None, T=70, D=16, decay="none"),
    "mh_scalar": dict(B=2, H=3, T=100, D=16, decay="scalar"),
    "mh_head": dict(B=2, H=4, T=137, D=32, decay="head"),
    "mh_bht": dict(B=2, H=2, T=80, D=16, decay="bht"),
    "bt_decay": dict(B=2, H=None, T=67, D=8, decay="bt"),
    "mask_len": dict(B=2, H=2, T=150, D=16, decay="none", mask="len"),
    "mask_4d_decay": dict(B=2, H=2, T=96, D=8, decay="head", mask="4d"),
    "d64_mask": dict(B=1, H=1, T=160, D=64, decay="none", mask="len"),
}

STREAM_SPLIT = 128


def _rng(name: str) -> np.random.Generator:
    return np.random.default_rng(zlib.crc32(name.encode()))


def engine_inputs(B, T, D):
    """q, k, v, dO as float32 [B,T,D] (N(0,1) * 0.5)."""
    g = np.random.default_rng(T + D)
    return [(g.standard_normal((B, T, D)) * 0.5).astype(np.float32) for _ in range(4)]


def config1_inputs(seed: int = 0):
    """B=1, N=1024, D=256 float32 U[0,1) (the README example's shape)."""
    g = np.random.default_rng(seed)
    return [g.random((1, 1024, 256), dtype=np.float32) for _ in range(3)]


def lengths_mask(B, T, g):
    lens = np.linspace(T, T // 2, B).astype(np.int64) if B > 1 else np.array([T * 3 // 4])
    g.shuffle(lens)
    return (np.arange(T)[None, :] < lens[:, None])


def autograd_inputs(spec):
    """q, k, v, dO (float64), w (or None for no decay) and a mask (or None)."""
    name = repr(sorted(spec.items()))
    g = _rng(name)
    B, H, T, D = spec["B"], spec["H"], spec["T"], spec["D"]
    shape = (B, T, D) if H is None else (B, H, T, D)
    q, k, v, dO = (g.standard_normal(shape) for _ in range(4))
    Hh = 1 if H is None else H
    decay = spec.get("decay", "none")
    if decay == "none":
        w = None
    elif decay == "scalar":
        w = np.array(2.5)
    elif decay == "head":
        w = np.linspace(1.0, 4.0, Hh)
    elif decay == "bt":
        w = g.standard_normal((B, T)) + 2.0
    elif decay == "bht":
        w = g.standard_normal((B, Hh, T)) + 2.0
    else:
        raise ValueError(decay)
    mask = None
    if spec.get("mask") == "len":
        mask = lengths_mask(B, T, g)
    elif spec.get("mask") == "4d":
        m2 = lengths_mask(B, T, g)
        mask = np.broadcast_to(m2[:, None, None, :], (B, 1, T, T)).copy()
    return q, k, v, dO, w, mask


def stream_inputs():
    g = _rng("stream")
    return [g.standard_normal((1, 2, 4 * STREAM_SPLIT, 16)) for _ in range(3)]


# ---------------------------------------------------------------------------
# Block cases: one pre-LayerNorm transformer block of the reference's audio
# model (python/subq_audio/model.py:97-135: LayerNorm -> SubQLinearAttention
# -> residual -> LayerNorm -> Linear/GELU/Linear -> residual) at d_model 768,
# 12 heads of 64, data-dependent decay gating, MSE loss to seeded targets.
# ---------------------------------------------------------------------------
BLOCK_CASES = {
    "block_causal": dict(B=2, T=512, d=768, H=12, Hkv=12, ffn=3072, causal=True, mask=False),
    "block_bidir_gqa_mask": dict(B=2, T=384, d=768, H=12, Hkv=4, ffn=3072, causal=False, mask=True),
}
BLOCK_ROW_STEP = 64  # output / input-gradient rows kept in the fixture (float32): every 64th position
BLOCK_HEAD = 256     # leading elements of each flattened parameter gradient kept


def make_block(attn_cls, spec):
    """The block with ``attn_cls`` (the reference's SubQLinearAttention or this
    package's) as its attention; parameter names are the same for both."""
    import torch.nn as nn

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            d = spec["d"]
            self.input_layernorm = nn.LayerNorm(d, eps=1e-5)
            self.self_attn = attn_cls(d, num_heads=spec["H"], num_key_value_heads=spec["Hkv"],
                                      is_causal=spec["causal"])
            self.post_attention_layernorm = nn.LayerNorm(d, eps=1e-5)
            self.fc1 = nn.Linear(d, spec["ffn"])
            self.fc2 = nn.Linear(spec["ffn"], d)
            self.act = nn.GELU()

        def forward(self, x, attention_mask=None):
            h = x + self.self_attn(self.input_layernorm(x), attention_mask=attention_mask)[0]
            return h + self.fc2(self.act(self.fc1(self.post_attention_layernorm(h))))

    return Block()


def block_params(name, block):
    """Seeded values for every parameter of ``block`` (float64 numpy, by name):
    Linear weights N(0, 1/fan_in), biases N(0, 0.02^2), norm weights 1 + N(0,
    0.1^2), norm biases N(0, 0.1^2), raw decay logit(0.99) + N(0, 0.5^2)."""
    g = _rng("params/" + name)
    out = {}
    for pname, p in sorted(block.named_parameters()):
        shape = tuple(p.shape)
        if pname.endswith("raw_decay"):
            val = np.log(0.99 / 0.01) + 0.5 * g.standard_normal(shape)
        elif "norm" in pname and pname.endswith("weight"):
            val = 1.0 + 0.1 * g.standard_normal(shape)
        elif "norm" in pname:
            val = 0.1 * g.standard_normal(shape)
        elif pname.endswith("weight"):
            val = g.standard_normal(shape) / np.sqrt(shape[-1])
        else:
            val = 0.02 * g.standard_normal(shape)
        out[pname] = val
    return out


def load_block_params(block, values):
    import torch

    with torch.no_grad():
        for pname, p in block.named_parameters():
            p.copy_(torch.from_numpy(values[pname]).to(p.dtype))


def block_inputs(name, spec):
    """x ~ N(0,1) [B, T, d], targets ~ N(0,1), a key-padding mask (or None),
    and one unit direction per parameter gradient (for projections)."""
    g = _rng("inputs/" + name)
    B, T, d = spec["B"], spec["T"], spec["d"]
    x = g.standard_normal((B, T, d))
    y = g.standard_normal((B, T, d))
    mask = lengths_mask(B, T, g) if spec["mask"] else None
    return x, y, mask


def block_direction(name, pname, shape):
    r = _rng(f"dir/{name}/{pname}").standard_normal(shape)
    return r / np.linalg.norm(r)
