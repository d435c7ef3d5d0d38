"""One pre-LayerNorm block of the audio model (d_model 768, 12 heads of 64,
data-dependent decay gating, FFN 3072 GELU; the reference's
python/subq_audio/model.py:97-135 pattern) with this package's
SubQLinearAttention, against the same block with the reference's layer
(python/subq_audio/autograd.py:663-772). The fixture block_cases.npz holds the
reference block's float64 loss, output rows, input-gradient rows and, for
every parameter, its gradient's norm, projection on a seeded unit direction
and leading values (tests/golden/make_golden.py, from seeded weights and
inputs in golden_inputs.py).

float64 on the GPU: log(gamma) crosses the C ABI as float32, so the block
agrees to ~1e-7 relative; tolerance 1e-5. bf16 autocast (the training
setting, float32 weights): the bf16 roundings of every projection bound the
agreement; tolerances in BF16_TOL.
"""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from subq_audio.autograd import SubQLinearAttention

pytestmark = pytest.mark.gpu

TOL64 = 1e-5
BF16_TOL = {"loss": 1e-2, "out": 3e-2, "dx": 5e-2, "norm": 5e-2, "proj": 5e-2, "head": 1e-1}


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _run(name, dtype):
    spec = gi.BLOCK_CASES[name]
    torch.manual_seed(0)
    blk = gi.make_block(SubQLinearAttention, spec).to(torch.float64 if dtype == torch.float64 else torch.float32)
    gi.load_block_params(blk, gi.block_params(name, blk))
    blk = blk.cuda()
    x, y, mask = gi.block_inputs(name, spec)
    pd = torch.float64 if dtype == torch.float64 else torch.float32
    xt = torch.tensor(x, dtype=pd, device="cuda", requires_grad=True)
    yt = torch.tensor(y, dtype=pd, device="cuda")
    mt = None if mask is None else torch.tensor(mask, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16):
        o = blk(xt, attention_mask=mt)
        loss = torch.nn.functional.mse_loss(o.to(pd), yt)
    loss.backward()
    grads = {n: p.grad.double().cpu().numpy() for n, p in blk.named_parameters()}
    return float(loss.detach()), o.detach().double().cpu().numpy(), xt.grad.double().cpu().numpy(), grads


def _errors(name, dtype):
    ref = np.load(gi.__file__.replace("golden_inputs.py", "block_cases.npz"))
    loss, o, dx, grads = _run(name, dtype)
    st = gi.BLOCK_ROW_STEP
    e = {"loss": abs(loss - ref[f"{name}/loss"]) / abs(ref[f"{name}/loss"]),
         "out": _rel(o[:, ::st], ref[f"{name}/out_rows"]),
         "dx": _rel(dx[:, ::st], ref[f"{name}/dx_rows"]),
         "norm": 0.0, "proj": 0.0, "head": 0.0}
    worst = {}
    for pname, g in grads.items():
        n_ref = float(ref[f"{name}/g/{pname}/norm"])
        proj = float((g * gi.block_direction(name, pname, g.shape)).sum())
        pe = {"norm": abs(np.linalg.norm(g) - n_ref) / n_ref,
              "proj": abs(proj - float(ref[f"{name}/g/{pname}/proj"])) / n_ref,
              "head": _rel(g.reshape(-1)[:gi.BLOCK_HEAD], ref[f"{name}/g/{pname}/head"])}
        for key, val in pe.items():
            if val > e[key]:
                e[key], worst[key] = val, pname
    return e, worst


@pytest.mark.parametrize("name", list(gi.BLOCK_CASES))
def test_block_float64_matches_reference_layer(name):
    e, worst = _errors(name, torch.float64)
    for key, val in e.items():
        assert val < TOL64, f"{key}: {val:.3e} ({worst.get(key, '')})"


@pytest.mark.parametrize("name", list(gi.BLOCK_CASES))
def test_block_bf16_autocast_matches_reference_layer(name):
    e, worst = _errors(name, torch.bfloat16)
    print(name, {k: f"{v:.2e}" for k, v in e.items()}, worst)
    for key, val in e.items():
        assert val < BF16_TOL[key], f"{key}: {val:.3e} ({worst.get(key, '')})"
