"""Incremental decoding through a stack of layers with per-layer
past_key_values (subq_audio.cache, the reference's model.py:227-238 loop):
a prompt prefilled in one call and then one token per call, each call
carrying every layer's device-resident state, gives the outputs and final
states of one pass over the whole sequence. float32 (the one-token steps run
the token-recurrent kernel; the prefill the chunked kernels), tolerance 1e-4
of max |ref|; bf16 (tensor-core prefill) at 3e-2.
"""
import pytest
import torch
import torch.nn as nn

from subq_audio.autograd import SubQLinearAttention
from subq_audio.cache import StateCache, prepare_inputs_for_generation, run_layers

pytestmark = pytest.mark.gpu


class Block(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.ln = nn.LayerNorm(d)
        self.attn = SubQLinearAttention(d, heads, use_data_dependent_gating=True)

    def forward(self, h, past_state=None, attention_mask=None, use_cache=False):
        a, st = self.attn(self.ln(h), past_state=past_state, attention_mask=attention_mask, use_cache=use_cache)
        return h + a, st


def rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max())


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 3e-2)])
def test_prefill_then_single_tokens_equals_one_pass(dtype, tol):
    torch.manual_seed(0)
    d, heads, T, P = 256, 4, 200, 192
    blocks = nn.ModuleList([Block(d, heads) for _ in range(3)]).cuda().to(dtype)
    emb = nn.Embedding(100, d).cuda().to(dtype)
    ids = torch.randint(0, 100, (2, T), device="cuda")
    with torch.no_grad():
        full, full_cache = run_layers(blocks, emb(ids))
        out, past = run_layers(blocks, emb(ids[:, :P]))
        cache = StateCache()
        cache.step(past, P)
        outs = [out]
        for t in range(P, T):
            inp = prepare_inputs_for_generation(ids[:, :t + 1], past_key_values=cache.to_legacy())
            assert inp["input_ids"].shape == (2, 1)
            o, past = run_layers(blocks, emb(inp["input_ids"]), past_key_values=inp["past_key_values"])
            cache.step(past, 1)
            outs.append(o)
    assert cache.get_seq_length() == T
    assert rel(torch.cat(outs, dim=1), full) < tol
    for a, b in zip(cache.to_legacy(), full_cache):
        assert rel(a, b) < tol and rel(a.Z, b.Z) < tol
    # one state per layer, its size independent of the length
    assert cache.memory_bytes() == 3 * 2 * heads * (64 * 64 + 64) * 4


def test_reorder_follows_the_batch():
    torch.manual_seed(1)
    blocks = nn.ModuleList([Block(128, 2) for _ in range(2)]).cuda()
    x = torch.randn(3, 70, 128, device="cuda")
    idx = torch.tensor([2, 2, 0], device="cuda")
    with torch.no_grad():
        _, past = run_layers(blocks, x[:, :64])
        cache = StateCache(past, 64)
        cache.reorder(idx)
        o, _ = run_layers(blocks, x[idx, 64:], past_key_values=cache.to_legacy())
        ref, _ = run_layers(blocks, x[idx])
    assert rel(o, ref[:, 64:]) < 1e-4
