"""Known answers of the attention-mask normalisation (the rules of the
reference's subq_audio/autograd.py:57-105, its answers in
tests/test_mask_normalization.py:19-52): a 2-D/3-D/4-D bool, int or float mask
becomes the live-token mask [B, 1, T, 1] the kernels take; a 4-D mask marks a
token live when it is a live query and a live key, so a key-padding mask is
never dropped. The last case runs the kernels: a 2-D mask and the 4-D mask
made from it give the same output.
"""
import pytest
import torch

from subq_audio.autograd import _normalize_attention_mask, _token_mask, chunkwise_flash_linear_attention

B, T = 2, 6
# sequence 0 has 4 live tokens then 2 padded; sequence 1 is all live
LIVE = [[1, 1, 1, 1, 0, 0], [1, 1, 1, 1, 1, 1]]


def _live():
    return torch.tensor(LIVE, dtype=torch.bool)


def _norm(mask, T=T):
    out = _normalize_attention_mask(mask, torch.float32, T)
    assert out.shape == (mask.shape[0], 1, T, 1)
    return out.flatten(1).int().tolist()


def _lower():
    return torch.ones(T, T, dtype=torch.bool).tril()


CASES_4D = {
    # [B, 1, T, T] with every query row the key-padding row
    "key_padding": lambda: _live()[:, None, None, :].expand(B, 1, T, T),
    # causal (lower-triangular) AND key padding
    "causal_and_key_padding": lambda: _lower()[None, None] & _live()[:, None, None, :],
    # padded queries: whole rows off
    "query_padding": lambda: _live()[:, None, :, None].expand(B, 1, T, T),
}


@pytest.mark.parametrize("name", sorted(CASES_4D))
def test_four_d_masks_keep_the_padding(name):
    assert _norm(CASES_4D[name]()) == LIVE


def test_pure_causal_four_d_mask_keeps_every_token():
    assert _norm(_lower().expand(B, 1, T, T)) == [[1] * T] * B


def test_per_head_four_d_mask_reduces_to_one_row():
    m = _live()[:, None, None, :].expand(B, 3, T, T)
    assert _norm(m) == LIVE


def test_non_square_four_d_mask_is_rejected():
    with pytest.raises(ValueError):
        _normalize_attention_mask(torch.ones(B, 1, T, T + 2, dtype=torch.bool), torch.float32, T)


@pytest.mark.parametrize("kind", ["bool", "int", "float_mult", "float_additive"])
def test_two_d_masks_of_every_dtype(kind):
    live = _live()
    m = {"bool": live, "int": live.long(), "float_mult": live.float(),
         "float_additive": torch.where(live, 0.0, -1e9)}[kind]
    assert _norm(m) == LIVE
    # the kernels' form: [B, T] uint8
    tm = _token_mask(_normalize_attention_mask(m, torch.float32, T), B, T, torch.device("cpu"))
    assert tm.dtype == torch.uint8 and tm.tolist() == LIVE


def test_three_d_masks():
    live = _live()
    assert _norm(live[:, None, :]) == LIVE          # [B, 1, T]
    assert _norm(live[:, :, None]) == LIVE          # [B, T, 1]
    assert _norm(live[:, None, :].expand(B, T, T) & live[:, :, None]) == LIVE  # [B, T, T] query rows


@pytest.mark.gpu
def test_four_d_key_padding_equals_two_d_output():
    torch.manual_seed(0)
    q, k, v = (torch.randn(B, 2, T, 4) for _ in range(3))
    w = torch.tensor(0.5)
    out2, _ = chunkwise_flash_linear_attention(q, k, v, w, attention_mask=_live())
    out4, _ = chunkwise_flash_linear_attention(q, k, v, w, attention_mask=CASES_4D["key_padding"]())
    torch.testing.assert_close(out2, out4, rtol=0, atol=0)
    # padded tokens give zero output, live ones do not
    assert (out2[0, :, 4:] == 0).all() and (out2[0, :, :4].abs().sum() > 0)
