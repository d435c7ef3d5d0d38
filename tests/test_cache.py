"""Streaming-state formats (subq_audio.cache) on the host: the reference's
prepare_inputs_for_generation slicing (python/subq_audio/model.py:330-339),
the per-layer tuple threading of its model loop (:227-238), and the cache's
bookkeeping. The decode runs on the kernels are in test_cache_gpu.py."""
import torch

from subq_audio.cache import StateCache, prepare_inputs_for_generation, run_layers


def test_prepare_inputs_slices_to_the_last_token_once_cached():
    ids = torch.arange(10).view(2, 5)
    first = prepare_inputs_for_generation(ids)
    assert torch.equal(first["input_ids"], ids) and first["past_key_values"] is None and first["use_cache"]
    cache = (torch.zeros(1),)
    nxt = prepare_inputs_for_generation(ids, past_key_values=cache, use_cache=False)
    assert torch.equal(nxt["input_ids"], ids[:, -1:]) and nxt["past_key_values"] is cache
    assert nxt["use_cache"] is False


def test_run_layers_threads_one_state_per_layer():
    seen = []

    def layer(tag):
        def f(h, past_state=None, attention_mask=None, use_cache=False):
            seen.append((tag, past_state))
            return h + 1, f"{tag}-next"
        return f

    h, cache = run_layers([layer("a"), layer("b")], torch.zeros(1), past_key_values=("pa", "pb"))
    assert seen == [("a", "pa"), ("b", "pb")] and cache == ("a-next", "b-next") and h.item() == 2
    _, none = run_layers([layer("a")], torch.zeros(1), use_cache=False)
    assert none is None


def test_state_cache_bookkeeping_and_reorder():
    S = torch.arange(3 * 2 * 4 * 4, dtype=torch.float32).view(3, 2, 4, 4)
    S.Z = torch.arange(3 * 2 * 4, dtype=torch.float32).view(3, 2, 4, 1)
    c = StateCache()
    c.step((S, (S + 1, S.Z)), new_tokens=7)
    assert len(c) == 2 and c.get_seq_length() == 7
    c.step(c.to_legacy(), new_tokens=1)
    assert c.get_seq_length() == 8
    assert c.memory_bytes() == 2 * (S.numel() + S.Z.numel()) * 4
    c.reorder(torch.tensor([2, 0, 0]))
    S0 = c[0]
    assert torch.equal(S0, S[[2, 0, 0]]) and torch.equal(S0.Z, S.Z[[2, 0, 0]])
    assert torch.equal(c[1], (S + 1)[[2, 0, 0]])
    assert c[5] is None
    again = StateCache.from_legacy(c.to_legacy(), seen_tokens=8)
    assert len(again) == 2 and again.get_seq_length() == 8
