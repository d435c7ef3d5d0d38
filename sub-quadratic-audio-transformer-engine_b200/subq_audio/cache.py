"""Per-layer streaming states in the layout a Hugging Face style model keeps
them (the reference's SubQAudioModel, python/subq_audio/model.py:227-238 and
SubQAudioForCausalLM.prepare_inputs_for_generation, :330-339).

A model's ``past_key_values`` is a tuple with one entry per layer: that
layer's ``next_state`` as ``SubQLinearAttention`` returns it with
``use_cache=True`` (the float32 state S [B, H, D, D] on the device, with its
normaliser attached as ``S.Z``). ``run_layers`` threads such a tuple through
a stack of layers the way the reference's model loop does; ``StateCache``
holds it between generation steps (updating, batch reordering for beam
search, the count of tokens seen); ``prepare_inputs_for_generation`` slices
the prompt to its last token once a cache exists. The states stay on the
device between steps, so a one-token step runs the scan's token-recurrent
kernel on them directly.
"""
from __future__ import annotations

from typing import Any, Callable, Iterable, List, Optional, Sequence, Tuple

import torch

State = Any  # a layer's next_state: S [B, H, D, D] float32 with S.Z, or (S, Z)


def prepare_inputs_for_generation(input_ids: torch.Tensor, past_key_values: Optional[Sequence[State]] = None,
                                  **kwargs) -> dict:
    """The reference's slicing (model.py:330-339): with a cache, only the last
    token is fed; ``use_cache`` defaults to True."""
    if past_key_values is not None:
        input_ids = input_ids[:, -1:]
    return {"input_ids": input_ids, "past_key_values": past_key_values,
            "use_cache": kwargs.get("use_cache", True)}


def run_layers(layers: Iterable[Callable], hidden_states: torch.Tensor,
               past_key_values: Optional[Sequence[State]] = None, attention_mask: Optional[torch.Tensor] = None,
               use_cache: bool = True) -> Tuple[torch.Tensor, Optional[Tuple[State, ...]]]:
    """Layer i gets ``past_key_values[i]`` as ``past_state`` and returns
    ``(hidden_states, next_state)``; with ``use_cache`` the next states come
    back as a tuple, one per layer (model.py:227-238)."""
    next_cache: Optional[Tuple[State, ...]] = () if use_cache else None
    for idx, layer in enumerate(layers):
        layer_past = past_key_values[idx] if past_key_values is not None else None
        hidden_states, next_state = layer(hidden_states, past_state=layer_past, attention_mask=attention_mask,
                                          use_cache=use_cache)
        if use_cache:
            next_cache += (next_state,)
    return hidden_states, next_cache


def _split(state: State) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    if isinstance(state, tuple):
        return state[0], (state[1] if len(state) > 1 else None)
    return state, getattr(state, "Z", None)


class StateCache:
    """The per-layer states of one generation, between steps.

    ``cache[i]`` is layer i's state in the form the layer takes as
    ``past_state``; ``to_legacy()`` / ``from_legacy()`` convert to and from
    the plain tuple a model returns as ``past_key_values``.
    """

    def __init__(self, states: Optional[Sequence[State]] = None, seen_tokens: int = 0):
        self._states: List[Optional[State]] = list(states) if states is not None else []
        self._seen = int(seen_tokens)

    @classmethod
    def from_legacy(cls, past_key_values: Optional[Sequence[State]], seen_tokens: int = 0) -> "StateCache":
        return cls(past_key_values if past_key_values is not None else None, seen_tokens)

    def to_legacy(self) -> Tuple[State, ...]:
        return tuple(self._states)

    def __len__(self) -> int:
        return len(self._states)

    def __getitem__(self, idx: int) -> Optional[State]:
        return self._states[idx] if idx < len(self._states) else None

    def update(self, layer_idx: int, state: State) -> None:
        while len(self._states) <= layer_idx:
            self._states.append(None)
        self._states[layer_idx] = state

    def step(self, past_key_values: Sequence[State], new_tokens: int) -> None:
        """Takes a forward's returned tuple after it consumed ``new_tokens``."""
        for i, st in enumerate(past_key_values):
            self.update(i, st)
        self._seen += int(new_tokens)

    def get_seq_length(self) -> int:
        """Tokens consumed so far (the state itself does not grow with them)."""
        return self._seen

    def reorder(self, beam_idx: torch.Tensor) -> None:
        """Select batch rows (beam search): every state, and its normaliser,
        indexed along the batch dimension."""
        out = []
        for st in self._states:
            if st is None:
                out.append(None)
                continue
            S, Z = _split(st)
            idx = beam_idx.to(S.device)
            S2 = S.index_select(0, idx)
            if Z is not None:
                S2.Z = Z.index_select(0, idx.to(Z.device))
            out.append(S2)
        self._states = out

    def memory_bytes(self) -> int:
        """Device bytes held: fixed per layer, whatever the length."""
        total = 0
        for st in self._states:
            if st is None:
                continue
            S, Z = _split(st)
            total += S.numel() * S.element_size() + (Z.numel() * Z.element_size() if Z is not None else 0)
        return total
