"""Attention surgery: swap softmax self-attention blocks for SubQLinearAttention.

Behaviour follows the reference's python/subq_audio/surgery.py:
  * ``SubQAttentionOutput`` (:31-84): a tuple ``(out, None)`` or
    ``(out, None, past)`` that also behaves like the output tensor;
  * ``SubQBypassAttention`` (:86-150): the Hugging Face call contract around
    a ``SubQLinearAttention`` core;
  * ``bypass_transformer_with_subq`` (:161-331): finds modules whose name ends
    in one of ``target_select_suffixes`` and that own q/k/v/out Linear
    projections, infers heads, key-value heads and causality (a path or class
    name containing "encoder", or "bert" in the path, makes it bidirectional),
    copies the projection weights and zero-initialises the decay gate.
The layer-wise distillation trainer of that file is not part of this package.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .autograd import SubQLinearAttention

_Q_NAMES = ("q_proj", "query", "q", "in_proj_q")
_K_NAMES = ("k_proj", "key", "k", "in_proj_k")
_V_NAMES = ("v_proj", "value", "v", "in_proj_v")
_O_NAMES = ("out_proj", "o_proj", "dense", "proj", "c_proj")


class SubQAttentionOutput(tuple):
    """Tuple result that also acts as its first element (the attention output)."""

    def __new__(cls, output: torch.Tensor, attn_weights: Optional[torch.Tensor] = None,
                past_state: Optional[torch.Tensor] = None, return_tuple_arity: int = 2):
        items = (output, attn_weights, past_state) if return_tuple_arity == 3 else (output, attn_weights)
        obj = super().__new__(cls, items)
        obj.past_state = past_state
        return obj

    @property
    def output(self) -> torch.Tensor:
        return self[0]

    def __add__(self, other):
        return self[0] + other

    def __radd__(self, other):
        return other + self[0]

    def __sub__(self, other):
        return self[0] - other

    def __rsub__(self, other):
        return other - self[0]

    def __mul__(self, other):
        return self[0] * other

    def __rmul__(self, other):
        return other * self[0]

    def __truediv__(self, other):
        return self[0] / other

    def __rtruediv__(self, other):
        return other / self[0]

    def __getattr__(self, name):
        return getattr(self[0], name)


class SubQBypassAttention(nn.Module):
    """Hugging Face attention-block contract around a SubQLinearAttention core."""

    def __init__(self, core_attn: SubQLinearAttention, return_tuple_arity: int = 2):
        super().__init__()
        self.core = core_attn
        self.hidden_size = core_attn.hidden_size
        self.num_heads = core_attn.num_heads
        self.num_key_value_heads = core_attn.num_key_value_heads
        self.head_dim = core_attn.head_dim
        self.is_causal = core_attn.is_causal
        self.return_tuple_arity = return_tuple_arity
        self.q_proj, self.k_proj, self.v_proj = core_attn.q_proj, core_attn.k_proj, core_attn.v_proj
        self.out_proj, self.gate_proj, self.raw_decay = core_attn.out_proj, core_attn.gate_proj, core_attn.raw_decay

    @property
    def decay_factor(self) -> torch.Tensor:
        return self.core.decay_factor

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None, past_key_value: Optional[Any] = None,
                output_attentions: bool = False, use_cache: bool = False,
                cache_position: Optional[torch.Tensor] = None, **kwargs: Any) -> SubQAttentionOutput:
        past = past_key_value if isinstance(past_key_value, torch.Tensor) else None
        pos_emb = kwargs.pop("position_embeddings", None)
        self.core.is_causal = self.is_causal
        out, nxt = self.core(hidden_states=hidden_states, past_state=past, attention_mask=attention_mask,
                             use_cache=use_cache, position_embeddings=pos_emb, **kwargs)
        keep_past = self.return_tuple_arity == 3 or (use_cache and nxt is not None)
        return SubQAttentionOutput(out, None, nxt if keep_past else None,
                                   return_tuple_arity=self.return_tuple_arity)


def _linear_child(module: nn.Module, names: Tuple[str, ...]):
    for name, child in module.named_children():
        if isinstance(child, nn.Linear) and name.lower() in names:
            return name, child
    return None


def _first_attr(objs, names):
    for o in objs:
        if o is None:
            continue
        for n in names:
            val = getattr(o, n, None)
            if val:
                return val
    return None


def bypass_transformer_with_subq(model: nn.Module,
                                 target_select_suffixes: Tuple[str, ...] = ("self_attn", "attention", "attn"),
                                 decay_init: float = 0.99, use_data_dependent_gating: bool = True,
                                 copy_weights: bool = True, verbose: bool = False
                                 ) -> Tuple[nn.Module, List[Dict[str, Any]]]:
    """Replace every matching attention block in ``model`` (in place).

    Returns ``(model, replaced)`` with one metadata dict per replaced block.
    """
    replaced: List[Dict[str, Any]] = []
    cfg = getattr(model, "config", None)

    def visit(parent: nn.Module, prefix: str) -> None:
        for name, child in list(parent.named_children()):
            path = f"{prefix}.{name}" if prefix else name
            if isinstance(child, (SubQLinearAttention, SubQBypassAttention)):
                continue
            suffix_ok = (any(name.lower().endswith(s.lower()) for s in target_select_suffixes)
                         if target_select_suffixes else True)
            found = [_linear_child(child, n) for n in (_Q_NAMES, _K_NAMES, _V_NAMES, _O_NAMES)]
            if not (suffix_ok and all(found)):
                visit(child, path)
                continue
            (_, q), (_, k), (_, v), (_, o) = found
            hidden = q.in_features
            heads = (_first_attr([child], ("num_heads", "num_attention_heads", "n_heads"))
                     or _first_attr([cfg], ("num_attention_heads", "encoder_attention_heads")) or 1)
            head_dim = q.out_features // heads if hidden % heads else hidden // heads
            kv_heads = (_first_attr([child], ("num_key_value_heads", "num_key_value_groups"))
                        or _first_attr([cfg], ("num_key_value_heads",))
                        or (k.out_features // head_dim if head_dim > 0 else heads))
            if kv_heads <= 0 or heads % kv_heads:
                kv_heads = heads
            causal = getattr(child, "is_causal", None)
            if causal is None:
                if getattr(child, "is_decoder", None) is False:
                    causal = False
                else:
                    low = path.lower()
                    causal = not ("encoder" in low or "bert" in low or "encoder" in type(child).__name__.lower())
            bias = q.bias is not None
            core = SubQLinearAttention(hidden_size=hidden, num_heads=heads, num_key_value_heads=kv_heads,
                                       decay_init=decay_init, bias=bias,
                                       use_data_dependent_gating=use_data_dependent_gating,
                                       is_causal=causal).to(device=q.weight.device, dtype=q.weight.dtype)
            if copy_weights:
                with torch.no_grad():
                    for dst, src in ((core.q_proj, q), (core.k_proj, k), (core.v_proj, v), (core.out_proj, o)):
                        dst.weight.copy_(src.weight)
                        if bias and src.bias is not None and dst.bias is not None:
                            dst.bias.copy_(src.bias)
                    if core.gate_proj is not None:
                        core.gate_proj.weight.zero_()
                        if core.gate_proj.bias is not None:
                            core.gate_proj.bias.zero_()
            setattr(parent, name, SubQBypassAttention(core, return_tuple_arity=2))
            info = {"path": path, "hidden_size": hidden, "num_heads": heads, "num_key_value_heads": kv_heads,
                    "is_causal": causal, "has_bias": bias}
            replaced.append(info)
            if verbose:
                print(f"[Surgery] Replaced {path} -> SubQLinearAttention (H={heads}, KV_H={kv_heads}, "
                      f"D={hidden}, causal={causal})")

    visit(model, "")
    return model, replaced
