"""Linear-attention autograd surface of subq_audio, on the B200 kernels.

Same public names, signatures and semantics as the reference's
python/subq_audio/autograd.py: ``feature_map``, ``feature_map_prime``,
``chunkwise_flash_linear_attention`` (:379-438), ``SubQAttentionFunction``
(:547-660), ``SubQLinearAttention`` (:663-772). The scan itself runs in the
CUDA kernels of libsubq_b200.so; there is no torch fallback, and CPU tensors
are staged through the GPU.

Differences a caller can see:
  * the carried state S (and S.Z) is float32 whatever the input dtype (the
    reference keeps it in q.dtype, where a float16 Z overflows past ~65k
    tokens);
  * ``chunk_size`` is accepted for compatibility; the kernels choose their
    own tiling, and results do not depend on it beyond float rounding.
"""
from __future__ import annotations

import math
from typing import Any, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import library as _library  # noqa: F401  (registers torch.ops.subq_audio)
from . import ops

StateLike = Optional[Union[torch.Tensor, Tuple[torch.Tensor, ...]]]


def feature_map(x: torch.Tensor) -> torch.Tensor:
    """phi(x) = ELU(x) + 1 (positive feature map)."""
    return F.elu(x) + 1.0


def feature_map_prime(x: torch.Tensor) -> torch.Tensor:
    """phi'(x) = 1 for x > 0 else exp(x)."""
    return torch.where(x > 0.0, torch.ones_like(x), torch.exp(x))


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         unsqueeze_dim: int = 1) -> Tuple[torch.Tensor, torch.Tensor]:
    if cos.ndim == 3 and q.ndim == 4:
        cos = cos.unsqueeze(unsqueeze_dim)
        sin = sin.unsqueeze(unsqueeze_dim)
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


def _normalize_attention_mask(attention_mask: Optional[torch.Tensor], target_dtype: torch.dtype,
                              target_len: int) -> Optional[torch.Tensor]:
    """2-D/3-D/4-D bool/int/float mask -> active-token mask [B, 1, T, 1].

    Rules of the reference (autograd.py:57-105): bool as is; float masks are
    additive (< -1 means masked) or multiplicative (> 0 means live); a 4-D
    mask marks a token live when it is a live query and a live key.
    """
    if attention_mask is None:
        return None
    m = attention_mask
    if m.dtype == torch.bool:
        valid = m.to(dtype=target_dtype)
    elif torch.is_floating_point(m):
        valid = ((m >= -1.0) if bool((m < -1.0).any()) else (m > 0.0)).to(dtype=target_dtype)
    else:
        valid = (m != 0).to(dtype=target_dtype)
    if valid.ndim == 2:
        return valid[:, None, :, None]
    if valid.ndim == 3:
        if valid.shape[1] == 1 and valid.shape[2] == target_len:
            return valid.unsqueeze(-1)
        if valid.shape[2] == 1 and valid.shape[1] == target_len:
            return valid.unsqueeze(1)
        red = (valid.sum(dim=-1, keepdim=True) > 0).to(dtype=target_dtype)
        return red.unsqueeze(1) if red.shape[1] == target_len else red
    if valid.ndim == 4:
        if valid.shape[-2] != valid.shape[-1]:
            raise ValueError(f"4D attention_mask must be square [B, 1|H, T, T]; got {tuple(valid.shape)}")
        live_q = valid.sum(dim=-1) > 0
        live_k = valid.sum(dim=-2) > 0
        out = (live_q & live_k).to(dtype=target_dtype).unsqueeze(-1)
        return out[:, :1] if out.shape[1] > 1 else out
    return valid


def _token_mask(valid_mask: Optional[torch.Tensor], B: int, T: int, device) -> Optional[torch.Tensor]:
    """[B,1,T,1] active mask -> [B, T] uint8 for the kernels."""
    if valid_mask is None:
        return None
    m = valid_mask.reshape(valid_mask.shape[0], -1)[:, :T] if valid_mask.ndim != 4 else valid_mask[:, 0, :, 0]
    m = m.expand(B, T)
    return (m != 0).to(device=device, dtype=torch.uint8).contiguous()


def _log_gamma(decay_w: Any, B: int, H: int, T: int, device, dtype=torch.float32):
    """``-softplus(-w)`` in the reference's broadcast layout (autograd.py:310-333).

    Returns None for "no decay" (w is None), else a differentiable float32
    tensor of shape [] / [H] / [B,H,T].
    """
    if decay_w is None:
        return None
    w = decay_w if isinstance(decay_w, torch.Tensor) else torch.tensor(decay_w, device=device)
    w = w.to(device=device, dtype=dtype)
    lg = -F.softplus(-w)
    if w.ndim == 0:
        return lg
    if w.ndim == 1:
        if w.shape[0] == H:
            return lg
        return lg.view(1, 1, -1).expand(B, H, T)
    if w.ndim == 2:
        if w.shape[1] == T:
            return lg.view(B, 1, T).expand(B, H, T)
        return lg.view(B, H, 1).expand(B, H, T)
    if w.ndim == 3 and tuple(w.shape) == (B, H, T):
        return lg
    return lg.expand(B, H, T)


def _split_state(past_state: StateLike):
    if past_state is None:
        return None
    if isinstance(past_state, tuple):
        S = past_state[0]
        Z = past_state[1] if len(past_state) > 1 else None
    else:
        S = past_state
        Z = getattr(past_state, "Z", None)
    return (S, Z)


class _CausalScan(torch.autograd.Function):
    """One scan direction on the kernels (causal, or reverse time for the
    second direction of the bidirectional scan); differentiable in q, k, v,
    log_gamma. Runs the ``subq_audio::scan_fwd`` / ``scan_bwd`` operators
    (traceable: they carry fake kernels); the forward's handover buffer and
    output go to the backward, which then runs in one pass."""

    @staticmethod
    def forward(ctx, q, k, v, lg, mask_u8, S0, z0, want_state, reverse=False):
        lg_t = lg if isinstance(lg, torch.Tensor) else None
        if lg is not None and lg_t is None:
            lg_t = torch.tensor(float(lg), dtype=torch.float32, device=q.device)
        o, S, z, handover = torch.ops.subq_audio.scan_fwd(q, k, v, lg_t, mask_u8, S0, z0, reverse, want_state)
        ctx.reverse = reverse
        ctx.lg_is_tensor = isinstance(lg, torch.Tensor)
        ctx.lg_strided = lg_t is not None and lg_t.dim() == 3 and not lg_t.is_contiguous()
        ctx.save_for_backward(q, k, v, lg_t, mask_u8, S0, z0, o, handover)
        if want_state:
            ctx.mark_non_differentiable(S, z)
            return o, S, z
        return o, None, None

    @staticmethod
    def backward(ctx, do, _dS=None, _dz=None):
        q, k, v, lg, mask_u8, S0, z0, o, handover = ctx.saved_tensors
        need_lg = ctx.lg_is_tensor and ctx.needs_input_grad[3]
        # dO in any layout with a contiguous last dimension (the kernels take strides)
        dq, dk, dv, dlg = torch.ops.subq_audio.scan_bwd(q, k, v, do, lg, mask_u8, S0, z0, o, handover,
                                                        ctx.reverse, need_lg)
        glg = None
        if need_lg:
            glg = dlg.to(lg.dtype)
            if ctx.lg_strided:
                # the gradient in log(gamma)'s own memory order (a [B, H, N] view of a
                # gate projection's [B, N, H] output): the elementwise backward ops that
                # follow then see one layout, for which torch's fake (tracing) and real
                # kernels agree on the output strides
                glg = torch.empty_like(lg).copy_(glg)
            if lg.dim() == 0:
                glg = glg.sum()
            elif lg.dim() == 1:
                glg = glg.sum(dim=(0, 2))
        return dq, dk, dv, glg, None, None, None, None, None


class _HeadRMSNorm(torch.autograd.Function):
    """Per-head RMSNorm of the scan's output on the library's kernels
    (``subq_audio::head_rmsnorm_fwd`` / ``_bwd``): the reference's
    ``nn.RMSNorm(head_dim)`` and the transpose copy after it
    (python/subq_audio/autograd.py:763-769). The output is a [B, H, N, D] view
    of a [B, N, H, D] buffer, so the transpose back for the output projection
    is a view; the backward recomputes the row scale from x."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        y = torch.ops.subq_audio.head_rmsnorm_fwd(x, weight, eps)
        ctx.eps = eps
        ctx.save_for_backward(x, weight)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx, dw = torch.ops.subq_audio.head_rmsnorm_bwd(dy, x, w, ctx.eps)
        gw = dw.to(w.dtype) if (w is not None and ctx.needs_input_grad[1]) else None
        return dx, gw, None


def _to_device_inputs(q, k, v):
    if q.is_cuda:
        return q, k, v, None
    if not torch.cuda.is_available():
        raise RuntimeError("subq_audio needs a CUDA device: the scan runs only in its B200 kernels")
    dev = torch.device("cuda", torch.cuda.current_device())
    return q.to(dev), k.to(dev), v.to(dev), q.device


def _single_direction(q, k, v, decay_w, past_state, valid_mask, want_state, reverse=False):
    B, H, T, D = q.shape
    lg = _log_gamma(decay_w, B, H, T, q.device)
    mask_u8 = _token_mask(valid_mask, B, T, q.device)
    st = _split_state(past_state)
    S0 = Z0 = None
    if st is not None:
        S0, Z0 = st
        S0 = S0.detach().to(device=q.device, dtype=torch.float32).reshape(B, H, D, v.shape[-1]).contiguous()
        Z0 = None if Z0 is None else Z0.detach().to(device=q.device, dtype=torch.float32).reshape(B, H, D).contiguous()
    o, S_next, z_next = _CausalScan.apply(q, k, v, lg, mask_u8, S0, Z0, want_state, reverse)
    return o, S_next, z_next


def chunkwise_flash_linear_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, decay_w: Any,
                                     past_state: StateLike = None, chunk_size: int = 64,
                                     attention_mask: Optional[torch.Tensor] = None,
                                     is_causal: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """Normalised ELU+1 linear attention (reference autograd.py:379-438).

    ``q, k, v`` are [B,T,D] or [B,H,T,D]; ``decay_w`` is the decay logit
    (gamma = sigmoid(w)) as a scalar, [H], [B,T], [B,H] or [B,H,T], or None
    for gamma == 1. Returns ``(out, S_next)`` with ``S_next.Z`` attached.
    """
    out, S_next = _chunkwise(q, k, v, decay_w, past_state, attention_mask, is_causal)
    return out.contiguous(), S_next


def _chunkwise(q, k, v, decay_w, past_state, attention_mask, is_causal, want_state=True):
    """chunkwise_flash_linear_attention with ``out`` in q's memory order (a
    [B, H, T, D] view of a [B, T, H, D] buffer when q is a view of a
    projection's output), for callers that transpose it back. Without
    ``want_state`` the final state is not formed (None is returned for it)."""
    is_3d = q.ndim == 3
    if is_3d:
        q, k, v = q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1)
    q, k, v, home = _to_device_inputs(q, k, v)
    B, H, T, D = q.shape
    valid_mask = _normalize_attention_mask(
        attention_mask.to(q.device) if attention_mask is not None else None, q.dtype, T)
    out, S_next, z_next = _single_direction(q, k, v, decay_w, past_state, valid_mask, want_state)
    if not is_causal:
        # Bidirectional: add the reverse-time scan and remove the double-counted
        # diagonal (in normalised linear attention the self term is v). The
        # kernels run the reverse direction in place of the reference's scan of
        # time-flipped copies (the same decay between tokens, no copies).
        out_b, _, _ = _single_direction(q, k, v, decay_w, None, valid_mask, False, reverse=True)
        vq = v if v.shape[1] == q.shape[1] else v.repeat_interleave(q.shape[1] // v.shape[1], dim=1)
        diag = vq if valid_mask is None else vq * valid_mask.expand_as(vq)
        out = out + out_b - diag
        if valid_mask is not None:
            out = out * valid_mask.expand_as(out)
    if want_state:
        S_next = S_next.to(q.device)
        S_next.Z = z_next.unsqueeze(-1)
    if is_3d:
        out = out.squeeze(1)
    if home is not None:
        out = out.to(home)
    return out, S_next


def _reduce_dw(dlg: torch.Tensor, w: torch.Tensor, B: int, H: int, T: int) -> torch.Tensor:
    """d loss / d w from the per-token d loss / d log(gamma) (reference autograd.py:526-542)."""
    sg = torch.sigmoid(-w.to(torch.float32))
    if w.ndim == 0:
        return (dlg * sg).sum()
    if w.ndim == 1:
        if w.shape[0] == H:
            return (dlg * sg.view(1, H, 1)).sum(dim=(0, 2))
        return (dlg * sg.view(1, 1, -1)).sum(dim=(0, 1))
    if w.ndim == 2:
        if w.shape[1] == T:
            return (dlg * sg.view(B, 1, T)).sum(dim=1)
        return (dlg * sg.view(B, H, 1)).sum(dim=-1)
    if w.ndim == 3:
        return dlg * sg
    return dlg.sum()


def _direction_grads(q, k, v, w, do, valid_mask, reverse=False):
    B, H, T, D = q.shape
    lg = None if w is None else _log_gamma(w.detach(), B, H, T, q.device)
    mask_u8 = _token_mask(valid_mask, B, T, q.device)
    dq, dk, dv, dlg = ops.scan_backward(q, k, v, do.contiguous(), log_gamma=lg, mask=mask_u8, normalize=True,
                                        need_dlog_gamma=w is not None, reverse=reverse)
    dw = None if w is None else _reduce_dw(dlg, w, B, H, T)
    return dq, dk, dv, dw


class SubQAttentionFunction(torch.autograd.Function):
    """Analytic autograd bridge (reference autograd.py:547-660).

    ``apply(q, k, v, decay_w, chunk_size=64, attention_mask=None, is_causal=True)``.
    Saves exactly (q, k, v, decay_w): the backward recomputes the forward
    states in the kernels, so memory stays O(inputs).
    """

    @staticmethod
    def forward(ctx, q, k, v, decay_w, chunk_size: int = 64, attention_mask=None, is_causal: bool = True):
        if q.shape != k.shape or q.shape != v.shape:
            raise ValueError(f"Shape mismatch: Q:{q.shape}, K:{k.shape}, V:{v.shape}")
        with torch.no_grad():
            out, _ = chunkwise_flash_linear_attention(q, k, v, decay_w, chunk_size=chunk_size,
                                                      attention_mask=attention_mask, is_causal=is_causal)
        if decay_w is None:  # gamma == 1; a placeholder keeps save_for_backward uniform
            w_t = torch.zeros((), dtype=q.dtype, device=q.device)
        elif isinstance(decay_w, torch.Tensor):
            w_t = decay_w
        else:
            w_t = torch.tensor(decay_w, dtype=q.dtype, device=q.device)
        ctx.save_for_backward(q, k, v, w_t)
        ctx.is_3d = q.ndim == 3
        ctx.is_causal = is_causal
        ctx.decay_none = decay_w is None
        T = q.shape[-2]
        ctx.valid_mask = (_normalize_attention_mask(attention_mask, q.dtype, T)
                          if attention_mask is not None else None)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, w = ctx.saved_tensors
        home = None
        if not q.is_cuda:
            home = q.device
        q4, k4, v4, g4 = (x.unsqueeze(1) if ctx.is_3d else x for x in (q, k, v, grad_output))
        q4, k4, v4, _ = _to_device_inputs(q4, k4, v4)
        g4 = g4.to(q4.device)
        w_dev = None if ctx.decay_none else w.to(q4.device)
        vm = ctx.valid_mask.to(q4.device) if ctx.valid_mask is not None else None
        dQ, dK, dV, dw = _direction_grads(q4, k4, v4, w_dev, g4, vm)
        if not ctx.is_causal:  # the reverse-time direction (reference: on time-flipped copies)
            dQb, dKb, dVb, dwb = _direction_grads(q4, k4, v4, w_dev, g4, vm, reverse=True)
            g_m = g4 if vm is None else g4 * vm.expand_as(g4)
            dQ = dQ + dQb
            dK = dK + dKb
            dV = dV + dVb - g_m
            if dw is not None:
                dw = dw + dwb
        if ctx.is_3d:
            dQ, dK, dV = dQ.squeeze(1), dK.squeeze(1), dV.squeeze(1)
        dw_out = None if dw is None else dw.to(w.dtype).reshape(w.shape)
        grads = [dQ.contiguous(), dK.contiguous(), dV.contiguous(), dw_out]
        if home is not None:
            grads = [g.to(home) if g is not None else None for g in grads]
        return tuple(grads) + (None, None, None)


class SubQLinearAttention(nn.Module):
    """Linear-attention layer (reference autograd.py:663-772): q/k/v/out
    projections, optional RoPE, GQA, learnable base decay with optional
    data-dependent gating, per-head RMSNorm. The scan is the B200 kernel.
    """

    def __init__(self, hidden_size: int, num_heads: int = 1, num_key_value_heads: Optional[int] = None,
                 decay_init: float = 0.99, bias: bool = False, use_data_dependent_gating: bool = True,
                 is_causal: bool = True):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_key_value_heads = num_key_value_heads if num_key_value_heads is not None else num_heads
        self.head_dim = hidden_size // num_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.use_data_dependent_gating = use_data_dependent_gating
        self.is_causal = is_causal
        if self.head_dim * num_heads != hidden_size:
            raise ValueError(f"hidden_size {hidden_size} must be divisible by num_heads {num_heads}")
        if self.num_heads % self.num_key_value_heads != 0:
            raise ValueError(f"num_heads {num_heads} must be divisible by num_key_value_heads "
                             f"{self.num_key_value_heads}")
        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=bias)
        self.k_proj = nn.Linear(hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)
        self.out_proj = nn.Linear(hidden_size, hidden_size, bias=bias)
        self.head_norm = nn.RMSNorm(self.head_dim, eps=1e-5) if hasattr(nn, "RMSNorm") else None
        d0 = min(max(decay_init, 1e-4), 1.0 - 1e-4)
        self.raw_decay = nn.Parameter(torch.full((num_heads,), math.log(d0 / (1.0 - d0)), dtype=torch.float32))
        self.gate_proj = nn.Linear(hidden_size, num_heads, bias=bias) if use_data_dependent_gating else None

    @property
    def decay_factor(self) -> torch.Tensor:
        return torch.sigmoid(self.raw_decay)

    def _fused_projections(self, x: torch.Tensor):
        """q, k, v and the gate from ONE GEMM over the concatenated weights
        (rows padded to a multiple of 8, so every output row starts on a 16-byte
        boundary), returned as strided views of its [B, L, R] output. Against
        four nn.Linear calls this casts x once under autocast, and its backward
        forms dx in one GEMM instead of four GEMMs and three adds. The
        parameters stay the four Linear modules (the reference's state-dict
        names); their gradients come back through the concatenation. None when
        a projection is not a plain nn.Linear or the sizes do not align."""
        mods = [self.q_proj, self.k_proj, self.v_proj]
        if self.use_data_dependent_gating and self.gate_proj is not None:
            mods.append(self.gate_proj)
        if not x.is_cuda or any(type(m) is not nn.Linear for m in mods):
            return None
        outs = [m.out_features for m in mods]
        if any(o % 8 for o in outs[:3]):
            return None
        rows = sum(outs)
        pad = -rows % 8
        ws = [m.weight for m in mods]
        if len({(w.dtype, w.device) for w in ws}) != 1:
            return None
        if pad:
            ws.append(ws[0].new_zeros(pad, ws[0].shape[1]))
        has_bias = [m.bias is not None for m in mods]
        bias = None
        if any(has_bias):
            bs = [m.bias if m.bias is not None else ws[0].new_zeros(o) for m, o in zip(mods, outs)]
            if pad:
                bs.append(ws[0].new_zeros(pad))
            bias = torch.cat(bs)
        y = F.linear(x, torch.cat(ws), bias)
        # split, not slicing: its backward writes the one [B, L, R] gradient with a
        # single concatenation (a slice's backward zero-fills a full-size gradient
        # per slice and then sums them)
        return list(torch.split(y, outs + ([pad] if pad else []), dim=-1))[:len(outs)]

    def forward(self, hidden_states: torch.Tensor, past_state: StateLike = None,
                attention_mask: Optional[torch.Tensor] = None, use_cache: bool = False,
                position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, **kwargs: Any):
        B, L, _ = hidden_states.shape
        fused = self._fused_projections(hidden_states)
        if fused is not None:
            q, k, v = fused[:3]
            gate_lin = fused[3] if len(fused) > 3 else None
        else:
            q, k, v = self.q_proj(hidden_states), self.k_proj(hidden_states), self.v_proj(hidden_states)
            gate_lin = None
        Q = q.view(B, L, self.num_heads, self.head_dim).transpose(1, 2)
        K = k.view(B, L, self.num_key_value_heads, self.head_dim).transpose(1, 2)
        V = v.view(B, L, self.num_key_value_heads, self.head_dim).transpose(1, 2)
        if position_embeddings is not None:
            cos, sin = position_embeddings
            Q, K = apply_rotary_pos_emb(Q, K, cos, sin)
        # grouped K/V (num_key_value_groups > 1) go to the kernels as they are:
        # query head h reads K/V head h // groups, and the backward sums dK, dV
        # over each group (the reference's repeat_interleave, autograd.py:746-748)
        if self.use_data_dependent_gating and self.gate_proj is not None:
            gate = (gate_lin if gate_lin is not None else self.gate_proj(hidden_states)).transpose(1, 2)
            decay_w = self.raw_decay.view(1, self.num_heads, 1) + gate
        else:
            decay_w = self.raw_decay
        # the scan writes out in Q's memory order ([B, L, H, D] under the [B, H, L, D]
        # view), so the transpose back below needs no copy
        out, next_state = _chunkwise(Q, K, V, decay_w, past_state, attention_mask, self.is_causal,
                                     want_state=use_cache)
        if ops.head_rmsnorm_supported(out):
            # the library's per-head RMSNorm (float32 math with the float32 weight);
            # it writes [B, L, H, D] memory, so the transpose back is a view
            w = self.head_norm.weight if self.head_norm is not None else None
            eps = self.head_norm.eps if (self.head_norm is not None and self.head_norm.eps is not None) else 1e-5
            out = _HeadRMSNorm.apply(out, w, eps)
            out = out.transpose(1, 2).reshape(B, L, self.hidden_size)
        else:
            if self.head_norm is not None:
                out = self.head_norm(out)
            else:
                out = out * torch.rsqrt(out.pow(2).mean(-1, keepdim=True) + 1e-5)
            out = out.transpose(1, 2).contiguous().view(B, L, self.hidden_size)
        return self.out_proj(out), (next_state if use_cache else None)


SubQuadraticAttention = SubQLinearAttention
