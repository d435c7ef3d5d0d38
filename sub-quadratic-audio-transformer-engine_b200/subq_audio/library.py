"""The scan as torch operators: ``torch.ops.subq_audio.scan_fwd`` and
``torch.ops.subq_audio.scan_bwd`` (normalised form, the model path of
``SubQLinearAttention`` / ``chunkwise_flash_linear_attention``).

Registered with ``torch.library`` with fake (meta) kernels, so a model that
calls them can be traced by ``torch.compile`` / ``torch.export`` without a
graph break: the fake kernels give the outputs' shapes, dtypes and memory
order (the output follows q's memory order, as ``ops.scan_forward`` writes
it) and the size of the forward's handover buffer, which is a function of
the shapes only. The real kernels are the C-ABI calls of ``ops``.

    o, S, z, handover = torch.ops.subq_audio.scan_fwd(q, k, v, log_gamma, mask, S0, z0, reverse, want_state)
    dq, dk, dv, dlog_gamma = torch.ops.subq_audio.scan_bwd(q, k, v, dout, log_gamma, mask, S0, z0, o,
                                                           handover, reverse, need_dlog_gamma)

``log_gamma`` is None or float32 ([], [H] or [B, H, N]); ``mask`` None or a
uint8 / bool [B, N]; ``S0`` [B, H, d, e] and ``z0`` [B, H, d] float32 or
None. Outputs that a call does not produce (S, z without ``want_state``, the
handover off the tensor-core path, d log(gamma) without ``need_dlog_gamma``)
are empty tensors.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _capi, ops

Tensor = torch.Tensor
_FAKE_PTR = 1 << 16  # a 16-byte-aligned stand-in address: the size query reads no memory


def _handover_bytes(q: Tensor, k: Tensor, v: Tensor, log_gamma: Optional[Tensor], mask: Optional[Tensor],
                    reverse: bool) -> int:
    """Bytes of the forward's handover buffer for these shapes and strides
    (subq_segment_states_bytes; no tensor data is read)."""
    B, H, N, d = q.shape
    a = _capi.FwdArgs()
    desc = a.desc
    desc.batch, desc.heads, desc.seq_len, desc.head_dim, desc.value_dim = B, H, N, d, v.shape[-1]
    desc.kv_heads = v.shape[1] if v.shape[1] != H else 0
    desc.dtype = ops._DTYPES[q.dtype]
    desc.normalize = 1
    desc.scale = 1.0 / math.sqrt(d)
    desc.clamp_min = 1e-5
    desc.path = _capi.SUBQ_PATH_AUTO
    desc.reverse = 1 if reverse else 0
    if log_gamma is not None:
        desc.decay_mode = _capi.SUBQ_DECAY_PER_TOKEN
        desc.log_gamma = _FAKE_PTR
    if mask is not None:
        desc.mask = _FAKE_PTR
        desc.mask_stride_b = N
    # (o is allocated in q's memory order; the size depends on its strides only
    # through their alignment, which q's share)
    for name, t in (("q", q), ("k", k), ("v", v), ("o", q)):
        t4 = getattr(a, name)
        t4.data = _FAKE_PTR
        t4.stride_b, t4.stride_h, t4.stride_n = t.stride(0), t.stride(1), t.stride(2)
    with torch.cuda.device(q.device):
        return _capi.segment_states_bytes(a)


def _empty_f32(ref: Tensor, shape) -> Tensor:
    return torch.empty(shape, dtype=torch.float32, device=ref.device)


@torch.library.custom_op("subq_audio::scan_fwd", mutates_args=(), device_types="cuda")
def scan_fwd(q: Tensor, k: Tensor, v: Tensor, log_gamma: Optional[Tensor], mask: Optional[Tensor],
             S0: Optional[Tensor], z0: Optional[Tensor], reverse: bool,
             want_state: bool) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    seg = ops.SegmentStates()
    state = None if S0 is None else (S0, z0)
    o, st = ops.scan_forward(q, k, v, log_gamma=log_gamma, mask=mask, normalize=True, state=state,
                             return_state=want_state, reverse=reverse, segments=seg)
    S, z = st if want_state else (_empty_f32(q, (0,)), _empty_f32(q, (0,)))
    handover = seg.buf if seg.buf is not None else torch.empty(0, dtype=torch.uint8, device=q.device)
    return o, S, z, handover


@scan_fwd.register_fake
def _scan_fwd_fake(q, k, v, log_gamma, mask, S0, z0, reverse, want_state):
    B, H, N, d = q.shape
    e = v.shape[-1]
    o = ops._empty_in_order(q, (B, H, N, e), q.dtype)
    if want_state:
        S, z = _empty_f32(q, (B, H, d, e)), _empty_f32(q, (B, H, d))
    else:
        S, z = _empty_f32(q, (0,)), _empty_f32(q, (0,))
    nbytes = _handover_bytes(q, k, v, log_gamma, mask, reverse)
    return o, S, z, torch.empty(nbytes, dtype=torch.uint8, device=q.device)


@torch.library.custom_op("subq_audio::scan_bwd", mutates_args=(), device_types="cuda")
def scan_bwd(q: Tensor, k: Tensor, v: Tensor, dout: Tensor, log_gamma: Optional[Tensor], mask: Optional[Tensor],
             S0: Optional[Tensor], z0: Optional[Tensor], o: Tensor, handover: Tensor, reverse: bool,
             need_dlog_gamma: bool) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    seg = None
    if handover.numel() > 0:
        seg = ops.SegmentStates()
        seg.buf = handover
    state = None if S0 is None else (S0, z0)
    dq, dk, dv, dlg = ops.scan_backward(q, k, v, dout, log_gamma=log_gamma, mask=mask, normalize=True, state=state,
                                        need_dlog_gamma=need_dlog_gamma, reverse=reverse, segments=seg,
                                        forward_out=o if seg is not None else None)
    if dlg is None:
        dlg = _empty_f32(q, (0,))
    return dq, dk, dv, dlg


@scan_bwd.register_fake
def _scan_bwd_fake(q, k, v, dout, log_gamma, mask, S0, z0, o, handover, reverse, need_dlog_gamma):
    B, H, N, _ = q.shape
    dq = ops._empty_in_order(q, tuple(q.shape), q.dtype)
    dk = ops._empty_in_order(k, tuple(k.shape), q.dtype)
    dv = ops._empty_in_order(v, tuple(v.shape), q.dtype)
    dlg = _empty_f32(q, (B, H, N) if need_dlog_gamma else (0,))
    return dq, dk, dv, dlg


# Per-head RMSNorm of the scan's output (the module epilogue):
#     y = torch.ops.subq_audio.head_rmsnorm_fwd(x, weight, eps)
#     dx, dweight = torch.ops.subq_audio.head_rmsnorm_bwd(dy, x, weight, eps)
# y is a [B, H, N, D] view of a [B, N, H, D] buffer; dweight is float32 [D]
# (empty without a weight).
@torch.library.custom_op("subq_audio::head_rmsnorm_fwd", mutates_args=(), device_types="cuda")
def head_rmsnorm_fwd(x: Tensor, weight: Optional[Tensor], eps: float) -> Tensor:
    return ops.head_rmsnorm(x, weight, eps)


@head_rmsnorm_fwd.register_fake
def _head_rmsnorm_fwd_fake(x, weight, eps):
    B, H, N, D = x.shape
    return x.new_empty((B, N, H, D)).transpose(1, 2)


@torch.library.custom_op("subq_audio::head_rmsnorm_bwd", mutates_args=(), device_types="cuda")
def head_rmsnorm_bwd(dy: Tensor, x: Tensor, weight: Optional[Tensor], eps: float) -> Tuple[Tensor, Tensor]:
    dx, dw = ops.head_rmsnorm_backward(dy, x, weight, eps, need_dweight=weight is not None)
    return dx, (dw if dw is not None else _empty_f32(x, (0,)))


@head_rmsnorm_bwd.register_fake
def _head_rmsnorm_bwd_fake(dy, x, weight, eps):
    dx = ops._empty_in_order(x, tuple(x.shape), x.dtype)
    return dx, _empty_f32(x, (x.shape[-1],) if weight is not None else (0,))
