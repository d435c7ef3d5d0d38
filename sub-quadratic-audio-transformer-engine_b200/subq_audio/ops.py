"""Torch-facing launchers of the B200 scan kernels (through the C ABI).

Tensors are [B, H, N, D] CUDA tensors (any strides with a contiguous last
dimension). Computation is stream-ordered on torch's current stream; the
only host work is argument packing. There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple, Union

import torch

from . import _capi

_DTYPES = {torch.float32: _capi.SUBQ_FP32, torch.float16: _capi.SUBQ_FP16, torch.bfloat16: _capi.SUBQ_BF16,
           torch.float64: _capi.SUBQ_FP64}
_PATHS = {"auto": _capi.SUBQ_PATH_AUTO, "exact": _capi.SUBQ_PATH_EXACT, "tensorcore": _capi.SUBQ_PATH_TENSORCORE,
          "chunked": _capi.SUBQ_PATH_CHUNKED}

LogGamma = Union[None, float, torch.Tensor]


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise RuntimeError("subq_audio scan kernels run on CUDA tensors only (there is no CPU path)")


def _t4(t: Optional[torch.Tensor]) -> _capi.Tensor4:
    out = _capi.Tensor4()
    if t is None:
        return out
    if t.dim() != 4:
        raise ValueError(f"expected a [B, H, N, D] tensor, got shape {tuple(t.shape)}")
    sb, sh, sn, sd = t.stride()
    if sd != 1 and t.shape[-1] > 1:
        raise ValueError("the last dimension must be contiguous")
    out.data = t.data_ptr()
    out.stride_b, out.stride_h, out.stride_n = sb, sh, sn
    return out


def _inner_contig(t: torch.Tensor) -> torch.Tensor:
    return t if (t.shape[-1] <= 1 or t.stride(-1) == 1) else t.contiguous()


def _empty_in_order(ref: torch.Tensor, shape, dtype: torch.dtype) -> torch.Tensor:
    """An empty [B, H, N, x] tensor whose memory runs over B, H and N in the
    same order as ``ref``'s. For q, k, v that are [B, H, N, x] views of a
    projection's [B, N, H * x] output, the results are views of a [B, N, H, x]
    buffer, so the transpose back to [B, N, H * x] needs no copy."""
    st = ref.stride()
    order = sorted(range(3), key=lambda i: (-st[i], i))  # outermost first
    if order == [0, 1, 2]:
        return torch.empty(shape, dtype=dtype, device=ref.device)
    buf = torch.empty([shape[i] for i in order] + [shape[3]], dtype=dtype, device=ref.device)
    return buf.permute(*([order.index(i) for i in range(3)] + [3]))


def _check_kv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """k [B, Hkv, N, d] and v [B, Hkv, N, e] with Hkv a divisor of q's H (grouped K/V)."""
    B, H, N, d = q.shape
    if (k.dim() != 4 or v.dim() != 4 or k.shape[0] != B or k.shape[2] != N or k.shape[3] != d
            or v.shape[:3] != k.shape[:3] or k.shape[1] < 1 or H % k.shape[1] != 0):
        raise ValueError(f"shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")


def _desc(q: torch.Tensor, v: torch.Tensor, log_gamma: LogGamma, mask: Optional[torch.Tensor],
          normalize: bool, scale: Optional[float], clamp_min: float, flush_subnormal: bool,
          path: str, keep: list, reverse: bool = False) -> _capi.ScanDesc:
    B, H, N, d = q.shape
    desc = _capi.ScanDesc()
    desc.batch, desc.heads, desc.seq_len, desc.head_dim, desc.value_dim = B, H, N, d, v.shape[-1]
    desc.kv_heads = v.shape[1] if v.shape[1] != H else 0  # grouped K/V (GQA)
    desc.reverse = 1 if reverse else 0
    if q.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {q.dtype}; use float32, float16, bfloat16 or float64")
    desc.dtype = _DTYPES[q.dtype]
    desc.normalize = 1 if normalize else 0
    desc.scale = float(scale) if scale is not None else (1.0 / math.sqrt(d) if normalize else 1.0)
    desc.clamp_min = float(clamp_min)
    desc.flush_subnormal = 1 if flush_subnormal else 0
    desc.path = _PATHS[path]
    if log_gamma is None:
        desc.decay_mode = _capi.SUBQ_DECAY_NONE
    elif isinstance(log_gamma, (float, int)):
        desc.decay_mode = _capi.SUBQ_DECAY_SCALAR
        desc.log_gamma_scalar = float(log_gamma)
    else:
        lg = log_gamma.detach()
        if lg.device != q.device:
            raise ValueError("log_gamma must be on the device of q")
        lg = lg.to(torch.float32)
        if lg.dim() == 0:
            lg = lg.reshape(1).expand(H)
        if lg.dim() == 1 and lg.shape[0] == H:
            desc.decay_mode = _capi.SUBQ_DECAY_PER_HEAD
        else:
            lg = lg.expand(B, H, N)
            desc.decay_mode = _capi.SUBQ_DECAY_PER_TOKEN
        lg = lg.contiguous()
        keep.append(lg)
        desc.log_gamma = lg.data_ptr()
    if mask is not None:
        m = mask.detach()
        if m.dim() != 2 or m.shape[0] != B or m.shape[1] != N:
            raise ValueError(f"mask must be [B, N] = [{B}, {N}], got {tuple(m.shape)}")
        if m.device != q.device:
            raise ValueError("mask must be on the device of q")
        if m.dtype == torch.bool and m.stride(1) == 1:
            m = m.view(torch.uint8)  # same bytes (0/1), no conversion launch
        elif m.dtype != torch.uint8 or m.stride(1) != 1:
            m = (m != 0).to(torch.uint8).contiguous()
        keep.append(m)
        desc.mask = m.data_ptr()
        desc.mask_stride_b = m.stride(0)
    return desc


def _workspace(nbytes: int, device: torch.device, keep: list) -> Tuple[int, int]:
    if nbytes == 0:
        return 0, 0
    buf = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    keep.append(buf)
    ptr = buf.data_ptr()
    return (ptr + 255) // 256 * 256, nbytes


class SegmentStates:
    """Carrier of what a forward hands to the backward of the same inputs:
    pass one instance as ``segments=`` to ``scan_forward`` (which fills it on
    the tensor-core path: the states at the start of each segment and, without
    decay, the state before every chunk and the per-token normalisers) and
    then to ``scan_backward``. With the forward's output as well (``out``, set
    by ``scan_forward``, or ``forward_out=`` of ``scan_backward``) an
    undecayed backward runs in one pass from them; a decayed one skips
    recomputing the segment states. The forward must be the same call's:
    a carrier from other inputs gives wrong gradients."""

    def __init__(self) -> None:
        self.buf: Optional[torch.Tensor] = None
        self.out: Optional[torch.Tensor] = None


def scan_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, log_gamma: LogGamma = None,
                 mask: Optional[torch.Tensor] = None, normalize: bool = True, scale: Optional[float] = None,
                 clamp_min: float = 1e-5, state: Optional[Tuple[torch.Tensor, Optional[torch.Tensor]]] = None,
                 return_state: bool = False, flush_subnormal: bool = False, path: str = "auto",
                 out: Optional[torch.Tensor] = None, reverse: bool = False,
                 segments: Optional[SegmentStates] = None):
    """Causal scan. Returns ``(o, (S, z) | None)``; S [B,H,d,e] and z [B,H,d] are float32.
    ``k`` and ``v`` may have fewer heads than ``q`` (a divisor of H: grouped K/V,
    query head h reading K/V head h // (H // Hkv)); the backward then returns
    dk, dv summed over each group. ``reverse=True`` scans in reverse time
    (token t sees itself and the later tokens; the state runs from the end)."""
    _require_cuda(q, k, v)
    q, k, v = _inner_contig(q), _inner_contig(k), _inner_contig(v)
    _check_kv(q, k, v)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k and v must share one dtype")
    B, H, N, d = q.shape
    e = v.shape[-1]
    keep: list = []
    with torch.cuda.device(q.device):
        o = out if out is not None else _empty_in_order(q, (B, H, N, e), q.dtype)
        a = _capi.FwdArgs()
        a.desc = _desc(q, v, log_gamma, mask, normalize, scale, clamp_min, flush_subnormal, path, keep, reverse)
        a.q, a.k, a.v, a.o = _t4(q), _t4(k), _t4(v), _t4(o)
        S_out = z_out = None
        if state is not None:
            S_in, z_in = state[0], (state[1] if len(state) > 1 else None)
            S_in = S_in.detach().to(torch.float32).reshape(B, H, d, e).contiguous()
            keep.append(S_in)
            a.state_in = S_in.data_ptr()
            if z_in is not None:
                z_in = z_in.detach().to(torch.float32).reshape(B, H, d).contiguous()
                keep.append(z_in)
                a.norm_in = z_in.data_ptr()
        if return_state:
            S_out = torch.empty((B, H, d, e), dtype=torch.float32, device=q.device)
            z_out = torch.zeros((B, H, d), dtype=torch.float32, device=q.device)
            a.state_out = S_out.data_ptr()
            if normalize:
                a.norm_out = z_out.data_ptr()
        a.stream = torch.cuda.current_stream(q.device).cuda_stream
        a.workspace, a.workspace_bytes = _workspace(_capi.fwd_workspace_bytes(a), q.device, keep)
        if segments is not None:
            nbytes = _capi.segment_states_bytes(a)
            segments.buf = torch.empty(nbytes, dtype=torch.uint8, device=q.device) if nbytes else None
            if segments.buf is not None:
                a.segment_states = segments.buf.data_ptr()
            segments.out = o
        _capi.fwd(a)
    return o, ((S_out, z_out) if return_state else None)


def scan_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dout: torch.Tensor, *,
                  log_gamma: LogGamma = None, mask: Optional[torch.Tensor] = None, normalize: bool = True,
                  scale: Optional[float] = None, clamp_min: float = 1e-5,
                  state: Optional[Tuple[torch.Tensor, Optional[torch.Tensor]]] = None,
                  need_dlog_gamma: bool = False, flush_subnormal: bool = False, path: str = "auto",
                  reverse: bool = False, segments: Optional[SegmentStates] = None,
                  forward_out: Optional[torch.Tensor] = None):
    """Gradients of ``scan_forward``. Returns ``(dq, dk, dv, dlog_gamma | None)``;
    dlog_gamma is float32 [B,H,N] (d loss / d log gamma_t per token).
    ``segments`` (and ``forward_out``, else ``segments.out``) come from the
    forward of the same call; see ``SegmentStates``."""
    _require_cuda(q, k, v, dout)
    q, k, v, dout = _inner_contig(q), _inner_contig(k), _inner_contig(v), _inner_contig(dout)
    _check_kv(q, k, v)
    if dout.dtype != q.dtype:
        dout = dout.to(q.dtype)
    B, H, N, d = q.shape
    e = v.shape[-1]
    keep: list = []
    with torch.cuda.device(q.device):
        dq = _empty_in_order(q, (B, H, N, d), q.dtype)
        dk = _empty_in_order(k, tuple(k.shape), q.dtype)  # [B, Hkv, N, d]: summed per K/V group
        dv = _empty_in_order(v, tuple(v.shape), q.dtype)
        a = _capi.BwdArgs()
        a.desc = _desc(q, v, log_gamma, mask, normalize, scale, clamp_min, flush_subnormal, path, keep, reverse)
        a.q, a.k, a.v, a.dout = _t4(q), _t4(k), _t4(v), _t4(dout)
        a.dq, a.dk, a.dv = _t4(dq), _t4(dk), _t4(dv)
        if state is not None:
            S_in = state[0].detach().to(torch.float32).reshape(B, H, d, e).contiguous()
            keep.append(S_in)
            a.state_in = S_in.data_ptr()
            if len(state) > 1 and state[1] is not None:
                z_in = state[1].detach().to(torch.float32).reshape(B, H, d).contiguous()
                keep.append(z_in)
                a.norm_in = z_in.data_ptr()
        dlg = None
        if need_dlog_gamma:
            dlg = torch.empty((B, H, N), dtype=torch.float32, device=q.device)
            a.dlog_gamma = dlg.data_ptr()
        a.stream = torch.cuda.current_stream(q.device).cuda_stream
        if segments is not None and segments.buf is not None and segments.buf.device == q.device:
            a.segment_states = segments.buf.data_ptr()
            fo = forward_out if forward_out is not None else segments.out
            if fo is not None:
                if tuple(fo.shape) != (B, H, N, e) or fo.dtype != q.dtype or fo.device != q.device:
                    raise ValueError("forward_out must be the forward's [B, H, N, e] output")
                fo = _inner_contig(fo)
                keep.append(fo)
                a.out = _t4(fo)
        # (after the handover fields: they decide the kernel path and its workspace)
        a.workspace, a.workspace_bytes = _workspace(_capi.bwd_workspace_bytes(a), q.device, keep)
        _capi.bwd(a)
    return dq, dk, dv, dlg


class DecodeStep:
    """Streaming decode over preallocated device buffers: the serving loop of
    the scan, with the float32 state carried on the device and updated in
    place (the C3 streaming case at its finest grain, one call per new token
    or a few tokens).

    ``q, k`` [B, H, T, d], ``v`` [B, H, T, e] and ``out`` [B, H, T, e] hold the
    step's T new tokens (usually T = 1); ``S`` [B, H, d, e] and, for the
    normalised form, ``z`` [B, H, d] are contiguous float32 state buffers.
    ``log_gamma`` is None, a float, a float32 [H] tensor or a contiguous
    float32 [B, H, T] tensor; ``mask`` a contiguous bool/uint8 [B, T] tensor.
    ``step()`` enqueues one scan call on the current stream: out = the scan of
    the new tokens from (S, z), then (S, z) <- the state after them. It
    allocates nothing and does not synchronise, so a CUDA graph can capture
    it; refill q, k, v (and log_gamma, mask) in place between steps.
    Short steps run on the token-recurrent kernel (see ``subq_fwd``'s path
    choice).
    """

    def __init__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, S: torch.Tensor,
                 z: Optional[torch.Tensor] = None, *, log_gamma: LogGamma = None, mask: Optional[torch.Tensor] = None,
                 normalize: bool = True, scale: Optional[float] = None, clamp_min: float = 1e-5, path: str = "auto"):
        _require_cuda(q, k, v, out, S)
        B, H, T, d = q.shape
        e = v.shape[-1]
        _check_kv(q, k, v)
        Hkv = k.shape[1]
        for name, t, shape in (("k", k, (B, Hkv, T, d)), ("v", v, (B, Hkv, T, e)), ("out", out, (B, H, T, e))):
            if tuple(t.shape) != shape or t.dtype != q.dtype or t.stride(-1) != 1:
                raise ValueError(f"{name} must be {shape} of {q.dtype} with a contiguous last dimension")
        if q.stride(-1) != 1:
            raise ValueError("q must have a contiguous last dimension")
        if S.dtype != torch.float32 or tuple(S.shape) != (B, H, d, e) or not S.is_contiguous():
            raise ValueError(f"S must be a contiguous float32 [{B}, {H}, {d}, {e}] tensor")
        if normalize and (z is None or z.dtype != torch.float32 or tuple(z.shape) != (B, H, d)
                          or not z.is_contiguous()):
            raise ValueError(f"z must be a contiguous float32 [{B}, {H}, {d}] tensor for the normalised form")
        self._keep: list = [q, k, v, out, S, z]
        a = _capi.FwdArgs()
        a.desc = _desc(q, v, log_gamma, mask, normalize, scale, clamp_min, False, path, self._keep)
        # the step must read the caller's buffers, not copies made at set-up
        if isinstance(log_gamma, torch.Tensor) and a.desc.log_gamma != log_gamma.data_ptr():
            raise ValueError("log_gamma must be a contiguous float32 [H] or [B, H, T] tensor")
        if mask is not None and a.desc.mask != mask.data_ptr():
            raise ValueError("mask must be a contiguous bool or uint8 [B, T] tensor")
        a.q, a.k, a.v, a.o = _t4(q), _t4(k), _t4(v), _t4(out)
        a.state_in = a.state_out = S.data_ptr()
        if normalize:
            a.norm_in = a.norm_out = z.data_ptr()
        self.device = q.device
        with torch.cuda.device(q.device):
            a.workspace, a.workspace_bytes = _workspace(_capi.fwd_workspace_bytes(a), q.device, self._keep)
        self._args = a

    def step(self) -> None:
        self._args.stream = torch.cuda.current_stream(self.device).cuda_stream
        _capi.fwd(self._args)


def feature_map_(x: torch.Tensor) -> torch.Tensor:
    """In-place phi(x) = ELU(x) + 1 on a contiguous CUDA tensor (run_feature_map)."""
    _require_cuda(x)
    if not x.is_contiguous():
        raise ValueError("feature_map_ needs a contiguous tensor")
    with torch.cuda.device(x.device):
        _capi.check(_capi.load().subq_feature_map(x.data_ptr(), x.numel(), _DTYPES[x.dtype],
                                                   torch.cuda.current_stream(x.device).cuda_stream))
    return x


def check_device_status(device: Optional[torch.device] = None) -> None:
    """Synchronises the current stream of ``device`` (default: the current
    device) and raises ``SubqError`` when, since the last check, a bounded
    device-side wait of a tensor-core kernel gave up (SUBQ_ERR_TIMEOUT) or a
    backward was given the handover of another call's forward
    (SUBQ_ERR_STATE): the outputs of the calls in between are then not valid.
    The scan launches themselves never synchronise; callers check at their own
    synchronisation points (``AudioTransformerEngine`` does)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        st = _capi.device_status(torch.cuda.current_stream(dev).cuda_stream)
    if st == _capi.SUBQ_ERR_TIMEOUT:
        raise _capi.SubqError(st, "a bounded device-side wait of a tensor-core kernel gave up "
                                  "(SUBQ_ERR_TIMEOUT); the outputs since the last check are not valid")
    if st != _capi.SUBQ_OK:
        raise _capi.SubqError(st, f"device status {st}: a backward was given the forward state of another "
                                  "call; its gradients are not valid")


_RMS_DIMS = (8, 16, 32, 64, 128, 256)


def head_rmsnorm_supported(x: torch.Tensor) -> bool:
    """True when the per-head RMSNorm kernels take x ([B, H, N, D] CUDA,
    float32/float16/bfloat16, D in 8..256 a power of two)."""
    return (x.is_cuda and x.dim() == 4 and x.shape[-1] in _RMS_DIMS
            and x.dtype in (torch.float32, torch.float16, torch.bfloat16))


def _rows16(t: torch.Tensor) -> torch.Tensor:
    """t itself when its rows start on 16-byte boundaries, else a contiguous copy."""
    es = t.element_size()
    if (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
            and all((s * es) % 16 == 0 for s in t.stride()[:3])):
        return t
    return t.contiguous()


def _rms_args(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float, keep: list) -> _capi.RmsArgs:
    B, H, N, D = x.shape
    a = _capi.RmsArgs()
    a.batch, a.heads, a.seq_len, a.head_dim = B, H, N, D
    a.dtype = _DTYPES[x.dtype]
    a.eps = float(eps)
    a.x = _t4(x)
    if weight is not None:
        w = weight.detach().to(device=x.device, dtype=torch.float32).contiguous()
        if w.shape != (D,):
            raise ValueError(f"weight must have shape ({D},), got {tuple(weight.shape)}")
        keep.append(w)
        a.weight = w.data_ptr()
    a.stream = torch.cuda.current_stream(x.device).cuda_stream
    return a


def head_rmsnorm(x: torch.Tensor, weight: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """Per-head RMSNorm y = x * rsqrt(mean(x^2, -1) + eps) * weight of a
    [B, H, N, D] scan output (float32 math). y is a [B, H, N, D] view of a
    [B, N, H, D] buffer, so ``y.transpose(1, 2).reshape(B, N, H * D)`` -- the
    output projection's input -- is a view, not a copy."""
    _require_cuda(x)
    if not head_rmsnorm_supported(x):
        raise ValueError(f"head_rmsnorm needs a [B, H, N, D] float32/float16/bfloat16 tensor with D in {_RMS_DIMS}")
    x = _rows16(x)
    B, H, N, D = x.shape
    y = torch.empty(B, N, H, D, dtype=x.dtype, device=x.device).transpose(1, 2)
    keep: list = []
    with torch.cuda.device(x.device):
        a = _rms_args(x, weight, eps, keep)
        a.y = _t4(y)
        _capi.head_rmsnorm_fwd(a)
    return y


def head_rmsnorm_backward(dy: torch.Tensor, x: torch.Tensor, weight: Optional[torch.Tensor] = None,
                          eps: float = 1e-5, need_dweight: bool = True
                          ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Gradients of ``head_rmsnorm``: dx (in x's memory order, x's dtype) and,
    with a weight and ``need_dweight``, d weight (float32 [D])."""
    _require_cuda(dy, x)
    if not head_rmsnorm_supported(x) or dy.shape != x.shape or dy.dtype != x.dtype:
        raise ValueError("head_rmsnorm_backward needs dy and x of one supported shape and dtype")
    x, dy = _rows16(x), _rows16(dy)
    D = x.shape[-1]
    dx = _empty_in_order(x, tuple(x.shape), x.dtype)
    dw = torch.empty(D, dtype=torch.float32, device=x.device) if (need_dweight and weight is not None) else None
    keep: list = []
    with torch.cuda.device(x.device):
        a = _rms_args(x, weight, eps, keep)
        a.dy, a.dx = _t4(dy), _t4(dx)
        if dw is not None:
            a.dweight = dw.data_ptr()
            nbytes = _capi.head_rmsnorm_bwd_workspace_bytes(a)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
            a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
            keep.append(ws)
        _capi.head_rmsnorm_bwd(a)
    return dx, dw


def last_path() -> str:
    return {0: "auto", 1: "exact", 2: "tensorcore", 3: "chunked"}.get(_capi.last_path(), "?")


def last_launches() -> int:
    return _capi.last_launches()
