"""Engine wrapper and distributed helpers (reference python/subq_audio/engine.py).

``AudioTransformerEngine`` keeps the reference's dispatch rules
(engine.py:46-146):
  * torch float16/bfloat16 tensors (and CPU torch tensors) -> the normalised
    scan with decay gamma = decay_factor (``chunkwise_flash_linear_attention``);
  * CUDA float32 tensors -> the unnormalised engine scan on device pointers
    (``SubQEngine.forward_raw`` / ``backward_raw``);
  * NumPy arrays -> ``SubQEngine.forward`` / ``backward`` (host staging).
All of them execute in the B200 kernels.
"""
from __future__ import annotations

import math
import os
from typing import Any, Dict, Optional, Tuple, Union

import numpy as np

from . import _C

TensorLike = Union[np.ndarray, Any]


def _decay_logit(decay_factor: float) -> float:
    g = min(max(float(decay_factor), 1e-7), 1.0 - 1e-7)
    return math.log(g / (1.0 - g))


class AudioTransformerEngine:
    """Polymorphic front end over the native ``SubQEngine``."""

    def __init__(self, vram_capacity: int = 32 * 1024 * 1024, device_id: int = 0) -> None:
        self._vram_capacity = vram_capacity
        self._device_id = device_id
        self._engine = _C.SubQEngine(vram_capacity, device_id)

    @property
    def device_id(self) -> int:
        return self._device_id

    def load_weights(self, filepath: str) -> None:
        if not os.path.exists(filepath):
            raise FileNotFoundError(f"Model weight file not found: {filepath}")
        self._engine.load(filepath)

    @property
    def device_info(self) -> Dict[str, Any]:
        return _C.get_device_info()

    def forward(self, Q: TensorLike, K: TensorLike, V: TensorLike, decay_factor: float = 0.99) -> TensorLike:
        if hasattr(Q, "is_cuda"):
            import torch

            if not isinstance(Q, torch.Tensor):
                raise TypeError(f"Expected torch.Tensor, got {type(Q)}")
            if Q.dtype in (torch.float16, torch.bfloat16) or not Q.is_cuda:
                from .autograd import chunkwise_flash_linear_attention

                w = torch.tensor(_decay_logit(decay_factor), dtype=torch.float32)
                out, _ = chunkwise_flash_linear_attention(Q, K, V, decay_w=w)
                return out.to(dtype=Q.dtype)
            if Q.is_cuda and getattr(K, "is_cuda", False) and getattr(V, "is_cuda", False):
                Qc, Kc, Vc = Q.contiguous().float(), K.contiguous().float(), V.contiguous().float()
                O = torch.empty_like(Qc)
                B, N, D = Qc.shape
                from . import ops

                ops.check_device_status(Qc.device)  # synchronises the inputs' stream
                self._engine.forward_raw(Qc.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), O.data_ptr(),
                                         int(B), int(N), int(D), float(decay_factor))
                return O.to(Q.dtype)
        Qn = np.ascontiguousarray(Q, dtype=np.float32)
        Kn = np.ascontiguousarray(K, dtype=np.float32)
        Vn = np.ascontiguousarray(V, dtype=np.float32)
        return self._engine.forward(Qn, Kn, Vn, float(decay_factor))

    def backward(self, dO: TensorLike, Q: TensorLike, K: TensorLike, V: TensorLike,
                 decay_factor: float = 0.99) -> Tuple[TensorLike, TensorLike, TensorLike, float]:
        if hasattr(Q, "is_cuda"):
            import torch

            if Q.dtype in (torch.float16, torch.bfloat16) or not Q.is_cuda:
                from .autograd import SubQAttentionFunction

                q = Q.detach().clone().requires_grad_(True)
                k = K.detach().clone().requires_grad_(True)
                v = V.detach().clone().requires_grad_(True)
                gamma = min(max(float(decay_factor), 1e-7), 1.0 - 1e-7)
                w = torch.tensor(_decay_logit(decay_factor), dtype=torch.float32, device=Q.device,
                                 requires_grad=True)
                out = SubQAttentionFunction.apply(q, k, v, w)
                (out * dO).sum().backward()
                dw = float(w.grad.item()) if w.grad is not None else 0.0
                if q.is_cuda:  # (.item() has synchronised) a device-side wait that gave up raises here
                    from . import ops

                    ops.check_device_status(q.device)
                return (q.grad.contiguous().to(Q.dtype), k.grad.contiguous().to(Q.dtype),
                        v.grad.contiguous().to(Q.dtype), dw / (gamma * (1.0 - gamma)))
            if Q.is_cuda and getattr(dO, "is_cuda", False):
                dOc, Qc, Kc, Vc = (x.contiguous().float() for x in (dO, Q, K, V))
                dQ, dK, dV = torch.empty_like(Qc), torch.empty_like(Kc), torch.empty_like(Vc)
                B, N, D = Qc.shape
                from . import ops

                ops.check_device_status(Qc.device)  # synchronises the inputs' stream
                d_decay = self._engine.backward_raw(dOc.data_ptr(), Qc.data_ptr(), Kc.data_ptr(), Vc.data_ptr(),
                                                    dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(),
                                                    int(B), int(N), int(D), float(decay_factor))
                return dQ.to(Q.dtype), dK.to(Q.dtype), dV.to(Q.dtype), float(d_decay)
        dOn, Qn, Kn, Vn = (np.ascontiguousarray(x, dtype=np.float32) for x in (dO, Q, K, V))
        return self._engine.backward(dOn, Qn, Kn, Vn, float(decay_factor))


def setup_distributed(backend: Optional[str] = None, init_method: Optional[str] = None,
                      timeout_s: Optional[float] = None) -> Tuple[int, int, int]:
    """Initialise torch.distributed from RANK/LOCAL_RANK/WORLD_SIZE (NCCL on GPUs, else gloo)."""
    import datetime

    import torch
    import torch.distributed as dist

    if dist.is_initialized():
        rank = dist.get_rank()
        return rank, int(os.environ.get("LOCAL_RANK", rank)), dist.get_world_size()
    rank = int(os.environ.get("RANK", 0))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    world_size = int(os.environ.get("WORLD_SIZE", 1))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() and dist.is_nccl_available() else "gloo"
    if torch.cuda.is_available() and backend == "nccl":
        torch.cuda.set_device(local_rank)
    kwargs = {}
    if timeout_s is not None:
        kwargs["timeout"] = datetime.timedelta(seconds=timeout_s)
    dist.init_process_group(backend=backend, init_method=init_method, rank=rank, world_size=world_size, **kwargs)
    return rank, local_rank, world_size


def cleanup_distributed() -> None:
    import torch.distributed as dist

    if dist.is_initialized():
        dist.destroy_process_group()


def wrap_model_ddp(model: Any, device_id: Optional[int] = None, find_unused_parameters: bool = False,
                   bucket_cap_mb: int = 25, gradient_as_bucket_view: bool = False) -> Any:
    import torch
    from torch.nn.parallel import DistributedDataParallel as DDP

    ids = [device_id] if torch.cuda.is_available() and device_id is not None else None
    return DDP(model, device_ids=ids, output_device=device_id if ids else None,
               find_unused_parameters=find_unused_parameters, bucket_cap_mb=bucket_cap_mb,
               gradient_as_bucket_view=gradient_as_bucket_view)


def create_distributed_dataloader(dataset: Any, batch_size: int, rank: Optional[int] = None,
                                  world_size: Optional[int] = None, shuffle: bool = True, num_workers: int = 0,
                                  pin_memory: bool = True, drop_last: bool = False, **kwargs: Any) -> Any:
    import torch
    from torch.utils.data import DataLoader, DistributedSampler

    sampler = DistributedSampler(dataset, num_replicas=world_size, rank=rank, shuffle=shuffle, drop_last=drop_last)
    return DataLoader(dataset, batch_size=batch_size, sampler=sampler, num_workers=num_workers,
                      pin_memory=(pin_memory and torch.cuda.is_available()), **kwargs)
