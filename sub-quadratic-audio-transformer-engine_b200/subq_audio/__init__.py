"""Sub-Quadratic Audio Transformer Engine — causal ELU+1 linear attention on B200.

Drop-in for the reference package's hot path: the native module ``_C``
(``SubQEngine``, ``get_device_info``), the autograd surface
(``SubQAttentionFunction``, ``chunkwise_flash_linear_attention``,
``SubQLinearAttention``), attention surgery and the DDP helpers. Every scan
runs in the sm_100a kernels of ``libsubq_b200.so``.
"""
import sys
from typing import List, Optional

from . import _C
from ._C import SubQEngine, get_device_info

AudioStreamBuffer = None  # the streaming-ingest ring buffer is not part of this package
from .engine import (
    AudioTransformerEngine,
    cleanup_distributed,
    create_distributed_dataloader,
    setup_distributed,
    wrap_model_ddp,
)
from .autograd import (
    SubQAttentionFunction,
    SubQLinearAttention,
    SubQuadraticAttention,
    chunkwise_flash_linear_attention,
)
from .surgery import SubQAttentionOutput, SubQBypassAttention, bypass_transformer_with_subq

sys.modules.setdefault("subq_engine", _C)

__version__ = "0.1.0+b200"

Engine = AudioTransformerEngine
_default_engine: Optional[AudioTransformerEngine] = None


def _get_default_engine() -> AudioTransformerEngine:
    global _default_engine
    if _default_engine is None:
        _default_engine = AudioTransformerEngine()
    return _default_engine


def load(filepath: str) -> None:
    """Load weights into the default engine."""
    _get_default_engine().load_weights(filepath)


def generate(Q, K, V, decay_factor: float = 0.99):
    """Attention output from the default engine."""
    return _get_default_engine().forward(Q, K, V, decay_factor)


__all__: List[str] = [
    "_C", "SubQEngine", "AudioStreamBuffer", "get_device_info", "AudioTransformerEngine", "Engine",
    "SubQuadraticAttention", "SubQLinearAttention", "SubQAttentionFunction", "chunkwise_flash_linear_attention",
    "bypass_transformer_with_subq", "SubQBypassAttention", "SubQAttentionOutput",
    "setup_distributed", "cleanup_distributed", "wrap_model_ddp", "create_distributed_dataloader",
    "load", "generate", "__version__",
]
