"""Type stub of the subq_audio._C native module (B200 build)."""
from typing import Any, Dict, Optional, Tuple

import numpy as np
import numpy.typing as npt

def get_device_info() -> Dict[str, Any]:
    """{'backend': 'CUDA' | 'CPU', 'architecture': 'SM 10.0' | 'Host', 'memory_size': int,
    'bfloat16_supported': bool}"""
    ...

def abi_version() -> int: ...

class SubQEngine:
    """Device-resident engine: one arena (cudaMalloc once) holding the carried
    float32 state and all scratch; scans run in the sm_100a kernels."""

    def __init__(self, vram_capacity: int = 33554432, device_id: int = 0) -> None: ...
    @property
    def device_id(self) -> int: ...
    def load(self, filepath: str) -> None:
        """Load a safetensors file into the arena. RuntimeError('Loader Error: ...') on malformed files."""
        ...
    def forward(self, Q: npt.NDArray[np.float32], K: npt.NDArray[np.float32], V: npt.NDArray[np.float32],
                decay_factor: float = 0.99, *, carry_state: bool = False,
                normalize: bool = False) -> npt.NDArray[np.float32]:
        """[B, N, D] float32 scan S = gamma S + phi(k) v^T, O = phi(q) S (normalize=False);
        carry_state=True continues from the previous call's state."""
        ...
    def forward_raw(self, q_ptr: int, k_ptr: int, v_ptr: int, o_ptr: int, batch: int, seq_len: int,
                    d_model: int, decay_factor: float = 0.99, *, carry_state: bool = False,
                    normalize: bool = False) -> None: ...
    def backward(self, dO: npt.NDArray[np.float32], Q: npt.NDArray[np.float32], K: npt.NDArray[np.float32],
                 V: npt.NDArray[np.float32], decay_factor: float = 0.99
                 ) -> Tuple[npt.NDArray[np.float32], npt.NDArray[np.float32], npt.NDArray[np.float32], float]: ...
    def backward_raw(self, do_ptr: int, q_ptr: int, k_ptr: int, v_ptr: int, dq_ptr: int, dk_ptr: int,
                     dv_ptr: int, batch: int, seq_len: int, d_model: int, decay_factor: float = 0.99) -> float: ...
    def reset_state(self) -> None: ...
    def state(self) -> Optional[npt.NDArray[np.float32]]: ...
