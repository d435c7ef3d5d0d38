"""Device-side timeouts reach the caller. Every wait of the tensor-core
kernels is bounded: when one gives up, the kernel records SUBQ_ERR_TIMEOUT in
the device status word and returns. These tests make such a wait run out on
purpose - a barrier that nothing arrives at, with the poll limit shortened
(subq_selftest_wait_timeout) - and check that every product-level checkpoint
reports it and clears it. No GPU fault is involved.
"""
import numpy as np
import pytest
import torch

from subq_audio import _C, _capi, ops
from subq_audio.engine import AudioTransformerEngine

pytestmark = pytest.mark.gpu


def _time_out():
    _capi.selftest_wait_timeout(polls=64, stream=torch.cuda.current_stream().cuda_stream)


def test_status_word_records_and_clears_a_timeout():
    torch.cuda.synchronize()
    assert _capi.device_status() == _capi.SUBQ_OK
    _time_out()
    assert _capi.device_status() == _capi.SUBQ_ERR_TIMEOUT
    assert _capi.device_status() == _capi.SUBQ_OK  # read and cleared in one step


def test_ops_check_raises_on_a_timeout():
    x = torch.randn(1, 2, 300, 64, device="cuda", dtype=torch.bfloat16)
    ops.scan_forward(x, x, x)
    ops.check_device_status()  # nothing recorded
    _time_out()
    with pytest.raises(_capi.SubqError) as err:
        ops.check_device_status()
    assert err.value.code == _capi.SUBQ_ERR_TIMEOUT
    ops.check_device_status()  # cleared


def test_engine_reports_a_timeout_as_engine_error():
    eng = _C.SubQEngine()
    Q = np.random.default_rng(0).random((1, 64, 16), dtype=np.float32)
    eng.forward(Q, Q, Q, 0.99)
    _time_out()
    with pytest.raises(RuntimeError, match="Engine Forward Error: .*SUBQ_ERR_TIMEOUT"):
        eng.forward(Q, Q, Q, 0.99)
    eng.forward(Q, Q, Q, 0.99)  # the word was cleared by the failing call
    _time_out()
    with pytest.raises(RuntimeError, match="Engine Backward Error: .*SUBQ_ERR_TIMEOUT"):
        eng.backward(Q, Q, Q, Q, 0.99)


def test_transformer_engine_backward_reports_a_timeout():
    eng = AudioTransformerEngine()
    Q = torch.randn(1, 200, 64, device="cuda", dtype=torch.bfloat16)
    eng.backward(Q, Q, Q, Q)
    _time_out()
    with pytest.raises(_capi.SubqError):
        eng.backward(Q, Q, Q, Q)
