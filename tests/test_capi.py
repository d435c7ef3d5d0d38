"""The C ABI library: loads, exports every declared symbol, mirrors the header's
struct layout, and rejects bad arguments before touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

import subq_audio
from subq_audio import _capi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "kernels.hpp")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(subq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    declared = _declared_functions()
    assert declared, "no declarations found"
    assert set(declared) == set(_capi.EXPORTED)
    out = subprocess.run(["nm", "-D", "--defined-only", _capi.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s(subq_\w+)", out))
    for name in declared:
        assert name in exported, name
        assert hasattr(lib, name)


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "kernels.hpp"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu %zu %zu %zu\\n\", sizeof(subq_tensor4), sizeof(subq_scan_desc),"
        " sizeof(subq_fwd_args), sizeof(subq_bwd_args), offsetof(subq_scan_desc, log_gamma),"
        " offsetof(subq_fwd_args, state_in), offsetof(subq_bwd_args, dlog_gamma),"
        " offsetof(subq_bwd_args, out));return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-x", "c", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    got = list(map(int, subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()))
    want = [ctypes.sizeof(_capi.Tensor4), ctypes.sizeof(_capi.ScanDesc), ctypes.sizeof(_capi.FwdArgs),
            ctypes.sizeof(_capi.BwdArgs), _capi.ScanDesc.log_gamma.offset, _capi.FwdArgs.state_in.offset,
            _capi.BwdArgs.dlog_gamma.offset, _capi.BwdArgs.out.offset]
    assert got == want


def _fwd_args(B=1, H=1, N=8, d=4, e=4, dtype=_capi.SUBQ_FP32):
    a = _capi.FwdArgs()
    a.desc.batch, a.desc.heads, a.desc.seq_len, a.desc.head_dim, a.desc.value_dim = B, H, N, d, e
    a.desc.dtype = dtype
    a.desc.scale = 1.0
    a.desc.clamp_min = 1e-5
    for name, width in (("q", d), ("k", d), ("v", e), ("o", e)):
        t = getattr(a, name)
        t.data = 0x1000
        t.stride_b, t.stride_h, t.stride_n = H * N * width, N * width, width
    return a


def test_abi_version_and_error_text():
    lib = _capi.load()
    assert lib.subq_abi_version() == 5
    a = _fwd_args()
    a.desc.head_dim = 0
    assert lib.subq_fwd(ctypes.byref(a)) == _capi.SUBQ_ERR_INVALID_ARGUMENT
    assert b"positive" in lib.subq_last_error()


@pytest.mark.parametrize("field,value,code", [
    ("dtype", 9, _capi.SUBQ_ERR_INVALID_ARGUMENT),
    ("decay_mode", 7, _capi.SUBQ_ERR_INVALID_ARGUMENT),
    ("batch", -1, _capi.SUBQ_ERR_INVALID_ARGUMENT),
    ("head_dim", 512, _capi.SUBQ_ERR_UNSUPPORTED),
    ("path", 5, _capi.SUBQ_ERR_INVALID_ARGUMENT),
])
def test_forward_rejects_bad_descriptions(field, value, code):
    a = _fwd_args()
    setattr(a.desc, field, value)
    assert _capi.load().subq_fwd(ctypes.byref(a)) == code


def test_grouped_kv_heads_must_divide_heads():
    lib = _capi.load()
    a = _fwd_args(H=4)
    a.desc.kv_heads = 3
    assert lib.subq_fwd(ctypes.byref(a)) == _capi.SUBQ_ERR_INVALID_ARGUMENT
    assert b"kv_heads" in lib.subq_last_error()
    a.desc.kv_heads = -1
    assert lib.subq_fwd(ctypes.byref(a)) == _capi.SUBQ_ERR_INVALID_ARGUMENT


def test_grouped_kv_backward_workspace_holds_per_head_gradients():
    """With kv_heads < heads the backward needs room for dk, dv per query head
    (summed per group afterwards): the workspace grows by 2 x B x H x N x d
    elements over the same call without grouping (exact path, float32)."""
    lib = _capi.load()
    B, H, N, d = 2, 4, 16, 8

    def bwd_args(kv):
        a = _capi.BwdArgs()
        a.desc.batch, a.desc.heads, a.desc.seq_len, a.desc.head_dim, a.desc.value_dim = B, H, N, d, d
        a.desc.dtype, a.desc.scale, a.desc.clamp_min, a.desc.path = _capi.SUBQ_FP32, 1.0, 1e-5, 1
        a.desc.kv_heads = kv
        for i, name in enumerate(("q", "k", "v", "dout", "dq", "dk", "dv")):
            t = getattr(a, name)
            t.data = 0x10000 * (i + 1)
            t.stride_b, t.stride_h, t.stride_n = H * N * d, N * d, d
        return a

    plain = lib.subq_bwd_workspace_bytes(ctypes.byref(bwd_args(0)))
    grouped = lib.subq_bwd_workspace_bytes(ctypes.byref(bwd_args(2)))
    assert plain > 0 and grouped - plain >= 2 * B * H * N * d * 4


def test_forward_rejects_null_and_misaligned_tensors():
    lib = _capi.load()
    a = _fwd_args()
    a.q.data = 0
    assert lib.subq_fwd(ctypes.byref(a)) == _capi.SUBQ_ERR_INVALID_ARGUMENT
    a = _fwd_args()
    a.k.data = 0x1002
    assert lib.subq_fwd(ctypes.byref(a)) == _capi.SUBQ_ERR_INVALID_ARGUMENT
    a = _fwd_args()
    a.desc.decay_mode = _capi.SUBQ_DECAY_PER_TOKEN
    assert lib.subq_fwd(ctypes.byref(a)) == _capi.SUBQ_ERR_INVALID_ARGUMENT
    assert lib.subq_fwd(None) == _capi.SUBQ_ERR_INVALID_ARGUMENT


def test_backward_rejects_aliased_gradients():
    """Gradient outputs aliasing inputs raise, as the reference's backward does
    (src/kernels/attention_backward.cpp:51-56)."""
    lib = _capi.load()
    b = _capi.BwdArgs()
    b.desc.batch = b.desc.heads = 1
    b.desc.seq_len, b.desc.head_dim, b.desc.value_dim = 8, 4, 4
    b.desc.scale, b.desc.clamp_min = 1.0, 1e-5
    for i, name in enumerate(("q", "k", "v", "dout", "dq", "dk", "dv")):
        t = getattr(b, name)
        t.data = 0x10000 * (i + 1)
        t.stride_b, t.stride_h, t.stride_n = 32, 32, 4
    b.dk.data = b.k.data
    assert lib.subq_bwd(ctypes.byref(b)) == _capi.SUBQ_ERR_ALIAS
    assert b"must not alias" in lib.subq_last_error()


def test_workspace_query_without_device():
    b = _capi.BwdArgs()
    b.desc.batch, b.desc.heads, b.desc.seq_len, b.desc.head_dim, b.desc.value_dim = 2, 3, 100, 16, 16
    b.desc.scale, b.desc.clamp_min = 0.25, 1e-5
    for i, name in enumerate(("q", "k", "v", "dout", "dq", "dk", "dv")):
        t = getattr(b, name)
        t.data = 0x10000 * (i + 1)
        t.stride_b, t.stride_h, t.stride_n = 3 * 100 * 16, 100 * 16, 16
    b.desc.path = _capi.SUBQ_PATH_EXACT
    need = _capi.bwd_workspace_bytes(b)
    assert need >= 3 * 4 * 2 * 3 * 100 and need % 256 == 0


def test_product_has_no_cpu_path():
    import torch

    q = torch.randn(1, 1, 8, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        subq_audio.ops.scan_forward(q, q, q)
