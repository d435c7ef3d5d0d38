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


def _rms_args(B=2, H=3, N=5, D=64, dtype=_capi.SUBQ_BF16):
    a = _capi.RmsArgs()
    a.batch, a.heads, a.seq_len, a.head_dim, a.dtype, a.eps = B, H, N, D, dtype, 1e-5
    for i, name in enumerate(("x", "y", "dy", "dx")):
        t = getattr(a, name)
        t.data = 0x100000 * (i + 1)
        t.stride_b, t.stride_h, t.stride_n = N * H * D, D, H * D  # [B, N, H, D] memory
    return a


def test_rmsnorm_struct_layout_matches_header(tmp_path):
    src = tmp_path / "rms.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "kernels.hpp"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu\\n\", sizeof(subq_rmsnorm_args),"
        " offsetof(subq_rmsnorm_args, x), offsetof(subq_rmsnorm_args, weight),"
        " offsetof(subq_rmsnorm_args, workspace_bytes), offsetof(subq_rmsnorm_args, stream));return 0;}\n")
    exe = tmp_path / "rms"
    subprocess.run(["gcc", "-x", "c", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    got = list(map(int, subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()))
    R = _capi.RmsArgs
    assert got == [ctypes.sizeof(R), R.x.offset, R.weight.offset, R.workspace_bytes.offset, R.stream.offset]


@pytest.mark.parametrize("change,code,text", [
    (lambda a: setattr(a, "head_dim", 48), _capi.SUBQ_ERR_UNSUPPORTED, b"head_dim"),
    (lambda a: setattr(a, "dtype", _capi.SUBQ_FP64), _capi.SUBQ_ERR_INVALID_ARGUMENT, b"float32"),
    (lambda a: setattr(a, "eps", -1.0), _capi.SUBQ_ERR_INVALID_ARGUMENT, b"eps"),
    (lambda a: setattr(a.x, "stride_n", 3 * 64 + 4), _capi.SUBQ_ERR_INVALID_ARGUMENT, b"16-byte"),
    (lambda a: setattr(a.y, "data", 0x100008), _capi.SUBQ_ERR_INVALID_ARGUMENT, b"16-byte"),
    (lambda a: setattr(a.x, "data", 0), _capi.SUBQ_ERR_INVALID_ARGUMENT, b"null"),
    (lambda a: setattr(a, "seq_len", -1), _capi.SUBQ_ERR_INVALID_ARGUMENT, b"negative"),
])
def test_rmsnorm_rejects_bad_arguments_before_the_gpu(change, code, text):
    lib = _capi.load()
    a = _rms_args()
    change(a)
    assert lib.subq_head_rmsnorm_fwd(ctypes.byref(a)) == code
    assert text in lib.subq_last_error()
    assert lib.subq_head_rmsnorm_fwd(None) == _capi.SUBQ_ERR_INVALID_ARGUMENT


def test_rmsnorm_backward_workspace_is_the_cta_partials():
    """dweight needs one D-float partial per CTA: min(ceil(rows / (256 / (D / 8))), 1184) of them,
    rounded up to 256 bytes; no workspace without dweight."""
    lib = _capi.load()
    for B, H, N, D in [(2, 3, 5, 64), (4, 12, 16384, 64), (1, 1, 1, 8), (1, 2, 700, 256)]:
        a = _rms_args(B, H, N, D)
        assert lib.subq_head_rmsnorm_bwd_workspace_bytes(ctypes.byref(a)) == 0
        a.dweight = 0x900000
        rows, rpb = B * H * N, 256 // (D // 8)
        blocks = min(-(-rows // rpb), 148 * 8)
        want = -(-blocks * D * 4 // 256) * 256
        assert lib.subq_head_rmsnorm_bwd_workspace_bytes(ctypes.byref(a)) == want


def test_chunked_forward_workspace_and_path_choice():
    """float32 calls of 64 tokens or more take the chunked forward under AUTO:
    per 64-token chunk and sequence a block of 17,152 + 512 (round32(d) + 4)
    bytes, the normaliser copy, and in the chunk-parallel form (few sequences)
    d (e + 1) floats of chunk states; shorter calls run on the exact path with
    no workspace; an explicit CHUNKED request the path cannot take is refused."""
    lib = _capi.load()

    def ws(B, H, N, d, e, path=_capi.SUBQ_PATH_AUTO, dtype=_capi.SUBQ_FP32):
        a = _fwd_args(B, H, N, d, e, dtype)
        a.desc.path = path
        return lib.subq_fwd_workspace_bytes(ctypes.byref(a))

    block = lambda d: 17152 + 512 * ((d + 31) // 32 * 32 + 4)  # noqa: E731
    zcopy = lambda B, H, d: -(-B * H * d * 4 // 16) * 16  # noqa: E731
    assert ws(1, 1, 640, 64, 64) == 10 * block(64) + zcopy(1, 1, 64) + 10 * 64 * 65 * 4   # chunk-parallel
    assert ws(4, 8, 640, 64, 64) == 32 * 10 * block(64) + zcopy(4, 8, 64)                 # sequential walk
    assert ws(1, 1, 63, 64, 64) == 0                                                      # exact path
    assert ws(64, 64, 65536, 64, 64) == 0  # over 4 GiB of chunk workspace: the exact path, which needs none
    assert ws(1, 1, 63, 64, 64, path=_capi.SUBQ_PATH_CHUNKED) == block(64) + zcopy(1, 1, 64) + 64 * 65 * 4
    a = _fwd_args(1, 1, 100, 8, 8, _capi.SUBQ_FP64)
    a.desc.path = _capi.SUBQ_PATH_CHUNKED
    assert lib.subq_fwd(ctypes.byref(a)) == _capi.SUBQ_ERR_UNSUPPORTED
    assert b"chunked" in lib.subq_last_error()
