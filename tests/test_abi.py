"""The C ABI without a GPU: libfp8gq.so builds and loads, exports every entry
point include/fp8gq.h declares, and rejects bad arguments before it touches a
device (no compute call is made here)."""
import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "fp8gq.h"


def declared_entry_points():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fp8gq_[a-z_0-9]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from fp8gq import _lib
    return _lib.load()


def test_header_declares_the_entry_points():
    names = declared_entry_points()
    for want in ("fp8gq_fused_gemv_quant", "fp8gq_gemv_quant_row", "fp8gq_gemv_quant_tm",
                 "fp8gq_fused_swiglu_q_gemm", "fp8gq_group_quant", "fp8gq_swiglu_group_quant",
                 "fp8gq_workspace_bytes", "fp8gq_status_string", "fp8gq_version", "fp8gq_device_error"):
        assert want in names


def test_library_exports_every_declared_symbol(lib):
    from fp8gq import _lib
    for name in declared_entry_points():
        assert hasattr(lib, name), f"{name} declared in include/fp8gq.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in fp8gq._lib"


def test_version_and_status_strings(lib):
    assert lib.fp8gq_version() == 2
    for code in range(0, 11):
        assert lib.fp8gq_status_string(code)
    assert b"unknown" in lib.fp8gq_status_string(1234)


def _call_row(lib, x=1 << 20, w=1 << 20, ws=1 << 20, out=1 << 20, N=256, K=256, ldw=256, ldws=2):
    return lib.fp8gq_gemv_quant_row(x, w, ldw, ws, ldws, out, N, K, None, None, None)


def test_null_pointers_rejected(lib):
    assert _call_row(lib, x=None) == 1
    assert _call_row(lib, w=None) == 1
    assert lib.fp8gq_group_quant(None, 128, 1, 128, 1 << 20, 1 << 20, None) == 1


def test_shapes_rejected(lib):
    assert _call_row(lib, N=200) == 2
    assert _call_row(lib, K=100, ldw=128) == 2
    assert _call_row(lib, N=0) == 2
    args = [1 << 20, 256, 1 << 20, 256, 1 << 20, 2, 1 << 20, 256]
    assert lib.fp8gq_fused_gemv_quant(*args, 0, 256, 256, None, None, None, 0, None) == 2


def test_strides_and_alignment_rejected(lib):
    assert _call_row(lib, ldw=128) == 4          # ldw < K
    assert _call_row(lib, ldws=1) == 4           # ldws < K/128
    assert _call_row(lib, x=(1 << 20) + 8) == 3  # x not 16-byte aligned
    assert _call_row(lib, ldw=264) == 3          # ldw not a multiple of 16


def test_device_error_needs_pointer(lib):
    assert lib.fp8gq_device_error(None, 0) == 1


def test_valid_arguments_need_a_b200(lib):
    """Well-formed arguments reach the device check, which fails without a GPU
    (and on any GPU that is not compute capability 10.x)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _call_row(lib) == 6


def test_python_ops_refuse_cpu_tensors():
    import torch
    import fp8gq
    x = torch.zeros(1, 128, dtype=torch.bfloat16)
    w = torch.zeros(128, 128, dtype=torch.float8_e4m3fn)
    s = torch.ones(1, 1)
    with pytest.raises(ValueError, match="CUDA"):
        fp8gq.fused_gemv_quant(x, w, s)


def test_fp8gq_error_carries_status():
    from fp8gq._lib import Fp8gqError
    e = Fp8gqError(3, "fp8gq_gemv_quant_row")
    assert e.status == 3 and "FP8GQ_ERR_ALIGNMENT" in str(e)


def test_weight_checks_and_strides():
    """The host-side weight checks of every op (CPU tensors: no device is
    touched): dtypes, K against the activation, multiples of 128, contiguity
    along K, the scale shape; and the row strides they return."""
    import torch
    from fp8gq import ops
    w = torch.zeros(256, 384, dtype=torch.float8_e4m3fn)
    s = torch.ones(2, 3)
    assert ops._check_weight_strides(w, s, 384) == (256, 384, 3)
    wide = torch.zeros(256, 512, dtype=torch.float8_e4m3fn)[:, :384]          # row stride 512
    assert ops._check_weight_strides(wide, s, 384) == (256, 512, 3)
    assert ops._check_weight(w, s, 384) == 256
    with pytest.raises(TypeError):
        ops._check_weight_strides(w.view(torch.uint8), s, 384)
    with pytest.raises(TypeError):
        ops._check_weight_strides(w, s.double(), 384)
    with pytest.raises(ops.ShapeError):
        ops._check_weight_strides(w, s, 256)                                     # K mismatch
    with pytest.raises(ops.ShapeError):
        ops._check_weight_strides(torch.zeros(200, 384, dtype=torch.float8_e4m3fn), s, 384)
    with pytest.raises(ValueError):
        ops._check_weight_strides(torch.zeros(384, 256, dtype=torch.float8_e4m3fn).t(), s, 384)
    with pytest.raises(ops.ShapeError):
        ops._check_weight_strides(w, torch.ones(2, 2), 384)                       # scale shape
