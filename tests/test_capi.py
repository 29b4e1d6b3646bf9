"""The C ABI (include/qatf.h) without a GPU: the library loads, exports exactly the
declared entry points, and rejects bad arguments before touching the device."""

import ctypes
import re
from pathlib import Path

import pytest

from qatfactory_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "qatf.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|int64_t|uint64_t|const char \*)\s*(qatf_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_bound_entry_points():
    assert declared_symbols() == set(_native.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = _native.load_library()
    for name in sorted(declared_symbols()):
        assert hasattr(lib, name), name


def test_status_strings_and_version():
    lib = _native.load_library()
    assert lib.qatf_version() >= 100
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert lib.qatf_status_string(code)
    assert lib.qatf_status_string(-99) == b"unknown status"


P = ctypes.c_void_p(16)  # never dereferenced: every call below fails validation first


@pytest.mark.parametrize(
    "call",
    [
        lambda L: L.qatf_nvfp4_qdq(P, 2, -1, 16, 16, P, P, None, None),
        lambda L: L.qatf_nvfp4_qdq(P, 2, 4, 16, 8, P, P, None, None),  # ld < cols
        lambda L: L.qatf_nvfp4_qdq(P, 2, 4, 16, 16, None, P, None, None),  # no tensor amax
        lambda L: L.qatf_mxfp4_qdq_ceil(P, 2, 4, 48, 48, P, None),  # cols % 32
        lambda L: L.qatf_nvfp4_pack(P, 2, 4, 40, 40, P, P, P, P, None, None),  # cols % 16
        lambda L: L.qatf_mxfp4_pack(P, 2, 4, 48, 48, P, P, None, None),  # cols % 32
        lambda L: L.qatf_q4k_encode(P, 2, 4, 300, 300, 1, None, None, None, None),  # cols % 256
        lambda L: L.qatf_q4k_encode(P, 2, 4, 256, 256, 7, None, None, None, None),  # method
        lambda L: L.qatf_q4k_dequant(P, 4, 100, P, None),
        lambda L: L.qatf_e2m1_pack_rows(P, 2, 3, P, None),  # odd cols
        lambda L: L.qatf_ste_backward(None, 2, 8, P, P, None),
        lambda L: L.qatf_tensor_amax(P, 2, 8, None, None),
        lambda L: L.qatf_nvfp4_dequant(P, P, P, 2, 24, P, None),
        lambda L: L.qatf_mxfp4_dequant(P, P, 2, 48, P, None),
    ],
)
def test_invalid_arguments_are_rejected_before_launch(call):
    assert call(_native.load_library()) == -1


def test_empty_tensors_are_a_no_op():
    L = _native.load_library()
    assert L.qatf_nvfp4_qdq(None, 2, 0, 16, 16, P, None, None, None) == 0
    assert L.qatf_mxfp4_qdq_even(None, 2, 5, 0, 0, None, None, None) == 0
    assert L.qatf_q4k_encode(None, 2, 0, 256, 256, 1, None, None, None, None) == 0


def test_unknown_dtype_code():
    L = _native.load_library()
    # validation passes, dtype dispatch fails before any launch
    assert L.qatf_mxfp4_qdq_even(P, 9, 1, 32, 32, P, None, None) == -2


def test_rejected_calls_launch_nothing():
    L = _native.load_library()
    before = _native.launch_count()
    assert L.qatf_nvfp4_qdq(P, 2, 4, 16, 8, P, P, None, None) == -1
    assert L.qatf_mxfp4_qdq_even(None, 2, 5, 0, 0, None, None, None) == 0
    assert L.qatf_mxfp4_qdq_even(P, 9, 1, 32, 32, P, None, None) == -2
    assert _native.launch_count() == before


def test_gemm_entry_points_reject_unsupported_shapes_before_launch():
    L = _native.load_library()
    assert L.qatf_nvfp4_operand(P, 2, 100, 64, P, 0, P, P, None, None, None) == -6  # rows % 128
    assert L.qatf_nvfp4_operand(P, 2, 128, 64, P, 1, P, P, None, None, None) == -6  # B side: rows % 256
    assert L.qatf_nvfp4_operand(P, 2, 128, 64, P, 0, P, P, None, None, None) == -6  # A side: cols % 128
    assert L.qatf_nvfp4_operand(P, 2, 256, 48, P, 1, P, P, None, None, None) == -6  # cols % 64
    assert L.qatf_nvfp4_operand(P, 0, 128, 256, P, 0, P, P, None, None, None) == -2  # BF16 only
    assert L.qatf_nvfp4_operand(P, 2, 128, 256, None, 0, P, P, None, None, None) == -1  # no amax
    assert L.qatf_nvfp4_operand(P, 2, 128, 64, P, 5, P, P, None, None, None) == -1  # role
    assert L.qatf_nvfp4_gemm(P, P, P, P, P, P, 100, 256, 256, P, P, None) == -6
    assert L.qatf_nvfp4_gemm(P, P, P, P, P, P, 128, 128, 256, P, P, None) == -6  # N % 256
    assert L.qatf_nvfp4_gemm(P, P, P, P, P, P, 128, 256, 256, P, None, None) == -1  # no error word
    assert L.qatf_bf16_gemm(P, 7, P, 0, 128, 256, 64, None, P, P, None) == -1  # layout code
    assert L.qatf_bf16_gemm(P, 0, P, 0, 128, 256, 48, None, P, P, None) == -6  # K % 64


def test_mxfp4_gemm_entry_points_reject_unsupported_arguments_before_launch():
    L = _native.load_library()
    before = _native.launch_count()
    # qatf_mxfp4_operand(x, dtype, rows, cols, role, rule, codes, scales, deq, mask, stream)
    assert L.qatf_mxfp4_operand(P, 2, 100, 256, 0, 0, P, P, None, None, None) == -6  # A side: rows % 128
    assert L.qatf_mxfp4_operand(P, 2, 128, 128, 0, 0, P, P, None, None, None) == -6  # A side: cols % 256
    assert L.qatf_mxfp4_operand(P, 2, 128, 128, 1, 0, P, P, None, None, None) == -6  # B side: rows % 256
    assert L.qatf_mxfp4_operand(P, 2, 256, 64, 1, 1, P, P, None, None, None) == -6  # B side: cols % 128
    assert L.qatf_mxfp4_operand(P, 2, 128, 256, 2, 0, P, P, None, None, None) == -1  # role
    assert L.qatf_mxfp4_operand(P, 2, 128, 256, 0, 5, P, P, None, None, None) == -1  # rule
    assert L.qatf_mxfp4_operand(P, 0, 128, 256, 0, 1, P, P, None, None, None) == -2  # BF16 only
    assert L.qatf_mxfp4_operand(P, 2, 128, 256, 0, 1, None, P, None, None, None) == -1  # no codes
    assert L.qatf_mxfp4_operand(None, 2, 0, 256, 0, 1, None, None, None, None, None) == 0  # empty
    # qatf_mxfp4_gemm(a_codes, a_scales, b_codes, b_scales, m, n, k, out, err, stream)
    assert L.qatf_mxfp4_gemm(P, P, P, P, 100, 256, 256, P, P, None) == -6  # M % 128
    assert L.qatf_mxfp4_gemm(P, P, P, P, 128, 128, 256, P, P, None) == -6  # N % 256
    assert L.qatf_mxfp4_gemm(P, P, P, P, 128, 256, 128, P, P, None) == -6  # K % 256
    assert L.qatf_mxfp4_gemm(P, P, P, P, 128, 256, 256, P, None, None) == -1  # no error word
    assert L.qatf_mxfp4_gemm(P, P, P, P, 0, 256, 256, P, P, None) == 0  # empty
    assert _native.launch_count() == before


def test_gemm_grids_beyond_32_bit_tile_counts_are_refused():
    """The GEMM kernels number their 128 x 256 output tiles with 32-bit ints: a call whose tile
    count would not fit is refused up front (every size here is within the other limits)."""

    L = _native.load_library()
    m, n, k = 128 * 65535, 1 << 30, 256  # 65,535 x 4,194,304 tiles
    assert L.qatf_nvfp4_gemm(P, P, P, P, P, P, m, n, k, P, P, None) == -6
    assert L.qatf_mxfp4_gemm(P, P, P, P, m, n, k, P, P, None) == -6
    assert L.qatf_bf16_gemm(P, 0, P, 0, m, n, k, None, P, P, None) == -6
