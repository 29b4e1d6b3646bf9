"""CPU oracle for the fake-quantization path -- TEST INFRASTRUCTURE ONLY.

A ctypes front end over ``oracle/qatf_oracle.c``, the plain-C restatement of the
reference's PyTorch CPU quantizers (qatfactory/quant/formats/nvfp4.py, mxfp4.py, q4_k.py).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
this package, and only as the checker or the timed CPU baseline; the product path
(``qatfactory_b200``) never imports it and has no CPU fallback.

Parity pin: the C functions are checked against golden vectors produced by the reference
itself (``tests/golden/make_golden.py`` imports the reference in the build container and
records its outputs) and against the reference tests' known answers
(``tests/test_oracle_golden.py``).

All functions take and return CPU ``torch.Tensor`` objects; inputs may be float32,
float16 or bfloat16 and are read in their own dtype, as the reference does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (system gcc, -ffp-contract=off)."""

    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(_LIB_PATH))
    vp, i64, f32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
    sigs = {
        "oracle_tensor_amax": (f32, [vp, i32, i64]),
        "oracle_nvfp4_qdq": (None, [vp, i32, i64, i64, f32, vp, vp]),
        "oracle_nvfp4_pack": (None, [vp, i32, i64, i64, f32, vp, vp, vp, vp]),
        "oracle_nvfp4_dequant": (None, [vp, vp, f32, i64, i64, vp]),
        "oracle_mxfp4_qdq_even": (None, [vp, i32, i64, i64, vp, vp]),
        "oracle_mxfp4_qdq_ceil": (None, [vp, i32, i64, i64, vp]),
        "oracle_mxfp4_pack": (None, [vp, i32, i64, i64, vp, vp, vp]),
        "oracle_mxfp4_dequant": (None, [vp, vp, i64, i64, vp]),
        "oracle_ste_backward": (None, [vp, i32, i64, vp, vp]),
        "oracle_q4k_encode": (None, [vp, i32, i64, i64, i32, vp, vp, vp]),
        "oracle_q4k_dequant": (None, [vp, i64, i64, vp]),
        "oracle_float_to_bf16": (ctypes.c_uint16, [f32]),
        "oracle_float_to_half": (ctypes.c_uint16, [f32]),
        "oracle_cast_e4m3": (f32, [f32]),
        "oracle_round_to_e2m1": (f32, [f32]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _c(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cpu":
        raise ValueError("the oracle runs on CPU tensors only")
    return t.contiguous()


def _code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {t.dtype}") from exc


def set_num_threads(n: int) -> None:
    """OpenMP thread count of the oracle (used by the CPU-baseline timing)."""

    os.environ["OMP_NUM_THREADS"] = str(int(n))
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(int(n))
    except OSError:  # pragma: no cover - libgomp ships with the system gcc
        pass


def tensor_amax(x: torch.Tensor) -> torch.Tensor:
    x = _c(x)
    return torch.tensor(_load().oracle_tensor_amax(x.data_ptr(), _code(x), x.numel()), dtype=torch.float32)


def nvfp4_qdq(x: torch.Tensor, tensor_amax: torch.Tensor | float | None = None):
    """``_fake_quantize_nvfp4_torch`` (nvfp4.py:465-501) -> (quantized, in_range bool)."""

    x = _c(x)
    rows, cols = x.shape
    amax = float(tensor_amax) if tensor_amax is not None else float(tensor_amax_of(x))
    y = torch.empty_like(x)
    mask = torch.empty(x.shape, dtype=torch.uint8)
    _load().oracle_nvfp4_qdq(x.data_ptr(), _code(x), rows, cols, amax, y.data_ptr(), mask.data_ptr())
    return y, mask.bool()


def tensor_amax_of(x: torch.Tensor) -> float:
    return float(tensor_amax(x))


def nvfp4_pack(x: torch.Tensor, tensor_amax: torch.Tensor | float | None = None, recon: bool = True):
    """``quantize_nvfp4`` (nvfp4.py:400-462) -> (packed u8, scales e4m3 bytes, scale_2, recon)."""

    x = _c(x)
    rows, cols = x.shape
    amax = float(tensor_amax) if tensor_amax is not None else tensor_amax_of(x)
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8)
    scales = torch.empty(rows, cols // 16, dtype=torch.uint8)
    s2 = torch.empty((), dtype=torch.float32)
    rc = torch.empty_like(x) if recon else None
    _load().oracle_nvfp4_pack(
        x.data_ptr(), _code(x), rows, cols, amax, packed.data_ptr(), scales.data_ptr(), s2.data_ptr(),
        rc.data_ptr() if rc is not None else None,
    )
    return packed, scales, s2, rc


def nvfp4_dequant(packed: torch.Tensor, scales: torch.Tensor, scale_2) -> torch.Tensor:
    packed, scales = _c(packed), _c(scales.view(torch.uint8))
    rows, cols = packed.shape[0], packed.shape[1] * 2
    out = torch.empty(rows, cols, dtype=torch.float32)
    _load().oracle_nvfp4_dequant(packed.data_ptr(), scales.data_ptr(), float(scale_2), rows, cols, out.data_ptr())
    return out


def mxfp4_qdq_even(x: torch.Tensor):
    """``_fake_quantize_mxfp4_torch`` (mxfp4.py:154-174) -> (quantized, in_range bool)."""

    x = _c(x)
    rows, cols = x.shape
    y = torch.empty_like(x)
    mask = torch.empty(x.shape, dtype=torch.uint8)
    _load().oracle_mxfp4_qdq_even(x.data_ptr(), _code(x), rows, cols, y.data_ptr(), mask.data_ptr())
    return y, mask.bool()


def mxfp4_qdq_ceil(x: torch.Tensor) -> torch.Tensor:
    """``_fake_quantize_mxfp4_activation_torch`` (mxfp4.py:205-222), flattened to 2-D."""

    shape = x.shape
    x = _c(x.reshape(-1, shape[-1]))
    rows, cols = x.shape
    if cols % 32:
        raise ValueError("MXFP4 activation quantization needs a last dim divisible by 32")
    y = torch.empty_like(x)
    _load().oracle_mxfp4_qdq_ceil(x.data_ptr(), _code(x), rows, cols, y.data_ptr())
    return y.reshape(shape)


def mxfp4_pack(x: torch.Tensor, recon: bool = True):
    """``quantize_mxfp4`` (mxfp4.py:126-151) -> (packed u8, biased E8M0 scales u8, recon)."""

    x = _c(x)
    rows, cols = x.shape
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8)
    scales = torch.empty(rows, cols // 32, dtype=torch.uint8)
    rc = torch.empty_like(x) if recon else None
    _load().oracle_mxfp4_pack(
        x.data_ptr(), _code(x), rows, cols, packed.data_ptr(), scales.data_ptr(), rc.data_ptr() if rc is not None else None
    )
    return packed, scales, rc


def mxfp4_dequant(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    packed, scales = _c(packed), _c(scales)
    rows, cols = packed.shape[0], packed.shape[1] * 2
    out = torch.empty(rows, cols, dtype=torch.float32)
    _load().oracle_mxfp4_dequant(packed.data_ptr(), scales.data_ptr(), rows, cols, out.data_ptr())
    return out


def ste_backward(grad: torch.Tensor, in_range: torch.Tensor) -> torch.Tensor:
    """``grad_output * in_range`` (nvfp4.py:39-41)."""

    grad = _c(grad)
    mask = _c(in_range.to(torch.uint8))
    out = torch.empty_like(grad)
    _load().oracle_ste_backward(grad.data_ptr(), _code(grad), grad.numel(), mask.data_ptr(), out.data_ptr())
    return out


Q4K_METHODS = {"grid_search": 0, "minmax": 1}


def q4k_encode(x: torch.Tensor, method: str = "grid_search"):
    """``quantize_q4_k`` + ``fake_quantize_q4_k`` (q4_k.py:245-340).

    Returns (packed block_q4_K bytes [rows, cols/256*144], reconstruction, in_range bool).
    """

    x = _c(x)
    rows, cols = x.shape
    if cols % 256:
        raise ValueError("Q4_K needs in_features divisible by 256")
    blocks = torch.empty(rows, cols // 256 * 144, dtype=torch.uint8)
    recon = torch.empty_like(x)
    mask = torch.empty(x.shape, dtype=torch.uint8)
    _load().oracle_q4k_encode(
        x.data_ptr(), _code(x), rows, cols, Q4K_METHODS[method], recon.data_ptr(), mask.data_ptr(), blocks.data_ptr()
    )
    return blocks, recon, mask.bool()


def q4k_dequant(blocks: torch.Tensor, in_features: int) -> torch.Tensor:
    blocks = _c(blocks)
    rows = blocks.shape[0]
    out = torch.empty(rows, in_features, dtype=torch.float32)
    _load().oracle_q4k_dequant(blocks.data_ptr(), rows, in_features, out.data_ptr())
    return out


def float_to_bf16_bits(v: float) -> int:
    return int(_load().oracle_float_to_bf16(v))


def float_to_half_bits(v: float) -> int:
    return int(_load().oracle_float_to_half(v))


def cast_e4m3(v: float) -> float:
    return float(_load().oracle_cast_e4m3(v))


def round_to_e2m1(v: float) -> float:
    return float(_load().oracle_round_to_e2m1(v))
