"""ctypes binding of libqatf.so (the sm_100a kernels) and thin torch-tensor wrappers.

Every wrapper takes CUDA tensors, checks what the C ABI cannot (device, dtype, layout),
launches on the tensor's device and current stream, and raises ``RuntimeError`` with the
library's status text when a call fails.  There is no fallback: if the shared library is
missing or the tensors are not on an sm_100 GPU, the call fails loudly.
"""

from __future__ import annotations

import contextlib
import ctypes
import threading
from pathlib import Path

import torch

_PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = _PKG_DIR / "libqatf.so"

_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
Q4K_METHOD_CODE = {"grid_search": 0, "minmax": 1}

_lock = threading.Lock()
_lib = None
_checked_devices: set[int] = set()

_SIGNATURES = {
    "qatf_version": (ctypes.c_int, []),
    "qatf_status_string": (ctypes.c_char_p, ["i"]),
    "qatf_launch_count": (ctypes.c_uint64, []),
    "qatf_tensor_amax": (ctypes.c_int, ["p", "i", "l", "p", "p"]),
    "qatf_tensor_amax_update": (ctypes.c_int, ["p", "i", "l", "p", "p"]),
    "qatf_fp8_block_dequant": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "l", "l", "p", "i", "p"]),
    "qatf_nvfp4_qdq_shadow": (ctypes.c_int, ["p", "l", "l", "p", "p", "p", "p"]),
    "qatf_tensor_amax_batched": (ctypes.c_int, ["p", "i", "l", "l", "p", "p"]),
    "qatf_nvfp4_qdq": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p", "p", "p"]),
    "qatf_nvfp4_qdq_experts": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p", "p", "p"]),
    "qatf_nvfp4_fake_quant": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p", "p", "p"]),
    "qatf_nvfp4_fake_quant_noalloc": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p", "p"]),
    "qatf_nvfp4_pack": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p", "p", "p", "p", "p"]),
    "qatf_nvfp4_dequant": (ctypes.c_int, ["p", "p", "p", "l", "l", "p", "p"]),
    "qatf_mxfp4_qdq_even": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p", "p"]),
    "qatf_mxfp4_qdq_ceil": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p"]),
    "qatf_mxfp4_pack": (ctypes.c_int, ["p", "i", "l", "l", "l", "p", "p", "p", "p"]),
    "qatf_mxfp4_dequant": (ctypes.c_int, ["p", "p", "l", "l", "p", "p"]),
    "qatf_ste_backward": (ctypes.c_int, ["p", "i", "l", "p", "p", "p"]),
    "qatf_e2m1_pack_rows": (ctypes.c_int, ["p", "l", "l", "p", "p"]),
    "qatf_e2m1_unpack_rows": (ctypes.c_int, ["p", "l", "l", "p", "p"]),
    "qatf_q4k_encode": (ctypes.c_int, ["p", "i", "l", "l", "l", "i", "p", "p", "p", "p"]),
    "qatf_q4k_dequant": (ctypes.c_int, ["p", "l", "l", "p", "p"]),
    "qatf_nvfp4_operand": (ctypes.c_int, ["p", "i", "l", "l", "p", "i", "p", "p", "p", "p", "p"]),
    "qatf_nvfp4_operand_tracked": (ctypes.c_int, ["p", "i", "l", "l", "p", "i", "p", "p", "p", "p", "p", "p"]),
    "qatf_nvfp4_gemm": (ctypes.c_int, ["p", "p", "p", "p", "p", "p", "l", "l", "l", "p", "p", "p"]),
    "qatf_mxfp4_operand": (ctypes.c_int, ["p", "i", "l", "l", "i", "i", "p", "p", "p", "p", "p"]),
    "qatf_mxfp4_gemm": (ctypes.c_int, ["p", "p", "p", "p", "l", "l", "l", "p", "p", "p"]),
    "qatf_nvfp4_linear_fwd": (ctypes.c_int, ["p", "p", "p", "p", "p", "l", "l", "l", "p", "p", "p", "p", "p", "p", "p",
                                             "p"]),
    "qatf_bf16_gemm": (ctypes.c_int, ["p", "i", "p", "i", "l", "l", "l", "p", "p", "p", "p"]),
    "qatf_bf16_gemm_workspace_size": (ctypes.c_int64, ["l", "l", "l"]),
    "qatf_bf16_gemm_ws": (ctypes.c_int, ["p", "i", "p", "i", "l", "l", "l", "p", "p", "p", "p", "l", "p"]),
    "qatf_kd_forward_kl": (ctypes.c_int, ["p", "p", "i", "l", "l", "l", "l", "f", "p", "p", "p", "f", "p"]),
}
_CTYPE = {"p": ctypes.c_void_p, "i": ctypes.c_int, "l": ctypes.c_int64, "f": ctypes.c_float}


def load_library() -> ctypes.CDLL:
    """Load libqatf.so once; raise if it was not built (``__graft_entry__.build()``)."""

    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the CUDA library first (python -c 'import __graft_entry__ as g; g.build()')"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = [_CTYPE[a] for a in args]
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def launch_count() -> int:
    """Kernels launched by libqatf.so in this process so far (``qatf_launch_count``)."""

    return int(load_library().qatf_launch_count())


def _check(status: int, what: str) -> None:
    if status != 0:
        text = load_library().qatf_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {text} (status {status})")


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise RuntimeError(
                "qatfactory_b200 kernels run on CUDA tensors only (there is no CPU path); "
                f"got a tensor on {t.device}"
            )
        if t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    index = dev.index if dev.index is not None else torch.cuda.current_device()
    if index not in _checked_devices:
        major, minor = torch.cuda.get_device_capability(index)
        if major != 10:
            raise RuntimeError(f"libqatf.so is built for sm_100a (B200); device {index} is sm_{major}{minor}")
        _checked_devices.add(index)
    return dev


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16") from exc


# the current stream of a device as a raw pointer, without building a torch.cuda.Stream object
# (the wrappers run once per quantized tensor, so their host cost shows in eager calls)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_NO_SWITCH = contextlib.nullcontext()


def _stream(dev: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(dev.index if dev.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(dev).cuda_stream


def _scalar_f32(t: torch.Tensor) -> torch.Tensor:
    """A one-element tensor as a contiguous FP32 scalar (no new tensor when it already is one)."""

    if t.dtype == torch.float32 and t.numel() == 1 and t.is_contiguous():
        return t.detach()
    return t.detach().to(torch.float32).reshape(()).contiguous()


def _on(dev: torch.device):
    """Context that makes ``dev`` the current device for a launch: nothing when it already is."""

    if dev.index is None or dev.index == torch.cuda.current_device():
        return _NO_SWITCH
    return torch.cuda.device(dev)


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def mask_nbytes(numel: int) -> int:
    return (numel + 7) // 8


def unpack_mask(mask_bits: torch.Tensor, numel: int, shape) -> torch.Tensor:
    """Expand a bit mask (bit e%8 of byte e//8) into a bool tensor of ``shape``."""

    bits = mask_bits.to(torch.int32).unsqueeze(-1)
    shifts = torch.arange(8, device=mask_bits.device, dtype=torch.int32)
    flat = ((bits >> shifts) & 1).reshape(-1)[:numel].bool()
    return flat.reshape(shape)


def _as_2d(x: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    """(tensor, rows, cols, ld) with unit column stride; copies only when needed."""

    if x.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(x.shape)}")
    if x.stride(1) != 1 or (x.shape[0] > 1 and x.stride(0) < x.shape[1]):
        x = x.contiguous()
    rows, cols = x.shape
    ld = x.stride(0) if rows > 1 else cols
    return x, rows, cols, max(ld, cols)


# ------------------------------------------------------------------------ wrappers


def tensor_amax(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """max |x| as an FP32 0-dim tensor on x's device (NaN-propagating)."""

    dev = _require_cuda(x)
    x = x.contiguous()
    if out is None:
        out = torch.empty((), dtype=torch.float32, device=dev)
    with _on(dev):
        _check(load_library().qatf_tensor_amax(x.data_ptr(), _dtype_code(x), x.numel(), out.data_ptr(), _stream(dev)),
               "qatf_tensor_amax")
    return out


_FP8_FORMAT = {torch.float8_e4m3fn: 0, torch.float8_e5m2: 1}


def fp8_block_dequant(weight: torch.Tensor, scale_inv: torch.Tensor, dtype: torch.dtype = torch.bfloat16):
    """``(float(weight) * scale_inv[block]).to(dtype)`` for FP8 codes ``[..., rows, cols]`` and a
    scale grid ``[..., scale_rows, scale_cols]`` (leading dimensions broadcast to the weight's)."""

    dev = _require_cuda(weight, scale_inv)
    if weight.dtype not in _FP8_FORMAT:
        raise ValueError(f"FP8 block dequantization takes float8_e4m3fn / float8_e5m2 codes, got {weight.dtype}")
    if weight.ndim < 2 or scale_inv.ndim < 2:
        raise ValueError("FP8 weights and scale grids must be at least 2-D")
    rows, cols = weight.shape[-2:]
    srows, scols = scale_inv.shape[-2:]
    if rows % srows or cols % scols:
        raise ValueError(f"FP8 weight shape ({rows}, {cols}) is not divisible by its scale grid ({srows}, {scols}).")
    lead = weight.shape[:-2]
    scales = scale_inv.to(torch.float32).expand(*lead, srows, scols).contiguous()
    codes = weight.contiguous().view(torch.uint8)
    out = torch.empty(weight.shape, dtype=dtype, device=dev)
    batches = codes.numel() // max(rows * cols, 1)
    with _on(dev):
        _check(load_library().qatf_fp8_block_dequant(codes.data_ptr(), _FP8_FORMAT[weight.dtype], batches, rows, cols,
                                                     scales.data_ptr(), srows, scols, out.data_ptr(),
                                                     _dtype_code(out), _stream(dev)), "qatf_fp8_block_dequant")
    return out


def tensor_amax_update(x: torch.Tensor, running: torch.Tensor) -> torch.Tensor:
    """running = max(running, max |x|) in place (one launch); ``running`` is an FP32 0-dim
    tensor on x's device holding an earlier maximum of absolute values."""

    dev = _require_cuda(x, running)
    if running.dtype != torch.float32 or running.numel() != 1 or not running.is_contiguous():
        raise ValueError("running amax must be a contiguous FP32 tensor of one element")
    x = x.contiguous()
    with _on(dev):
        _check(load_library().qatf_tensor_amax_update(x.data_ptr(), _dtype_code(x), x.numel(), running.data_ptr(),
                                                      _stream(dev)), "qatf_tensor_amax_update")
    return running


def nvfp4_qdq_shadow(latent: torch.Tensor, tensor_amax: torch.Tensor, out: torch.Tensor,
                     mask: torch.Tensor) -> None:
    """out (FP32) = NVFP4 fake quantization of latent.to(bfloat16), widened back to FP32, and
    its STE mask bits; latent and out FP32 [rows, cols] contiguous (cols % 16 == 0)."""

    dev = _require_cuda(latent, tensor_amax, out, mask)
    if latent.dtype != torch.float32 or out.dtype != torch.float32 or latent.shape != out.shape:
        raise ValueError("shadow quantization takes FP32 latent and output tensors of one shape")
    if latent.dim() != 2 or not latent.is_contiguous() or not out.is_contiguous():
        raise ValueError("shadow quantization takes dense 2-D tensors")
    rows, cols = latent.shape
    if mask.dtype != torch.uint8 or mask.numel() < mask_nbytes(rows * cols):
        raise ValueError("mask must be a uint8 buffer of ceil(numel / 8) bytes")
    amax = _scalar_f32(tensor_amax)
    with _on(dev):
        _check(load_library().qatf_nvfp4_qdq_shadow(latent.data_ptr(), rows, cols, amax.data_ptr(), out.data_ptr(),
                                                    mask.data_ptr(), _stream(dev)), "qatf_nvfp4_qdq_shadow")


def tensor_amax_batched(x: torch.Tensor) -> torch.Tensor:
    """max |x[b]| over each leading-dimension slice, FP32 [x.shape[0]] (NaN-propagating)."""

    dev = _require_cuda(x)
    x = x.contiguous()
    batches = x.shape[0]
    out = torch.empty(batches, dtype=torch.float32, device=dev)
    with _on(dev):
        _check(load_library().qatf_tensor_amax_batched(x.data_ptr(), _dtype_code(x), batches,
                                                       x.numel() // max(batches, 1), out.data_ptr(), _stream(dev)),
               "qatf_tensor_amax_batched")
    return out


def nvfp4_qdq(x: torch.Tensor, tensor_amax: torch.Tensor, want_mask: bool = True):
    """NVFP4 QDQ of a 2-D tensor with a device FP32 tensor amax -> (y dense, mask bits)."""

    dev = _require_cuda(x, tensor_amax)
    x, rows, cols, ld = _as_2d(x)
    amax = _scalar_f32(tensor_amax)
    y = torch.empty((rows, cols), dtype=x.dtype, device=dev)
    mask = torch.empty(mask_nbytes(rows * cols), dtype=torch.uint8, device=dev) if want_mask else None
    with _on(dev):
        _check(load_library().qatf_nvfp4_qdq(x.data_ptr(), _dtype_code(x), rows, cols, ld, amax.data_ptr(),
                                             y.data_ptr(), _ptr(mask), _stream(dev)), "qatf_nvfp4_qdq")
    return y, mask


def nvfp4_qdq_experts(x: torch.Tensor, tensor_amax: torch.Tensor, want_mask: bool = True):
    """NVFP4 QDQ of a 3-D expert tensor [E, rows, cols] with an FP32 amax per expert [E]
    -> (y [E, rows, cols], mask bits over the flattened tensor)."""

    dev = _require_cuda(x, tensor_amax)
    x = x.contiguous()
    experts, rows, cols = x.shape
    amax = tensor_amax.detach().to(torch.float32).reshape(experts).contiguous()
    y = torch.empty_like(x)
    mask = torch.empty(mask_nbytes(x.numel()), dtype=torch.uint8, device=dev) if want_mask else None
    with _on(dev):
        _check(load_library().qatf_nvfp4_qdq_experts(x.data_ptr(), _dtype_code(x), experts, rows, cols,
                                                     amax.data_ptr(), y.data_ptr(), _ptr(mask), _stream(dev)),
               "qatf_nvfp4_qdq_experts")
    return y, mask


def nvfp4_fake_quant(x: torch.Tensor, amax_scratch: torch.Tensor | None = None, want_mask: bool = True):
    """NVFP4 QDQ with the tensor amax computed on the device -> (y, mask bits, amax)."""

    dev = _require_cuda(x)
    x = x.contiguous()
    rows, cols = x.shape
    if amax_scratch is None:
        amax_scratch = torch.empty((), dtype=torch.float32, device=dev)
    y = torch.empty((rows, cols), dtype=x.dtype, device=dev)
    mask = torch.empty(mask_nbytes(rows * cols), dtype=torch.uint8, device=dev) if want_mask else None
    with _on(dev):
        _check(load_library().qatf_nvfp4_fake_quant(x.data_ptr(), _dtype_code(x), rows, cols, cols,
                                                    amax_scratch.data_ptr(), y.data_ptr(), _ptr(mask), _stream(dev)),
               "qatf_nvfp4_fake_quant")
    return y, mask, amax_scratch


def mxfp4_qdq_even(x: torch.Tensor, want_mask: bool = True):
    dev = _require_cuda(x)
    x, rows, cols, ld = _as_2d(x)
    y = torch.empty((rows, cols), dtype=x.dtype, device=dev)
    mask = torch.empty(mask_nbytes(rows * cols), dtype=torch.uint8, device=dev) if want_mask else None
    with _on(dev):
        _check(load_library().qatf_mxfp4_qdq_even(x.data_ptr(), _dtype_code(x), rows, cols, ld, y.data_ptr(),
                                                  _ptr(mask), _stream(dev)), "qatf_mxfp4_qdq_even")
    return y, mask


def mxfp4_qdq_ceil(x: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(x)
    x, rows, cols, ld = _as_2d(x)
    y = torch.empty((rows, cols), dtype=x.dtype, device=dev)
    with _on(dev):
        _check(load_library().qatf_mxfp4_qdq_ceil(x.data_ptr(), _dtype_code(x), rows, cols, ld, y.data_ptr(),
                                                  _stream(dev)), "qatf_mxfp4_qdq_ceil")
    return y


def ste_backward(grad: torch.Tensor, mask_bits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """grad * mask; ``out=grad`` (a contiguous tensor) applies the mask in place."""

    dev = _require_cuda(grad, mask_bits)
    if out is not None and (out.shape != grad.shape or out.dtype != grad.dtype or not out.is_contiguous()):
        raise ValueError("ste_backward output must be a contiguous tensor of the gradient's shape and dtype")
    grad = grad.contiguous()
    out = torch.empty_like(grad) if out is None else out
    with _on(dev):
        _check(load_library().qatf_ste_backward(grad.data_ptr(), _dtype_code(grad), grad.numel(), mask_bits.data_ptr(),
                                                out.data_ptr(), _stream(dev)), "qatf_ste_backward")
    return out


def nvfp4_pack(x: torch.Tensor, tensor_amax: torch.Tensor, recon: bool = True):
    """-> (packed u8 [r, c/2], scales u8 [r, c/16], weight_scale_2 fp32 [], recon | None)."""

    dev = _require_cuda(x, tensor_amax)
    x, rows, cols, ld = _as_2d(x)
    amax = _scalar_f32(tensor_amax)
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((rows, cols // 16), dtype=torch.uint8, device=dev)
    s2 = torch.empty((), dtype=torch.float32, device=dev)
    rc = torch.empty((rows, cols), dtype=x.dtype, device=dev) if recon else None
    with _on(dev):
        _check(load_library().qatf_nvfp4_pack(x.data_ptr(), _dtype_code(x), rows, cols, ld, amax.data_ptr(),
                                              packed.data_ptr(), scales.data_ptr(), s2.data_ptr(), _ptr(rc),
                                              _stream(dev)), "qatf_nvfp4_pack")
    return packed, scales, s2, rc


def nvfp4_dequant(packed: torch.Tensor, scales: torch.Tensor, scale_2: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(packed, scales, scale_2)
    packed, scales = packed.contiguous(), scales.contiguous().view(torch.uint8)
    s2 = _scalar_f32(scale_2)
    rows, cols = packed.shape[0], packed.shape[1] * 2
    out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
    with _on(dev):
        _check(load_library().qatf_nvfp4_dequant(packed.data_ptr(), scales.data_ptr(), s2.data_ptr(), rows, cols,
                                                 out.data_ptr(), _stream(dev)), "qatf_nvfp4_dequant")
    return out


def mxfp4_pack(x: torch.Tensor, recon: bool = True):
    dev = _require_cuda(x)
    x, rows, cols, ld = _as_2d(x)
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((rows, cols // 32), dtype=torch.uint8, device=dev)
    rc = torch.empty((rows, cols), dtype=x.dtype, device=dev) if recon else None
    with _on(dev):
        _check(load_library().qatf_mxfp4_pack(x.data_ptr(), _dtype_code(x), rows, cols, ld, packed.data_ptr(),
                                              scales.data_ptr(), _ptr(rc), _stream(dev)), "qatf_mxfp4_pack")
    return packed, scales, rc


def mxfp4_dequant(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(packed, scales)
    packed, scales = packed.contiguous(), scales.contiguous()
    rows, cols = packed.shape[0], packed.shape[1] * 2
    out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
    with _on(dev):
        _check(load_library().qatf_mxfp4_dequant(packed.data_ptr(), scales.data_ptr(), rows, cols, out.data_ptr(),
                                                 _stream(dev)), "qatf_mxfp4_dequant")
    return out


def e2m1_pack_rows(nibbles: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(nibbles)
    nibbles = nibbles.contiguous()
    rows, cols = nibbles.shape
    out = torch.empty((rows, cols // 2), dtype=torch.uint8, device=dev)
    with _on(dev):
        _check(load_library().qatf_e2m1_pack_rows(nibbles.data_ptr(), rows, cols, out.data_ptr(), _stream(dev)),
               "qatf_e2m1_pack_rows")
    return out


def e2m1_unpack_rows(packed: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(packed)
    packed = packed.contiguous()
    rows, pcols = packed.shape
    out = torch.empty((rows, pcols * 2), dtype=torch.uint8, device=dev)
    with _on(dev):
        _check(load_library().qatf_e2m1_unpack_rows(packed.data_ptr(), rows, pcols, out.data_ptr(), _stream(dev)),
               "qatf_e2m1_unpack_rows")
    return out


def q4k_encode(x: torch.Tensor, method: str, *, recon: bool = True, mask: bool = True, blocks: bool = True):
    """-> (blocks u8 [r, c/256*144] | None, recon | None, mask bits | None)."""

    if method not in Q4K_METHOD_CODE:
        raise ValueError(f"Unknown Q4_K method {method!r}; supported: {tuple(Q4K_METHOD_CODE)}.")
    dev = _require_cuda(x)
    x, rows, cols, ld = _as_2d(x)
    blk = torch.empty((rows, cols // 256 * 144), dtype=torch.uint8, device=dev) if blocks else None
    rc = torch.empty((rows, cols), dtype=x.dtype, device=dev) if recon else None
    mk = torch.empty(mask_nbytes(rows * cols), dtype=torch.uint8, device=dev) if mask else None
    with _on(dev):
        _check(load_library().qatf_q4k_encode(x.data_ptr(), _dtype_code(x), rows, cols, ld, Q4K_METHOD_CODE[method],
                                              _ptr(rc), _ptr(mk), _ptr(blk), _stream(dev)), "qatf_q4k_encode")
    return blk, rc, mk


def q4k_dequant(blocks: torch.Tensor, in_features: int) -> torch.Tensor:
    dev = _require_cuda(blocks)
    blocks = blocks.contiguous()
    rows = blocks.shape[0]
    out = torch.empty((rows, in_features), dtype=torch.float32, device=dev)
    with _on(dev):
        _check(load_library().qatf_q4k_dequant(blocks.data_ptr(), rows, in_features, out.data_ptr(), _stream(dev)),
               "qatf_q4k_dequant")
    return out


# ------------------------------------------------------------------ W4A4 GEMM operands
K_MAJOR = 0
MN_MAJOR = 1
_GEMM_ERR: dict[int, torch.Tensor] = {}


def gemm_error_word(dev: torch.device) -> torch.Tensor:
    """The device int the tcgen05 GEMMs set when a bounded wait expires (zero while healthy).

    The word is sticky: once set, every later GEMM on the device returns at once with its
    output unwritten.  ``nvfp4_gemm`` and ``bf16_gemm`` watch it (``_gemm_watch``) and raise;
    ``check_gemm_errors`` reads it synchronously and ``reset_gemm_error_word`` clears it."""

    index = dev.index if dev.index is not None else torch.cuda.current_device()
    if index not in _GEMM_ERR:
        _GEMM_ERR[index] = torch.zeros((), dtype=torch.int32, device=torch.device("cuda", index))
    return _GEMM_ERR[index]


class GemmTimeoutError(RuntimeError):
    """A tcgen05 GEMM's bounded wait expired; its output (and every later GEMM's on the same
    device until ``reset_gemm_error_word``) was left unwritten."""


_GEMM_WATCH: dict[int, list] = {}


def _gemm_raise(index: int, value: int) -> None:
    raise GemmTimeoutError(
        f"a tcgen05 GEMM on cuda:{index} gave up on a bounded wait (error word {value}); its output and those "
        "of the GEMMs launched after it are unwritten. Call qatfactory_b200._native.reset_gemm_error_word(device) "
        "before retrying the step.")


def _gemm_watch(dev: torch.device) -> None:
    """Raise if an earlier GEMM on ``dev`` set the error word, then queue a 4-byte copy of the
    word into pinned host memory behind the GEMM just launched.  The copy is stream-ordered and
    the host never waits for it: a failure is reported by the first GEMM call after the copy
    lands (``check_gemm_errors`` reports it at once, with a synchronisation).  Skipped while the
    stream is being captured into a CUDA graph."""

    if torch.cuda.is_current_stream_capturing():
        return
    index = dev.index if dev.index is not None else torch.cuda.current_device()
    ent = _GEMM_WATCH.get(index)
    if ent is None:
        ent = _GEMM_WATCH[index] = [torch.zeros((), dtype=torch.int32).pin_memory(), torch.cuda.Event(), False]
    host, event, in_flight = ent
    if in_flight:
        if not event.query():
            return  # the previous copy has not landed yet; it is checked on a later call
        ent[2] = False
        if int(host) != 0:
            _gemm_raise(index, int(host))
    host.copy_(gemm_error_word(dev), non_blocking=True)
    event.record(torch.cuda.current_stream(dev))
    ent[2] = True


def check_gemm_errors(dev: torch.device) -> None:
    """Synchronise ``dev`` and raise ``GemmTimeoutError`` if a tcgen05 GEMM's bounded wait expired."""

    value = int(gemm_error_word(dev).item())
    if value != 0:
        _gemm_raise(dev.index if dev.index is not None else torch.cuda.current_device(), value)


def reset_gemm_error_word(dev: torch.device) -> None:
    """Clear the sticky error word after a ``GemmTimeoutError`` (synchronises ``dev`` first)."""

    torch.cuda.synchronize(dev)
    gemm_error_word(dev).zero_()
    torch.cuda.synchronize(dev)
    index = dev.index if dev.index is not None else torch.cuda.current_device()
    if index in _GEMM_WATCH:
        _GEMM_WATCH[index][0].zero_()
        _GEMM_WATCH[index][2] = False


OPERAND_A = 0
OPERAND_B = 1


def nvfp4_operand(x: torch.Tensor, tensor_amax: torch.Tensor, role: int = OPERAND_A, deq: bool = True,
                  mask: bool = True, running_amax: torch.Tensor | None = None):
    """BF16 [rows, cols] -> (codes u8 [rows, cols/2], block scales u8 in the layout of ``role``
    (``OPERAND_A`` for the GEMM's A side, ``OPERAND_B`` for its B side), deq BF16 | None,
    mask bits | None).  ``running_amax`` (FP32, one element, x's device) is raised in place to
    max(running_amax, max |x|) by the same pass."""

    dev = _require_cuda(x, tensor_amax) if running_amax is None else _require_cuda(x, tensor_amax, running_amax)
    if running_amax is not None and (running_amax.dtype != torch.float32 or running_amax.numel() != 1
                                     or not running_amax.is_contiguous()):
        raise ValueError("running amax must be a contiguous FP32 tensor of one element")
    x = x.contiguous()
    rows, cols = x.shape
    amax = _scalar_f32(tensor_amax)
    codes = torch.empty((rows, cols // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty(rows * (cols // 16) * 4, dtype=torch.uint8, device=dev)
    d = torch.empty_like(x) if deq else None
    m = torch.empty(mask_nbytes(rows * cols), dtype=torch.uint8, device=dev) if mask else None
    with _on(dev):
        _check(load_library().qatf_nvfp4_operand_tracked(x.data_ptr(), _dtype_code(x), rows, cols, amax.data_ptr(),
                                                         role, codes.data_ptr(), scales.data_ptr(), _ptr(d), _ptr(m),
                                                         _ptr(running_amax), _stream(dev)),
               "qatf_nvfp4_operand")
    return codes, scales, d, m


def nvfp4_gemm(a_codes, a_scales, a_amax, b_codes, b_scales, b_amax) -> torch.Tensor:
    """out[M, N] BF16 = (a_amax/2688)(b_amax/2688) sum_k A[m,k] B[n,k] on NVFP4 operands (A from
    ``nvfp4_operand(..., OPERAND_A)``, B from ``nvfp4_operand(..., OPERAND_B)``)."""

    dev = _require_cuda(a_codes, a_scales, b_codes, b_scales)
    m, k = a_codes.shape[0], a_codes.shape[1] * 2
    n = b_codes.shape[0]
    if b_codes.shape[1] * 2 != k:
        raise ValueError("NVFP4 GEMM operands disagree on K")
    aa = _scalar_f32(a_amax)
    ba = _scalar_f32(b_amax)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    with _on(dev):
        _check(load_library().qatf_nvfp4_gemm(a_codes.data_ptr(), a_scales.data_ptr(), aa.data_ptr(),
                                              b_codes.data_ptr(), b_scales.data_ptr(), ba.data_ptr(), m, n, k,
                                              out.data_ptr(), gemm_error_word(dev).data_ptr(), _stream(dev)),
               "qatf_nvfp4_gemm")
        _gemm_watch(dev)
    return out


MXFP4_EVEN, MXFP4_CEIL = 0, 1  # QATF_MXFP4_EVEN / QATF_MXFP4_CEIL


def mxfp4_operand(x: torch.Tensor, role: int = OPERAND_A, rule: int = MXFP4_CEIL, deq: bool = True,
                  mask: bool = True):
    """BF16 [rows, cols] -> (codes u8 [rows, cols/2], E8M0 block-32 scales u8 in the layout of
    ``role``, deq BF16 | None, mask bits | None) for ``mxfp4_gemm``; ``rule`` is ``MXFP4_EVEN``
    (weights) or ``MXFP4_CEIL`` (activations: the mask is all true)."""

    dev = _require_cuda(x)
    x = x.contiguous()
    rows, cols = x.shape
    codes = torch.empty((rows, cols // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty(rows * (cols // 32) * 4, dtype=torch.uint8, device=dev)
    d = torch.empty_like(x) if deq else None
    m = torch.empty(mask_nbytes(rows * cols), dtype=torch.uint8, device=dev) if mask else None
    with _on(dev):
        _check(load_library().qatf_mxfp4_operand(x.data_ptr(), _dtype_code(x), rows, cols, role, rule,
                                                 codes.data_ptr(), scales.data_ptr(), _ptr(d), _ptr(m), _stream(dev)),
               "qatf_mxfp4_operand")
    return codes, scales, d, m


def mxfp4_gemm(a_codes, a_scales, b_codes, b_scales) -> torch.Tensor:
    """out[M, N] BF16 = sum_k A[m,k] B[n,k] on MXFP4 operands (A from
    ``mxfp4_operand(..., OPERAND_A)``, B from ``mxfp4_operand(..., OPERAND_B)``)."""

    dev = _require_cuda(a_codes, a_scales, b_codes, b_scales)
    m, k = a_codes.shape[0], a_codes.shape[1] * 2
    n = b_codes.shape[0]
    if b_codes.shape[1] * 2 != k:
        raise ValueError("MXFP4 GEMM operands disagree on K")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    with _on(dev):
        _check(load_library().qatf_mxfp4_gemm(a_codes.data_ptr(), a_scales.data_ptr(), b_codes.data_ptr(),
                                              b_scales.data_ptr(), m, n, k, out.data_ptr(),
                                              gemm_error_word(dev).data_ptr(), _stream(dev)),
               "qatf_mxfp4_gemm")
        _gemm_watch(dev)
    return out


def nvfp4_linear_sync_words(m: int, k: int) -> int:
    """QATF_NVFP4_LINEAR_SYNC_WORDS: one readiness counter per (128-row tile, 256-column K
    stage) plus one work counter."""

    return (m // 128) * (k // 256) + 1


def nvfp4_linear_fwd(x: torch.Tensor, x_amax: torch.Tensor, w_codes: torch.Tensor, w_scales: torch.Tensor,
                     w_amax: torch.Tensor, deq: bool = True, mask: bool = True):
    """W4A4 forward with the activation quantizer inside the FP4 GEMM (one launch): BF16 x
    [M, K] with static tensor amax x_amax, weight operand from
    ``nvfp4_operand(w, w_amax, OPERAND_B)`` -> (out BF16 [M, N], x codes, x scales (A layout),
    x deq BF16 | None, x mask bits | None).  Codes, scales, deq and mask equal
    ``nvfp4_operand(x, x_amax, OPERAND_A)``'s, and out equals ``nvfp4_gemm`` on them."""

    dev = _require_cuda(x, x_amax, w_codes, w_scales, w_amax)
    x = x.contiguous()
    if x.dim() != 2 or x.dtype != torch.bfloat16:
        raise ValueError("nvfp4_linear_fwd expects a 2-D BF16 activation")
    m, k = x.shape
    n = w_codes.shape[0]
    if w_codes.shape[1] * 2 != k:
        raise ValueError("NVFP4 linear operands disagree on K")
    xa = _scalar_f32(x_amax)
    wa = _scalar_f32(w_amax)
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty(m * (k // 16) * 4, dtype=torch.uint8, device=dev)
    d = torch.empty_like(x) if deq else None
    mk = torch.empty(mask_nbytes(m * k), dtype=torch.uint8, device=dev) if mask else None
    sync = torch.empty(nvfp4_linear_sync_words(m, k), dtype=torch.int32, device=dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    with _on(dev):
        _check(load_library().qatf_nvfp4_linear_fwd(x.data_ptr(), xa.data_ptr(), w_codes.data_ptr(),
                                                    w_scales.data_ptr(), wa.data_ptr(), m, n, k, codes.data_ptr(),
                                                    scales.data_ptr(), _ptr(d), _ptr(mk), sync.data_ptr(),
                                                    out.data_ptr(), gemm_error_word(dev).data_ptr(), _stream(dev)),
               "qatf_nvfp4_linear_fwd")
        _gemm_watch(dev)
    return out, codes, scales, d, mk


def bf16_gemm(a: torch.Tensor, a_layout: int, b: torch.Tensor, b_layout: int,
              mask_bits: torch.Tensor | None = None, split_k: bool = True) -> torch.Tensor:
    """out[M, N] BF16 = A B^T (FP32 accumulation) times the optional STE mask over out.

    A is [M, K] (K_MAJOR) or [K, M] (MN_MAJOR); B is [N, K] (K_MAJOR) or [K, N] (MN_MAJOR).
    ``split_k`` lets a mostly idle last wave of tiles run as K-slices through a workspace
    (``qatf_bf16_gemm_ws``; FP32 summation order differs there); False gives every tile whole."""

    dev = _require_cuda(a, b)
    a = a.contiguous()
    b = b.contiguous()
    m, k = (a.shape[0], a.shape[1]) if a_layout == K_MAJOR else (a.shape[1], a.shape[0])
    n, kb = (b.shape[0], b.shape[1]) if b_layout == K_MAJOR else (b.shape[1], b.shape[0])
    if k != kb:
        raise ValueError(f"BF16 GEMM operands disagree on K: {k} vs {kb}")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    with _on(dev):
        lib = load_library()
        # a last wave that would leave most SM pairs idle is split along K into a workspace
        ws_bytes = int(lib.qatf_bf16_gemm_workspace_size(m, n, k)) if split_k else 0
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
        _check(lib.qatf_bf16_gemm_ws(a.data_ptr(), a_layout, b.data_ptr(), b_layout, m, n, k, _ptr(mask_bits),
                                     out.data_ptr(), gemm_error_word(dev).data_ptr(), _ptr(ws), ws_bytes,
                                     _stream(dev)),
               "qatf_bf16_gemm")
        _gemm_watch(dev)
    return out


def kd_forward_kl(student: torch.Tensor, teacher: torch.Tensor, temperature: float = 1.0,
                  row_valid: torch.Tensor | None = None, want_grad: bool = True, grad_scale: float = 1.0):
    """2-D logits [rows, vocab] (unit column stride) -> (per-row KL FP32 [rows], gradient wrt the
    student logits [rows, vocab] in the student's dtype, or None)."""

    dev = _require_cuda(student, teacher)
    if student.shape != teacher.shape or student.dtype != teacher.dtype:
        raise ValueError("student and teacher logits must have the same shape and dtype")
    if student.stride(1) != 1:
        student = student.contiguous()
    if teacher.stride(1) != 1:
        teacher = teacher.contiguous()
    rows, vocab = student.shape
    row_loss = torch.empty(rows, dtype=torch.float32, device=dev)
    grad = torch.empty((rows, vocab), dtype=student.dtype, device=dev) if want_grad else None
    valid = None if row_valid is None else row_valid.to(torch.uint8).contiguous()
    with _on(dev):
        _check(load_library().qatf_kd_forward_kl(student.data_ptr(), teacher.data_ptr(), _dtype_code(student), rows,
                                                 vocab, student.stride(0), teacher.stride(0), float(temperature),
                                                 _ptr(valid), row_loss.data_ptr(), _ptr(grad), float(grad_scale),
                                                 _stream(dev)),
               "qatf_kd_forward_kl")
    return row_loss, grad
