"""The allocation-free NVFP4 entry point, qatf_nvfp4_fake_quant_noalloc, called through the
C ABI.

It serves callers that cannot allocate device memory (a C/cgo/JNI host that binds only
libqatf.so and has no device allocator, or a runtime whose memory pool must not see
cudaMalloc inside a step): instead of a caller-owned amax word it reduces the tensor amax in
a static array inside the library.  Its results must equal those of the allocating entry
point, qatf_nvfp4_fake_quant, bit for bit (the tolerance of every parity test here is zero),
on consecutive calls that reuse the static array.  Collected last (file name) so that a run
stopping at the first failure has already run every other test.
"""

import pytest
import torch

from qatfactory_b200 import _native

pytestmark = pytest.mark.gpu

QATF_F32, QATF_F16, QATF_BF16 = 0, 1, 2
QATF_ERR_UNSUPPORTED = -6
_CODE = {torch.float32: QATF_F32, torch.float16: QATF_F16, torch.bfloat16: QATF_BF16}
_BITS = {torch.float32: torch.int32, torch.float16: torch.int16, torch.bfloat16: torch.int16}


def _call_noalloc(x: torch.Tensor):
    lib = _native.load_library()
    rows, cols = x.shape
    y = torch.empty((rows, cols), dtype=x.dtype, device=x.device)
    mask = torch.empty((x.numel() + 7) // 8, dtype=torch.uint8, device=x.device)
    status = lib.qatf_nvfp4_fake_quant_noalloc(x.data_ptr(), _CODE[x.dtype], rows, cols, cols, y.data_ptr(),
                                               mask.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert status == 0, lib.qatf_status_string(status)
    return y, mask


def _input(shape, dtype, scale, misaligned):
    g = torch.Generator().manual_seed(shape[0])
    n = shape[0] * shape[1]
    flat = (torch.randn(n + 1, generator=g) * scale).to(dtype).cuda()
    # a view one element into its storage: not 16-byte aligned, so both entry points take
    # their scalar (unvectorised) paths
    x = flat[1:].view(shape) if misaligned else flat[:n].view(shape)
    assert (x.data_ptr() % 16 != 0) == misaligned
    return x


@pytest.mark.parametrize("shape,dtype,scale,misaligned", [
    ((4096, 4096), torch.bfloat16, 0.02, False),
    ((257, 1000), torch.bfloat16, 3.0, False),
    ((3000, 528), torch.float32, 1e-3, False),
    ((1024, 768), torch.float16, 0.5, False),
    ((255, 1024), torch.bfloat16, 0.02, True),
    ((129, 2048), torch.float16, 4.0, True),
    ((77, 320), torch.float32, 1e-2, True),
])
def test_noalloc_matches_allocating_entry_point_on_consecutive_calls(shape, dtype, scale, misaligned):
    x = _input(shape, dtype, scale, misaligned)
    y_ref, mask_ref, amax_ref = _native.nvfp4_fake_quant(x)
    for _ in range(2):  # the second call reuses the static array left by the first
        y, mask = _call_noalloc(x)
        torch.cuda.synchronize()
        assert torch.equal(y.view(_BITS[dtype]), y_ref.view(_BITS[dtype]))
        assert torch.equal(mask, mask_ref)


def test_noalloc_rejects_tensors_beyond_its_static_scratch():
    lib = _native.load_library()
    dummy = 256  # never dereferenced: the size check comes first
    status = lib.qatf_nvfp4_fake_quant_noalloc(dummy, QATF_BF16, 1 << 20, 1 << 10, 1 << 10, dummy, None, None)
    assert status == QATF_ERR_UNSUPPORTED
