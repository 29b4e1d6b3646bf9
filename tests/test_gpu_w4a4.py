"""W4A4 NVFP4 linear on the tensor cores: the operand quantizer against the CPU oracle (bit
exact), the block-scaled FP4 GEMM against the exact product of its operands and against the
reference's BF16 matmul of the dequantized operands (relative Frobenius error <= 1e-2, the
north-star tolerance for GEMMs), and the BF16 GEMMs of the backward pass."""

import numpy as np
import pytest
import torch

import oracle
from qatfactory_b200 import _native, workloads

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float64)


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def _lane_word_offset(lane: torch.Tensor, word: torch.Tensor) -> torch.Tensor:
    """Byte offset of word `word` (0..7) of `lane` (0..127) in a 4 KB 128x256b block."""

    return (lane // 8) * 256 + (lane % 8) * 16 + (word // 4) * 128 + (word % 4) * 4


def role_a_layout(scales: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Row-major [rows, cols/16] block scales -> the A-side layout (4 KB per 128 rows x 128
    columns; row r's word for K-block kb is word 4(kb%2) + (r/32)%4 of the lanes r%32 + 32q)."""

    sc = scales.reshape(rows, cols // 64, 4).cpu()
    out = torch.zeros(rows * (cols // 16) * 4, dtype=torch.uint8)
    r = torch.arange(rows).reshape(-1, 1)
    kb = torch.arange(cols // 64).reshape(1, -1)
    blk = ((r // 128) * (cols // 128) + kb // 2) * 4096
    for q in range(4):
        base = blk + _lane_word_offset(r % 32 + 32 * q, 4 * (kb % 2) + (r // 32) % 4)
        for s in range(4):
            out[(base + s).reshape(-1)] = sc[:, :, s].reshape(-1)
    return out


def role_b_layout(scales: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Row-major [rows, cols/16] block scales -> the B-side layout (4 KB per 256 rows x 64
    columns; the word of row r sits as word (r/32)%8 in each of the lanes r%32 + 32q)."""

    sc = scales.reshape(rows, cols // 64, 4).cpu()
    out = torch.zeros(rows * (cols // 16) * 4, dtype=torch.uint8)
    r = torch.arange(rows).reshape(-1, 1)
    kb = torch.arange(cols // 64).reshape(1, -1)
    blk = ((r // 256) * (cols // 64) + kb) * 4096
    for q in range(4):
        base = blk + _lane_word_offset(r % 32 + 32 * q, (r // 32) % 8)
        for s in range(4):
            out[(base + s).reshape(-1)] = sc[:, :, s].reshape(-1)
    return out


def decode(codes: torch.Tensor, scales_rm: torch.Tensor, amax: float) -> torch.Tensor:
    """Exact FP64 value of an NVFP4 operand: E2M1 code * E4M3 scale * amax / 2688."""

    c = codes.cpu().to(torch.int64)
    nib = torch.stack([c & 0xF, c >> 4], dim=-1).reshape(c.shape[0], -1)
    val = E2M1[nib & 7] * torch.where(nib & 8 > 0, -1.0, 1.0).double()
    sc = scales_rm.cpu().view(torch.float8_e4m3fn).double().repeat_interleave(16, dim=1)
    gs = float(np.float32(amax) / np.float32(2688.0))
    return val * sc * gs


def operand_input(rows, cols, seed):
    x = workloads.student_t_outliers((rows, cols), seed=seed, outlier_seed=seed + 1).to(torch.bfloat16)
    x[3, :32] = 0  # zero blocks
    x[5, 16:32] = 1e-32  # a block below 2^-100 relative: the exact per-element path
    return x


@pytest.mark.parametrize("rows,cols,role", [(128, 128, 0), (256, 1024, 0), (256, 1024, 1), (384, 4096, 0),
                                           (512, 4096, 1), (256, 64, 1)])
def test_operand_matches_oracle_pack_and_qdq(rows, cols, role):
    x = operand_input(rows, cols, seed=40 + rows)
    amax = x.float().abs().amax()
    codes, scales, deq, mask = _native.nvfp4_operand(x.to(DEV), amax.to(DEV), role)
    o_packed, o_scales, _, _ = oracle.nvfp4_pack(x, amax)
    o_y, o_mask = oracle.nvfp4_qdq(x, amax)
    assert torch.equal(codes.cpu(), o_packed)
    layout = role_a_layout if role == _native.OPERAND_A else role_b_layout
    assert torch.equal(scales.cpu(), layout(o_scales.view(torch.uint8), rows, cols))
    assert torch.equal(deq.cpu().view(torch.int16), o_y.view(torch.int16))
    want = torch.from_numpy(np.packbits(o_mask.reshape(-1).numpy().astype(np.uint8), bitorder="little"))
    assert torch.equal(mask.cpu(), want)


@pytest.mark.parametrize("role", [0, 1])
def test_operand_zero_amax(role):
    x = operand_input(256, 256, seed=77)
    codes, scales, deq, mask = _native.nvfp4_operand(x.to(DEV), torch.zeros((), device=DEV), role)
    assert int(codes.count_nonzero()) == 0
    layout = role_a_layout if role == _native.OPERAND_A else role_b_layout
    ones = torch.ones(256, 256 // 16, dtype=torch.uint8)
    assert torch.equal(scales.cpu(), layout(ones, 256, 256))  # 2^-9 for every block (nvfp4.py:427-435)
    assert int(deq.count_nonzero()) == 0
    assert bool((mask == 0xFF).all())


def _nvfp4_case(m, n, k, seed):
    x = operand_input(m, k, seed).to(DEV)
    w = workloads.normal((n, k), 0.02, seed=seed + 7).to(torch.bfloat16).to(DEV)
    xa, wa = x.float().abs().amax(), w.float().abs().amax()
    ax = _native.nvfp4_operand(x, xa, _native.OPERAND_A)
    aw = _native.nvfp4_operand(w, wa, _native.OPERAND_B)
    return x, w, xa, wa, ax, aw


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (256, 512, 2048), (384, 768, 1280)])
def test_nvfp4_gemm_matches_exact_product_and_bf16_reference(m, n, k):
    x, w, xa, wa, (cx, sx, dx, _), (cw, sw, dw, _) = _nvfp4_case(m, n, k, seed=m + n + k)
    out = _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    o_pk_x, o_sc_x, _, _ = oracle.nvfp4_pack(x.cpu(), xa.cpu())
    o_pk_w, o_sc_w, _, _ = oracle.nvfp4_pack(w.cpu(), wa.cpu())
    exact = decode(o_pk_x, o_sc_x.view(torch.uint8), float(xa)) @ decode(o_pk_w, o_sc_w.view(torch.uint8), float(wa)).T
    assert rel_fro(out.cpu(), exact) < 4e-3  # BF16 rounding of the output only
    ref = (dx.float() @ dw.float().T).to(torch.bfloat16)  # reference: BF16 matmul of dequantized operands
    assert rel_fro(out.cpu(), ref.cpu()) < 1e-2


def test_nvfp4_gemm_config4_forward():
    xb, wb, _ = workloads.config4_inputs()
    x, w = xb.to(DEV), wb.to(DEV)
    xa, wa = _native.tensor_amax(x), _native.tensor_amax(w)
    cx, sx, dx, _ = _native.nvfp4_operand(x, xa, _native.OPERAND_A)
    cw, sw, dw, _ = _native.nvfp4_operand(w, wa, _native.OPERAND_B)
    out = _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa)
    ref = torch.nn.functional.linear(dx, dw)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    assert rel_fro(out, ref) < 1e-2


@pytest.mark.parametrize("a_layout", [_native.K_MAJOR, _native.MN_MAJOR])
@pytest.mark.parametrize("b_layout", [_native.K_MAJOR, _native.MN_MAJOR])
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("m", [256, 384])  # CTA-pair tiles (M % 256 == 0) and single-CTA tiles
def test_bf16_gemm_layouts(a_layout, b_layout, masked, m):
    n, k = 512, 576
    g = torch.Generator().manual_seed(a_layout * 4 + b_layout * 2 + masked + m)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, generator=g).to(torch.bfloat16)
    mask = torch.rand(m * n, generator=g) < 0.9
    bits = torch.from_numpy(np.packbits(mask.numpy().astype(np.uint8), bitorder="little")).to(DEV)
    a_st = a if a_layout == _native.K_MAJOR else a.T.contiguous()
    b_st = b if b_layout == _native.K_MAJOR else b.T.contiguous()
    out = _native.bf16_gemm(a_st.to(DEV), a_layout, b_st.to(DEV), b_layout, bits if masked else None)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    ref = a.double() @ b.double().T
    if masked:
        ref = ref * mask.reshape(m, n).double()
        assert bool((out.cpu()[~mask.reshape(m, n)] == 0).all())
    assert rel_fro(out.cpu(), ref) < 4e-3


def test_w4a4_backward_gemms_config4():
    xb, wb, dyb = workloads.config4_inputs()
    x, w, dy = xb.to(DEV), wb.to(DEV), dyb.to(DEV)
    xa, wa = _native.tensor_amax(x), _native.tensor_amax(w)
    _, _, dx_q, mx = _native.nvfp4_operand(x, xa)
    _, _, dw_q, mw = _native.nvfp4_operand(w, wa)
    grad_x = _native.bf16_gemm(dy, _native.K_MAJOR, dw_q, _native.MN_MAJOR, mx)
    grad_w = _native.bf16_gemm(dy, _native.MN_MAJOR, dx_q, _native.MN_MAJOR, mw)
    ref_x = (dy @ dw_q) * _native.unpack_mask(mx, x.numel(), x.shape)
    ref_w = (dy.T @ dx_q) * _native.unpack_mask(mw, w.numel(), w.shape)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    assert rel_fro(grad_x, ref_x) < 1e-2
    assert rel_fro(grad_w, ref_w) < 1e-2


def test_nvfp4_linear_w4a4_forward_backward_matches_reference_formulation():
    """NVFP4Linear with W4A4 on the tensor cores vs the reference's own formulation,
    F.linear(fake_quantize_nvfp4_activation(x), fake_quantize_nvfp4(w)) with STE autograd."""

    from qatfactory_b200.quant.formats.nvfp4 import (NVFP4Linear, fake_quantize_nvfp4,
                                                      fake_quantize_nvfp4_activation)

    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 768, bias=True, device=DEV, dtype=torch.bfloat16)
    q = NVFP4Linear.from_linear(lin)
    q._quantize_activations = True
    x = workloads.student_t_outliers((2, 128, 512), seed=9, outlier_seed=10).to(DEV).requires_grad_(True)
    y = q(x)
    g = torch.randn_like(y)
    y.backward(g)
    gx, gw, gb = x.grad.clone(), q.weight.grad.clone(), q.bias.grad.clone()

    x2 = x.detach().clone().requires_grad_(True)
    w2 = q.weight.detach().clone().requires_grad_(True)
    b2 = q.bias.detach().clone().requires_grad_(True)
    ref = torch.nn.functional.linear(fake_quantize_nvfp4_activation(x2, q._input_amax_static),
                                     fake_quantize_nvfp4(w2), b2)
    ref.backward(g)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    assert rel_fro(y.detach(), ref.detach()) < 1e-2
    assert rel_fro(gx, x2.grad) < 1e-2
    assert rel_fro(gw, w2.grad) < 1e-2
    assert rel_fro(gb, b2.grad) < 1e-2


@pytest.mark.parametrize("lead,k,n", [((7,), 512, 768), ((2, 100), 4112, 1000), ((130,), 48, 40), ((3, 128), 256, 256)])
def test_w4a4_off_tile_shapes_are_padded_onto_the_tensor_cores(lead, k, n, monkeypatch):
    """Token rows % 128, in features % 256 and out features % 256 are zero-padded to the GEMM
    tiles (the last case needs none): the tensor-core GEMM runs, outputs and all three gradients
    agree with the reference formulation within 1e-2, and the running input maximum is the
    maximum of the real input."""

    from qatfactory_b200.quant.formats.nvfp4 import (NVFP4Linear, fake_quantize_nvfp4,
                                                      fake_quantize_nvfp4_activation)

    calls = []
    gemm = _native.nvfp4_gemm
    monkeypatch.setattr(_native, "nvfp4_gemm", lambda *a, **kw: calls.append(1) or gemm(*a, **kw))
    torch.manual_seed(1)
    lin = torch.nn.Linear(k, n, bias=True, device=DEV, dtype=torch.bfloat16)
    q = NVFP4Linear.from_linear(lin)
    q._quantize_activations = True
    q._track_input_amax = True
    q.train()
    x = workloads.student_t_outliers((*lead, k), seed=19, outlier_seed=20).to(DEV).requires_grad_(True)
    with torch.no_grad():
        q(x * 0.5)  # bootstraps the static input scale and the running maximum below max |x|
    y = q(x)  # raises the running maximum inside the (padded) operand pass
    assert y.shape == (*lead, n) and calls == [1, 1]
    g = torch.randn_like(y)
    y.backward(g)

    x2 = x.detach().clone().requires_grad_(True)
    w2 = q.weight.detach().clone().requires_grad_(True)
    b2 = q.bias.detach().clone().requires_grad_(True)
    ref = torch.nn.functional.linear(fake_quantize_nvfp4_activation(x2, q._input_amax_static),
                                     fake_quantize_nvfp4(w2), b2)
    ref.backward(g)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    assert rel_fro(y.detach(), ref.detach()) < 1e-2
    assert rel_fro(x.grad, x2.grad) < 1e-2
    assert rel_fro(q.weight.grad, w2.grad) < 1e-2
    assert rel_fro(q.bias.grad, b2.grad) < 1e-2
    assert float(q._input_amax) == float(x.detach().float().abs().max())


def test_gemms_as_the_first_cuda_work_of_a_fresh_thread():
    """Autograd runs the backward on its own thread; the GEMMs must not rely on a context made
    current by earlier CUDA work on the calling thread."""

    import threading

    a = torch.randn(256, 256, device=DEV).to(torch.bfloat16)
    b = torch.randn(256, 256, device=DEV).to(torch.bfloat16)
    x = workloads.normal((256, 256), 1.0, seed=3).to(DEV)
    w = workloads.normal((256, 256), 0.02, seed=4).to(DEV)
    xa, wa = x.float().abs().amax(), w.float().abs().amax()
    cx, sx, _, _ = _native.nvfp4_operand(x, xa, _native.OPERAND_A)
    cw, sw, _, _ = _native.nvfp4_operand(w, wa, _native.OPERAND_B)
    torch.cuda.synchronize()
    results = {}

    def worker():
        try:
            results["bf16"] = _native.bf16_gemm(a, _native.K_MAJOR, b, _native.MN_MAJOR)
            results["fp4"] = _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa)
            torch.cuda.synchronize()
        except Exception as exc:  # surfaced in the main thread
            results["error"] = exc

    th = threading.Thread(target=worker)
    th.start()
    th.join()
    assert "error" not in results, results.get("error")
    assert rel_fro(results["bf16"], a.float() @ b.float()) < 4e-3
    assert results["fp4"].shape == (256, 256)


def test_expired_wait_word_is_reported_by_the_gemm_wrappers_and_can_be_reset():
    """The GEMMs' sticky error word (set here from the host, as an expired bounded wait would
    set it; no kernel waits on anything) makes every later GEMM return with its output
    unwritten: the wrappers must raise GemmTimeoutError instead of passing garbage on, and
    reset_gemm_error_word must bring the device back."""

    g = torch.Generator().manual_seed(41)
    a = (torch.randn(128, 256, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    b = (torch.randn(256, 256, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    good = _native.bf16_gemm(a, _native.K_MAJOR, b, _native.K_MAJOR)
    _native.check_gemm_errors(DEV)
    word = _native.gemm_error_word(DEV)
    try:
        word.fill_(1)
        torch.cuda.synchronize()
        with pytest.raises(_native.GemmTimeoutError):
            for _ in range(3):  # the first call queues the copy of the word; a later one reports it
                _native.bf16_gemm(a, _native.K_MAJOR, b, _native.K_MAJOR)
                torch.cuda.synchronize()
        with pytest.raises(_native.GemmTimeoutError):
            _native.check_gemm_errors(DEV)
    finally:
        _native.reset_gemm_error_word(DEV)
    again = _native.bf16_gemm(a, _native.K_MAJOR, b, _native.K_MAJOR)
    _native.check_gemm_errors(DEV)
    assert torch.equal(again, good)


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (256, 512, 2048), (384, 768, 1280), (1152, 512, 512)])
def test_fused_linear_forward_equals_operand_pass_then_gemm(m, n, k):
    """One launch that quantizes X inside the FP4 GEMM gives exactly the two-launch result: the
    same codes, A-layout scales, deq and mask as the operand pass, and the same output bits."""

    x, w, xa, wa, (cx, sx, dx, mx), (cw, sw, dw, _) = _nvfp4_case(m, n, k, seed=3 * m + n + k)
    ref = _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa)
    for _ in range(2):  # the second call reuses the allocator's blocks: the sync words are cleared per call
        out, fc, fs, fd, fm = _native.nvfp4_linear_fwd(x, xa, cw, sw, wa)
        torch.cuda.synchronize()
        assert torch.equal(fc, cx) and torch.equal(fs, sx)
        assert torch.equal(fd.view(torch.int16), dx.view(torch.int16)) and torch.equal(fm, mx)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    _native.check_gemm_errors(DEV)


def test_fused_linear_forward_config4_and_zero_amax():
    x, w, _ = workloads.config4_inputs()
    x, w = x.to(DEV), w.to(DEV)
    xa, wa = x.float().abs().amax(), w.float().abs().amax()
    cx, sx, dx, mx = _native.nvfp4_operand(x, xa, _native.OPERAND_A)
    cw, sw, _, _ = _native.nvfp4_operand(w, wa, _native.OPERAND_B)
    out, fc, fs, fd, fm = _native.nvfp4_linear_fwd(x, xa, cw, sw, wa)
    ref = _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa)
    torch.cuda.synchronize()
    assert torch.equal(fc, cx) and torch.equal(fs, sx) and torch.equal(fm, mx)
    assert torch.equal(fd.view(torch.int16), dx.view(torch.int16))
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    # a zero activation amax: zero codes, zero deq, all-true mask, zero output (nvfp4.py:427-435, :493-494)
    out0, fc0, _, fd0, fm0 = _native.nvfp4_linear_fwd(x[:256], torch.zeros((), device=DEV), cw, sw, wa)
    torch.cuda.synchronize()
    assert int(fc0.count_nonzero()) == 0 and int(fd0.count_nonzero()) == 0 and bool((fm0 == 0xFF).all())
    assert int(out0.count_nonzero()) == 0
    _native.check_gemm_errors(DEV)


@pytest.mark.parametrize("m,n,k", [(6144, 4096, 4096), (2048, 1024, 2048)])
def test_bf16_gemm_split_k_tail_matches_whole_tiles(m, n, k):
    """A last wave split into K-slices (workspace path) agrees with whole tiles to FP32
    summation order, with the STE mask applied identically."""

    g = torch.Generator().manual_seed(m + n)
    a = torch.randn(k, m, generator=g).to(torch.bfloat16).to(DEV)  # MN-major A, like wgrad's dY
    b = (torch.randn(k, n, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    mask = torch.randint(0, 256, (m * n // 8,), generator=g, dtype=torch.uint8).to(DEV)
    lib = _native.load_library()
    ws = int(lib.qatf_bf16_gemm_workspace_size(m, n, k))
    whole = _native.bf16_gemm(a, _native.MN_MAJOR, b, _native.MN_MAJOR, mask, split_k=False)
    split = _native.bf16_gemm(a, _native.MN_MAJOR, b, _native.MN_MAJOR, mask)
    ref = (a.float().T @ b.float()) * _native.unpack_mask(mask, m * n, (m, n)).float()
    _native.check_gemm_errors(DEV)
    assert rel_fro(split.float(), ref) < 4e-3 and rel_fro(whole.float(), ref) < 4e-3
    assert torch.equal((split == 0), (whole == 0)) or rel_fro(split.float(), whole.float()) < 1e-3
    if ws:  # the split path ran: most tiles are whole and bit-identical
        same = (split.view(torch.int16) == whole.view(torch.int16)).float().mean()
        assert float(same) > 0.5


@pytest.mark.parametrize("role", [0, 1])
def test_operand_pass_raises_the_running_amax(role):
    """qatf_nvfp4_operand_tracked: identical outputs, and running = max(running, max |x|)."""

    x = operand_input(256, 1024, seed=91).to(DEV)
    amax = x.float().abs().amax()
    plain = _native.nvfp4_operand(x, amax, role)
    for start, expect in ((0.0, amax), (1e6, torch.tensor(1e6))):
        running = torch.tensor(start, device=DEV)
        tracked = _native.nvfp4_operand(x, amax, role, running_amax=running)
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(plain, tracked))
        assert float(running) == float(expect)
    x[100, 7] = float("nan")
    running = torch.tensor(2.0, device=DEV)
    _native.nvfp4_operand(x, amax, role, running_amax=running)
    assert bool(torch.isnan(running))


def test_nvfp4_linear_w4a4_running_input_amax_over_steps():
    """The W4A4 running input maximum (nvfp4.py:634-648): the bootstrap forward sets it, later
    forwards raise it inside the operand pass (tensor-core shapes) or by one update launch (off-tile
    shapes), and a loaded value is copied, never mutated."""

    from qatfactory_b200.quant.formats.nvfp4 import NVFP4Linear

    torch.manual_seed(1)
    lin = torch.nn.Linear(512, 768, bias=False, device=DEV, dtype=torch.bfloat16)
    q = NVFP4Linear.from_linear(lin)
    q._quantize_activations = True
    q._track_input_amax = True
    q.train()
    xs = [workloads.student_t_outliers((128, 512), seed=s, outlier_seed=s + 1).to(DEV) * f
          for s, f in ((20, 1.0), (22, 3.0), (24, 0.5))]
    xs.append(torch.randn(3, 512, device=DEV, dtype=torch.bfloat16) * 40)  # off-tile rows: update launch
    expect = None
    for x in xs:
        q(x)
        cur = x.float().abs().amax()
        expect = cur if expect is None else torch.maximum(expect, cur)
        torch.cuda.synchronize()
        assert float(q._input_amax) == float(expect)
    loaded = torch.tensor(1e4, device=DEV)
    q._input_amax = loaded
    q(xs[0])
    assert float(loaded) == 1e4 and float(q._input_amax) == 1e4 and q._input_amax is not loaded
