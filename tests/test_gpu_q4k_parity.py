"""GPU parity of the Q4_K encoder/decoder (through libqatf.so) with the reference.

The reference's own Triton encoder agrees with its torch encoder on only ~99.4% of
weights (reference tests/quant/test_q4_k.py:96-111, :135-150); the bar here is 100%:
blocks, reconstruction and STE mask bit for bit, for both level-1 methods, against the
reference's outputs (golden fixtures, min-max digests) and against the IEEE-arithmetic
oracle.  The single documented gap: the reference host's torch.sqrt is not correctly
rounded, which moves 8 of 753,664 grid-search super-blocks of layer 0.
"""

import hashlib
import json

import pytest
import torch

import oracle
from qatfactory_b200 import _native, workloads
from qatfactory_b200.quant import (
    dequantize_q4_k,
    fake_quantize_q4_k,
    get_quant_format,
    pack_deploy_weight,
    quantize_q4_k,
    v_head_reorder_perm,
)
from tests.golden.fixtures import GOLDEN_DIR, load_cases

pytestmark = pytest.mark.gpu

Q4K = load_cases(GOLDEN_DIR / "q4k_golden.npz")
DIGESTS = json.loads((GOLDEN_DIR / "digests.json").read_text())
DEV = "cuda"
METHODS = ("minmax", "grid_search")


def bits(t):
    t = t.detach().cpu()
    return t.view(torch.int16) if t.dtype in (torch.bfloat16, torch.float16) else (
        t.view(torch.int32) if t.dtype == torch.float32 else t)


def digest(t):
    t = t.detach().cpu().contiguous().reshape(-1)
    return hashlib.sha256(t.view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("name", sorted(Q4K))
def test_q4k_golden(name):
    c = Q4K[name]
    x = c["x"].to(DEV)
    blocks, recon, mask = _native.q4k_encode(x, c["method"])
    assert torch.equal(blocks.cpu(), c["blocks"])
    assert torch.equal(bits(recon), bits(c["recon"]))
    assert torch.equal(_native.unpack_mask(mask, x.numel(), x.shape).cpu(), c["mask"])
    assert torch.equal(bits(dequantize_q4_k(blocks, x.shape[1])), bits(c["dequant"]))


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("dtype,scale", ((torch.bfloat16, 0.05), (torch.bfloat16, 1e-3), (torch.float32, 1.0), (torch.float16, 0.1)))
def test_random_weights_match_oracle_exactly(method, dtype, scale):
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(256, 2048, generator=g) * scale).to(dtype)
    blocks, recon, mask = _native.q4k_encode(w.to(DEV), method)
    ref_blocks, ref_recon, ref_mask = oracle.q4k_encode(w, method)
    assert torch.equal(blocks.cpu(), ref_blocks)
    assert torch.equal(bits(recon), bits(ref_recon))
    assert torch.equal(_native.unpack_mask(mask, w.numel(), w.shape).cpu(), ref_mask)


@pytest.mark.parametrize("method", METHODS)
def test_self_consistency_and_fake_quant(method):
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(64, 1024, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    r = quantize_q4_k(w, method=method)
    assert torch.equal(dequantize_q4_k(r.packed_weight, w.shape[1]).to(r.reconstruction.dtype), r.reconstruction)
    assert torch.equal(fake_quantize_q4_k(w, method=method), r.reconstruction)


def test_ste_gradient_is_the_mask():
    g = torch.Generator().manual_seed(2)
    w = torch.randn(4, 512, generator=g).to(DEV).requires_grad_()
    fake_quantize_q4_k(w).sum().backward()
    _, _, ref_mask = oracle.q4k_encode(w.detach().cpu(), "grid_search")
    assert torch.equal(w.grad.cpu(), ref_mask.float())


def test_col_perm_fake_quant_matches_deploy_pack():
    g = torch.Generator().manual_seed(3)
    col_perm = v_head_reorder_perm(2, 2, 128)
    w = (torch.randn(64, col_perm.numel(), generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    fq = fake_quantize_q4_k(w, col_perm=col_perm)
    deploy = pack_deploy_weight(w, col_perm=col_perm)
    inverse = torch.empty_like(col_perm)
    inverse[col_perm] = torch.arange(col_perm.numel())
    un = dequantize_q4_k(deploy, col_perm.numel()).index_select(1, inverse.to(DEV))
    assert torch.equal(un.to(fq.dtype), fq)


def test_format_pack_hook_shapes():
    fmt = get_quant_format("q4_k")
    packed = fmt.pack_weight(torch.randn(4, 256, dtype=torch.bfloat16, device=DEV))
    assert packed.dtype == torch.uint8 and packed.shape == (4, 144)


def test_row_strided_input():
    g = torch.Generator().manual_seed(4)
    wide = (torch.randn(32, 1024, generator=g) * 0.05).to(torch.bfloat16)
    view = wide.to(DEV)[:, 256:768]
    for method in METHODS:
        blocks, recon, _ = _native.q4k_encode(view, method)
        ref_blocks, ref_recon, _ = oracle.q4k_encode(wide[:, 256:768].contiguous(), method)
        assert torch.equal(blocks.cpu(), ref_blocks)
        assert torch.equal(bits(recon), bits(ref_recon))


def test_config3_layer0_minmax_matches_reference_digests():
    for name, w in workloads.config3_layer(0):
        r = quantize_q4_k(w.to(DEV), method="minmax")
        assert digest(r.packed_weight) == DIGESTS[f"config3/layer0/{name}/minmax/blocks"], name
        assert digest(r.reconstruction) == DIGESTS[f"config3/layer0/{name}/minmax/recon"], name


def test_config3_layer0_grid_search_matches_ieee_oracle_digests():
    """Grid search equals the IEEE-arithmetic restatement bit for bit.  The reference itself
    weights each sub-block with torch.sqrt, which on its host is not correctly rounded, so
    it agrees on 99.9997% of the weights (8 of 753,664 super-blocks of layer 0 differ); the
    recorded agreement is checked here too."""

    for name, w in workloads.config3_layer(0):
        r = quantize_q4_k(w.to(DEV), method="grid_search")
        assert digest(r.packed_weight) == DIGESTS[f"config3/layer0/{name}/grid_search/oracle_blocks"], name
        assert digest(r.reconstruction) == DIGESTS[f"config3/layer0/{name}/grid_search/oracle_recon"], name
    agree = DIGESTS["config3/layer0/grid_search/reference_agreement"]
    assert agree["superblocks_differ"] / agree["superblocks"] < 2e-5


def test_config3_size_independent_roundtrip_on_a_later_layer():
    """encode -> decode reproduces the reconstruction bit for bit at full size (layer 35)."""

    for name, w in workloads.config3_layer(35):
        r = quantize_q4_k(w.to(DEV), method="minmax")
        assert torch.equal(dequantize_q4_k(r.packed_weight, w.shape[1]).to(torch.bfloat16), r.reconstruction), name


def _stack_digests(part: str):
    p = GOLDEN_DIR / f"config3_stack_{part}.json"
    return json.loads(p.read_text()) if p.exists() else None


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(memoryview(t.contiguous().reshape(-1).view(torch.uint8).numpy())).hexdigest()


@pytest.mark.timeout(1800)
def test_config3_all_layers_match_reference_and_oracle_digests():
    """Configuration 3 as configured: all 36 layers x 7 linears (6.95 G weights).  Min-max
    blocks and reconstruction equal the reference's quantize_q4_k digests, and grid-search
    blocks and reconstruction equal the IEEE oracle's, tensor by tensor.  The inputs are drawn
    on the host (the reference's bits) a few layers ahead on worker threads, and the outputs
    are hashed on worker threads while the GPU encodes the next tensors."""

    from concurrent.futures import ThreadPoolExecutor

    minmax = _stack_digests("minmax")
    grid = _stack_digests("grid")
    assert minmax is not None, "tests/golden/config3_stack_minmax.json is missing"
    layers = workloads.QWEN3_8B_LAYERS
    # grid-search oracle digests are recorded layer by layer (the oracle's search runs for
    # hours on a CPU); every recorded layer is checked
    grid_layers = set() if grid is None else {l for l in range(layers)
                                             if f"layer{l}/grid_search/reference_agreement" in grid}
    mismatches, checked = [], 0
    with ThreadPoolExecutor(8) as pool:
        ahead = 3
        gens = {l: pool.submit(workloads.config3_layer, l) for l in range(min(ahead, layers))}
        pending = []
        for l in range(layers):
            layer = gens.pop(l).result()
            if l + ahead < layers:
                gens[l + ahead] = pool.submit(workloads.config3_layer, l + ahead)
            for name, w in layer:
                wd = w.to(DEV)
                methods = [("minmax", minmax, "blocks", "recon")]
                if l in grid_layers:
                    methods.append(("grid_search", grid, "oracle_blocks", "oracle_recon"))
                for method, want, kb, kr in methods:
                    blocks, recon, _ = _native.q4k_encode(wd, method, mask=False)
                    key = f"layer{l}/{name}/{method}"
                    pending.append((f"{key}/{kb}", want[f"{key}/{kb}"], pool.submit(_sha, blocks.cpu())))
                    pending.append((f"{key}/{kr}", want[f"{key}/{kr}"], pool.submit(_sha, recon.cpu())))
            del layer, wd
            for key, expect, fut in pending:  # bound host memory: settle this layer's hashes
                checked += 1
                if fut.result() != expect:
                    mismatches.append(key)
            pending = []
    assert checked == (layers + len(grid_layers)) * 7 * 2
    assert not mismatches, mismatches[:10]
    if grid_layers:
        agree = [grid[f"layer{l}/grid_search/reference_agreement"] for l in sorted(grid_layers)]
        differ = sum(a["superblocks_differ"] for a in agree)
        total = sum(a["superblocks"] for a in agree)
        assert total == len(grid_layers) * 27131904 // layers
        assert differ / total < 2e-5  # the documented torch.sqrt gap of the reference's grid search
