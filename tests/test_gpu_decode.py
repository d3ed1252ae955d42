"""GPU parity tests of the fused decode path (``rpfq_wide_linear_sm100`` with
``dense == NULL``): the packed codes are decoded inside the GEMM, so the
layer reads only the packed planes.

Bar: max|y - y_ref| / max|y_ref| <= 1e-3 against the float64 product of the
oracle's fp16 coefficient planes (the same bar as the prepacked path), and
the same bar between the fused and the prepacked path on identical inputs.
Gammas vary per 256-column block so that the block indexing is exercised.
"""

import numpy as np
import pytest
import torch

from oracle import packed_ref as pr
from tests.helpers import rel_err, to_numpy_packed

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _ops():
    from rpfq_review_b200 import ops
    return ops


def _layer(n_c, k_c, stages, seed, device):
    """random_packed with per-block gamma factors (fp16-exact powers of two
    times a few mantissas), so that each 256-column block decodes differently."""
    from rpfq_review_b200.packing import PackedLayer, random_packed
    base = random_packed(n_c, k_c, seed=seed, stages=stages)
    g = torch.Generator().manual_seed(seed + 1)
    planes = {}
    for name, (c, gr, gi) in base.planes.items():
        f = torch.tensor([0.5, 0.75, 1.0, 1.25, 2.0], dtype=torch.float32)
        fr = f[torch.randint(0, 5, gr.shape, generator=g)]
        fi = f[torch.randint(0, 5, gi.shape, generator=g)]
        planes[name] = (c, (gr.float() * fr).half(), (gi.float() * fi).half())
    return PackedLayer(n_c, k_c, stages, base.code_bits, planes, base.bias).to(device)


def _reference(layer, x, act_bits=None, gelu=False, residual=None):
    n_c, k_c = layer.n_c, layer.k_c
    dense = pr.dense_fp16_from_planes(pr.coefficient_planes(to_numpy_packed(layer), n_c, k_c))
    y = pr.wide_linear(x.cpu().numpy(), dense, layer.bias.cpu().numpy(), act_bits)
    if gelu:
        y = pr.gelu_erf(y)
    if residual is not None:
        y = y + residual.cpu().double().numpy()
    return y


SHAPES = [
    (1, 64, 64, 2),        # one token, one row block
    (7, 40, 200, 2),       # ragged rows in the last block, K tail inside a stage
    (128, 384, 384, 2),    # one full sub-tile, two gamma blocks
    (197, 1152, 384, 2),   # a ViT qkv layer at batch 1 (two sub-tiles)
    (256, 96, 520, 2),     # largest m, three gamma blocks, K tail
    (129, 8, 8, 2),        # 8 complex rows, one partial stage; m just over a sub-tile
    (200, 48, 64, 1),      # one residual stage
    (33, 64, 136, 4),      # four stages: all eight planes
    (16, 4736, 64, 2),     # enough rows for the 32-row blocks
    (16, 9472, 72, 2),     # enough rows for the 64-row blocks
]


@pytest.mark.parametrize("m,n_c,k_c,stages", SHAPES)
def test_fused_decode_matches_oracle(cuda, m, n_c, k_c, stages):
    ops = _ops()
    layer = _layer(n_c, k_c, stages, seed=m * 131 + n_c + k_c, device=cuda)
    g = torch.Generator().manual_seed(m + n_c)
    x = torch.randn((m, 2 * k_c), generator=g).half().to(cuda)
    y = ops.wide_linear(x, layer, None)
    torch.cuda.synchronize()
    ref = _reference(layer, x)
    assert rel_err(y.cpu().numpy(), ref) <= TOL
    y_dense = ops.wide_linear(x, layer, ops.prepack(layer))
    assert rel_err(y.cpu().numpy(), y_dense.cpu().double().numpy()) <= TOL


@pytest.mark.parametrize("m", [5, 197])
def test_fused_decode_epilogues(cuda, m):
    ops = _ops()
    n_c, k_c = 384, 384
    layer = _layer(n_c, k_c, 2, seed=77 + m, device=cuda)
    g = torch.Generator().manual_seed(m)
    x = torch.randn((m, 2 * k_c), generator=g).half().to(cuda)
    # bias + GELU, fp16 out
    y = ops.wide_linear(x, layer, None, activation="gelu")
    assert rel_err(y.cpu().numpy(), _reference(layer, x, gelu=True)) <= TOL
    # fp16 residual added in place
    r16 = torch.randn((m, 2 * n_c), generator=g).half().to(cuda)
    want = _reference(layer, x, residual=r16)
    ops.wide_linear(x, layer, None, residual=r16, out=r16)
    assert rel_err(r16.cpu().numpy(), want) <= TOL
    # fp32 output with an fp32 residual in place (the ViT residual stream)
    r32 = torch.randn((m, 2 * n_c), generator=g).to(cuda)
    want = _reference(layer, x, residual=r32)
    ops.wide_linear(x, layer, None, residual=r32, out=r32)
    assert rel_err(r32.cpu().numpy(), want) <= TOL
    # activation quantization in front (same quantized x as the prepacked path)
    yq = ops.wide_linear(x, layer, None, act_bits=4)
    yq_dense = ops.wide_linear(x, layer, ops.prepack(layer), act_bits=4)
    assert rel_err(yq.cpu().numpy(), _reference(layer, x, act_bits=4)) <= TOL
    assert rel_err(yq.cpu().numpy(), yq_dense.cpu().double().numpy()) <= TOL


def test_fused_decode_strided_rows(cuda):
    """x and y as row slices of wider buffers (ldx, ldy > row length)."""
    ops = _ops()
    n_c, k_c, m = 64, 128, 50
    layer = _layer(n_c, k_c, 2, seed=5, device=cuda)
    xb = torch.randn((m, 2 * k_c + 64), generator=torch.Generator().manual_seed(3)).half().to(cuda)
    x = xb[:, 32:32 + 2 * k_c]
    yb = torch.zeros((m, 2 * n_c + 16), dtype=torch.float16, device=cuda)
    y = yb[:, 8:8 + 2 * n_c]
    ops.wide_linear(x, layer, None, out=y)
    assert rel_err(y.cpu().numpy(), _reference(layer, x)) <= TOL
    assert torch.count_nonzero(yb[:, :8]) == 0 and torch.count_nonzero(yb[:, 8 + 2 * n_c:]) == 0


def test_fused_decode_empty_and_limits(cuda):
    ops = _ops()
    layer = _layer(64, 64, 2, seed=9, device=cuda)
    y = ops.wide_linear(torch.empty((0, 128), dtype=torch.float16, device=cuda), layer, None)
    assert y.shape == (0, 128)
    with pytest.raises(ValueError, match="dense coefficients are required"):
        ops.wide_linear(torch.zeros((ops.FUSED_DECODE_MAX_ROWS + 1, 128), dtype=torch.float16, device=cuda),
                        layer, None)
    from rpfq_review_b200.packing import random_packed
    wide = random_packed(64, 64, seed=4, code_bits=3, device=cuda)
    with pytest.raises(NotImplementedError, match="2-bit codes only"):
        ops.wide_linear(torch.zeros((4, 128), dtype=torch.float16, device=cuda), wide, None)


def test_packed_module_without_dense_cache(cuda):
    """PackedPhaseLinear(cache_dense=False): the fused path for short inputs,
    a temporary dense matrix for long ones; no cache is kept either way."""
    from rpfq_review_b200 import PackedPhaseLinear
    layer = _layer(192, 384, 2, seed=21, device=cuda)
    cached = PackedPhaseLinear.from_packed(layer, enable_act_quant=True, act_num_bits=4, activation="gelu")
    lean = PackedPhaseLinear.from_packed(layer, enable_act_quant=True, act_num_bits=4, activation="gelu",
                                         cache_dense=False)
    g = torch.Generator().manual_seed(8)
    for m in (3, 197, 300):
        x = torch.randn((m, 768), generator=g).half().to(cuda)
        a, b = cached(x), lean(x)
        assert rel_err(b.cpu().numpy(), a.cpu().double().numpy()) <= TOL
    assert lean.dense is None


def test_fused_decode_no_device_errors(cuda):
    from rpfq_review_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


# ViT-B layers at one image (m = 197) and shapes whose row blocks leave most
# SMs idle: the fused decode splits K over a cluster of CTAs per row block.
SPLIT_SHAPES = [
    (197, 384, 1536, 2, "residual"),  # fc2: 24 row blocks x 6 splits
    (197, 384, 384, 2, "residual"),   # proj: 24 x 3
    (197, 1152, 384, 2, "none"),      # qkv: 72 x 2
    (198, 192, 768, 2, "gelu"),       # DeiT-S fc1-like, 12 blocks
    (5, 64, 520, 2, "none"),          # K tail inside a stage, ragged rows
    (256, 40, 1024, 1, "residual"),   # one stage, ragged last block
]


@pytest.mark.parametrize("m,n_c,k_c,stages,epi", SPLIT_SHAPES)
@pytest.mark.parametrize("split_k", [0, 2, 8])
def test_fused_decode_split_k(cuda, m, n_c, k_c, stages, epi, split_k):
    """Split-K against the oracle and the unsplit kernel (the partials are
    summed in a fixed order: two calls are bit-identical)."""
    ops = _ops()
    layer = _layer(n_c, k_c, stages, seed=m * 7 + n_c + k_c, device=cuda)
    g = torch.Generator().manual_seed(m + k_c)
    x = torch.randn((m, 2 * k_c), generator=g).half().to(cuda)
    res = torch.randn((m, 2 * n_c), generator=g).float().to(cuda) if epi == "residual" else None
    act = "gelu" if epi == "gelu" else "none"

    def run(split):
        out = res.clone() if res is not None else None
        return ops.wide_linear(x, layer, None, residual=out, out=out, activation=act,
                               out_dtype=torch.float32 if res is not None else torch.float16, split_k=split)

    y = run(split_k)
    y2 = run(split_k)
    y1 = run(1)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    ref = _reference(layer, x, gelu=epi == "gelu", residual=res)
    assert rel_err(y.cpu().numpy(), ref) <= TOL
    assert rel_err(y.cpu().double().numpy(), y1.cpu().double().numpy()) <= TOL
    from rpfq_review_b200 import _lib
    assert _lib.device_error() == 0
