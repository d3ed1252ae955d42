"""GPU tests of the torch operator with the packed-layer schema,
``torch.ops.rpfq.wide_linear(x, codes, gamma_re, gamma_im, bias, n_c, k_c,
act_bits, gelu)`` (registered like the reference's ``Library("quant",
"DEF")`` op, RPFQ-ViT-main/quant_models/kernel.py:599-605): called with the
reference's packed tensors, compared with the CPU oracle on both of its
paths — the fused decode for at most 256 rows and the cached decode + GEMM
above — with activation quantization and GELU, 3-D inputs, a head-sized
layer whose dims are not multiples of 8, and 4-bit codes."""

import numpy as np
import pytest
import torch

from oracle import packed_ref as pr
from tests.helpers import rel_err, to_numpy_packed

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _lists(layer):
    names = [f"u_s{i}" for i in range(layer.stages)] + [f"w_s{i}" for i in range(layer.stages)]
    return ([layer.planes[n][0] for n in names], [layer.planes[n][1] for n in names],
            [layer.planes[n][2] for n in names])


def _reference(layer, x, act_bits, gelu, code_bits=2):
    np_layer = to_numpy_packed(layer)
    if code_bits == 2:
        dense = pr.dense_weight_from_packed(np_layer, layer.n_c, layer.k_c)
    else:  # the extension's oracle: the fp16 coefficient planes
        dense = pr.dense_fp16_from_planes(pr.coefficient_planes(np_layer, layer.n_c, layer.k_c,
                                                                code_bits=code_bits)).astype(np.float32)
    y = pr.wide_linear(x.reshape(-1, x.shape[-1]), dense, np_layer["bias"].astype(np.float32),
                       act_bits=act_bits or None)
    return pr.gelu_erf(y) if gelu else y


@pytest.mark.parametrize("shape", [(1, 768), (197, 768), (4, 197, 768), (1576, 768)])
@pytest.mark.parametrize("act_bits,gelu", [(0, False), (4, False), (0, True), (4, True)])
def test_packed_op_matches_oracle(cuda, shape, act_bits, gelu):
    from rpfq_review_b200 import ops
    from rpfq_review_b200.packing import random_packed
    layer = random_packed(384, 384, seed=31, device=cuda)
    codes, gre, gim = _lists(layer)
    g = torch.Generator().manual_seed(sum(shape) + act_bits)
    x = torch.randn(*shape, generator=g).half()
    before = dict(ops.dense_cache_stats)
    y = torch.ops.rpfq.wide_linear(x.to(cuda), codes, gre, gim, layer.bias, 384, 384, act_bits, gelu)
    assert y.shape == (*shape[:-1], 768) and y.dtype == torch.float16
    ref = _reference(layer, x.float().numpy(), act_bits, gelu)
    assert rel_err(y.float().cpu().numpy().reshape(ref.shape), ref) < TOL
    rows = int(np.prod(shape[:-1]))
    decoded = ops.dense_cache_stats["decodes"] - before["decodes"] + ops.dense_cache_stats["hits"] - before["hits"]
    assert decoded == (0 if rows <= ops.FUSED_DECODE_MAX_ROWS else 1)


def test_packed_op_caches_the_decode(cuda):
    from rpfq_review_b200 import ops
    from rpfq_review_b200.packing import random_packed
    layer = random_packed(256, 384, seed=32, device=cuda)
    codes, gre, gim = _lists(layer)
    x = torch.randn(1000, 768, generator=torch.Generator().manual_seed(1)).half().to(cuda)
    before = dict(ops.dense_cache_stats)
    y1 = torch.ops.rpfq.wide_linear(x, codes, gre, gim, layer.bias, 256, 384)
    y2 = torch.ops.rpfq.wide_linear(x, codes, gre, gim, layer.bias, 256, 384)
    assert torch.equal(y1, y2)
    assert ops.dense_cache_stats["decodes"] - before["decodes"] == 1
    assert ops.dense_cache_stats["hits"] - before["hits"] == 1
    codes[0].bitwise_xor_(1)  # a plane written in place decodes again
    torch.ops.rpfq.wide_linear(x, codes, gre, gim, layer.bias, 256, 384)
    assert ops.dense_cache_stats["decodes"] - before["decodes"] == 2


@pytest.mark.parametrize("n_c,k_c,code_bits,rows", [(500, 384, 2, 8), (192, 200, 4, 300), (192, 200, 4, 5)])
def test_packed_op_dense_path_shapes(cuda, n_c, k_c, code_bits, rows):
    """Layers the fused decode does not take (n_c = 500: the 1000-class head;
    4-bit codes) go through the decoded matrix at any row count."""
    from rpfq_review_b200.packing import random_packed
    layer = random_packed(n_c, k_c, seed=33, code_bits=code_bits, device=cuda)
    codes, gre, gim = _lists(layer)
    x = torch.randn(rows, 2 * k_c, generator=torch.Generator().manual_seed(2)).half()
    y = torch.ops.rpfq.wide_linear(x.to(cuda), codes, gre, gim, layer.bias, n_c, k_c, 0, False)
    ref = _reference(layer, x.float().numpy(), 0, False, code_bits)
    assert rel_err(y.float().cpu().numpy(), ref) < TOL


def test_packed_op_rejects_bad_arguments(cuda):
    from rpfq_review_b200.packing import random_packed
    layer = random_packed(64, 64, seed=34, device=cuda)
    codes, gre, gim = _lists(layer)
    x = torch.zeros(4, 128, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        torch.ops.rpfq.wide_linear(x, codes[:3], gre[:3], gim[:3], None, 64, 64)  # odd plane count
    with pytest.raises(ValueError):
        torch.ops.rpfq.wide_linear(x, codes, gre, gim, torch.zeros(3, dtype=torch.float16, device=cuda), 64, 64)
    with pytest.raises(ValueError):
        torch.ops.rpfq.wide_linear(torch.zeros(4, 100, dtype=torch.float16, device=cuda), codes, gre, gim, None, 64, 64)
