"""GPU tests of the GEMM's narrow tail: when the CTA-pair tiles leave a last
wave at most half full, those tiles are cut into 4 (or 2) column pieces of 64
(or 128) columns dealt out over the idle pairs. Each case checks the plan
(rpfq_gemm_plan_sm100), the result against float64, and that it is
bit-identical to whole 256 x 256 tiles (cta_pair = 2 forced): every output
element is still accumulated over all of K in one pass, in the same order."""

import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3

# (m, n, k, epilogue, pieces): ViT-B at 32 images per GPU (m = 6304: proj / fc2
# 75 pair tiles, qkv 225, fc1 300 on 74 pairs), 64 images (12608), a ragged m,
# and a last wave of 34 tiles that takes two pieces per tile.
CASES = [
    (6304, 768, 768, "residual_f32", 4),
    (6304, 2304, 768, "none", 4),
    (6304, 3072, 768, "gelu", 4),
    (6304, 768, 3072, "residual_f32", 4),
    (12608, 768, 3072, "residual_f32", 4),
    (6301, 2304, 768, "none", 4),
    (3072, 2304, 768, "none", 2),
    (6304, 3072, 768, "f32", 4),
]


def _inputs(m, n, k, epi, dev):
    g = torch.Generator().manual_seed(m * 5 + n * 3 + k)
    x = torch.randn(m, k, generator=g).half()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, generator=g) * 0.1).half()
    r = torch.randn(m, n, generator=g) if epi == "residual_f32" else None
    return x.to(dev), w.to(dev), b.to(dev), (r.to(dev) if r is not None else None)


@pytest.mark.parametrize("m,n,k,epi,pieces", CASES)
def test_narrow_tail(cuda, m, n, k, epi, pieces):
    from rpfq_review_b200 import _lib, ops
    out_dtype = torch.float32 if epi in ("residual_f32", "f32") else torch.float16
    plan = ops.gemm_plan(m, n, k, out_dtype=out_dtype, residual=epi == "residual_f32", device=cuda)
    assert plan["cta_pair"] == 2 and plan["pieces"] == pieces and plan["stream_k_tiles"] == 0, plan
    assert 0 < plan["tail_tiles"] * pieces <= plan["units"]
    whole = ops.gemm_plan(m, n, k, out_dtype=out_dtype, residual=epi == "residual_f32", cta_pair=2, device=cuda)
    assert whole["pieces"] == 0
    x, w, b, r = _inputs(m, n, k, epi, cuda)
    act = "gelu" if epi == "gelu" else "none"

    def run(cta_pair):
        out = r.clone() if r is not None else None
        return ops.gemm(x, w, b, residual=out, out=out, out_dtype=out_dtype, activation=act, cta_pair=cta_pair)

    y = run(0)
    y_whole = run(2)
    torch.cuda.synchronize(cuda)
    lin = x.double() @ w.double().T + b.double()
    ref = torch.nn.functional.gelu(lin) if epi == "gelu" else lin
    if r is not None:
        ref = ref + r.double()
    assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) < TOL
    assert torch.equal(y, y_whole), "narrow tail and whole tiles differ"
    assert _lib.device_error() == 0


@pytest.mark.parametrize("m,n,k", [(401408, 384, 96), (401408, 288, 96), (100352, 576, 192)])
def test_partial_width_keeps_block_n_picker(cuda, m, n, k):
    """Swin-T stage-1/2 layers (n not a multiple of 256) whose pair tiles would
    leave a short last wave keep the tile width of the wave model: 256-wide
    tiles over 288 or 384 columns waste a quarter or more of every tile."""
    from rpfq_review_b200 import ops
    plan = ops.gemm_plan(m, n, k, device=cuda)
    assert plan["pieces"] == 0 and plan["stream_k_tiles"] == 0, plan
