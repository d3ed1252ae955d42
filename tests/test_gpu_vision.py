"""GPU parity tests of the vision-aware activation quantizer
(``rpfq_vision_act_quant_sm100``; VisionAwareActivationQuantizer,
quant_rpfq_vit_vision.py:26-171).

Bar: the saliency mask equal to the reference's and the quantized fp16
values bit-identical to fp16(reference output), on the golden fixtures made
by the reference class itself (golden_vision.npz) and on larger seeded
batches against the oracle restatement. The drop-in layer is held to the
layer bar (1e-3 of max|y|) against F.linear on the oracle's quantized input.
"""

import os

import numpy as np
import pytest
import torch

from oracle import packed_ref as pr
from oracle import vision_ref as vr
from tests.helpers import rel_err

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["vitb", "nocls", "all_salient", "no_salient", "grid4", "zero_token", "fallback_tokens", "fallback_2d"]


def _run(x, params, cuda, **kw):
    from rpfq_review_b200 import ops
    ratio, clip, wgt, cls = params
    return ops.vision_act_quant(x.to(cuda), ratio, clip, wgt, bool(cls), return_mask=True, **kw)


@pytest.mark.parametrize("name", CASES)
def test_vision_quant_matches_reference_golden(cuda, name):
    g = np.load(os.path.join(GOLD, "golden_vision.npz"))
    params = tuple(float(v) for v in g[f"{name}.params"])
    xr, xi = g[f"{name}.x_real"], g[f"{name}.x_imag"]
    x = torch.from_numpy(np.concatenate([xr, xi], axis=-1))  # fp16 [.., 2 k_c]
    y, mask = _run(x, params, cuda)
    assert np.array_equal(mask.cpu().numpy().astype(np.uint8), g[f"{name}.mask"])
    want = np.concatenate([g[f"{name}.q_real"], g[f"{name}.q_imag"]], axis=-1).astype(np.float16)
    assert np.array_equal(y.cpu().numpy().view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("b,t,k_c,ratio", [(4, 197, 384, 0.25), (2, 577, 64, 0.4), (1, 2, 8, 0.5),
                                          (2, 1 + 64 * 64, 8, 0.25), (3, 50, 1536, 0.1)])
def test_vision_quant_matches_oracle(cuda, b, t, k_c, ratio):
    gen = torch.Generator().manual_seed(t + k_c)
    mag = torch.exp(torch.randn(b, t, 1, generator=gen) * 0.7)
    x = (torch.randn(b, t, 2 * k_c, generator=gen) * mag).half()
    params = (ratio, 0.75, 0.5, 1.0)
    y, mask = _run(x, params, cuda)
    xf = x.float().numpy()
    qr, qi, m = vr.vision_act_quant(xf[..., :k_c], xf[..., k_c:], ratio, 0.75, 0.5, True)
    assert np.array_equal(mask.cpu().numpy(), m)
    want = np.concatenate([qr, qi], axis=-1).astype(np.float16)
    assert np.array_equal(y.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_vision_quant_in_place_and_errors(cuda):
    from rpfq_review_b200 import ops
    x = (torch.randn(2, 197, 96, generator=torch.Generator().manual_seed(3))).half().to(cuda)
    want = ops.vision_act_quant(x)
    ops.vision_act_quant(x, out=x)
    assert torch.equal(x, want)
    with pytest.raises(ValueError, match=r"salient_token_ratio must be in \[0, 1\]"):
        ops.vision_act_quant(x, salient_token_ratio=1.5)
    with pytest.raises(ValueError, match="background_clip_ratio must be > 0"):
        ops.vision_act_quant(x, background_clip_ratio=0.0)


def test_vision_aware_drop_in_layer(cuda):
    """VisionAwareQATLinearComplexPhase on [B, T, K] against F.linear of the
    oracle-quantized input with the exporter-packed dense weight."""
    from rpfq_review_b200 import VisionAwareQATLinearComplexPhase
    gen = torch.Generator().manual_seed(11)
    n_c, k_c = 96, 64
    layer = VisionAwareQATLinearComplexPhase("complex_phase_v2", "complex_phase_v2", True, 4, False, 32,
                                             in_features=2 * k_c, out_features=2 * n_c, bias=True)
    with torch.no_grad():
        layer.weight.copy_(torch.randn(2 * n_c, 2 * k_c, generator=gen) * 0.05)
        layer.bias.copy_(torch.randn(2 * n_c, generator=gen) * 0.01)
    layer = layer.to(cuda)
    x = (torch.randn(2, 197, 2 * k_c, generator=gen) * torch.exp(torch.randn(2, 197, 1, generator=gen))).half()
    y = layer(x.to(cuda)).float().cpu().numpy()
    xf = x.float().numpy()
    qr, qi, _ = vr.vision_act_quant(xf[..., :k_c], xf[..., k_c:])
    packed = pr.pack_linear(layer.weight.detach().cpu().numpy(), layer.bias.detach().cpu().numpy(), 2)
    dense = pr.dense_weight_from_packed(packed, n_c, k_c)
    ref = pr.wide_linear(np.concatenate([qr, qi], -1).reshape(-1, 2 * k_c), dense,
                         packed["bias"].astype(np.float32)).reshape(2, 197, 2 * n_c)
    assert rel_err(y, ref) < 1e-3
    with pytest.raises(ValueError, match="energy_score_weight"):
        VisionAwareQATLinearComplexPhase(energy_score_weight=2.0, in_features=8, out_features=8)
