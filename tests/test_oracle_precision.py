"""The precision floor of the parity bars (CPU only).

configs[1] runs the layers with fp16 activations and the reference runtime
keeps an fp16 coefficient cache. Rounding the all-float32 reference forward's
own coefficients and activations to fp16 (``oracle.vit_ref`` with
``fp16=True`` / ``fp16_act=True``) moves its ViT-B/16 logits by this much,
before any GPU arithmetic: the distance of every fp16-activation
implementation from the float32 reference starts here, which is why the GPU
model tests hold the fp16-precision reference to 1e-3 and the float32 one
to 1.5e-3.
"""

import torch

from oracle import vit_ref
from tests.helpers import rel_err


def test_fp16_rounding_floor_of_the_float32_reference():
    from rpfq_review_b200.vit import VIT_B16, PackedViT
    model = PackedViT(VIT_B16, "cpu", seed=0, prepack=False)  # packed on the host (exporter algorithm)
    w32 = vit_ref.extract_weights(model, torch.float32)
    w16 = vit_ref.extract_weights(model, torch.float32, fp16=True)
    images = torch.randn(3, 3, 224, 224, generator=torch.Generator().manual_seed(7)).half()
    ref32 = vit_ref.vit_forward(w32, VIT_B16, images.float())
    coeff = rel_err(vit_ref.vit_forward(w16, VIT_B16, images.float()).numpy(), ref32.numpy())
    act = rel_err(vit_ref.vit_forward(w32, VIT_B16, images.float(), fp16_act=True).numpy(), ref32.numpy())
    both = rel_err(vit_ref.vit_forward(w16, VIT_B16, images.float(), fp16_act=True).numpy(), ref32.numpy())
    print(f"fp16 coefficients {coeff:.3e}, fp16 activations {act:.3e}, both {both:.3e}")
    # measured: 6.3e-4, 6.9e-4, 8.5e-4 (seed 7)
    assert 4e-4 < coeff < 1e-3 and 4e-4 < act < 1e-3 and 6e-4 < both < 1.2e-3
