"""GPU tests of the short-sequence attention kernel (``rpfq_attention_sm100``)
against float64 softmax(q k^T / sqrt(64)) v on the same fp16 qkv.

Bar: max|out - ref| / max|ref| <= 3e-3 (P is rounded to fp16 for the second
tensor-core product, the output to fp16), for the ViT / DeiT token counts and
the tile edges (1, 17, 64, 128, 129, 208, 209, 224, 256 tokens; up to 208
keys the second half of each row keeps its P after S in TMEM, above that it
waits for the first half)."""

import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


def _ref(qkv: torch.Tensor, heads: int) -> torch.Tensor:
    B, L, three_d = qkv.shape
    d = three_d // 3
    x = qkv.double().view(B, L, 3, heads, 64).permute(2, 0, 3, 1, 4)
    q, k, v = x[0], x[1], x[2]
    att = torch.softmax(q @ k.transpose(-2, -1) / 8.0, dim=-1)
    return (att @ v).transpose(1, 2).reshape(B, L, d)


@pytest.mark.parametrize("B,L,H", [(3, 197, 12), (2, 198, 6), (2, 1, 2), (2, 64, 4), (2, 128, 3), (1, 129, 1),
                                   (2, 256, 2), (4, 197, 16), (2, 208, 3), (2, 209, 2), (3, 224, 2), (2, 17, 5)])
def test_attention_matches_fp64(cuda, B, L, H):
    from rpfq_review_b200 import ops
    g = torch.Generator().manual_seed(B * 1000 + L * 10 + H)
    qkv = (torch.randn(B, L, 3 * 64 * H, generator=g) * 1.5).half()
    out = ops.attention(qkv.to(cuda), H)
    ref = _ref(qkv, H)
    assert rel_err(out.cpu().numpy(), ref.numpy()) <= 3e-3


def test_attention_strided_output_and_errors(cuda):
    from rpfq_review_b200 import ops
    H, L = 4, 197
    qkv = torch.randn(2, L, 3 * 64 * H, generator=torch.Generator().manual_seed(1)).half().to(cuda)
    buf = torch.zeros(2, L, 64 * H + 32, dtype=torch.float16, device=cuda)
    out = buf[..., 16:16 + 64 * H]
    ops.attention(qkv, H, out=out)
    assert rel_err(out.cpu().numpy(), _ref(qkv.cpu(), H).numpy()) <= 3e-3
    assert torch.count_nonzero(buf[..., :16]) == 0 and torch.count_nonzero(buf[..., 16 + 64 * H:]) == 0
    with pytest.raises(NotImplementedError, match="tokens"):
        ops.attention(torch.zeros(1, 257, 3 * 64, dtype=torch.float16, device=cuda), 1)
    from rpfq_review_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("L,H,plants", [(197, 2, ((150, 8.0),)), (197, 3, ((40, 4.0), (170, 8.0))),
                                        (256, 1, ((100, 1.1), (230, 1.25))), (129, 2, ((128, 6.0),))])
def test_attention_raised_reference(cuda, L, H, plants):
    """Keys after the first chunk of 32 whose logits exceed that chunk's by far
    more than the one-pass softmax's 2^12 margin, for half of the query rows
    (q = +u + noise) and not for the other half (q = -u + noise): the rows that
    raise their reference rescale the weights already written, the others keep
    theirs, within one warp. plants: (key, a) sets k[key] = a u for every head."""
    from rpfq_review_b200 import ops
    g = torch.Generator().manual_seed(L * 7 + H)
    B, d = 2, 64 * H
    u = torch.where(torch.rand(64, generator=g) < 0.5, -1.0, 1.0)
    sign = torch.where(torch.arange(L) % 2 == 0, 1.0, -1.0)
    x = torch.randn(B, L, 3, H, 64, generator=g) * 0.7
    x[:, :, 0] += sign.view(1, L, 1, 1) * u
    for key, a in plants:
        x[:, key, 1] = a * u
    qkv = x.reshape(B, L, 3 * d).half()
    out = ops.attention(qkv.to(cuda), H)
    ref = _ref(qkv, H)
    assert rel_err(out.cpu().numpy(), ref.numpy()) <= 3e-3
    from rpfq_review_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
