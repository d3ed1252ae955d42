"""GPU tests of the Swin window-attention kernel (``rpfq_window_attention_sm100``)
against float64 softmax(q k^T / sqrt(32) + bias + mask) v on the same fp16 qkv.

Bar: max|out - ref| / max|ref| <= 3e-3 (P is rounded to fp16 for the second
tensor-core product, the output to fp16), for the Swin-T head counts (3, 6,
12, 24: odd counts leave the second head slot of the last pair empty), odd
window counts (the last pair has one window), unshifted (bias only) and
shifted (bias + per-window mask) blocks."""

import math

import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


def _bias_mask(bias: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
    """[nh, 49, 49] bias (+ [nW, 49, 49] mask) -> the kernel's operand."""
    from rpfq_review_b200 import ops
    m = bias[None] if mask is None else bias[None] + mask[:, None]
    return ops.window_bias_layout(m)


def _ref(qkv: torch.Tensor, heads: int, bias: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
    W = qkv.shape[0] // 49
    x = qkv.double().view(W, 49, 3, heads, 32).permute(2, 0, 3, 1, 4)
    q, k, v = x[0], x[1], x[2]
    att = q @ k.transpose(-2, -1) / math.sqrt(32) + bias.double()[None]
    if mask is not None:
        nw = mask.shape[0]
        att = att + mask.double()[torch.arange(W) % nw][:, None]
    return (torch.softmax(att, dim=-1) @ v).transpose(1, 2).reshape(W * 49, heads * 32)


@pytest.mark.parametrize("windows,heads,shifted", [(128, 3, False), (64, 3, True), (33, 6, True), (16, 12, False),
                                                   (5, 24, True), (1, 24, False), (2, 3, False), (7, 1, True)])
def test_window_attention_matches_fp64(cuda, windows, heads, shifted):
    from rpfq_review_b200 import ops
    from rpfq_review_b200.swin import shift_mask
    g = torch.Generator().manual_seed(windows * 100 + heads)
    qkv = (torch.randn(windows * 49, 3 * 32 * heads, generator=g) * 1.5).half()
    bias = torch.randn(heads, 49, 49, generator=g) * 0.5
    mask = None
    if shifted:
        full = shift_mask(14, 7, 3)  # 4 windows per image, the shifted regions
        mask = full
    out = ops.window_attention(qkv.to(cuda), heads, _bias_mask(bias, mask).to(cuda))
    ref = _ref(qkv, heads, bias, mask)
    assert rel_err(out.cpu().numpy(), ref.numpy()) <= 3e-3
    from rpfq_review_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_window_attention_strided_output_and_errors(cuda):
    from rpfq_review_b200 import ops
    heads, windows = 6, 9
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(windows * 49, 3 * 32 * heads, generator=g).half().to(cuda)
    bias = torch.randn(heads, 49, 49, generator=g)
    buf = torch.zeros(windows * 49, 32 * heads + 64, dtype=torch.float16, device=cuda)
    out = buf[:, 32:32 + 32 * heads]
    ops.window_attention(qkv, heads, _bias_mask(bias, None).to(cuda), out=out)
    assert rel_err(out.cpu().numpy(), _ref(qkv.cpu(), heads, bias, None).numpy()) <= 3e-3
    assert torch.count_nonzero(buf[:, :32]) == 0 and torch.count_nonzero(buf[:, 32 + 32 * heads:]) == 0
    with pytest.raises(ValueError, match="windows"):
        ops.window_attention(qkv[:50], heads, _bias_mask(bias, None).to(cuda))
    with pytest.raises(ValueError, match="bias_mask"):
        ops.window_attention(qkv, heads, torch.zeros(1, heads, 49, 64, device=cuda))
