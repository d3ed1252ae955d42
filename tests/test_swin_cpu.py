"""CPU tests of the Swin harness's index bookkeeping (window partition,
cyclic-shift mask, relative position index) and of the model's flop count;
the CPU reference forward runs on the seeded weights."""

import pytest
import torch

from rpfq_review_b200.swin import (SWIN_T, relative_position_index, shift_mask, window_partition,
                                   window_reverse)


def test_window_partition_round_trip_and_order():
    x = torch.arange(2 * 14 * 14 * 3, dtype=torch.float32).view(2, 14, 14, 3)
    w = window_partition(x, 7)
    assert w.shape == (2 * 4, 49, 3)
    # window 1 of image 0 is rows 0..6, columns 7..13; its first token is (0, 7)
    assert torch.equal(w[1, 0], x[0, 0, 7])
    assert torch.equal(w[1, 8], x[0, 1, 8])
    assert torch.equal(window_reverse(w, 7, 14), x)


def test_relative_position_index():
    idx = relative_position_index(7)
    assert idx.shape == (49, 49)
    assert int(idx.min()) == 0 and int(idx.max()) == 13 * 13 - 1
    # offset (0, 0) sits at the centre of the 13 x 13 table
    assert torch.all(idx.diagonal() == 6 * 13 + 6)
    # position 0 = (0, 0), position 48 = (6, 6): offset (-6, -6) -> 0; the reverse -> 168
    assert int(idx[0, 48]) == 0 and int(idx[48, 0]) == 168


def test_shift_mask_regions():
    m = shift_mask(56, 7, 3)
    assert m.shape == (64, 49, 49)
    # windows that do not touch the wrapped strips see no mask
    assert torch.count_nonzero(m[0]) == 0
    # the last window holds 4 regions: 16 + 12 + 12 + 9 positions
    last = m[-1]
    sizes = sorted(int((last[i] == 0).sum()) for i in range(49))
    assert set(sizes) == {16, 12, 9}
    assert set(torch.unique(m).tolist()) == {0.0, -100.0}


def test_swin_t_flops_per_image():
    # 4335.3 M multiply-adds of the linears (blocks, patch merging, head)
    assert SWIN_T.gemm_flops_per_image() == pytest.approx(8.6706e9, rel=1e-3)


def test_swin_reference_forward_runs_on_cpu():
    from oracle import swin_ref
    from rpfq_review_b200.swin import PackedSwin
    model = PackedSwin(SWIN_T, "cpu", seed=0, prepack=False)
    w = swin_ref.extract_weights(model)
    images = torch.randn(1, 3, 224, 224, generator=torch.Generator().manual_seed(0))
    logits = swin_ref.swin_forward(w, SWIN_T, images)
    assert logits.shape == (1, 1000) and torch.isfinite(logits).all()


def test_window_order_equals_roll_then_partition():
    from rpfq_review_b200.swin import window_order
    for r, ws, sh in ((56, 7, 3), (14, 7, 0), (28, 7, 3), (7, 7, 0)):
        x = torch.arange(r * r * 2, dtype=torch.float32).view(1, r, r, 2)
        rolled = torch.roll(x, shifts=(-sh, -sh), dims=(1, 2)) if sh else x
        want = window_partition(rolled, ws).reshape(-1, 2)
        perm = window_order(r, ws, sh)
        assert torch.equal(x.view(r * r, 2)[perm], want)
        # scattering back through the same permutation undoes partition and shift
        back = torch.zeros(r * r, 2).index_add_(0, perm, want)
        assert torch.equal(back, x.view(r * r, 2))


def test_inverse_gather_equals_scatter_add():
    """The norm2 pass adds the attention branch (window order) back through
    the inverse gather: x[n] + o[inverse[n]] equals the scatter
    x.index_add_(perm, o) it replaced, per image of a batch."""
    from rpfq_review_b200.swin import window_order
    B = 2
    for r, ws, sh in ((56, 7, 3), (28, 7, 0), (14, 7, 3), (7, 7, 0)):
        perm = window_order(r, ws, sh)
        base = torch.arange(B)[:, None] * (r * r)
        inverse = (base + torch.argsort(perm)[None]).reshape(-1)
        g = torch.Generator().manual_seed(r + sh)
        x = torch.randn(B, r * r, 5, generator=g)
        o = torch.randn(B * r * r, 5, generator=g)  # window order
        want = x.clone().index_add_(1, perm, o.view(B, r * r, 5))
        got = x.reshape(-1, 5) + o[inverse]
        assert torch.equal(got.view(B, r * r, 5), want)


def test_window_bias_layout():
    """window_bias_layout: key column j of query row i at [.., j // 4, i, j % 4],
    scaled by log2(e), -inf in the padding keys 49..63."""
    import math

    from rpfq_review_b200.ops import window_bias_layout
    g = torch.Generator().manual_seed(0)
    bias = torch.randn(3, 2, 49, 49, generator=g)
    t = window_bias_layout(bias)
    assert t.shape == (3, 2, 16, 49, 4) and t.dtype == torch.float32
    full = t.permute(0, 1, 3, 2, 4).reshape(3, 2, 49, 64)
    assert torch.allclose(full[..., :49], bias * math.log2(math.e))
    assert torch.isneginf(full[..., 49:]).all()
    assert float(t[1, 1, 12 // 4, 5, 12 % 4]) == float(bias[1, 1, 5, 12] * math.log2(math.e))
