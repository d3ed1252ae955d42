"""CPU tests of PackedViT's host-side token bookkeeping: the int32 tables with
which the first LayerNorm pass assembles the residual stream
[class (+ distillation) tokens, patch embeddings] + position embedding."""

import types

import torch

from rpfq_review_b200.vit import DEIT_S16, VIT_B16, PackedViT


def _tables(cfg, B):
    fake = types.SimpleNamespace(cfg=cfg)
    return PackedViT._token_index(fake, B, torch.device("cpu"))


def test_token_tables_vit_b():
    rows, tok = _tables(VIT_B16, 3)
    L, n_p = VIT_B16.tokens, 196
    assert rows.dtype == torch.int32 and tok.dtype == torch.int32 and rows.shape == (3 * L,)
    for b in range(3):
        assert int(rows[b * L]) == 0 and int(tok[b * L]) == 0  # every image reads the one class-token row
        for t in (1, 2, 195, 196):
            assert int(rows[b * L + t]) == 1 + b * n_p + t - 1
            assert int(tok[b * L + t]) == t


def test_token_tables_deit_distilled_and_cache():
    cfg = DEIT_S16
    fake = types.SimpleNamespace(cfg=cfg)
    rows, tok = PackedViT._token_index(fake, 2, torch.device("cpu"))
    L = cfg.tokens
    assert L == 198
    assert rows[:2].tolist() == [0, 1] and rows[L:L + 2].tolist() == [0, 1]
    assert int(rows[L + 2]) == 2 + 196  # image 1's first patch sits after image 0's 196
    assert int(rows.max()) == 2 + 2 * 196 - 1  # the source buffer holds 2 + B * 196 rows
    again = PackedViT._token_index(fake, 2, torch.device("cpu"))
    assert again[0] is rows  # kept per batch size
    other = PackedViT._token_index(fake, 5, torch.device("cpu"))
    assert other[0].shape == (5 * L,) and len(fake._token_index_cache) == 1
