"""CPU tests of PackedViT's host-side token bookkeeping: the int32 tables with
which the first LayerNorm pass assembles the residual stream
[class (+ distillation) tokens, patch embeddings] + position embedding, the
class-token rows the final norm gathers, and the constant fp32 buffers kept
across calls (class-token rows of the source buffer, position table)."""

import types

import torch

from rpfq_review_b200.vit import DEIT_S16, VIT_B16, PackedViT


def _fake(cfg, seed=0):
    g = torch.Generator().manual_seed(seed)
    ntok = 2 if cfg.distilled else 1
    return types.SimpleNamespace(cfg=cfg, cls_tokens=torch.randn(1, ntok, cfg.dim, generator=g).half(),
                                 pos_embed=torch.randn(1, cfg.tokens, cfg.dim, generator=g).half())


def _tables(cfg, B):
    return PackedViT._token_index(_fake(cfg), B, torch.device("cpu"))


def test_token_tables_vit_b():
    rows, tok, cls_rows, src, pos = _tables(VIT_B16, 3)
    L, n_p = VIT_B16.tokens, 196
    assert rows.dtype == torch.int32 and tok.dtype == torch.int32 and rows.shape == (3 * L,)
    for b in range(3):
        assert int(rows[b * L]) == 0 and int(tok[b * L]) == 0  # every image reads the one class-token row
        for t in (1, 2, 195, 196):
            assert int(rows[b * L + t]) == 1 + b * n_p + t - 1
            assert int(tok[b * L + t]) == t
    assert cls_rows.tolist() == [0, L, 2 * L] and cls_rows.dtype == torch.int32
    assert src.shape == (1 + 3 * n_p, VIT_B16.dim) and src.dtype == torch.float32
    assert pos.shape == (L, VIT_B16.dim) and pos.dtype == torch.float32


def test_token_tables_deit_distilled_and_cache():
    cfg = DEIT_S16
    fake = _fake(cfg, 1)
    rows, tok, cls_rows, src, pos = PackedViT._token_index(fake, 2, torch.device("cpu"))
    L = cfg.tokens
    assert L == 198
    assert rows[:2].tolist() == [0, 1] and rows[L:L + 2].tolist() == [0, 1]
    assert int(rows[L + 2]) == 2 + 196  # image 1's first patch sits after image 0's 196
    assert int(rows.max()) == 2 + 2 * 196 - 1  # the source buffer holds 2 + B * 196 rows
    assert cls_rows.tolist() == [0, 1, L, L + 1]
    assert torch.equal(src[:2], fake.cls_tokens[0].float())  # filled once, at creation
    assert torch.equal(pos, fake.pos_embed[0].float())
    again = PackedViT._token_index(fake, 2, torch.device("cpu"))
    assert again[0] is rows and again[3] is src  # kept per batch size
    other = PackedViT._token_index(fake, 5, torch.device("cpu"))
    assert other[0].shape == (5 * L,)
    # every batch size keeps its entry (a graph captured at one size still uses it)
    assert PackedViT._token_index(fake, 2, torch.device("cpu"))[3] is src and len(fake._token_index_cache) == 2
    fake.cls_tokens.add_(1.0)  # a changed class token rebuilds the buffers, the stale entries go
    fresh = PackedViT._token_index(fake, 5, torch.device("cpu"))
    assert fresh[3] is not other[3] and torch.equal(fresh[3][:2], fake.cls_tokens[0].float())
    assert len(fake._token_index_cache) == 1
