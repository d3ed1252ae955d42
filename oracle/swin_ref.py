"""CPU reference forward of Swin-T (TEST INFRASTRUCTURE ONLY).

The reference runs timm's SwinTransformer with every linear swapped for the
complex-phase layer (RPFQ-ViT-main/quant_models/quant_rpfq_swin.py:64-91);
timm is not available here, so the forward is restated from the
architecture's definition, in float32 with explicit attention: 4x4 patch
embedding + LayerNorm; per block LN -> window partition (cyclic shift on odd
blocks) -> qkv -> softmax(q k^T / sqrt(d_h) + relative position bias + shift
mask) v -> proj -> reverse shift -> residual; LN -> fc1 -> exact GELU -> fc2
-> residual; patch merging (2x2 concat, LN, reduction); final LN, token mean,
head. Every quantized linear uses the dense weight reconstructed from its
packed planes (``oracle.packed_ref.dense_weight_from_packed``). The window /
mask helpers are the product's (pure index bookkeeping, checked separately
by their own unit test); the arithmetic here is independent.

``fp16`` / ``fp16_act`` as in ``oracle.vit_ref``: the coefficients rounded
through fp16 (the runtime's fp16 coefficient cache) and the activations the
benchmarked configuration keeps in fp16 (LayerNorm outputs, qkv, softmax
probabilities, attention output, GELU output, the pooled features) rounded,
with a float32 residual stream and float32 accumulation.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import packed_ref as pr
from .vit_ref import packed_to_numpy


def extract_weights(model, dtype=torch.float32, linears: bool = True, fp16: bool = False) -> dict:
    """Dense reference weights of a ``rpfq_review_b200.swin.PackedSwin``
    (``linears=False``: everything but the packed linears; ``fp16``: the
    coefficients rounded through fp16)."""
    w = {"patch_w": model.patch_w.to(dtype).cpu(), "patch_b": model.patch_b.to(dtype).cpu(),
         "patch_norm_w": model.patch_norm_w.to(dtype).cpu(), "patch_norm_b": model.patch_norm_b.to(dtype).cpu(),
         "norm_w": model.norm_w.to(dtype).cpu(), "norm_b": model.norm_b.to(dtype).cpu()}
    for name, mod in (model.quantized_linears() if linears else ()):
        np_layer = packed_to_numpy(mod.packed())
        dense = pr.dense_weight_from_packed(np_layer, mod.n_c, mod.k_c)
        if fp16:
            dense = dense.astype(np.float16).astype(np.float32)
        w[name] = (torch.from_numpy(dense).to(dtype), torch.from_numpy(np_layer["bias"].astype(np.float32)).to(dtype))
    for s, stage in enumerate(model.stages):
        w[f"layers.{s}.rel_index"] = stage.rel_index.cpu()
        for i, blk in enumerate(stage.blocks):
            for n in ("norm1_w", "norm1_b", "norm2_w", "norm2_b", "rel_table"):
                w[f"layers.{s}.blocks.{i}.{n}"] = getattr(blk, n).detach().to(dtype).cpu()
        if hasattr(stage, "reduction"):
            w[f"layers.{s}.merge_norm_w"] = stage.merge_norm_w.to(dtype).cpu()
            w[f"layers.{s}.merge_norm_b"] = stage.merge_norm_b.to(dtype).cpu()
    return w


def swin_forward(w: dict, cfg, images: torch.Tensor, lin=None, fp16_act: bool = False) -> torch.Tensor:
    """Logits ``[B, classes]``; ``lin(name, t)`` overrides the packed linears
    (default: F.linear with the dense weights in ``w``)."""
    from rpfq_review_b200.swin import shift_mask, window_partition, window_reverse

    def r16(t):
        return t.half().float() if fp16_act else t

    x = images.float()
    b = x.shape[0]
    p = cfg.patch
    patches = x.reshape(b, 3, cfg.img // p, p, cfg.img // p, p).permute(0, 2, 4, 1, 3, 5).reshape(b, -1, 3 * p * p)
    dims, res = cfg.dims(), cfg.resolutions()
    x = F.linear(patches, w["patch_w"], w["patch_b"])
    x = F.layer_norm(x, (dims[0],), w["patch_norm_w"], w["patch_norm_b"], cfg.eps)

    if lin is None:
        def lin(name, t):
            W, bias = w[name]
            return F.linear(t, W, bias)

    for s, depth in enumerate(cfg.depths):
        c, nh, r = dims[s], cfg.heads[s], res[s]
        hd = c // nh
        ws, shift = cfg.stage_window(s)
        L = ws * ws
        idx = w[f"layers.{s}.rel_index"].reshape(-1)
        for i in range(depth):
            pre = f"layers.{s}.blocks.{i}"
            sh = shift if i % 2 == 1 else 0
            h = r16(F.layer_norm(x, (c,), w[f"{pre}.norm1_w"], w[f"{pre}.norm1_b"], cfg.eps)).view(b, r, r, c)
            if sh:
                h = torch.roll(h, shifts=(-sh, -sh), dims=(1, 2))
            win = window_partition(h, ws)
            qkv = r16(lin(f"{pre}.qkv", win)).view(win.shape[0], L, 3, nh, hd).permute(2, 0, 3, 1, 4)
            q, k, v = qkv[0], qkv[1], qkv[2]
            att = torch.matmul(q, k.transpose(-2, -1)) * (hd ** -0.5)
            bias = w[f"{pre}.rel_table"][idx].reshape(L, L, nh).permute(2, 0, 1)
            att = att + bias[None]
            if sh:
                nw = (r // ws) ** 2
                m = shift_mask(r, ws, sh)
                att = (att.view(b, nw, nh, L, L) + m[None, :, None]).view(-1, nh, L, L)
            a = r16(torch.matmul(r16(torch.softmax(att, dim=-1)), v).transpose(1, 2).reshape(win.shape[0], L, c))
            o = window_reverse(lin(f"{pre}.proj", a), ws, r)
            if sh:
                o = torch.roll(o, shifts=(sh, sh), dims=(1, 2))
            x = x + o.reshape(b, r * r, c)
            h = r16(F.layer_norm(x, (c,), w[f"{pre}.norm2_w"], w[f"{pre}.norm2_b"], cfg.eps))
            x = x + lin(f"{pre}.fc2", r16(F.gelu(lin(f"{pre}.fc1", h), approximate="none")))
        if s + 1 < len(cfg.depths):
            xs = x.view(b, r, r, c)
            cat = torch.cat([xs[:, 0::2, 0::2], xs[:, 1::2, 0::2], xs[:, 0::2, 1::2], xs[:, 1::2, 1::2]], dim=-1)
            h = r16(F.layer_norm(cat.reshape(b, -1, 4 * c), (4 * c,), w[f"layers.{s}.merge_norm_w"],
                                 w[f"layers.{s}.merge_norm_b"], cfg.eps))
            x = lin(f"layers.{s + 1}.downsample.reduction", h)
    h = r16(F.layer_norm(x, (dims[-1],), w["norm_w"], w["norm_b"], cfg.eps))
    return lin("head", r16(h.mean(dim=1)))
