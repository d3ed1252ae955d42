"""CPU reference forward of the ViT / DeiT models (TEST INFRASTRUCTURE ONLY).

Restates the reference's pure-torch runtime forward with export-reconstructed
weights, ``forward_runtime_path`` and ``capture_runtime_block_trace``
(RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:589-688): patch embed,
cls token (+ dist token for DeiT, quant_rpfq_deit.py:26), position embedding,
per block LN -> qkv -> softmax(q k^T / sqrt(d_h)) v -> proj + residual ->
LN -> fc1 -> exact GELU (audit…py:624) -> fc2 + residual, final LN, head on
the class token (DeiT: mean of the two heads at eval). Every quantized
linear uses the dense weight reconstructed from its packed planes by
``oracle.packed_ref.dense_weight_from_packed`` (the exporter's
``quantized_forward_weight``), i.e. the deployment path in float32/float64.

``fp16=True`` (``extract_weights``) rounds the dense coefficients through
fp16, i.e. the reference runtime's fused fp16 coefficient cache
(RPFQ-ViTAndroid/app/src/main/cpp/kernels/phase_linear_cache.cpp:84-133,
round-to-nearest-even here); ``fp16_act=True`` (``vit_forward``) rounds the
activations that configs[1] keeps in fp16 — every LayerNorm output (GEMM
input), the qkv output, the softmax probabilities, the attention output and
the GELU output — while the residual stream and every accumulation stay
float32. Together they give the reference forward at the precision the
benchmarked configuration specifies ("fp16 activations").
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import packed_ref as pr


def packed_to_numpy(layer) -> dict:
    out = {}
    for name, (c, gr, gi) in layer.planes.items():
        out[f"{name}.codes"] = c.cpu().numpy()
        out[f"{name}.gamma_real"] = gr.cpu().numpy()
        out[f"{name}.gamma_imag"] = gi.cpu().numpy()
    out["bias"] = layer.bias.cpu().numpy()
    return out


def extract_weights(model, dtype=torch.float32, fp16: bool = False) -> dict:
    """Dense reference weights of a ``rpfq_review_b200.vit.PackedViT``
    (``fp16``: the coefficients rounded through fp16)."""
    w = {"patch_w": model.patch_w.to(dtype).cpu(), "patch_b": model.patch_b.to(dtype).cpu(),
         "cls_tokens": model.cls_tokens.to(dtype).cpu(), "pos_embed": model.pos_embed.to(dtype).cpu(),
         "norm_w": model.norm_w.to(dtype).cpu(), "norm_b": model.norm_b.to(dtype).cpu()}
    for name, mod in model.quantized_linears():
        np_layer = packed_to_numpy(mod.packed())
        dense = pr.dense_weight_from_packed(np_layer, mod.n_c, mod.k_c)
        if fp16:
            dense = dense.astype(np.float16).astype(np.float32)
        w[name] = (torch.from_numpy(dense).to(dtype), torch.from_numpy(np_layer["bias"].astype(np.float32)).to(dtype))
    for i, blk in enumerate(model.blocks):
        for n in ("norm1_w", "norm1_b", "norm2_w", "norm2_b"):
            w[f"blocks.{i}.{n}"] = getattr(blk, n).detach().to(dtype).cpu()
    return w


def vit_forward(w: dict, cfg, images: torch.Tensor, act_bits: int = 0, fp16_act: bool = False) -> torch.Tensor:
    """Logits ``[B, classes]`` of the reference forward on CPU (``fp16_act``:
    the fp16 activations of configs[1], see the module docstring)."""
    dtype = w["patch_w"].dtype

    def r16(t):
        return t.half().to(t.dtype) if fp16_act else t

    x = images.to(dtype)
    B = x.shape[0]
    p = cfg.patch
    patches = x.reshape(B, 3, cfg.img // p, p, cfg.img // p, p).permute(0, 2, 4, 1, 3, 5)
    patches = patches.reshape(B, -1, 3 * p * p)
    x = F.linear(patches, w["patch_w"], w["patch_b"])
    x = torch.cat((w["cls_tokens"].expand(B, -1, -1), x), dim=1) + w["pos_embed"]
    d, H = cfg.dim, cfg.heads
    hd = d // H

    def lin(name, t):
        W, b = w[name]
        if act_bits:
            t = torch.from_numpy(pr.act_quant(t.float().numpy(), act_bits)).to(dtype)
        return F.linear(t, W, b)

    L = x.shape[1]
    for i in range(cfg.depth):
        h = r16(F.layer_norm(x, (d,), w[f"blocks.{i}.norm1_w"], w[f"blocks.{i}.norm1_b"], cfg.eps))
        qkv = r16(lin(f"blocks.{i}.qkv", h))
        q, k, v = qkv.chunk(3, dim=-1)
        q = q.reshape(B, L, H, hd).transpose(1, 2)
        k = k.reshape(B, L, H, hd).transpose(1, 2)
        v = v.reshape(B, L, H, hd).transpose(1, 2)
        att = r16(torch.softmax(torch.matmul(q, k.transpose(-2, -1)) * (hd ** -0.5), dim=-1))
        a = r16(torch.matmul(att, v).transpose(1, 2).reshape(B, L, d))
        x = x + lin(f"blocks.{i}.proj", a)
        h = r16(F.layer_norm(x, (d,), w[f"blocks.{i}.norm2_w"], w[f"blocks.{i}.norm2_b"], cfg.eps))
        x = x + lin(f"blocks.{i}.fc2", r16(F.gelu(lin(f"blocks.{i}.fc1", h), approximate="none")))
    ntok = 2 if cfg.distilled else 1
    cls = r16(F.layer_norm(x[:, :ntok], (d,), w["norm_w"], w["norm_b"], cfg.eps))
    logits = lin("head", cls[:, 0])
    if cfg.distilled:
        logits = (logits + lin("head_dist", cls[:, 1])) / 2
    return logits
