"""CPU restatement (numpy) of the reference's vision-aware activation
quantizer — TEST INFRASTRUCTURE ONLY: imported by tests/, never by the
product package.

Follows ``VisionAwareActivationQuantizer`` in
RPFQ-ViT-main/quant_models/quant_rpfq_vit_vision.py (cited as VQ:line):

* token energy = mean over channels of sqrt(re^2 + im^2 + EPS)        VQ:80
* contrast = mean |energy difference| to the 4-neighbours on the patch
  grid (up, down, left, right, in that summation order)             VQ:83-98
* score = w * energy / mean(energy) + (1 - w) * contrast / mean(contrast),
  means clamped at EPS                                               VQ:99-106
* the ceil(P * ratio) (at least 1 when ratio > 0) highest-scoring patches
  are salient; the CLS token is salient iff protect_cls_token      VQ:108-143
* salient tokens: per-token int8 scale 127 / max(amax, EPS); the others
  share one per-image scale 127 / max(background amax * clip, EPS), the
  background amax taken over tokens and channels                   VQ:63-64,145-167;
  ``127.0 / t`` evaluates as ``t.reciprocal() * 127`` (torch Tensor.__rdiv__)
* q = round_half_even(x * scale).clamp(-128, 127) / scale, returned in the
  straight-through form x + (q - x)                                  VQ:57-60
* inputs that are not [B, 1 + g*g, C] use the per-token scale for every
  token                                                             VQ:112-118,151-154

Every step is float32 as in the reference except the energy / contrast
means, which are accumulated in float64: they only order the patches, and a
different rounding moves a score by far less than the gap between
neighbouring scores of any fixture.
"""

from __future__ import annotations

import math

import numpy as np

EPS = np.float32(1e-6)


def _grid(tokens: int) -> int:
    p = tokens - 1
    if p <= 0:
        return 0
    g = math.isqrt(p)
    return g if g * g == p else 0


def saliency_scores(x_re: np.ndarray, x_im: np.ndarray, g: int, energy_weight: float) -> np.ndarray:
    """[B, P] scores of the patch tokens (x without the CLS token)."""
    xr = x_re.astype(np.float32)
    xi = x_im.astype(np.float32)
    e = np.sqrt(xr * xr + xi * xi + EPS).astype(np.float64).mean(axis=-1)  # [B, P]
    b = e.shape[0]
    grid = e.reshape(b, g, g)
    contrast = np.zeros_like(grid)
    count = np.zeros_like(grid)
    vd = np.abs(grid[:, 1:, :] - grid[:, :-1, :])
    contrast[:, 1:, :] += vd
    contrast[:, :-1, :] += vd
    count[:, 1:, :] += 1
    count[:, :-1, :] += 1
    hd = np.abs(grid[:, :, 1:] - grid[:, :, :-1])
    contrast[:, :, 1:] += hd
    contrast[:, :, :-1] += hd
    count[:, :, 1:] += 1
    count[:, :, :-1] += 1
    contrast = contrast / np.maximum(count, 1.0)
    en = grid / np.maximum(grid.mean(axis=(1, 2), keepdims=True), float(EPS))
    cn = contrast / np.maximum(contrast.mean(axis=(1, 2), keepdims=True), float(EPS))
    return (energy_weight * en + (1.0 - energy_weight) * cn).reshape(b, -1)


def saliency_mask(x_re: np.ndarray, x_im: np.ndarray, ratio: float, energy_weight: float,
                  protect_cls: bool) -> np.ndarray:
    """[B, T] bool; all True for inputs without a square patch grid."""
    if x_re.ndim != 3:
        return np.ones(x_re.shape[:-1], bool)
    b, t, _ = x_re.shape
    g = _grid(t)
    if g == 0:
        return np.ones((b, t), bool)
    scores = saliency_scores(x_re[:, 1:], x_im[:, 1:], g, energy_weight)
    p = scores.shape[1]
    k = 0 if ratio <= 0.0 else min(p, max(1, math.ceil(p * ratio)))
    mask = np.zeros((b, t), bool)
    mask[:, 0] = protect_cls
    for i in range(b):
        order = np.lexsort((np.arange(p), -scores[i]))  # score descending, then index
        mask[i, 1 + order[:k]] = True
    return mask


def _scale(amax: np.ndarray) -> np.ndarray:
    """``127.0 / t`` in torch is ``t.reciprocal() * 127`` (Tensor.__rdiv__):
    two float32 roundings."""
    r = (np.float32(1.0) / np.maximum(amax, EPS)).astype(np.float32)
    return (r * np.float32(127.0)).astype(np.float32)


def _quantize(x: np.ndarray, scale: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    q = np.clip(np.rint(x * scale), -128, 127).astype(np.float32) / scale
    return (x + (q - x)).astype(np.float32)


def vision_act_quant(x_re: np.ndarray, x_im: np.ndarray, ratio: float = 0.25, clip: float = 0.75,
                     energy_weight: float = 0.5, protect_cls: bool = True):
    """Returns (q_re, q_im, mask) as the reference's forward (float32)."""
    mask = saliency_mask(x_re, x_im, ratio, energy_weight, protect_cls)
    outs = []
    for x in (x_re.astype(np.float32), x_im.astype(np.float32)):
        amax = np.abs(x).max(axis=-1)
        tok_scale = _scale(amax)
        if x.ndim == 3:
            bg = np.where(mask, np.float32(0.0), amax).max(axis=-1, keepdims=True).astype(np.float32)
            bg_scale = _scale((bg * np.float32(clip)).astype(np.float32))
            scale = np.where(mask, tok_scale, bg_scale)
        else:
            scale = tok_scale
        outs.append(_quantize(x, scale[..., None]))
    return outs[0], outs[1], mask
