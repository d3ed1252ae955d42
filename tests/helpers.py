"""Shared test helpers: convert product-side packed layers to the oracle's
numpy dict form and compare results."""

from __future__ import annotations

import numpy as np
import torch


def to_numpy_packed(layer) -> dict:
    out = {}
    for name, (c, gr, gi) in layer.planes.items():
        out[f"{name}.codes"] = c.cpu().numpy()
        out[f"{name}.gamma_real"] = gr.cpu().numpy()
        out[f"{name}.gamma_imag"] = gi.cpu().numpy()
    if layer.bias is not None:
        out["bias"] = layer.bias.cpu().numpy()
    return out


def from_numpy_packed(d: dict, n_c: int, k_c: int, device, code_bits: int = 2):
    from rpfq_review_b200.packing import PackedLayer
    stages = 0
    while f"u_s{stages}.codes" in d:
        stages += 1
    planes = {}
    for tag in ("u", "w"):
        for s in range(stages):
            n = f"{tag}_s{s}"
            planes[n] = tuple(torch.from_numpy(np.ascontiguousarray(d[f"{n}.{k}"])).to(device)
                              for k in ("codes", "gamma_real", "gamma_imag"))
    bias = torch.from_numpy(np.ascontiguousarray(d["bias"])).to(device) if "bias" in d else None
    return PackedLayer(n_c, k_c, stages, code_bits, planes, bias)


def rel_err(y, ref) -> float:
    """The parity tests' normalised measure: max|y - ref| / max|ref|."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def elem_rel_err(y, ref, floor: float = 1e-3) -> float:
    """Element-wise relative error: max over elements of
    |y - ref| / max(|ref|, floor * max|ref|). The floor keeps elements that
    cancel to near zero from dividing by their own rounding noise."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.maximum(np.abs(ref), floor * max(np.abs(ref).max(), 1e-30))
    return float((np.abs(y - ref) / den).max())
