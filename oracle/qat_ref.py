"""CPU oracle: the reference's QAT forward of the complex-phase layer (TEST
INFRASTRUCTURE ONLY — only ``tests/`` and ``bench.py``'s CPU legs may import
it; the CUDA path never does).

``QATLinearComplexPhase.forward`` (``RPFQ-ViT-main/quant_models/quant_i.py:
513-554``) re-quantizes the float weight on every call: the 2 x 2 block split
into U / W (``:519-527``), the residual axial quantizer of each
(``_residual_quantize`` with ``_quantize_phase_axis``, ``:93-118, 65-83``,
masks ``:36-62``, scales ``_safe_mean_abs`` ``:29-33``), the reassembly
(``:534-544``), optional ``ActivationQuantSTE`` (``:442-455``) and
``F.linear``. This restatement runs the same torch CPU float32 operations in
the same order, so its masks and scales are the reference's bit for bit.

Unlike the exporter (``export_rpfq_vit_to_mlx.py:189-289``), whose stage
values are ``±1 / fp16(1 / scale)`` and whose scale clamp is 1e-6, the QAT
forward keeps each stage's value at the float32 scale (clamp 1e-5).
:func:`stage_codes` returns the axis decisions of each stage in the
exporter's code numbering so the two paths can be compared stage by stage.
"""

from __future__ import annotations

import numpy as np
import torch


def _safe_mean_abs(x: torch.Tensor, mask: torch.Tensor, min_val: float = 1e-5) -> torch.Tensor:
    """quant_i.py:29-33."""
    mask_f = mask.to(dtype=x.dtype)
    return ((x.abs() * mask_f).sum() / mask_f.sum().clamp_min(1.0)).clamp_min(min_val)


def _axis_masks(w_real: torch.Tensor, w_imag: torch.Tensor):
    """quant_i.py:36-62: dominant axis, ties resolved by quadrant."""
    abs_real, abs_imag = w_real.abs(), w_imag.abs()
    real_dominant = abs_real > abs_imag
    imag_dominant = abs_imag > abs_real
    tie = ~(real_dominant | imag_dominant)
    zero_tie = tie & (w_real == 0) & (w_imag == 0)
    tie_q1 = tie & (w_real > 0) & (w_imag > 0)
    tie_q2 = tie & (w_real < 0) & (w_imag > 0)
    tie_q3 = tie & (w_real < 0) & (w_imag < 0)
    tie_q4 = tie & (w_real > 0) & (w_imag < 0)
    real_pos = (real_dominant & (w_real >= 0)) | tie_q4 | zero_tie
    real_neg = (real_dominant & (w_real < 0)) | tie_q2
    imag_pos = (imag_dominant & (w_imag >= 0)) | tie_q1
    imag_neg = (imag_dominant & (w_imag < 0)) | tie_q3
    return real_pos, real_neg, imag_pos, imag_neg


def _quantize_phase_axis(w_real: torch.Tensor, w_imag: torch.Tensor):
    """quant_i.py:65-83: {±s_re, 0} or {0, ±s_im} with float32 scales; also
    the stage's codes (0: -1, 1: +1, 2: -i, 3: +i, the exporter's numbering)."""
    real_pos, real_neg, imag_pos, imag_neg = _axis_masks(w_real, w_imag)
    real_mean = _safe_mean_abs(w_real, real_pos | real_neg)
    imag_mean = _safe_mean_abs(w_imag, imag_pos | imag_neg)
    qw_real = torch.zeros_like(w_real)
    qw_imag = torch.zeros_like(w_imag)
    qw_real = torch.where(real_pos, real_mean, qw_real)
    qw_real = torch.where(real_neg, -real_mean, qw_real)
    qw_imag = torch.where(imag_pos, imag_mean, qw_imag)
    qw_imag = torch.where(imag_neg, -imag_mean, qw_imag)
    codes = torch.zeros(w_real.shape, dtype=torch.uint8)
    codes[real_pos] = 1
    codes[imag_neg] = 2
    codes[imag_pos] = 3
    return qw_real, qw_imag, codes, (float(real_mean), float(imag_mean))


def _residual_quantize(w_real: torch.Tensor, w_imag: torch.Tensor, steps: int, force_codes=None):
    """quant_i.py:93-118. ``force_codes`` (test instrument) replaces the axis
    decision of stage s by the given codes while keeping the float32 scales of
    the QAT path, to isolate where the exporter's result departs from it."""
    q_real = torch.zeros_like(w_real)
    q_imag = torch.zeros_like(w_imag)
    r_real, r_imag = w_real, w_imag
    stages = []
    for s in range(steps):
        if force_codes is not None and force_codes[s] is not None:
            c = torch.from_numpy(np.asarray(force_codes[s])).to(torch.uint8)
            real_pos, real_neg, imag_neg, imag_pos = (c == 1), (c == 0), (c == 2), (c == 3)
            real_mean = _safe_mean_abs(r_real, real_pos | real_neg)
            imag_mean = _safe_mean_abs(r_imag, imag_pos | imag_neg)
            step_real = torch.where(real_pos, real_mean, torch.where(real_neg, -real_mean, torch.zeros_like(r_real)))
            step_imag = torch.where(imag_pos, imag_mean, torch.where(imag_neg, -imag_mean, torch.zeros_like(r_imag)))
            stages.append((c, (float(real_mean), float(imag_mean))))
        else:
            step_real, step_imag, c, scales = _quantize_phase_axis(r_real, r_imag)
            stages.append((c, scales))
        q_real = q_real + step_real
        q_imag = q_imag + step_imag
        r_real = r_real - step_real
        r_imag = r_imag - step_imag
    return q_real, q_imag, stages


def quantized_weight(weight: np.ndarray, steps: int = 2, force_codes: dict | None = None):
    """The QAT forward's quantized weight ``q_weight`` (quant_i.py:513-544)
    and, per plane ``u`` / ``w``, the list of (codes, (scale_re, scale_im))
    of each stage. ``force_codes`` maps ``"u"`` / ``"w"`` to per-stage codes
    (or None) for :func:`_residual_quantize`."""
    w = torch.from_numpy(np.ascontiguousarray(weight, dtype=np.float32))
    half_out, half_in = w.shape[0] // 2, w.shape[1] // 2
    a11, a12 = w[:half_out, :half_in], w[:half_out, half_in:]
    a21, a22 = w[half_out:, :half_in], w[half_out:, half_in:]
    u_real, u_imag = 0.5 * (a11 + a22), 0.5 * (a21 - a12)
    w_real, w_imag = 0.5 * (a11 - a22), 0.5 * (a12 + a21)
    fc = force_codes or {}
    uq_r, uq_i, u_st = _residual_quantize(u_real, u_imag, steps, fc.get("u"))
    wq_r, wq_i, w_st = _residual_quantize(w_real, w_imag, steps, fc.get("w"))
    q = torch.cat((torch.cat((wq_r + uq_r, wq_i - uq_i), dim=1),
                   torch.cat((wq_i + uq_i, -wq_r + uq_r), dim=1)), dim=0)
    return q, {"u": u_st, "w": w_st}


def act_quant(x: torch.Tensor, num_bits: int) -> torch.Tensor:
    """ActivationQuantSTE.forward, quant_i.py:442-455."""
    half = x.shape[-1] // 2
    qmax, qmin = (1 << (num_bits - 1)) - 1, -(1 << (num_bits - 1))
    outs = []
    for part in (x[..., :half], x[..., half:]):
        scale = float(qmax) / part.abs().amax(dim=-1, keepdim=True).clamp_min(1e-5)
        outs.append((part * scale).round().clamp(qmin, qmax) / scale)
    return torch.cat(outs, dim=-1)


def forward(weight: np.ndarray, bias: np.ndarray | None, x: np.ndarray, act_bits: int = 0, steps: int = 2,
            force_codes: dict | None = None) -> np.ndarray:
    """QATLinearComplexPhase.forward with ``complex_phase_v{steps}`` for U and
    W (quant_i.py:513-554), float32 on the CPU."""
    q, _ = quantized_weight(weight, steps, force_codes)
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    if act_bits:
        xt = act_quant(xt, act_bits)
    b = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, dtype=np.float32))
    return torch.nn.functional.linear(xt, q, b).numpy()
