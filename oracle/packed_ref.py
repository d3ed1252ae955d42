"""CPU oracle for the packed complex-phase linear layer (TEST INFRASTRUCTURE ONLY).

This module is a numpy restatement of the reference's algorithm for the packed
complex-phase GEMM. It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it. The CUDA path in ``rpfq_review_b200`` never calls into it.

Every function cites the reference file:line it follows. Paths are relative to
the reference project root (Fmylalala/RPFQ-review):

* ``EXP``  = ``RPFQ-ViTApple/scripts/export_rpfq_vit_to_mlx.py``
* ``QI``   = ``RPFQ-ViT-main/quant_models/quant_i.py``
* ``PL``   = ``RPFQ-ViTAndroid/app/src/main/cpp/ops/phase_linear.cpp``
* ``PLC``  = ``RPFQ-ViTAndroid/app/src/main/cpp/kernels/phase_linear_cache.cpp``

Pinning: the exporter functions restated here are checked against golden
vectors produced by the reference exporter itself (``tests/golden``), and the
decode / wide-linear functions against the reference's C++ runtime compiled
from its own sources (``oracle/_ref``).

Layout conventions (identical to the reference):

* A real ``Linear(in=K, out=N)`` is a complex map ``K_c = K/2 -> N_c = N/2``.
  Real columns ``[0, K_c)`` carry Re(x), ``[K_c, K)`` carry Im(x); outputs
  use the same split.
* Packed weights: per stage ``s`` and per U/W, ``codes`` uint8
  ``[N_cP, K_cP/4]`` (2-bit codes, element j at bits ``2*(j%4)``), and fp16
  ``gamma_real`` / ``gamma_imag`` ``[N_cP, K_cP/256]`` holding ``1/scale``.
  Codebook: 0 -> -1, 1 -> +1, 2 -> -i, 3 -> +i.
"""

from __future__ import annotations

import numpy as np

BLOCK_SIZE = 256  # EXP:28
PLANE_NAMES = ("u_s0", "u_s1", "w_s0", "w_s1")  # EXP:409-419 key order


def round_up(value: int, multiple: int) -> int:
    """EXP:75-76."""
    return ((value + multiple - 1) // multiple) * multiple


# --------------------------------------------------------------------------
# Exporter (packer) restatement
# --------------------------------------------------------------------------

def safe_mean_abs(x: np.ndarray, mask: np.ndarray, min_value: float) -> np.float32:
    """Masked mean |x| clamped below (EXP:121-124 with 1e-6; QI:29-33 with 1e-5).

    The sum is accumulated in float64 and rounded once to float32; torch's
    float32 reduction can differ in the last bit, which only matters when the
    fp16 gamma sits exactly on a rounding boundary.
    """
    m = mask.astype(np.float64)
    total = float((np.abs(x.astype(np.float64)) * m).sum())
    count = max(float(m.sum()), 1.0)
    mean = np.float32(np.float32(total) / np.float32(count))
    return np.float32(max(mean, np.float32(min_value)))


def axis_masks(w_real: np.ndarray, w_imag: np.ndarray):
    """Dominant-axis masks with quadrant tie-breaking (EXP:127-145, QI:36-62)."""
    abs_real = np.abs(w_real)
    abs_imag = np.abs(w_imag)
    real_dom = abs_real > abs_imag
    imag_dom = abs_imag > abs_real
    tie = ~(real_dom | imag_dom)
    zero_tie = tie & (w_real == 0) & (w_imag == 0)
    tie_q1 = tie & (w_real > 0) & (w_imag > 0)
    tie_q2 = tie & (w_real < 0) & (w_imag > 0)
    tie_q3 = tie & (w_real < 0) & (w_imag < 0)
    tie_q4 = tie & (w_real > 0) & (w_imag < 0)
    real_pos = (real_dom & (w_real >= 0)) | tie_q4 | zero_tie
    real_neg = (real_dom & (w_real < 0)) | tie_q2
    imag_pos = (imag_dom & (w_imag >= 0)) | tie_q1
    imag_neg = (imag_dom & (w_imag < 0)) | tie_q3
    return real_pos, real_neg, imag_pos, imag_neg


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """Four 2-bit codes per byte, low bits first (EXP:148-159)."""
    out_dim, in_dim = codes.shape
    if in_dim % 4 != 0:
        raise ValueError(f"Expected packed width to be divisible by 4, got {in_dim}")
    c = codes.reshape(out_dim, in_dim // 4, 4).astype(np.uint8)
    return (c[:, :, 0] | (c[:, :, 1] << 2) | (c[:, :, 2] << 4) | (c[:, :, 3] << 6)).astype(np.uint8)


def unpack_codes(packed: np.ndarray, out_dim: int, in_dim: int) -> np.ndarray:
    """Inverse of :func:`pack_codes` (EXP:234-240; PL:15-19 ``get2BitCode``)."""
    p = packed.reshape(out_dim, in_dim // 4)
    c = np.stack([(p >> s) & 0x03 for s in (0, 2, 4, 6)], axis=-1)
    return c.reshape(out_dim, in_dim).astype(np.uint8)


def phase_quantize_axis(w_real, w_imag, padded_out_dim=None, padded_in_dim=None):
    """One axial stage: codes + fp16 gammas (EXP:189-224)."""
    out_dim, in_dim = w_real.shape
    padded_out_dim = padded_out_dim or out_dim
    padded_in_dim = padded_in_dim or in_dim
    if padded_in_dim % BLOCK_SIZE != 0:
        raise ValueError(f"Expected padded input dim aligned to block size, got {padded_in_dim}")
    real_pos, real_neg, imag_pos, imag_neg = axis_masks(w_real, w_imag)
    scale_real = safe_mean_abs(w_real, real_pos | real_neg, 1e-6)
    scale_imag = safe_mean_abs(w_imag, imag_pos | imag_neg, 1e-6)
    codes = np.zeros((padded_out_dim, padded_in_dim), dtype=np.uint8)
    valid = codes[:out_dim, :in_dim]
    valid[real_pos] = 1
    valid[imag_neg] = 2
    valid[imag_pos] = 3
    blocks = padded_in_dim // BLOCK_SIZE
    # EXP:222-223: 1.0 / float(scale) is a python float64 division, then fp16.
    g_re = np.full((padded_out_dim, blocks), np.float16(1.0 / float(scale_real)), dtype=np.float16)
    g_im = np.full((padded_out_dim, blocks), np.float16(1.0 / float(scale_imag)), dtype=np.float16)
    return pack_codes(codes), g_re, g_im


def dequantize_axis(codes_packed, gamma_real, gamma_imag, out_dim, in_dim):
    """codes -> (+-1 or 0) / gamma in float32 (EXP:227-254)."""
    codes = unpack_codes(codes_packed, out_dim, in_dim)
    w_real = np.zeros((out_dim, in_dim), dtype=np.float32)
    w_imag = np.zeros((out_dim, in_dim), dtype=np.float32)
    w_real[codes == 0] = -1.0
    w_real[codes == 1] = 1.0
    w_imag[codes == 2] = -1.0
    w_imag[codes == 3] = 1.0
    gr = np.repeat(gamma_real.astype(np.float32), BLOCK_SIZE, axis=1)[:, :in_dim]
    gi = np.repeat(gamma_imag.astype(np.float32), BLOCK_SIZE, axis=1)[:, :in_dim]
    return (w_real / gr).astype(np.float32), (w_imag / gi).astype(np.float32)


def residual_phase_quantize(w_real, w_imag, stages, padded_out_dim=None, padded_in_dim=None):
    """Residual axial quantization over ``stages`` steps (EXP:257-289)."""
    res_r = w_real.astype(np.float32).copy()
    res_i = w_imag.astype(np.float32).copy()
    vo, vi = w_real.shape
    po = padded_out_dim or vo
    pi = padded_in_dim or vi
    out = []
    for _ in range(stages):
        codes, g_re, g_im = phase_quantize_axis(res_r, res_i, po, pi)
        dr, di = dequantize_axis(codes, g_re, g_im, po, pi)
        res_r = (res_r - dr[:vo, :vi]).astype(np.float32)
        res_i = (res_i - di[:vo, :vi]).astype(np.float32)
        out.append((codes, g_re, g_im))
    return out


def widely_linear_decompose(weight: np.ndarray):
    """A -> (U, W) with y = U x + W conj(x) (EXP:317-333, QI:519-527)."""
    n, k = weight.shape
    if n % 2 or k % 2:
        raise ValueError(f"Complex decomposition requires even dims, got {weight.shape}")
    ho, hi = n // 2, k // 2
    w = weight.astype(np.float32)
    a11, a12, a21, a22 = w[:ho, :hi], w[:ho, hi:], w[ho:, :hi], w[ho:, hi:]
    half = np.float32(0.5)
    u = (half * (a11 + a22), half * (a21 - a12))
    ww = (half * (a11 - a22), half * (a12 + a21))
    return u, ww


def pack_linear(weight: np.ndarray, bias, stages: int = 2):
    """Float weight -> exporter-layout packed dict (EXP:384-423).

    Returns ``{"u_s0.codes": ..., "u_s0.gamma_real": ..., ..., "bias": fp16}``.
    """
    n, k = weight.shape
    n_cp = round_up(n // 2, BLOCK_SIZE)
    k_cp = round_up(k // 2, BLOCK_SIZE)
    (ur, ui), (wr, wi) = widely_linear_decompose(weight)
    out = {}
    for tag, (re, im) in (("u", (ur, ui)), ("w", (wr, wi))):
        for s, (codes, g_re, g_im) in enumerate(residual_phase_quantize(re, im, stages, n_cp, k_cp)):
            out[f"{tag}_s{s}.codes"] = codes
            out[f"{tag}_s{s}.gamma_real"] = g_re
            out[f"{tag}_s{s}.gamma_imag"] = g_im
    out["bias"] = (np.zeros(n, np.float32) if bias is None else np.asarray(bias, np.float32)).astype(np.float16)
    return out


# --------------------------------------------------------------------------
# Packed -> dense (deployment forward) restatement
# --------------------------------------------------------------------------

def stage_names(packed: dict) -> tuple[list[str], list[str]]:
    us = sorted({k.split(".")[0] for k in packed if k.startswith("u_s")})
    ws = sorted({k.split(".")[0] for k in packed if k.startswith("w_s")})
    return us, ws


def dense_weight_from_packed(packed: dict, n_c: int, k_c: int) -> np.ndarray:
    """Packed planes -> dense float32 ``[2 n_c, 2 k_c]`` (EXP:336-375).

    Same arithmetic as ``quantized_forward_weight``: stages summed into a zero
    accumulator in order, then ``A11 = Wr + Ur``, ``A12 = Wi - Ui``,
    ``A21 = Wi + Ui``, ``A22 = -Wr + Ur`` (EXP:365-368).
    """
    us, ws = stage_names(packed)
    codes0 = packed[us[0] + ".codes"]
    n_cp, k_cp = codes0.shape[0], codes0.shape[1] * 4

    def accumulate(names):
        acc_r = np.zeros((n_cp, k_cp), np.float32)
        acc_i = np.zeros((n_cp, k_cp), np.float32)
        for name in names:
            dr, di = dequantize_axis(packed[name + ".codes"], packed[name + ".gamma_real"],
                                     packed[name + ".gamma_imag"], n_cp, k_cp)
            acc_r += dr
            acc_i += di
        return acc_r[:n_c, :k_c], acc_i[:n_c, :k_c]

    ur, ui = accumulate(us)
    wr, wi = accumulate(ws)
    top = np.concatenate([wr + ur, wi - ui], axis=1)
    bot = np.concatenate([wi + ui, -wr + ur], axis=1)
    return np.concatenate([top, bot], axis=0).astype(np.float32)


def f32_to_f16_ties_away(s: np.ndarray) -> np.ndarray:
    """float32 -> fp16 rounding ties away from zero, as the reference's
    ``floatToHalfBits`` (PLC:58-82): truncate the mantissa and add one ulp
    when the first dropped bit is set; overflow -> inf; subnormals likewise."""
    bits = np.ascontiguousarray(s, dtype=np.float32).view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    exp = ((bits >> 23) & 0xFF) - 127 + 15
    mant = bits & 0x7FFFFF
    out = np.empty(bits.shape, np.int64)
    normal = (exp > 0) & (exp < 31)
    half = sign | (np.clip(exp, 0, 31) << 10) | (mant >> 13)
    half = half + ((mant & 0x1000) != 0)
    out[normal] = half[normal]
    out[exp >= 31] = (sign | 0x7C00)[exp >= 31]
    sub = exp <= 0
    tiny = sub & (exp < -10)
    out[tiny] = sign[tiny]
    mid = sub & ~tiny
    if mid.any():
        m = mant[mid] | 0x800000
        shift = 14 - exp[mid]
        hm = (m >> shift) + ((m >> (shift - 1)) & 1)
        out[mid] = sign[mid] | hm
    return out.astype(np.uint16).view(np.float16)


def unpack_bits(packed: np.ndarray, cols: int, code_bits: int) -> np.ndarray:
    """b-bit codes stored LSB-first as a bit stream per row (2-bit: four per
    byte exactly as :func:`pack_codes`). 3- and 4-bit widths are this build's
    extension for uniform 2^b phases; the reference defines only 2-bit codes."""
    rows = packed.shape[0]
    bits = np.unpackbits(packed.reshape(rows, -1), axis=1, bitorder="little")[:, : cols * code_bits]
    bits = bits.reshape(rows, cols, code_bits).astype(np.uint8)
    weights = (1 << np.arange(code_bits)).astype(np.uint8)
    return (bits * weights).sum(axis=-1).astype(np.uint8)


def phase_tables(code_bits: int):
    """float32 cos/sin of the uniform phases 2 pi c / 2^b, exact zeros kept."""
    n = 1 << code_bits
    ang = 2.0 * np.pi * np.arange(n) / n
    cs, sn = np.cos(ang), np.sin(ang)
    cs[np.abs(cs) < 1e-12] = 0.0
    sn[np.abs(sn) < 1e-12] = 0.0
    return cs.astype(np.float32), sn.astype(np.float32)


def decode_plane(packed: dict, name: str, n_c: int, k_c: int, code_bits: int = 2):
    """One plane -> float32 (re, im) on the valid region ``[n_c, k_c]``.

    2-bit: the reference codebook with ``1.0f / gamma`` (PL:82-83, PL:145-153).
    3/4-bit extension: ``(cos_c / gamma_real, sin_c / gamma_imag)`` with
    ``cos_c = cos(2 pi c / 2^b)`` in float32, each product rounded once.
    """
    codes_p = packed[name + ".codes"]
    k_cp = codes_p.shape[1] * 8 // code_bits
    codes = unpack_bits(codes_p, k_cp, code_bits)[:n_c, :k_c]
    inv_r = np.float32(1.0) / packed[name + ".gamma_real"].astype(np.float32)
    inv_i = np.float32(1.0) / packed[name + ".gamma_imag"].astype(np.float32)
    inv_r = np.repeat(inv_r, BLOCK_SIZE, axis=1)[:n_c, :k_c]
    inv_i = np.repeat(inv_i, BLOCK_SIZE, axis=1)[:n_c, :k_c]
    if code_bits == 2:
        zero = np.float32(0.0)
        re = np.where(codes == 0, -inv_r, np.where(codes == 1, inv_r, zero)).astype(np.float32)
        im = np.where(codes == 2, -inv_i, np.where(codes == 3, inv_i, zero)).astype(np.float32)
    else:
        cs, sn = phase_tables(code_bits)
        re = (cs[codes] * inv_r).astype(np.float32)
        im = (sn[codes] * inv_i).astype(np.float32)
    return re, im


def coefficient_planes(packed: dict, n_c: int, k_c: int, rounding: str = "rne",
                       code_bits: int = 2) -> dict[str, np.ndarray]:
    """Four fp16 coefficient planes, the B200 B operand (PLC:84-133).

    Follows ``buildFusedWideLinearCache``: per element the stage values are
    decoded with ``1.0f / gamma`` in float32 (PL:82-83) and summed left to
    right in float32 (PLC:119-126), U stages first, then W stages:

    * ``rr = u0Re + u1Re + w0Re + w1Re``   (x_re -> y_re)
    * ``ir = -u0Im - u1Im + w0Im + w1Im`` (x_im -> y_re)
    * ``ri = u0Im + u1Im + w0Im + w1Im``   (x_re -> y_im)
    * ``ii = u0Re + u1Re - w0Re - w1Re``   (x_im -> y_im)

    (the reference fixes 2 stages; other stage counts extend the same order).
    The reference converts to fp16 with ties rounded away from zero
    (``floatToHalfBits``, PLC:58-82): ``rounding="ties_away"`` reproduces it
    bit for bit. ``rounding="rne"`` (default) rounds to nearest even, the IEEE
    default; the two differ only on exact ties.
    """
    if rounding not in ("rne", "ties_away"):
        raise ValueError(f"unknown rounding {rounding!r}")
    us, ws = stage_names(packed)
    u0r, u0i = decode_plane(packed, us[0], n_c, k_c, code_bits)
    rr, ir, ri, ii = u0r, -u0i, u0i, u0r
    for name in us[1:]:
        re, im = decode_plane(packed, name, n_c, k_c, code_bits)
        rr, ir, ri, ii = rr + re, ir - im, ri + im, ii + re
    for name in ws:
        re, im = decode_plane(packed, name, n_c, k_c, code_bits)
        rr, ir, ri, ii = rr + re, ir + im, ri + im, ii - re
    cvt = (lambda a: a.astype(np.float16)) if rounding == "rne" else f32_to_f16_ties_away
    return {"rr": cvt(rr), "ir": cvt(ir), "ri": cvt(ri), "ii": cvt(ii)}


def dense_fp16_from_planes(planes: dict[str, np.ndarray]) -> np.ndarray:
    """Assemble the four planes into the dense fp16 ``[N, K]`` matrix that the
    GEMM consumes: ``[[rr, ir], [ri, ii]]`` (same block layout as EXP:369-375)."""
    top = np.concatenate([planes["rr"], planes["ir"]], axis=1)
    bot = np.concatenate([planes["ri"], planes["ii"]], axis=1)
    return np.concatenate([top, bot], axis=0)


# --------------------------------------------------------------------------
# Activation quantization and the layer forward
# --------------------------------------------------------------------------

def act_quant(x: np.ndarray, num_bits: int) -> np.ndarray:
    """Per-row symmetric quantization of the Re and Im halves (QI:442-455).

    ``s = qmax / max(amax, 1e-5)``; ``q = round_half_even(x * s)`` clamped to
    ``[qmin, qmax]``; returns ``q / s``. All steps in float32.

    ``float(qmax) / tensor`` in torch is evaluated as ``reciprocal(tensor) *
    qmax`` (two float32 roundings), which this restatement reproduces; the
    golden vectors of ``ActivationQuantSTE`` pin it bit for bit.
    """
    x = x.astype(np.float32)
    k_c = x.shape[-1] // 2
    qmax = np.float32((1 << (num_bits - 1)) - 1)
    qmin = np.float32(-(1 << (num_bits - 1)))
    out = np.empty_like(x)
    for lo, hi in ((0, k_c), (k_c, 2 * k_c)):
        part = x[..., lo:hi]
        amax = np.maximum(np.abs(part).max(axis=-1, keepdims=True), np.float32(1e-5)).astype(np.float32)
        s = ((np.float32(1.0) / amax).astype(np.float32) * qmax).astype(np.float32)
        q = np.clip(np.rint((part * s).astype(np.float32)), qmin, qmax).astype(np.float32)
        out[..., lo:hi] = (q / s).astype(np.float32)
    return out


def gelu_erf(x: np.ndarray) -> np.ndarray:
    """Exact (erf) GELU in float64, as F.gelu(approximate="none")."""
    from math import erf, sqrt
    v = np.vectorize(lambda t: 0.5 * t * (1.0 + erf(t / sqrt(2.0))))
    return v(x.astype(np.float64))


def wide_linear(x: np.ndarray, dense: np.ndarray, bias=None, act_bits: int | None = None) -> np.ndarray:
    """Layer forward ``F.linear(act_quant(x), W, b)`` in float64 (QI:546-554).

    ``dense`` is the float32 weight from :func:`dense_weight_from_packed` (the
    reference's deployment path) or the fp16 matrix from
    :func:`dense_fp16_from_planes` (the reference's fp16 runtime cache).
    """
    xx = x.astype(np.float32)
    if act_bits is not None:
        xx = act_quant(xx, act_bits)
    y = xx.astype(np.float64) @ dense.astype(np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y


def max_rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """``max|y - ref| / max|ref|`` — the relative-error measure used by the
    parity tests (the reference's own check is an absolute max, PL:225-245)."""
    ref = np.asarray(ref, np.float64)
    denom = max(float(np.abs(ref).max()), 1e-30)
    return float(np.abs(np.asarray(y, np.float64) - ref).max() / denom)


# --------------------------------------------------------------------------
# Synthetic packed layers (the benchmark's seeded workload), numpy flavour
# --------------------------------------------------------------------------

def random_packed_numpy(n_c: int, k_c: int, seed: int, stages: int = 2, bias_std: float = 0.01):
    """Seeded synthetic packed layer: uniform codes on the valid region, padding
    codes 0, per-row per-plane lognormal(0, 0.5) scales stored as fp16 1/s."""
    rng = np.random.default_rng(seed)
    n_cp, k_cp = round_up(n_c, BLOCK_SIZE), round_up(k_c, BLOCK_SIZE)
    out = {}
    for tag in ("u", "w"):
        for s in range(stages):
            codes = np.zeros((n_cp, k_cp), np.uint8)
            codes[:n_c, :k_c] = rng.integers(0, 4, size=(n_c, k_c), dtype=np.uint8)
            out[f"{tag}_s{s}.codes"] = pack_codes(codes)
            for part in ("gamma_real", "gamma_imag"):
                sc = rng.lognormal(0.0, 0.5, size=(n_cp, 1)).astype(np.float32)
                out[f"{tag}_s{s}.{part}"] = np.repeat((np.float32(1.0) / sc).astype(np.float16),
                                                      k_cp // BLOCK_SIZE, axis=1)
    out["bias"] = (rng.standard_normal(2 * n_c) * bias_std).astype(np.float16)
    return out
