"""Packed phase-code weight layout: packing float weights, seeded synthetic
layers, and the key/shape contract of the reference exporter.

The layout is the one the reference exporter writes and its mobile runtimes
read (RPFQ-ViTApple/scripts/export_rpfq_vit_to_mlx.py:148-159,189-224,384-423;
RPFQ-ViTAndroid/app/src/main/cpp/ops/phase_linear.cpp:42-117):

* per residual stage ``s`` of U and of W:
  ``{u,w}_s{s}.codes`` uint8 ``[n_cp, k_cp * code_bits / 8]`` (codes LSB-first;
  2-bit codebook 0:-1, 1:+1, 2:-i, 3:+i), ``{u,w}_s{s}.gamma_real`` and
  ``.gamma_imag`` fp16 ``[n_cp, k_cp / 256]`` holding ``1 / scale``;
* ``bias`` fp16 ``[2 n_c]``;
* ``n_cp``, ``k_cp`` = complex dims rounded up to 256; padding codes are 0.

Packing runs with torch ops on whatever device the weight lives on (it is
weight preparation, done once, not the inference hot path).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

BLOCK_SIZE = 256  # export_rpfq_vit_to_mlx.py:28

# quant_i.py:355-371 method name -> residual stages of the axial quantizer.
AXIAL_STAGES = {
    "complex_phase_v1": 1,
    "complex_phase_v2": 2,
    "complex_phase_v3": 3,
    "complex_phase_v4": 4,
}
SUPPORTED_QUANT_METHODS = (
    "complex_phase_v1",
    "complex_phase_v2",
    "complex_phase_v3",
    "complex_phase_v4",
    "complex_phase_new_v2",
    "complex_phase_next_v1",
)


def round_up(value: int, multiple: int) -> int:
    return ((value + multiple - 1) // multiple) * multiple


@dataclass
class PackedLayer:
    """One packed widely-linear layer (tensors on one device)."""

    n_c: int
    k_c: int
    stages: int
    code_bits: int
    planes: dict  # "u_s0" -> (codes, gamma_real, gamma_imag), ...
    bias: torch.Tensor | None  # fp16 [2 n_c]

    @property
    def n_cp(self) -> int:
        return int(self.planes["u_s0"][0].shape[0])

    @property
    def k_cp(self) -> int:
        return int(self.planes["u_s0"][0].shape[1] * 8 // self.code_bits)

    def plane_names(self, tag: str):
        return [f"{tag}_s{s}" for s in range(self.stages)]

    def to(self, device) -> "PackedLayer":
        planes = {k: tuple(t.to(device) for t in v) for k, v in self.planes.items()}
        bias = self.bias.to(device) if self.bias is not None else None
        return PackedLayer(self.n_c, self.k_c, self.stages, self.code_bits, planes, bias)

    def state_dict(self, prefix: str = "") -> dict:
        """Exporter keys (export_rpfq_vit_to_mlx.py:409-423)."""
        out = {}
        for name, (c, gr, gi) in self.planes.items():
            out[f"{prefix}{name}.codes"] = c
            out[f"{prefix}{name}.gamma_real"] = gr
            out[f"{prefix}{name}.gamma_imag"] = gi
        if self.bias is not None:
            out[f"{prefix}bias"] = self.bias
        return out

    @staticmethod
    def from_state_dict(sd: dict, prefix: str, in_features: int, out_features: int,
                        code_bits: int = 2) -> "PackedLayer":
        """Read an exporter-layout layer and validate shapes like the reference
        loader (phase_linear.cpp:42-88): codes ``[n_cp, k_cp/4]``, gammas
        ``[n_cp, k_cp/256]``, ``k_cp % 256 == 0``, no zero gamma."""
        if in_features % 2 or out_features % 2:
            raise ValueError("Complex-phase layers require even in/out features.")
        n_c, k_c = out_features // 2, in_features // 2
        stages = 0
        while f"{prefix}u_s{stages}.codes" in sd:
            stages += 1
        if stages == 0:
            raise ValueError(f"Missing packed tensor: {prefix}u_s0.codes")
        planes = {}
        for tag in ("u", "w"):
            for s in range(stages):
                name = f"{tag}_s{s}"
                try:
                    c = sd[f"{prefix}{name}.codes"]
                    gr = sd[f"{prefix}{name}.gamma_real"]
                    gi = sd[f"{prefix}{name}.gamma_imag"]
                except KeyError as e:
                    raise ValueError(f"Missing packed tensor: {e.args[0]}") from None
                n_cp = c.shape[0]
                k_cp = c.shape[1] * 8 // code_bits
                if k_cp % BLOCK_SIZE or n_cp < n_c or k_cp < k_c:
                    raise ValueError(f"Packed code shape mismatch for {prefix}{name}")
                if tuple(gr.shape) != (n_cp, k_cp // BLOCK_SIZE) or tuple(gi.shape) != (n_cp, k_cp // BLOCK_SIZE):
                    raise ValueError(f"Gamma row shape mismatch for {prefix}{name}")
                if bool((gr == 0).any()) or bool((gi == 0).any()):
                    raise ValueError(f"Zero gamma found in {prefix}{name}")
                planes[name] = (c.to(torch.uint8).contiguous(), gr.to(torch.float16).contiguous(),
                                gi.to(torch.float16).contiguous())
        bias = sd.get(f"{prefix}bias")
        if bias is not None:
            if bias.numel() != out_features:
                raise ValueError(f"WideLinear bias shape mismatch for {prefix}")
            bias = bias.to(torch.float16).contiguous()
        return PackedLayer(n_c, k_c, stages, code_bits, planes, bias)


# ---------------------------------------------------------------------------
# Exporter algorithm (torch): float weight -> packed axial codes
# ---------------------------------------------------------------------------

def _safe_mean_abs(x, mask, min_value=1e-6):
    """export_rpfq_vit_to_mlx.py:121-124."""
    m = mask.to(x.dtype)
    return ((x.abs() * m).sum() / m.sum().clamp_min(1.0)).clamp_min(min_value)


def _axis_masks(w_real, w_imag):
    """Dominant-axis masks with quadrant tie-breaking (export…py:127-145)."""
    abs_r, abs_i = w_real.abs(), w_imag.abs()
    real_dom = abs_r > abs_i
    imag_dom = abs_i > abs_r
    tie = ~(real_dom | imag_dom)
    zero_tie = tie & (w_real == 0) & (w_imag == 0)
    q1 = tie & (w_real > 0) & (w_imag > 0)
    q2 = tie & (w_real < 0) & (w_imag > 0)
    q3 = tie & (w_real < 0) & (w_imag < 0)
    q4 = tie & (w_real > 0) & (w_imag < 0)
    real_pos = (real_dom & (w_real >= 0)) | q4 | zero_tie
    real_neg = (real_dom & (w_real < 0)) | q2
    imag_pos = (imag_dom & (w_imag >= 0)) | q1
    imag_neg = (imag_dom & (w_imag < 0)) | q3
    return real_pos, real_neg, imag_pos, imag_neg


def pack_codes(codes: torch.Tensor) -> torch.Tensor:
    """Four 2-bit codes per byte, low bits first (export…py:148-159)."""
    out_dim, in_dim = codes.shape
    c = codes.reshape(out_dim, in_dim // 4, 4).to(torch.uint8)
    return (c[:, :, 0] | (c[:, :, 1] << 2) | (c[:, :, 2] << 4) | (c[:, :, 3] << 6)).to(torch.uint8)


def _phase_quantize_axis(w_real, w_imag, n_cp, k_cp):
    """export…py:189-224."""
    out_dim, in_dim = w_real.shape
    rp, rn, ip, inn = _axis_masks(w_real, w_imag)
    s_r = _safe_mean_abs(w_real, rp | rn)
    s_i = _safe_mean_abs(w_imag, ip | inn)
    codes = torch.zeros((n_cp, k_cp), dtype=torch.uint8, device=w_real.device)
    valid = codes[:out_dim, :in_dim]
    valid[rp] = 1
    valid[inn] = 2
    valid[ip] = 3
    blocks = k_cp // BLOCK_SIZE
    g_r = torch.full((n_cp, blocks), 1.0 / float(s_r), dtype=torch.float16, device=w_real.device)
    g_i = torch.full((n_cp, blocks), 1.0 / float(s_i), dtype=torch.float16, device=w_real.device)
    return pack_codes(codes), g_r, g_i


def _dequantize_axis(packed, g_r, g_i, out_dim, in_dim):
    """export…py:227-254."""
    p = packed.reshape(out_dim, in_dim // 4)
    codes = torch.stack([(p >> s) & 0x03 for s in (0, 2, 4, 6)], dim=-1).reshape(out_dim, in_dim)
    w_r = torch.zeros((out_dim, in_dim), dtype=torch.float32, device=packed.device)
    w_i = torch.zeros_like(w_r)
    w_r[codes == 0] = -1.0
    w_r[codes == 1] = 1.0
    w_i[codes == 2] = -1.0
    w_i[codes == 3] = 1.0
    gr = g_r.float().repeat_interleave(BLOCK_SIZE, dim=1)[:, :in_dim]
    gi = g_i.float().repeat_interleave(BLOCK_SIZE, dim=1)[:, :in_dim]
    return w_r / gr, w_i / gi


def pack_linear(weight: torch.Tensor, bias: torch.Tensor | None, stages: int = 2) -> PackedLayer:
    """Float ``[N, K]`` weight -> packed layer, the exporter's
    ``save_quantized_linear`` (export…py:384-423): widely-linear decomposition
    (export…py:317-333), then ``stages`` residual axial quantization steps
    (export…py:257-289) for U and for W.

    CUDA weights are packed by the GPU packer (``ops.pack_linear``, two
    kernels per stage, no host sync); CPU weights by the same algorithm in
    torch, the offline exporter's setting."""
    if weight.is_cuda:
        from . import ops
        return ops.pack_linear(weight, bias, stages)
    return pack_linear_torch(weight, bias, stages)


def pack_linear_torch(weight: torch.Tensor, bias: torch.Tensor | None, stages: int = 2) -> PackedLayer:
    """:func:`pack_linear` as torch tensor ops on the weight's device."""
    n, k = weight.shape
    if n % 2 or k % 2:
        raise ValueError(f"Complex decomposition requires even dims, got {tuple(weight.shape)}")
    n_c, k_c = n // 2, k // 2
    n_cp, k_cp = round_up(n_c, BLOCK_SIZE), round_up(k_c, BLOCK_SIZE)
    w = weight.detach().float()
    a11, a12, a21, a22 = w[:n_c, :k_c], w[:n_c, k_c:], w[n_c:, :k_c], w[n_c:, k_c:]
    parts = {
        "u": (0.5 * (a11 + a22), 0.5 * (a21 - a12)),
        "w": (0.5 * (a11 - a22), 0.5 * (a12 + a21)),
    }
    planes = {}
    for tag, (re, im) in parts.items():
        res_r, res_i = re.clone(), im.clone()
        for s in range(stages):
            codes, g_r, g_i = _phase_quantize_axis(res_r, res_i, n_cp, k_cp)
            d_r, d_i = _dequantize_axis(codes, g_r, g_i, n_cp, k_cp)
            res_r = res_r - d_r[:n_c, :k_c]
            res_i = res_i - d_i[:n_c, :k_c]
            planes[f"{tag}_s{s}"] = (codes, g_r, g_i)
    b = torch.zeros(n, device=weight.device) if bias is None else bias.detach()
    return PackedLayer(n_c, k_c, stages, 2, planes, b.to(torch.float16).contiguous())


# ---------------------------------------------------------------------------
# Seeded synthetic packed layers (the benchmark workload)
# ---------------------------------------------------------------------------

def pack_bits(codes: torch.Tensor, code_bits: int) -> torch.Tensor:
    """Pack integer codes ``[rows, cols]`` LSB-first into a bit stream per row
    (2-bit: four per byte, identical to :func:`pack_codes`)."""
    rows, cols = codes.shape
    if code_bits == 2:
        return pack_codes(codes)
    if (cols * code_bits) % 8:
        raise ValueError("row bit length must be a whole number of bytes")
    bits = torch.zeros((rows, cols * code_bits), dtype=torch.uint8)
    c = codes.to(torch.int64)
    for b in range(code_bits):
        bits[:, b::code_bits] = ((c >> b) & 1).to(torch.uint8)
    bits = bits.reshape(rows, -1, 8).to(torch.int64)
    weights = torch.tensor([1 << i for i in range(8)], dtype=torch.int64)
    return (bits * weights).sum(-1).to(torch.uint8)


def random_packed(n_c: int, k_c: int, seed: int, stages: int = 2, code_bits: int = 2,
                  bias_std: float = 0.01, device="cpu") -> PackedLayer:
    """Seeded synthetic packed layer on the benchmark's distribution: codes
    uniform over the 2^b phases on the valid ``[n_c, k_c]`` region, padding
    codes 0; per output row, per plane, separately for re and im, a scale
    ``s ~ lognormal(0, 0.5)`` stored as ``gamma = fp16(1/s)`` broadcast over
    the 256-column blocks; bias ~ N(0, bias_std^2) in fp16. Drawn on the CPU
    with a seeded torch.Generator, so every device sees the same layer."""
    g = torch.Generator().manual_seed(int(seed))
    n_cp, k_cp = round_up(n_c, BLOCK_SIZE), round_up(k_c, BLOCK_SIZE)
    blocks = k_cp // BLOCK_SIZE
    planes = {}
    for tag in ("u", "w"):
        for s in range(stages):
            codes = torch.zeros((n_cp, k_cp), dtype=torch.uint8)
            codes[:n_c, :k_c] = torch.randint(0, 1 << code_bits, (n_c, k_c), generator=g, dtype=torch.int64).to(
                torch.uint8)
            gam = []
            for _ in range(2):
                sc = torch.exp(torch.randn((n_cp, 1), generator=g) * 0.5)
                gam.append((1.0 / sc).to(torch.float16).repeat(1, blocks).contiguous())
            planes[f"{tag}_s{s}"] = (pack_bits(codes, code_bits), gam[0], gam[1])
    bias = (torch.randn(2 * n_c, generator=g) * bias_std).to(torch.float16)
    return PackedLayer(n_c, k_c, stages, code_bits, planes, bias).to(device)


def layer_seed(name: str, base: int = 0) -> int:
    """Stable per-layer seed from a layer name (FNV-1a, 31 bits)."""
    h = 2166136261
    for ch in f"{base}:{name}".encode():
        h = ((h ^ ch) * 16777619) & 0xFFFFFFFF
    return h & 0x7FFFFFFF


def phase_tables(code_bits: int):
    """cos/sin of the uniform phases 2 pi c / 2^b with exact zeros (the 3/4-bit
    extension; identical to the tables the CUDA library builds)."""
    n = 1 << code_bits
    cos, sin = [], []
    for c in range(n):
        a = 2.0 * math.pi * c / n
        cs, sn = math.cos(a), math.sin(a)
        cos.append(0.0 if abs(cs) < 1e-12 else cs)
        sin.append(0.0 if abs(sn) < 1e-12 else sn)
    return cos, sin
