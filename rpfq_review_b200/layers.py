"""Drop-in modules for the complex-phase linear layer.

* :class:`QATLinearComplexPhase` keeps the reference module's constructor and
  ``forward(x) -> y`` contract (RPFQ-ViT-main/quant_models/quant_i.py:475-554),
  so the model adapters' ``target_linear`` hook (quant_rpfq_vit.py:75-103,
  quant_rpfq_deit.py:65-92, quant_rpfq_swin.py:64-91) can instantiate it
  unchanged. Its float weight is packed with the exporter's algorithm (the
  deployment quantization) and cached until the weight changes.
* :class:`PackedPhaseLinear` holds the exporter's packed tensors as buffers
  under the exporter's keys (``u_s0.codes``, ``u_s0.gamma_real``, …,
  ``bias``), loads them from an exported state dict, and runs the B200 path.

Both run only on CUDA tensors through ``librpfq_b200.so``.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import ops
from .packing import AXIAL_STAGES, BLOCK_SIZE, SUPPORTED_QUANT_METHODS, PackedLayer, pack_linear, round_up


class PhasePlane(nn.Module):
    """Buffers of one residual stage: ``codes``, ``gamma_real``, ``gamma_imag``."""

    def __init__(self, n_cp: int, k_cp: int, code_bits: int = 2, device=None):
        super().__init__()
        self.register_buffer("codes", torch.zeros((n_cp, k_cp * code_bits // 8), dtype=torch.uint8, device=device))
        blocks = k_cp // BLOCK_SIZE
        self.register_buffer("gamma_real", torch.ones((n_cp, blocks), dtype=torch.float16, device=device))
        self.register_buffer("gamma_imag", torch.ones((n_cp, blocks), dtype=torch.float16, device=device))


class PackedPhaseLinear(nn.Module):
    """Inference layer over the packed phase-code layout.

    ``forward(x[..., in_features]) -> y[..., out_features]`` computes
    ``act(U x + W conj(x) + bias)`` (+ ``residual``) with optional activation
    quantization of x (``act_num_bits``). With ``cache_dense=True`` (the
    default; the reference runtime's fused fp16 cache) the dense fp16
    coefficients are decoded once on the GPU and kept as a non-persistent
    buffer. With ``cache_dense=False`` only the packed planes stay resident:
    calls of at most ``ops.FUSED_DECODE_MAX_ROWS`` rows decode the codes inside
    the GEMM, larger calls decode into a temporary dense matrix first.
    """

    def __init__(self, in_features: int, out_features: int, stages: int = 2, code_bits: int = 2,
                 enable_act_quant: bool = False, act_num_bits: int = 4, activation: str = "none",
                 rounding: str = "rne", cache_dense: bool = True, vision_quant: dict | None = None, device=None):
        super().__init__()
        if in_features % 2 or out_features % 2:
            raise ValueError("Complex-phase QAT requires even in/out features.")
        self.in_features, self.out_features = in_features, out_features
        self.n_c, self.k_c = out_features // 2, in_features // 2
        self.stages, self.code_bits = stages, code_bits
        self.act_bits = act_num_bits if enable_act_quant else 0
        self.activation = activation
        self.rounding = rounding
        self.cache_dense = cache_dense
        # vision-aware activation quantizer (quant_rpfq_vit_vision.py:26-171) in
        # place of ActivationQuantSTE: {salient_token_ratio, background_clip_ratio,
        # energy_score_weight, protect_cls_token}
        self.vision_quant = dict(vision_quant) if (vision_quant is not None and enable_act_quant) else None
        n_cp, k_cp = round_up(self.n_c, BLOCK_SIZE), round_up(self.k_c, BLOCK_SIZE)
        for tag in ("u", "w"):
            for s in range(stages):
                self.add_module(f"{tag}_s{s}", PhasePlane(n_cp, k_cp, code_bits, device))
        self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float16, device=device))
        self.register_buffer("dense", None, persistent=False)
        self._bias32 = None  # (version, fp32 copy of bias) for the epilogue

    # -- construction ---------------------------------------------------------
    @classmethod
    def from_packed(cls, layer: PackedLayer, **kw) -> "PackedPhaseLinear":
        dev = layer.planes["u_s0"][0].device
        m = cls(2 * layer.k_c, 2 * layer.n_c, layer.stages, layer.code_bits, device=dev, **kw)
        for name, (c, gr, gi) in layer.planes.items():
            plane = getattr(m, name)
            plane.codes.copy_(c)
            plane.gamma_real.copy_(gr)
            plane.gamma_imag.copy_(gi)
        if layer.bias is not None:
            m.bias.copy_(layer.bias)
        return m

    @classmethod
    def from_state_dict(cls, sd: dict, prefix: str, in_features: int, out_features: int, **kw):
        """Load an exporter-layout layer (keys ``{prefix}u_s0.codes`` …)."""
        return cls.from_packed(PackedLayer.from_state_dict(sd, prefix, in_features, out_features), **kw)

    @classmethod
    def from_linear(cls, linear: nn.Linear, stages: int = 2, **kw) -> "PackedPhaseLinear":
        """Pack a float ``nn.Linear`` with the exporter's algorithm."""
        return cls.from_packed(pack_linear(linear.weight, linear.bias, stages), **kw)

    def packed(self) -> PackedLayer:
        planes = {}
        for tag in ("u", "w"):
            for s in range(self.stages):
                p = getattr(self, f"{tag}_s{s}")
                planes[f"{tag}_s{s}"] = (p.codes, p.gamma_real, p.gamma_imag)
        return PackedLayer(self.n_c, self.k_c, self.stages, self.code_bits, planes, self.bias)

    # -- execution ------------------------------------------------------------
    @property
    def _aligned(self) -> bool:
        # The TMA path needs 16-byte row strides: real K and N multiples of 8.
        return self.in_features % 8 == 0 and self.out_features % 8 == 0

    def _bias_f32(self) -> torch.Tensor:
        """The fp16 bias widened to fp32 once (exact); refreshed when the
        bias tensor changes."""
        key = (self.bias.data_ptr(), self.bias._version, self.bias.device)
        if self._bias32 is None or self._bias32[0] != key:
            self._bias32 = (key, self.bias.float())
        return self._bias32[1]

    @property
    def _fused_decode_ok(self) -> bool:
        # the fused decode path stores 8 complex columns per vector
        return self.code_bits == 2 and self.n_c % 8 == 0 and self.k_c % 8 == 0

    def _decode_dense(self) -> torch.Tensor:
        dense = ops.prepack(self.packed(), self.rounding)
        if not self._aligned:
            n8, k8 = round_up(self.out_features, 8), round_up(self.in_features, 8)
            padded = torch.zeros((n8, k8), dtype=torch.float16, device=dense.device)
            padded[: self.out_features, : self.in_features] = dense
            dense = padded
        return dense

    def prepack(self) -> torch.Tensor:
        """Decode the packed planes once (K1). Layers whose real dims are not
        multiples of 8 keep a zero-padded copy ``[N8, K8]`` for the GEMM."""
        self.dense = self._decode_dense()
        return self.dense

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None, prequantized: bool = False) -> torch.Tensor:
        """``x[..., in_features]`` -> ``y[..., out_features]``.

        fp16 and fp32 inputs are supported; the output has the input's dtype
        unless ``out`` / ``out_dtype`` say otherwise (fp16 or fp32, written by
        the GEMM epilogue directly). ``residual`` (fp16 or fp32) is added in
        the epilogue and may be ``out`` itself. ``prequantized=True`` skips the
        activation quantization (already applied by the producer, e.g. the
        fused LayerNorm kernel)."""
        if out_dtype is None:
            out_dtype = out.dtype if out is not None else (x.dtype if x.dtype in (torch.float16, torch.float32)
                                                           else torch.float16)
        x16 = x if x.dtype == torch.float16 else x.to(torch.float16)
        act_bits = 0 if prequantized else self.act_bits
        if self.vision_quant is not None and not prequantized:
            # token saliency needs the [B, T, K] structure of the input
            x16 = ops.vision_act_quant(x16, **self.vision_quant)
            act_bits = 0
        rows = x.numel() // self.in_features if self.in_features else 0
        if not self.cache_dense and self._fused_decode_ok and rows <= ops.FUSED_DECODE_MAX_ROWS:
            return ops.wide_linear(x16, self.packed(), None, act_bits, self.activation, residual, out=out,
                                   out_dtype=out_dtype, bias=self._bias_f32())
        if self.cache_dense:
            if self.dense is None or self.dense.device != x.device:
                self.prepack()
            dense = self.dense
        else:
            dense = self._decode_dense()
        if self._aligned:
            return ops.wide_linear(x16, self.packed(), dense, act_bits, self.activation, residual, out=out,
                                   out_dtype=out_dtype, bias=self._bias_f32())
        y = self._forward_padded(x16, dense, residual, act_bits, out_dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def _forward_padded(self, x16: torch.Tensor, dense: torch.Tensor, residual: torch.Tensor | None,
                        act_bits: int, out_dtype: torch.dtype) -> torch.Tensor:
        """Layers whose K or N is not a multiple of 8: run the GEMM on
        zero-padded copies (x, bias, residual) and crop the output."""
        K, N = self.in_features, self.out_features
        n8, k8 = dense.shape
        lead = x16.shape[:-1]
        x2 = x16.reshape(-1, K)
        if act_bits:
            x2 = ops.act_quant(x2.contiguous(), act_bits)
        xp = torch.zeros((x2.shape[0], k8), dtype=torch.float16, device=x16.device)
        xp[:, :K] = x2
        bias = torch.zeros(n8, dtype=torch.float16, device=x16.device)
        bias[:N] = self.bias
        rp = None
        if residual is not None:
            rp = torch.zeros((x2.shape[0], n8), dtype=residual.dtype, device=x16.device)
            rp[:, :N] = residual.reshape(-1, N)
        y = ops.gemm(xp, dense, bias, rp, self.activation, out_dtype=out_dtype)
        return y[:, :N].contiguous().reshape(*lead, N)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, stages={self.stages}, "
                f"code_bits={self.code_bits}, act_bits={self.act_bits}, activation={self.activation}"
                + (f", vision_quant={self.vision_quant}" if self.vision_quant else ""))


class QATLinearComplexPhase(nn.Linear):
    """Drop-in for the reference ``QATLinearComplexPhase`` (quant_i.py:475-554).

    Same constructor and forward contract. The weight is quantized with the
    exporter's axial residual algorithm into the packed layout (what the
    deployed model runs) and the product runs on the B200 kernels; the packed
    form is rebuilt whenever the weight or bias changes.

    Error behaviour follows the reference: odd in/out features and unknown
    method names raise ``ValueError``. Methods whose weights the packed axial
    layout cannot represent (``complex_phase_new_v2``, ``complex_phase_next_v1``,
    different stage counts for U and W, ``enable_rotation=True``) raise
    ``NotImplementedError``: the reference exporter has no layout for them
    either (export_rpfq_vit_to_mlx.py:463-468 offers v1 and v2 only).
    """

    def __init__(self, quant_method_u: str = "complex_phase_v1", quant_method_w: str = "complex_phase_v1",
                 enable_act_quant: bool = True, act_num_bits: int = 4, enable_rotation: bool = False,
                 quant_group_size: int = 32, *args, **kwargs):
        super().__init__(*args, **kwargs)
        if self.in_features % 2 != 0 or self.out_features % 2 != 0:
            raise ValueError("Complex-phase QAT requires even in/out features.")
        for m in (quant_method_u, quant_method_w):
            if m not in SUPPORTED_QUANT_METHODS:
                raise ValueError(f"Unsupported quantization method: {m}")
            if m not in AXIAL_STAGES:
                raise NotImplementedError(f"{m} has no packed phase-code layout; use complex_phase_v1..v4")
        if AXIAL_STAGES[quant_method_u] != AXIAL_STAGES[quant_method_w]:
            raise NotImplementedError("the packed layout stores the same number of stages for U and W")
        if enable_rotation:
            raise NotImplementedError("the packed phase-code layout has no rotation; use enable_rotation=False")
        self.quant_method_u, self.quant_method_w = quant_method_u, quant_method_w
        self.stages = AXIAL_STAGES[quant_method_u]
        self.enable_act_quant = enable_act_quant
        self.act_num_bits = act_num_bits
        self.enable_rotation = enable_rotation
        self.quant_group_size = quant_group_size
        self._cache_key = None
        self._packed: PackedPhaseLinear | None = None

    def _key(self):
        b = self.bias
        return (self.weight.device, self.weight.data_ptr(), self.weight._version,
                None if b is None else (b.data_ptr(), b._version))

    def packed_module(self) -> PackedPhaseLinear:
        key = self._key()
        if self._packed is None or key != self._cache_key:
            with torch.no_grad():
                layer = pack_linear(self.weight, self.bias, self.stages)
            self._packed = PackedPhaseLinear.from_packed(layer, enable_act_quant=self.enable_act_quant,
                                                         act_num_bits=self.act_num_bits,
                                                         vision_quant=self._vision_quant())
            self._packed.prepack()
            self._cache_key = key
        return self._packed

    def _vision_quant(self) -> dict | None:
        return None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("QATLinearComplexPhase (B200) runs on CUDA tensors only")
        return self.packed_module()(x)


class VisionAwareQATLinearComplexPhase(QATLinearComplexPhase):
    """Drop-in for the reference ``VisionAwareQATLinearComplexPhase``
    (quant_rpfq_vit_vision.py:174-207): the complex-phase layer whose
    activation quantizer is the token-saliency one
    (``VisionAwareActivationQuantizer``, :26-171) — salient patch tokens (and
    CLS) keep per-token int8 scales, the rest share a clipped per-image scale.
    Inputs ``[B, 1 + g*g, K]`` get the saliency split, other shapes per-token
    int8 scales, as in the reference. Same constructor; ``enable_rotation``
    must be False (see :class:`QATLinearComplexPhase`)."""

    def __init__(self, quant_method_u: str = "complex_phase_v1", quant_method_w: str = "complex_phase_v1",
                 enable_act_quant: bool = True, act_num_bits: int = 4, enable_rotation: bool = False,
                 quant_group_size: int = 32, salient_token_ratio: float = 0.25, background_clip_ratio: float = 0.75,
                 energy_score_weight: float = 0.5, protect_cls_token: bool = True, *args, **kwargs):
        super().__init__(quant_method_u, quant_method_w, enable_act_quant, act_num_bits, enable_rotation,
                         quant_group_size, *args, **kwargs)
        if not 0.0 <= salient_token_ratio <= 1.0:
            raise ValueError("salient_token_ratio must be in [0, 1].")
        if background_clip_ratio <= 0.0:
            raise ValueError("background_clip_ratio must be > 0.")
        if not 0.0 <= energy_score_weight <= 1.0:
            raise ValueError("energy_score_weight must be in [0, 1].")
        self.salient_token_ratio = salient_token_ratio
        self.background_clip_ratio = background_clip_ratio
        self.energy_score_weight = energy_score_weight
        self.protect_cls_token = protect_cls_token

    def _vision_quant(self) -> dict | None:
        if not self.enable_act_quant:
            return None
        return dict(salient_token_ratio=self.salient_token_ratio, background_clip_ratio=self.background_clip_ratio,
                    energy_score_weight=self.energy_score_weight, protect_cls_token=self.protect_cls_token)
