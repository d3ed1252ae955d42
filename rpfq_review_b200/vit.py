"""ViT / DeiT inference harness whose every linear layer is a packed
complex-phase layer on the B200 path.

Architecture as in the reference models (RPFQ-ViT-main/quant_models/
quant_rpfq_vit.py:131-177 builds timm's VisionTransformer and swaps the
attention qkv / proj, the MLP fc1 / fc2 and the head for the complex-phase
layer; quant_rpfq_deit.py:26 adds the distillation token and head) and as the
reference's own runtime forward restates it
(RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:630-688): patch embed,
cls (+ dist) token, position embedding, pre-norm blocks
LN -> qkv -> softmax attention -> proj (+ residual) -> LN -> fc1 -> exact GELU
-> fc2 (+ residual), final LN, head on the class token.

On the GPU: every quantized linear is one tcgen05 GEMM launch over the
decoded coefficients with bias, GELU (fc1) and the residual add (proj, fc2)
fused into its epilogue; the patch embedding (a dense conv in the reference)
runs through the same GEMM on unfolded patches. LayerNorm (+ activation
quantization) is one kernel per row block; attention is PyTorch SDPA (cuDNN)
or, with ``attention="rpfq"``, the library's tcgen05 short-sequence kernel.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .layers import PackedPhaseLinear
from .packing import layer_seed, pack_linear, random_packed


@dataclass(frozen=True)
class ViTConfig:
    name: str
    dim: int
    depth: int
    heads: int
    mlp: int
    img: int = 224
    patch: int = 16
    classes: int = 1000
    distilled: bool = False
    eps: float = 1e-6  # timm ViT LayerNorm eps

    @property
    def tokens(self) -> int:
        return (self.img // self.patch) ** 2 + (2 if self.distilled else 1)

    def linear_shapes(self):
        """(name, out_features, in_features) of the quantized linears of one block."""
        d = self.dim
        return [("qkv", 3 * d, d), ("proj", d, d), ("fc1", self.mlp, d), ("fc2", d, self.mlp)]

    def gemm_flops_per_image(self) -> int:
        """Algorithmic flops of the complex-phase GEMMs per image: 2 M K N per
        linear, M = tokens (head: one class token per head)."""
        per_block = sum(2 * n * k for _, n, k in self.linear_shapes()) * self.tokens
        head = 2 * self.classes * self.dim * (2 if self.distilled else 1)
        return per_block * self.depth + head


VIT_B16 = ViTConfig("vit_base_patch16_224", dim=768, depth=12, heads=12, mlp=3072)
DEIT_S16 = ViTConfig("deit_small_distilled_patch16_224", dim=384, depth=12, heads=6, mlp=1536, distilled=True)
VIT_L16 = ViTConfig("vit_large_patch16_224", dim=1024, depth=24, heads=16, mlp=4096)
CONFIGS = {c.name: c for c in (VIT_B16, DEIT_S16, VIT_L16)}


def _trunc_normal(shape, std, gen):
    return torch.nn.init.trunc_normal_(torch.empty(shape), std=std, a=-2 * std, b=2 * std, generator=gen)


class PackedViT(nn.Module):
    """Inference ViT / DeiT with packed complex-phase linears.

    ``weights="random_init"``: timm-style random init (trunc-normal std 0.02,
    zero biases) of every float weight, then the exporter's 2-stage axial
    packing of every quantized linear (what "2-bit phase-quantized from random
    init" means for the reference). ``weights="synthetic"``: codes drawn
    uniformly over the 2^b phases with lognormal(0, 0.5) channel scales
    divided by ``sqrt(K)`` so activations stay in fp16 range (needed for the
    3/4-bit sweep, which the exporter cannot produce).
    Each layer's seed derives from its name and ``seed``.
    """

    def __init__(self, cfg: ViTConfig, device, seed: int = 0, act_bits: int = 0, weights: str = "random_init",
                 code_bits: int = 2, prepack: bool = True, vision_quant: dict | None = None,
                 attention: str = "sdpa"):
        super().__init__()
        self.cfg = cfg
        if attention not in ("sdpa", "rpfq"):
            raise ValueError(f"attention must be 'sdpa' or 'rpfq', got {attention!r}")
        # "rpfq": the library's tcgen05 short-sequence attention kernel (head
        # dim 64, <= 256 tokens); "sdpa": PyTorch scaled_dot_product_attention
        self.attention = attention
        # vision_quant: the reference's VisionAwareComplexVisionTransformer
        # (quant_rpfq_vit_vision.py:210-301): every packed linear quantizes its
        # input with the token-saliency quantizer (int8) instead of act_bits
        self.vision_quant = dict(vision_quant) if vision_quant is not None else None
        if self.vision_quant is not None:
            act_bits = 0
        self.act_bits = act_bits
        dev = torch.device(device)
        d = cfg.dim
        g = torch.Generator().manual_seed(layer_seed("embed", seed))
        pdim = 3 * cfg.patch * cfg.patch
        self.register_buffer("patch_w", _trunc_normal((d, pdim), 0.02, g).half().to(dev))
        self.register_buffer("patch_b", torch.zeros(d, dtype=torch.float16, device=dev))
        ntok = 2 if cfg.distilled else 1
        self.register_buffer("cls_tokens", _trunc_normal((1, ntok, d), 0.02, g).half().to(dev))
        self.register_buffer("pos_embed", _trunc_normal((1, cfg.tokens, d), 0.02, g).half().to(dev))

        def make(name, n_out, n_in, activation="none"):
            if weights == "random_init":
                gl = torch.Generator().manual_seed(layer_seed(name, seed))
                w = _trunc_normal((n_out, n_in), 0.02, gl).to(dev)
                layer = pack_linear(w, torch.zeros(n_out, device=dev), stages=2)
            elif weights == "synthetic":
                layer = random_packed(n_out // 2, n_in // 2, seed=layer_seed(name, seed), code_bits=code_bits,
                                      device=dev)
                scale = torch.tensor((n_in ** 0.5) * 2.0, device=dev)
                planes = {}
                for k, (c, gr, gi) in layer.planes.items():
                    planes[k] = (c, (gr.float() * scale).half(), (gi.float() * scale).half())
                layer.planes = planes
            else:
                raise ValueError(f"unknown weights mode {weights!r}")
            return PackedPhaseLinear.from_packed(layer, enable_act_quant=act_bits > 0 or vision_quant is not None,
                                                 act_num_bits=act_bits or 4, activation=activation,
                                                 vision_quant=vision_quant)

        self.blocks = nn.ModuleList()
        for i in range(cfg.depth):
            blk = nn.Module()
            blk.norm1_w = nn.Parameter(torch.ones(d, dtype=torch.float16, device=dev), requires_grad=False)
            blk.norm1_b = nn.Parameter(torch.zeros(d, dtype=torch.float16, device=dev), requires_grad=False)
            blk.norm2_w = nn.Parameter(torch.ones(d, dtype=torch.float16, device=dev), requires_grad=False)
            blk.norm2_b = nn.Parameter(torch.zeros(d, dtype=torch.float16, device=dev), requires_grad=False)
            blk.qkv = make(f"blocks.{i}.attn.qkv", 3 * d, d)
            blk.proj = make(f"blocks.{i}.attn.proj", d, d)
            blk.fc1 = make(f"blocks.{i}.mlp.fc1", cfg.mlp, d, activation="gelu")
            blk.fc2 = make(f"blocks.{i}.mlp.fc2", d, cfg.mlp)
            self.blocks.append(blk)
        self.register_buffer("norm_w", torch.ones(d, dtype=torch.float16, device=dev))
        self.register_buffer("norm_b", torch.zeros(d, dtype=torch.float16, device=dev))
        self.head = make("head", cfg.classes, d)
        self.head_dist = make("head_dist", cfg.classes, d) if cfg.distilled else None
        if prepack:
            for m in self.modules():
                if isinstance(m, PackedPhaseLinear):
                    m.prepack()

    def quantized_linears(self):
        for i, blk in enumerate(self.blocks):
            for n in ("qkv", "proj", "fc1", "fc2"):
                yield f"blocks.{i}.{n}", getattr(blk, n)
        yield "head", self.head
        if self.head_dist is not None:
            yield "head_dist", self.head_dist

    # ------------------------------------------------------------------ forward
    def _token_index(self, B: int, device):
        """Per-batch-size tables and buffers of the forward, kept across calls
        (built without caching while a CUDA graph is captured: the graph's
        memory pool must not back a cached tensor):

        * ``rows`` / ``tok``: int32 over the B x tokens rows of the residual
          stream, the source row of each token (class tokens first, then image
          b's patch embeddings at ntok + b * patches) and its position index;
        * ``cls_rows``: int32 over the B x ntok class-token rows of the stream;
        * ``src``: the fp32 token sources, the class-token rows filled once
          (the patch GEMM writes the rows below them on every call);
        * ``pos``: the position table in fp32.
        Constant per model, so the forward launches no cast or copy kernel
        (each would also cut the programmatic launch chain). Entries live as
        long as the model (a CUDA graph captured at one batch size keeps using
        its entry's buffers while other sizes run); only entries of an older
        class-token or position table are dropped."""
        versions = (self.cls_tokens._version, self.pos_embed._version)
        key = (B, str(device), versions)
        cache = self.__dict__.setdefault("_token_index_cache", {})
        if key in cache:
            return cache[key]
        L, n_p = self.cfg.tokens, (self.cfg.img // self.cfg.patch) ** 2
        ntok = L - n_p
        d = self.cfg.dim
        t = torch.arange(L, dtype=torch.int32, device=device).repeat(B)
        b = torch.arange(B, dtype=torch.int32, device=device).repeat_interleave(L)
        rows = torch.where(t < ntok, t, ntok + b * n_p + (t - ntok)).to(torch.int32)
        cls_rows = (torch.arange(B, dtype=torch.int32, device=device).repeat_interleave(ntok) * L +
                    torch.arange(ntok, dtype=torch.int32, device=device).repeat(B)).to(torch.int32)
        src = torch.empty((ntok + B * n_p, d), dtype=torch.float32, device=device)
        src[:ntok].copy_(self.cls_tokens[0])
        pos = self.pos_embed[0].float().contiguous()
        entry = (rows, t, cls_rows, src, pos)
        if torch.device(device).type != "cuda" or not torch.cuda.is_current_stream_capturing():
            for k in [k for k in cache if k[2] != versions]:
                del cache[k]
            cache[key] = entry
        return entry

    @torch.no_grad()
    def forward(self, images: torch.Tensor) -> torch.Tensor:
        """images ``[B, 3, 224, 224]`` (already normalised; fp16 or fp32) ->
        logits fp32 ``[B, classes]``.

        The residual stream is kept in fp32: LayerNorm reads it and writes the
        fp16 GEMM input (with the activation quantization fused in when
        enabled); proj and fc2 add their output to it in place in the GEMM
        epilogue. GEMM operands are fp16 with fp32 accumulation. With the
        vision-aware quantizer each packed linear quantizes its own
        ``[B, tokens, K]`` input (the saliency split needs the whole image)."""
        cfg = self.cfg
        B = images.shape[0]
        d, H = cfg.dim, cfg.heads
        hd = d // H
        ab = self.act_bits
        pre = self.vision_quant is None  # LayerNorm applied the quantizer
        patches = ops.patch_unfold(images, cfg.patch)
        n_p = patches.shape[1]
        ntok = cfg.tokens - n_p
        L = cfg.tokens
        # token sources: the class (+ distillation) token rows, then the patch
        # embeddings, which the patch GEMM writes straight below them
        rows, tok, cls_rows, src, pos = self._token_index(B, patches.device)
        ops.gemm(patches, self.patch_w, self.patch_b, out=src[ntok:].view(B, n_p, d))
        # residual stream x = [cls (+ dist), patches] + position embedding
        # (reference forward_runtime_path, audit_rpfq_vit_ios_parity.py:638-645),
        # assembled by the first LayerNorm pass: it gathers each token's source
        # row, adds its position row, writes x and normalizes it
        x = torch.empty((B, L, d), dtype=torch.float32, device=patches.device)
        for i, blk in enumerate(self.blocks):
            if i == 0:
                h, _ = ops.layernorm_ex(src, blk.norm1_w, blk.norm1_b, cfg.eps, ab, rows=rows, add=pos,
                                        add_rows=tok, out32=x, out32_prenorm=True)
            else:
                h = ops.layernorm(x, blk.norm1_w, blk.norm1_b, cfg.eps, ab)
            qkv = blk.qkv(h, prequantized=pre)
            if self.attention == "rpfq" and hd == 64 and L <= ops.ATTENTION_MAX_TOKENS:
                a = ops.attention(qkv.view(B, L, 3 * d), H)
            else:
                qkv = qkv.view(B, L, 3, H, hd).permute(2, 0, 3, 1, 4)
                a = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2]).transpose(1, 2).reshape(B, L, d)
            blk.proj(a, residual=x, out=x)
            h = ops.layernorm(x, blk.norm2_w, blk.norm2_b, cfg.eps, ab)
            blk.fc2(blk.fc1(h, prequantized=pre), residual=x, out=x)
        # final norm of the class-token rows only (a row gather, no strided copy)
        cls = ops.layernorm(x, self.norm_w, self.norm_b, cfg.eps, ab, rows=cls_rows,
                            out=torch.empty((B, ntok, d), dtype=torch.float16, device=x.device))
        logits = self.head(cls[:, 0], out_dtype=torch.float32, prequantized=pre)
        if self.head_dist is not None:
            logits = (logits + self.head_dist(cls[:, 1], out_dtype=torch.float32, prequantized=pre)) / 2
        return logits
