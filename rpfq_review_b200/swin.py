"""Swin Transformer inference harness whose every linear layer (attention qkv
/ proj, MLP fc1 / fc2, patch-merging reduction, head) is a packed
complex-phase layer on the B200 path.

The reference builds timm's SwinTransformer and swaps its linears for the
complex-phase layer through ``target_linear``
(RPFQ-ViT-main/quant_models/quant_rpfq_swin.py:64-91). timm is not part of
this build; the architecture is restated from its definition (Liu et al.,
"Swin Transformer", 2021): 4x4 patch embedding + LayerNorm, four stages of
pre-norm blocks with window attention (7x7 windows, a cyclic shift of 3 on
every second block, learned relative position bias), patch merging between
stages (2x2 neighbourhood concatenated in the order (0,0), (1,0), (0,1),
(1,1), LayerNorm, linear 4C -> 2C without bias), final LayerNorm, mean over
tokens, head.

On the GPU the packed linears run the tcgen05 GEMM with bias, GELU (fc1) and
the residual add (fc2) fused. Every LayerNorm (+ activation quantization) is
one pass of the ``rpfq_layernorm_ex_sm100`` kernel, whose row sources carry
the token bookkeeping: the norm1 pass gathers rows into the shifted window
order; the norm2 pass adds the attention branch (window order) back into the
residual stream through the inverse gather, in place, and normalizes the
updated rows; the patch-merging pass gathers the 2x2 neighbourhoods; the
patch-embedding norm writes the fp32 residual stream. Window attention is
the tcgen05 kernel ``rpfq_window_attention_sm100`` (or PyTorch SDPA with the
relative-position bias and shift mask as an additive mask).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .layers import PackedPhaseLinear
from .packing import layer_seed, pack_linear
from .vit import _trunc_normal


@dataclass(frozen=True)
class SwinConfig:
    name: str
    embed: int = 96
    depths: tuple = (2, 2, 6, 2)
    heads: tuple = (3, 6, 12, 24)
    window: int = 7
    patch: int = 4
    mlp_ratio: int = 4
    img: int = 224
    classes: int = 1000
    eps: float = 1e-5  # nn.LayerNorm default, as timm's Swin

    def dims(self):
        return [self.embed * 2 ** i for i in range(len(self.depths))]

    @property
    def tokens(self) -> int:
        """Tokens per image entering the first stage."""
        return (self.img // self.patch) ** 2

    @property
    def dim(self) -> int:
        """Width of the first stage."""
        return self.embed

    def resolutions(self):
        r0 = self.img // self.patch
        return [r0 // 2 ** i for i in range(len(self.depths))]

    def stage_window(self, s: int) -> tuple[int, int]:
        """(window, shift) of stage s: a stage whose resolution fits one window
        uses that window and no shift."""
        r = self.resolutions()[s]
        return (r, 0) if r <= self.window else (self.window, self.window // 2)

    def gemm_flops_per_image(self) -> int:
        """2 M K N summed over the packed linears of one image."""
        f = 0
        dims, res = self.dims(), self.resolutions()
        for s, depth in enumerate(self.depths):
            c, t = dims[s], res[s] ** 2
            f += depth * 2 * t * (3 * c * c + c * c + 2 * self.mlp_ratio * c * c)
            if s + 1 < len(self.depths):
                f += 2 * (res[s + 1] ** 2) * (4 * c) * (2 * c)
        return f + 2 * dims[-1] * self.classes


SWIN_T = SwinConfig("swin_tiny_patch4_window7_224")
SWIN_CONFIGS = {SWIN_T.name: SWIN_T}


def relative_position_index(ws: int) -> torch.Tensor:
    """[ws*ws, ws*ws] index into the (2 ws - 1)^2 bias table: (dy + ws - 1) *
    (2 ws - 1) + (dx + ws - 1) for the offset (dy, dx) between two window
    positions."""
    ys, xs = torch.meshgrid(torch.arange(ws), torch.arange(ws), indexing="ij")
    coords = torch.stack([ys.flatten(), xs.flatten()])  # [2, ws*ws]
    rel = coords[:, :, None] - coords[:, None, :]
    return (rel[0] + ws - 1) * (2 * ws - 1) + (rel[1] + ws - 1)


def shift_mask(res: int, ws: int, shift: int) -> torch.Tensor:
    """[num_windows, ws*ws, ws*ws] additive mask of a cyclically shifted
    window partition: 0 between positions of the same image region, -100
    across regions (the wrapped-around strips)."""
    label = torch.zeros(res, res)
    cuts = (slice(0, -ws), slice(-ws, -shift), slice(-shift, None))
    n = 0
    for hs in cuts:
        for wsl in cuts:
            label[hs, wsl] = n
            n += 1
    win = label.view(res // ws, ws, res // ws, ws).permute(0, 2, 1, 3).reshape(-1, ws * ws)
    diff = win[:, :, None] - win[:, None, :]
    return torch.where(diff == 0, 0.0, -100.0)


def window_order(res: int, ws: int, shift: int) -> torch.Tensor:
    """[res*res] source token of each position of the window-partitioned
    (cyclically shifted by -shift) layout: token t of window w comes from
    image position ((wy ws + i + shift) mod res, (wx ws + j + shift) mod res).
    The same permutation scatters the windows back (and undoes the shift)."""
    nw = res // ws
    wy, wx, i, j = torch.meshgrid(torch.arange(nw), torch.arange(nw), torch.arange(ws), torch.arange(ws),
                                  indexing="ij")
    y = (wy * ws + i + shift) % res
    x = (wx * ws + j + shift) % res
    return (y * res + x).reshape(-1)


def window_partition(x: torch.Tensor, ws: int) -> torch.Tensor:
    """[B, R, R, C] -> [B * (R/ws)^2, ws*ws, C] (windows in row-major order)."""
    b, r, _, c = x.shape
    x = x.view(b, r // ws, ws, r // ws, ws, c).permute(0, 1, 3, 2, 4, 5)
    return x.reshape(-1, ws * ws, c)


def window_reverse(w: torch.Tensor, ws: int, r: int) -> torch.Tensor:
    """Inverse of :func:`window_partition`."""
    c = w.shape[-1]
    b = w.shape[0] // ((r // ws) ** 2)
    x = w.view(b, r // ws, r // ws, ws, ws, c).permute(0, 1, 3, 2, 4, 5)
    return x.reshape(b, r, r, c)


class PackedSwin(nn.Module):
    """Inference Swin with packed complex-phase linears (random-init weights
    packed by the exporter's algorithm, as for :class:`PackedViT`).
    ``attention="rpfq"`` runs the library's tcgen05 window-attention kernel
    (7x7 windows, head dim 32), ``"sdpa"`` PyTorch SDPA with the bias as an
    additive mask."""

    def __init__(self, cfg: SwinConfig, device, seed: int = 0, act_bits: int = 0, prepack: bool = True,
                 attention: str = "rpfq"):
        super().__init__()
        if attention not in ("sdpa", "rpfq"):
            raise ValueError(f"attention must be 'sdpa' or 'rpfq', got {attention!r}")
        self.attention = attention
        self.cfg = cfg
        self.act_bits = act_bits
        dev = torch.device(device)
        g = torch.Generator().manual_seed(layer_seed("patch_embed", seed))
        pdim = 3 * cfg.patch * cfg.patch
        c0 = cfg.embed
        self.register_buffer("patch_w", _trunc_normal((c0, pdim), 0.02, g).half().to(dev))
        self.register_buffer("patch_b", torch.zeros(c0, dtype=torch.float16, device=dev))
        self.register_buffer("patch_norm_w", torch.ones(c0, dtype=torch.float16, device=dev))
        self.register_buffer("patch_norm_b", torch.zeros(c0, dtype=torch.float16, device=dev))

        def make(name, n_out, n_in, activation="none"):
            gl = torch.Generator().manual_seed(layer_seed(name, seed))
            w = _trunc_normal((n_out, n_in), 0.02, gl).to(dev)
            layer = pack_linear(w, torch.zeros(n_out, device=dev), stages=2)
            return PackedPhaseLinear.from_packed(layer, enable_act_quant=act_bits > 0, act_num_bits=act_bits or 4,
                                                 activation=activation)

        dims = cfg.dims()
        self.stages = nn.ModuleList()
        for s, depth in enumerate(cfg.depths):
            c, nh = dims[s], cfg.heads[s]
            ws, _ = cfg.stage_window(s)
            stage = nn.Module()
            stage.blocks = nn.ModuleList()
            for i in range(depth):
                blk = nn.Module()
                pre = f"layers.{s}.blocks.{i}"
                for n in ("norm1", "norm2"):
                    blk.register_buffer(f"{n}_w", torch.ones(c, dtype=torch.float16, device=dev))
                    blk.register_buffer(f"{n}_b", torch.zeros(c, dtype=torch.float16, device=dev))
                gb = torch.Generator().manual_seed(layer_seed(f"{pre}.attn.relative_position_bias_table", seed))
                blk.register_buffer("rel_table", _trunc_normal(((2 * ws - 1) ** 2, nh), 0.02, gb).to(dev))
                blk.qkv = make(f"{pre}.attn.qkv", 3 * c, c)
                blk.proj = make(f"{pre}.attn.proj", c, c)
                blk.fc1 = make(f"{pre}.mlp.fc1", cfg.mlp_ratio * c, c, activation="gelu")
                blk.fc2 = make(f"{pre}.mlp.fc2", c, cfg.mlp_ratio * c)
                stage.blocks.append(blk)
            stage.register_buffer("rel_index", relative_position_index(ws).to(dev))
            if s + 1 < len(cfg.depths):
                stage.register_buffer("merge_norm_w", torch.ones(4 * c, dtype=torch.float16, device=dev))
                stage.register_buffer("merge_norm_b", torch.zeros(4 * c, dtype=torch.float16, device=dev))
                stage.reduction = make(f"layers.{s + 1}.downsample.reduction", 2 * c, 4 * c)
            self.stages.append(stage)
        self.register_buffer("norm_w", torch.ones(dims[-1], dtype=torch.float16, device=dev))
        self.register_buffer("norm_b", torch.zeros(dims[-1], dtype=torch.float16, device=dev))
        self.head = make("head.fc", cfg.classes, dims[-1])
        self._masks: dict = {}
        self._orders: dict = {}
        if prepack:
            for m in self.modules():
                if isinstance(m, PackedPhaseLinear):
                    m.prepack()

    def quantized_linears(self):
        for s, stage in enumerate(self.stages):
            for i, blk in enumerate(stage.blocks):
                for n in ("qkv", "proj", "fc1", "fc2"):
                    yield f"layers.{s}.blocks.{i}.{n}", getattr(blk, n)
            if hasattr(stage, "reduction"):
                yield f"layers.{s + 1}.downsample.reduction", stage.reduction
        yield "head", self.head

    def attn_mask(self, s: int, i: int, batch: int) -> torch.Tensor:
        """Additive attention mask [B * nW, heads, L, L] of block i of stage s:
        relative position bias, plus the shift mask on shifted blocks.
        Cached per (stage, block, batch)."""
        key = (s, i, batch)
        m = self._masks.get(key)
        if m is None:
            cfg = self.cfg
            stage = self.stages[s]
            blk = stage.blocks[i]
            ws, shift = cfg.stage_window(s)
            r = cfg.resolutions()[s]
            nw = (r // ws) ** 2
            L = ws * ws
            bias = blk.rel_table[stage.rel_index.reshape(-1)].reshape(L, L, -1).permute(2, 0, 1)  # [nh, L, L]
            m = bias[None].expand(nw, -1, -1, -1)
            if shift and i % 2 == 1:
                m = m + shift_mask(r, ws, shift).to(m.device)[:, None]
            m = m[None].expand(batch, -1, -1, -1, -1).reshape(batch * nw, -1, L, L).to(torch.float16).contiguous()
            self._masks[key] = m
        return m

    def window_bias(self, s: int, i: int) -> torch.Tensor:
        """bias_mask of block i of stage s for the window attention kernel
        (``ops.window_bias_layout`` of the relative position bias + shift
        mask); bm_windows = 1 on unshifted blocks, the windows per image on
        shifted ones. Cached."""
        key = ("wb", s, i)
        m = self._masks.get(key)
        if m is None:
            cfg = self.cfg
            stage = self.stages[s]
            blk = stage.blocks[i]
            ws, shift = cfg.stage_window(s)
            r = cfg.resolutions()[s]
            L = ws * ws
            bias = blk.rel_table.float()[stage.rel_index.reshape(-1)].reshape(L, L, -1).permute(2, 0, 1)  # [nh, L, L]
            m = bias[None]
            if shift and i % 2 == 1:
                m = m + shift_mask(r, ws, shift).to(m.device)[:, None]
            m = ops.window_bias_layout(m)
            self._masks[key] = m
        return m

    def orders(self, s: int, shift: int, batch: int):
        """(perm [R*R] int64, rows [B*R*R] int32, inverse [B*R*R] int32) of
        stage s: the window order of the tokens, its per-image row gather for
        the LayerNorm kernel (window-order row -> natural row) and the inverse
        gather (natural row -> window-order row) that brings the attention
        branch back into the residual stream."""
        key = (s, shift, batch)
        o = self._orders.get(key)
        if o is None:
            cfg = self.cfg
            r = cfg.resolutions()[s]
            ws, _ = cfg.stage_window(s)
            dev = self.patch_w.device
            perm = window_order(r, ws, shift).to(dev)
            base = torch.arange(batch, device=dev)[:, None] * (r * r)
            rows = (base + perm[None]).reshape(-1).to(torch.int32)
            inverse = (base + torch.argsort(perm)[None]).reshape(-1).to(torch.int32)
            o = (perm, rows, inverse)
            self._orders[key] = o
        return o

    @torch.no_grad()
    def forward(self, images: torch.Tensor) -> torch.Tensor:
        """images ``[B, 3, 224, 224]`` -> logits fp32 ``[B, classes]``; the
        residual stream is fp32, GEMM operands fp16 with fp32 accumulation."""
        cfg = self.cfg
        ab = self.act_bits
        B = images.shape[0]
        dims, res = cfg.dims(), cfg.resolutions()
        emb = ops.gemm(ops.patch_unfold(images, cfg.patch), self.patch_w, self.patch_b, out_dtype=torch.float32)
        # patch-embedding LayerNorm in place: the residual stream starts as its fp32 output
        ops.layernorm_ex(emb, self.patch_norm_w, self.patch_norm_b, cfg.eps, fp16_out=False, out32=emb)
        x = emb
        for s, stage in enumerate(self.stages):
            c, nh, r = dims[s], cfg.heads[s], res[s]
            hd = c // nh
            ws, shift = cfg.stage_window(s)
            for i, blk in enumerate(stage.blocks):
                sh = shift if i % 2 == 1 else 0
                _, rows, inverse = self.orders(s, sh, B)
                # LayerNorm writes the tokens already shifted and window-partitioned
                win = ops.layernorm(x, blk.norm1_w, blk.norm1_b, cfg.eps, ab, rows=rows).view(-1, ws * ws, c)
                qkv = blk.qkv(win, prequantized=True)
                if self.attention == "rpfq" and ws * ws == ops.WINDOW_TOKENS and hd == ops.WINDOW_HEAD_DIM:
                    a = ops.window_attention(qkv.view(-1, 3 * c), nh, self.window_bias(s, i)).view(-1, ws * ws, c)
                else:
                    qkv = qkv.view(win.shape[0], ws * ws, 3, nh, hd).permute(2, 0, 3, 1, 4)
                    a = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], attn_mask=self.attn_mask(s, i, B))
                    a = a.transpose(1, 2).reshape(win.shape[0], ws * ws, c)
                o = blk.proj(a, out_dtype=torch.float32)
                # un-partition, un-shift and add to the residual stream (in place) in
                # the LayerNorm pass that also produces the MLP input
                h, _ = ops.layernorm_ex(x, blk.norm2_w, blk.norm2_b, cfg.eps, ab, add=o.view(-1, c),
                                        add_rows=inverse, out32=x, out32_prenorm=True)
                blk.fc2(blk.fc1(h.view(B, r * r, c), prequantized=True), residual=x, out=x)
            if hasattr(stage, "reduction"):
                # patch merging: the 2x2 neighbourhood concatenation rides on the LayerNorm's row gather
                h, _ = ops.layernorm_ex(x, stage.merge_norm_w, stage.merge_norm_b, cfg.eps, ab, merge_side=r)
                x = stage.reduction(h.view(B, (r // 2) ** 2, 4 * c), out_dtype=torch.float32, prequantized=True)
        h = ops.layernorm(x, self.norm_w, self.norm_b, cfg.eps)
        pooled = h.float().mean(dim=1).to(torch.float16)
        return self.head(pooled, out_dtype=torch.float32)
