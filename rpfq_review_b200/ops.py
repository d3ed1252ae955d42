"""PyTorch entry points over the C ABI (``include/rpfq_b200.h``).

Functional wrappers (:func:`prepack`, :func:`gemm`, :func:`act_quant`,
:func:`wide_linear`) and the ``torch.ops.rpfq`` operators, registered with
``torch.library`` in the same way the reference registers its GPU op
(``Library("quant", "DEF")`` + ``define`` + ``impl``,
RPFQ-ViT-main/quant_models/kernel.py:599-605). Every op has a CUDA
implementation only: calling one on CPU tensors fails in the dispatcher, and
a missing library raises — there is no fallback path.
"""

from __future__ import annotations

import ctypes
import os
import math

import torch

from . import _lib
from .packing import PackedLayer

_ACT = {"none": _lib.ACT_NONE, "gelu": _lib.ACT_GELU, None: _lib.ACT_NONE,
        _lib.ACT_NONE: _lib.ACT_NONE, _lib.ACT_GELU: _lib.ACT_GELU}
_ROUND = {"rne": _lib.ROUND_NEAREST_EVEN, "ties_away": _lib.ROUND_TIES_AWAY}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class LaunchTimer:
    """Optional instrumentation: a count of every kernel this library launches
    and, with ``events=True``, CUDA events around every GEMM launch. Events
    are created with ``external=True`` so that they become event-record nodes
    when the launches are captured into a CUDA graph (timings are then those
    of the last replay). Event nodes sit between the kernel nodes and so cut
    the programmatic (PDL) chaining of consecutive launches: time a graph
    captured with ``events=False`` and read GEMM times from a separate one."""

    def __init__(self, events: bool = True):
        self.gemm_events: list[tuple[torch.cuda.Event, torch.cuda.Event, int]] = []
        self.launches = 0
        self.events = events

    def gemm_ms_and_flops(self) -> tuple[float, int]:
        ms = sum(s.elapsed_time(e) for s, e, _ in self.gemm_events)
        return ms, sum(f for _, _, f in self.gemm_events)


_timer: LaunchTimer | None = None


def set_launch_timer(timer: LaunchTimer | None) -> None:
    global _timer
    _timer = timer


def _count_launch(n: int = 1) -> None:
    if _timer is not None:
        _timer.launches += n


# Largest row count of the fused decode path (``dense=None``); the C ABI
# rejects more.
FUSED_DECODE_MAX_ROWS = 256


def _p(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


# Split-K for small-M GEMMs: 0 = automatic, 1 = never, 2..8 = forced (the
# RPFQ_SPLIT_K environment variable sets the default of every call).
SPLIT_K = int(os.environ.get("RPFQ_SPLIT_K", "0"))

# One split-K workspace per (device, stream): calls on one stream run in
# order, so they can share it; calls on different streams may overlap.
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, split_k: int) -> tuple[int | None, int]:
    if split_k == 1:
        return None, 0
    key = (device.index if device.index is not None else torch.cuda.current_device(), _stream(device))
    ws = _workspaces.get(key)
    if ws is None:
        with torch.cuda.device(device):
            nbytes = int(_lib.lib().rpfq_gemm_workspace_bytes(0, 0, 0))
        # zeroed: the stream-K flag words at its end start at zero (the library
        # leaves them zero after every call)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws.data_ptr(), ws.numel()


def _require(t: torch.Tensor, name: str, dtype=torch.float16):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the packed phase-linear path has no CPU implementation)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


def _rows(x: torch.Tensor, k: int, name: str):
    """View ``x[..., k]`` as a 2-D row-major matrix with unit column stride."""
    if x.shape[-1] != k:
        raise ValueError(f"{name}: last dim {x.shape[-1]} != {k}")
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    ld = x2.stride(0) if x2.shape[0] > 1 else k
    return x2, ld


def layer_struct(layer: PackedLayer) -> _lib.RpfqPackedLinear:
    s = _lib.RpfqPackedLinear()
    s.n_c, s.k_c = layer.n_c, layer.k_c
    s.n_cp, s.k_cp = layer.n_cp, layer.k_cp
    s.stages, s.code_bits = layer.stages, layer.code_bits
    for i in range(layer.stages):
        for tag, arr in (("u", s.u), ("w", s.w)):
            c, gr, gi = layer.planes[f"{tag}_s{i}"]
            arr[i].codes, arr[i].gamma_real, arr[i].gamma_imag = c.data_ptr(), gr.data_ptr(), gi.data_ptr()
    return s


def prepack(layer: PackedLayer, rounding: str = "rne") -> torch.Tensor:
    """K1: packed planes -> dense fp16 ``[2 n_c, 2 k_c]`` = ``[[rr, ir], [ri, ii]]``."""
    c0 = layer.planes["u_s0"][0]
    _require(c0, "codes", torch.uint8)
    dev = c0.device
    out = torch.empty((2 * layer.n_c, 2 * layer.k_c), dtype=torch.float16, device=dev)
    s = layer_struct(layer)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().rpfq_prepack_sm100(ctypes.byref(s), out.data_ptr(), _ROUND[rounding], _stream(dev)),
                   "rpfq_prepack_sm100")
    return out


ATTENTION_MAX_TOKENS = 256


def attention(qkv: torch.Tensor, heads: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Self-attention of the qkv GEMM output ``[B, L, 3 d]`` (fp16, head dim
    64, L <= 256) through ``rpfq_attention_sm100`` -> ``[B, L, d]`` fp16:
    softmax(q k^T / 8) v per head, heads concatenated."""
    _require(qkv, "qkv")
    if qkv.dim() != 3 or qkv.shape[-1] != 3 * 64 * heads:
        raise ValueError(f"qkv must be [B, L, 3 * heads * 64], got {tuple(qkv.shape)} for {heads} heads")
    if not qkv.is_contiguous():
        qkv = qkv.contiguous()
    B, L, _ = qkv.shape
    d = 64 * heads
    if out is None:
        out = torch.empty((B, L, d), dtype=torch.float16, device=qkv.device)
    o2, ldo = _rows(out, d, "out")
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.lib().rpfq_attention_sm100(qkv.data_ptr(), B, L, heads, 64, o2.data_ptr(), ldo,
                                                   _stream(qkv.device)), "rpfq_attention_sm100")
    if B:
        _count_launch(1)
    return out


WINDOW_TOKENS = 49  # 7 x 7 Swin windows
WINDOW_HEAD_DIM = 32


def window_bias_layout(bias: torch.Tensor) -> torch.Tensor:
    """``[bm_windows, heads, 49, 49]`` additive attention bias (relative
    position bias + shift mask, natural units) -> the float32
    ``[bm_windows, heads, 16, 49, 4]`` operand of :func:`window_attention`
    (scaled by log2(e), -inf in the padding keys)."""
    n, h, L, L2 = bias.shape
    if L != WINDOW_TOKENS or L2 != WINDOW_TOKENS:
        raise ValueError("window_bias_layout: expects [bm_windows, heads, 49, 49]")
    full = torch.full((n, h, L, 64), float("-inf"), dtype=torch.float32, device=bias.device)
    full[..., :L] = bias.float() * 1.4426950408889634
    return full.view(n, h, L, 16, 4).permute(0, 1, 3, 2, 4).contiguous()


def window_attention(qkv: torch.Tensor, heads: int, bias_mask: torch.Tensor,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Swin window attention (``rpfq_window_attention_sm100``): ``qkv`` is the
    qkv GEMM output in window order, fp16 ``[windows * 49, 3 * 32 * heads]``;
    ``bias_mask`` fp32 ``[bm_windows, heads, 16, 49, 4]`` holds log2(e) times
    the relative position bias (+ shift mask) of query row i and key column j
    at ``[..., j // 4, i, j % 4]``, -inf in key columns 49..63 (window w uses
    entry ``w % bm_windows``; :func:`window_bias_layout` builds it from
    ``[bm_windows, heads, 49, 49]``). Returns fp16 ``[windows * 49, 32 * heads]``
    (or writes ``out``)."""
    _require(qkv, "qkv")
    if not bias_mask.is_cuda or bias_mask.dtype != torch.float32 or not bias_mask.is_contiguous():
        raise ValueError("window_attention: bias_mask must be a contiguous float32 CUDA tensor")
    d = WINDOW_HEAD_DIM * heads
    q2, ldq = _rows(qkv, 3 * d, "qkv")
    if ldq != 3 * d:
        raise ValueError("window_attention: qkv rows must be contiguous")
    rows = q2.shape[0]
    if rows % WINDOW_TOKENS:
        raise ValueError(f"window_attention: {rows} rows are not whole {WINDOW_TOKENS}-token windows")
    bm = bias_mask.shape
    if len(bm) != 5 or bm[1] != heads or bm[2] != 16 or bm[3] != WINDOW_TOKENS or bm[4] != 4:
        raise ValueError(f"window_attention: bias_mask must be [bm_windows, {heads}, 16, 49, 4], got {tuple(bm)}")
    if out is None:
        out = torch.empty((rows, d), dtype=torch.float16, device=qkv.device)
    o2, ldo = _rows(out, d, "out")
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.lib().rpfq_window_attention_sm100(
            q2.data_ptr(), rows // WINDOW_TOKENS, heads, WINDOW_HEAD_DIM, WINDOW_TOKENS, bias_mask.data_ptr(),
            bm[0], o2.data_ptr(), ldo, _stream(qkv.device)), "rpfq_window_attention_sm100")
    if rows:
        _count_launch()
    return out


def vision_act_quant(x: torch.Tensor, salient_token_ratio: float = 0.25, background_clip_ratio: float = 0.75,
                     energy_score_weight: float = 0.5, protect_cls_token: bool = True,
                     out: torch.Tensor | None = None, return_mask: bool = False):
    """Vision-aware activation quantization (``VisionAwareActivationQuantizer``,
    quant_rpfq_vit_vision.py:26-171) of fp16 ``x`` through
    ``rpfq_vision_act_quant_sm100``. ``x`` is ``[B, T, K]`` (saliency over each
    image's T tokens when T = 1 + g*g) or ``[M, K]`` (per-token int8 scales,
    the reference's fallback for inputs that are not 3-D). ``out`` may be ``x``."""
    _require(x, "x")
    if x.dim() == 3:
        images, tokens, K = x.shape
    elif x.dim() == 2:
        images, tokens, K = x.shape[0], 1, x.shape[1]
    else:
        raise ValueError(f"x must be [B, T, K] or [M, K], got {tuple(x.shape)}")
    x2, ldx = _rows(x, K, "x")
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    y2, ldy = _rows(out, K, "out")
    mask = torch.empty(x.shape[:-1], dtype=torch.uint8, device=x.device) if return_mask else None
    L = _lib.lib()
    ws_bytes = int(L.rpfq_vision_workspace_bytes(images, tokens))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    with torch.cuda.device(x.device):
        _lib.check(L.rpfq_vision_act_quant_sm100(
            x2.data_ptr(), ldx, y2.data_ptr(), ldy, images, tokens, K, float(salient_token_ratio),
            float(background_clip_ratio), float(energy_score_weight), int(bool(protect_cls_token)), _p(mask),
            _p(ws), ws_bytes, _stream(x.device)), "rpfq_vision_act_quant_sm100")
    if images:
        g = math.isqrt(tokens - 1) if tokens > 1 else 0
        _count_launch(3 if g and g * g == tokens - 1 else 1)
    return (out, mask.bool()) if return_mask else out


def pack_linear(weight: torch.Tensor, bias: torch.Tensor | None = None, stages: int = 2) -> PackedLayer:
    """The exporter's packing on the GPU (``save_quantized_linear``,
    export_rpfq_vit_to_mlx.py:384-423) through ``rpfq_pack_linear_sm100``:
    float ``[N, K]`` weight -> ``stages`` residual stages of 2-bit axial codes
    and fp16 gammas for U and W, bit-identical to the exporter; bias -> fp16."""
    if not weight.is_cuda:
        raise ValueError("weight must be a CUDA tensor (rpfq_pack_linear_sm100 packs on the GPU)")
    n, k = weight.shape
    if n % 2 or k % 2:
        raise ValueError(f"Complex decomposition requires even dims, got {tuple(weight.shape)}")
    from .packing import BLOCK_SIZE, round_up
    w = weight.detach().to(torch.float32)
    if w.stride(1) != 1 or w.data_ptr() % 4:
        w = w.contiguous()
    dev = w.device
    n_c, k_c = n // 2, k // 2
    n_cp, k_cp = round_up(n_c, BLOCK_SIZE), round_up(k_c, BLOCK_SIZE)
    outs = {"u": (_lib.RpfqPhasePlaneOut * stages)(), "w": (_lib.RpfqPhasePlaneOut * stages)()}
    planes = {}
    for tag in ("u", "w"):
        for i in range(stages):
            codes = torch.empty((n_cp, k_cp // 4), dtype=torch.uint8, device=dev)
            gr = torch.empty((n_cp, k_cp // BLOCK_SIZE), dtype=torch.float16, device=dev)
            gi = torch.empty_like(gr)
            outs[tag][i].codes, outs[tag][i].gamma_real, outs[tag][i].gamma_imag = (
                codes.data_ptr(), gr.data_ptr(), gi.data_ptr())
            planes[f"{tag}_s{i}"] = (codes, gr, gi)
    L = _lib.lib()
    ws_bytes = int(L.rpfq_pack_workspace_bytes(n_c, k_c))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.rpfq_pack_linear_sm100(w.data_ptr(), w.stride(0), n_c, k_c, stages, outs["u"], outs["w"],
                                            ws.data_ptr(), ws_bytes, _stream(dev)), "rpfq_pack_linear_sm100")
    b = torch.zeros(n, device=dev) if bias is None else bias.detach()
    return PackedLayer(n_c, k_c, stages, 2, planes, b.to(device=dev, dtype=torch.float16).contiguous())


def _flags(out: torch.Tensor, residual: torch.Tensor | None, bias: torch.Tensor | None = None) -> int:
    f = 0
    if bias is not None:
        if bias.dtype == torch.float32:
            f |= _lib.GEMM_BIAS_F32
        elif bias.dtype != torch.float16:
            raise ValueError(f"bias must be float16 or float32, got {bias.dtype}")
    if out.dtype == torch.float32:
        f |= _lib.GEMM_OUT_F32
    elif out.dtype != torch.float16:
        raise ValueError(f"out must be float16 or float32, got {out.dtype}")
    if residual is not None:
        if residual.dtype == torch.float32:
            f |= _lib.GEMM_RESIDUAL_F32
        elif residual.dtype != torch.float16:
            raise ValueError(f"residual must be float16 or float32, got {residual.dtype}")
    return f


def gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
         residual: torch.Tensor | None = None, activation="none", block_n: int = 0,
         out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16, cta_pair: int = 0,
         split_k: int | None = None) -> torch.Tensor:
    """K2: ``act(x @ w.T + bias) + residual`` with fp16 operands, fp32
    accumulation; ``residual`` and ``out`` may be fp16 or fp32 (and may be the
    same tensor for an in-place residual add). ``split_k``: 0 automatic (small
    M splits K over a cluster of CTAs), 1 never, 2..8 forced; None = ``SPLIT_K``."""
    _require(x, "x")
    _require(w, "w")
    n, k = w.shape
    if not w.is_contiguous():
        w = w.contiguous()
    x2, ldx = _rows(x, k, "x")
    m = x2.shape[0]
    if bias is not None:
        _require(bias, "bias", bias.dtype)
        bias = bias.contiguous()
    r2, ldr = (None, 0)
    if residual is not None:
        if not residual.is_cuda:
            raise ValueError("residual must be a CUDA tensor")
        r2, ldr = _rows(residual, n, "residual")
        if r2.shape[0] != m:
            raise ValueError("residual rows do not match x")
    if out is None:
        out = torch.empty((*x.shape[:-1], n), dtype=out_dtype, device=x.device)
    y2, ldy = _rows(out, n, "out")
    if y2.data_ptr() != out.data_ptr() or y2.shape[0] != m:
        raise ValueError("out must be a row-major view with unit column stride")
    split_k = SPLIT_K if split_k is None else int(split_k)
    ws, ws_bytes = _workspace(x.device, split_k)
    a = _lib.RpfqGemmArgs(x=x2.data_ptr(), ldx=ldx, w=w.data_ptr(), bias=_p(bias), residual=_p(r2), ldr=ldr,
                          y=y2.data_ptr(), ldy=ldy, m=m, n=n, k=k, activation=_ACT[activation], block_n=block_n,
                          flags=_flags(out, r2, bias), cta_pair=cta_pair, split_k=split_k, workspace=ws,
                          workspace_bytes=ws_bytes)
    timer = _timer if _timer is not None and _timer.events else None
    with torch.cuda.device(x.device):
        if timer is not None:
            ev0 = torch.cuda.Event(enable_timing=True, external=True)
            ev1 = torch.cuda.Event(enable_timing=True, external=True)
            ev0.record()
        _lib.check(_lib.lib().rpfq_gemm_sm100(ctypes.byref(a), _stream(x.device)), "rpfq_gemm_sm100")
        if timer is not None:
            ev1.record()
            timer.gemm_events.append((ev0, ev1, 2 * m * n * k))
    if m:
        _count_launch()
    return out


def gemm_plan(m: int, n: int, k: int, *, out_dtype: torch.dtype = torch.float16, residual: bool = False,
              block_n: int = 0, cta_pair: int = 0, split_k: int | None = None,
              device: torch.device | None = None) -> dict:
    """The tile plan :func:`gemm` runs for an ``[m, k] x [n, k]`` product on
    ``device`` with the same choices (``rpfq_gemm_plan_sm100``; nothing is
    launched): tile width, CTA pairs, K splits, stream-K tail, grid units."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    split_k = SPLIT_K if split_k is None else int(split_k)
    ws, ws_bytes = _workspace(device, split_k)
    f = (_lib.GEMM_OUT_F32 if out_dtype == torch.float32 else 0)
    if residual:
        f |= _lib.GEMM_RESIDUAL_F32 if out_dtype == torch.float32 else 0
    # placeholders: only alignment and strides are validated, nothing is read
    a = _lib.RpfqGemmArgs(x=256, ldx=k, w=256, bias=None, residual=256 if residual else None, ldr=n if residual else 0,
                          y=256, ldy=n, m=m, n=n, k=k, activation=0, block_n=block_n, flags=f, cta_pair=cta_pair,
                          split_k=split_k, workspace=ws, workspace_bytes=ws_bytes)
    plan = _lib.RpfqGemmPlan()
    with torch.cuda.device(device):
        _lib.check(_lib.lib().rpfq_gemm_plan_sm100(ctypes.byref(a), ctypes.byref(plan)), "rpfq_gemm_plan_sm100")
    return {f: getattr(plan, f) for f, _ in _lib.RpfqGemmPlan._fields_}


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float, act_bits: int = 0,
              out: torch.Tensor | None = None, rows: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm of an fp32 ``x[..., d]`` into fp16, with the activation
    quantization of the next packed GEMM fused in when ``act_bits > 0``.
    ``rows`` (int32 CUDA tensor of the flattened row count) gathers: output
    row r is the normalized input row ``rows[r]``."""
    if not x.is_cuda or x.dtype != torch.float32:
        raise ValueError("layernorm: x must be a float32 CUDA tensor")
    _require(weight, "weight")
    _require(bias, "bias")
    d = x.shape[-1]
    x2, ldx = _rows(x, d, "x")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    y2, ldy = _rows(out, d, "out")
    if rows is not None:
        _require(rows, "rows", torch.int32)
        if rows.numel() != y2.shape[0]:
            raise ValueError("layernorm: rows must hold one index per output row")
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().rpfq_layernorm_rows_sm100(
            x2.data_ptr(), ldx, x2.shape[0], _p(rows), weight.data_ptr(), bias.data_ptr(), y2.data_ptr(), ldy,
            y2.shape[0], d, float(eps), int(act_bits), _stream(x.device)), "rpfq_layernorm_rows_sm100")
    if y2.shape[0]:
        _count_launch()
    return out


def layernorm_ex(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float, act_bits: int = 0, *,
                 rows: torch.Tensor | None = None, merge_side: int = 0, add: torch.Tensor | None = None,
                 add_rows: torch.Tensor | None = None, out: torch.Tensor | None = None, fp16_out: bool = True,
                 out32: torch.Tensor | None = None, out32_prenorm: bool = False):
    """The LayerNorm pass with all its row sources and outputs
    (``rpfq_layernorm_ex_sm100``); returns ``(fp16 output or None, fp32
    output or None)``.

    Row sources: ``x`` rows as they are; ``rows`` gathers (output row r is
    input row ``rows[r]``); ``merge_side`` = s > 0 is Swin's 2x2 patch merging
    of an ``x`` of ``[images * s * s, c]`` tokens into ``[images * (s/2)^2, 4c]``
    rows; ``add`` adds ``add[add_rows[r]]`` (or ``add[r]``) to row r before the
    normalization and needs ``out32`` with ``out32_prenorm=True``, which then
    receives the updated rows (``out32`` may be ``x``: in place). ``out32``
    without ``out32_prenorm`` receives the normalized rows in fp32."""
    if not x.is_cuda or x.dtype != torch.float32:
        raise ValueError("layernorm: x must be a float32 CUDA tensor")
    _require(weight, "weight")
    _require(bias, "bias")
    c = x.shape[-1]
    x2, ldx = _rows(x, c, "x")
    if merge_side:
        d, m = 4 * c, x2.shape[0] // 4
    else:
        d, m = c, (rows.numel() if rows is not None else x2.shape[0])
    if rows is not None:
        _require(rows, "rows", torch.int32)
    if fp16_out and out is None:
        out = torch.empty((m, d), dtype=torch.float16, device=x.device)
    y2, ldy = _rows(out, d, "out") if out is not None else (None, 0)
    z2, ldz = _rows(out32, d, "out32") if out32 is not None else (None, 0)
    for t in (y2, z2):
        if t is not None and t.shape[0] != m:
            raise ValueError(f"layernorm: the outputs must have {m} rows")
    a2, lda = (None, 0)
    if add is not None:
        if not add.is_cuda or add.dtype != torch.float32:
            raise ValueError("layernorm: add must be a float32 CUDA tensor")
        a2, lda = _rows(add, d, "add")
    if add_rows is not None:
        _require(add_rows, "add_rows", torch.int32)
    args = _lib.RpfqLayerNormArgs(
        x=x2.data_ptr(), ldx=ldx, x_rows=x2.shape[0], rows=_p(rows), add=_p(a2), ld_add=lda,
        add_bound=a2.shape[0] if a2 is not None else 0, add_rows=_p(add_rows), weight=weight.data_ptr(),
        bias=bias.data_ptr(), y=_p(y2), ldy=ldy, y32=_p(z2), ldy32=ldz, m=m, d=d, eps=float(eps),
        act_bits=int(act_bits), merge_side=int(merge_side), y32_prenorm=int(bool(out32_prenorm)))
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().rpfq_layernorm_ex_sm100(ctypes.byref(args), _stream(x.device)),
                   "rpfq_layernorm_ex_sm100")
    if m:
        _count_launch()
    return out, out32


def patch_unfold(images: torch.Tensor, patch: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """images ``[B, C, H, W]`` (fp16 or fp32) -> fp16 patch rows ``[B, (H/P)(W/P), C P P]``
    in the CHW patch order of the reference's ``patchify_tensor``
    (``audit_rpfq_vit_ios_parity.py:125-134``), ``rpfq_patch_unfold_sm100``."""
    if not images.is_cuda or images.dtype not in (torch.float16, torch.float32) or images.dim() != 4:
        raise ValueError("patch_unfold: images must be a [B, C, H, W] float16 or float32 CUDA tensor")
    images = images.contiguous()
    B, C, H, W = images.shape
    if patch <= 0 or H % patch or W % patch:
        raise ValueError(f"patch_unfold: patch {patch} must divide the image size {H}x{W}")
    n, k = (H // patch) * (W // patch), C * patch * patch
    if out is None:
        out = torch.empty((B, n, k), dtype=torch.float16, device=images.device)
    o2, ldo = _rows(out, k, "out")
    if o2.data_ptr() != out.data_ptr() or o2.shape[0] != B * n:
        raise ValueError(f"patch_unfold: out must be a row-major view of {B * n} rows with unit column stride")
    if B == 0:
        return out
    with torch.cuda.device(images.device):
        _lib.check(_lib.lib().rpfq_patch_unfold_sm100(images.data_ptr(), int(images.dtype == torch.float32), B, C, H,
                                                      W, int(patch), o2.data_ptr(), ldo, _stream(images.device)),
                   "rpfq_patch_unfold_sm100")
    _count_launch()
    return out


def act_quant(x: torch.Tensor, num_bits: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row symmetric quantization of the Re / Im halves (ActivationQuantSTE)."""
    _require(x, "x")
    k = x.shape[-1]
    x2, ldx = _rows(x, k, "x")
    if out is None:
        out = torch.empty_like(x2)
    o2, ldo = _rows(out, k, "out")
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().rpfq_act_quant_sm100(x2.data_ptr(), ldx, o2.data_ptr(), ldo, x2.shape[0], k,
                                                   int(num_bits), _stream(x.device)), "rpfq_act_quant_sm100")
    if x2.shape[0]:
        _count_launch()
    return out.reshape(x.shape)


def wide_linear(x: torch.Tensor, layer: PackedLayer, dense: torch.Tensor | None, act_bits: int = 0,
                activation="none", residual: torch.Tensor | None = None,
                out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16,
                bias: torch.Tensor | None = None, split_k: int | None = None) -> torch.Tensor:
    """Whole layer through ``rpfq_wide_linear_sm100``: optional activation
    quantization, then the GEMM over the prepacked coefficients with bias and
    epilogue. ``x`` is fp16 ``[..., 2 k_c]``; ``residual`` / ``out`` fp16 or
    fp32 (``out`` may be ``residual`` for an in-place residual add).

    ``dense=None`` selects the fused decode path (at most ``FUSED_DECODE_MAX_ROWS``
    rows, 2-bit codes, ``n_c`` and ``k_c`` multiples of 8): the packed planes
    are decoded inside the GEMM and no dense matrix exists anywhere.

    ``bias`` (optional) replaces ``layer.bias`` for this call, e.g. the same
    values widened to fp32 once, which the epilogue adds without converting.
    ``split_k`` as in :func:`gemm` (both paths: the fused decode splits K over
    a cluster of CTAs per block of output rows when those blocks alone leave
    most SMs idle)."""
    _require(x, "x")
    if dense is not None:
        _require(dense, "dense")
    if bias is None:
        bias = layer.bias
    K, N = 2 * layer.k_c, 2 * layer.n_c
    x2, ldx = _rows(x, K, "x")
    m = x2.shape[0]
    r2, ldr = (None, 0)
    if residual is not None:
        if not residual.is_cuda:
            raise ValueError("residual must be a CUDA tensor")
        r2, ldr = _rows(residual, N, "residual")
    if out is None:
        out = torch.empty((*x.shape[:-1], N), dtype=out_dtype, device=x.device)
    y2, ldy = _rows(out, N, "out")
    if y2.data_ptr() != out.data_ptr() or y2.shape[0] != m:
        raise ValueError("out must be a row-major view with unit column stride")
    scratch = torch.empty((m, K), dtype=torch.float16, device=x.device) if act_bits else None
    s = layer_struct(layer)
    split_k = SPLIT_K if split_k is None else int(split_k)
    ws, ws_bytes = _workspace(x.device, split_k)
    a = _lib.RpfqWideLinearArgs(layer=ctypes.pointer(s), dense=_p(dense), x=x2.data_ptr(), ldx=ldx,
                                bias=_p(bias), residual=_p(r2), ldr=ldr, y=y2.data_ptr(), ldy=ldy, m=m,
                                act_bits=int(act_bits), activation=_ACT[activation], scratch=_p(scratch),
                                flags=_flags(out, r2, bias), split_k=split_k, workspace=ws,
                                workspace_bytes=ws_bytes)
    timer = _timer if _timer is not None and _timer.events else None
    with torch.cuda.device(x.device):
        if timer is not None:
            # With act_bits > 0 the span also holds the quantization kernel.
            ev0 = torch.cuda.Event(enable_timing=True, external=True)
            ev1 = torch.cuda.Event(enable_timing=True, external=True)
            ev0.record()
        _lib.check(_lib.lib().rpfq_wide_linear_sm100(ctypes.byref(a), _stream(x.device)), "rpfq_wide_linear_sm100")
        if timer is not None:
            ev1.record()
            timer.gemm_events.append((ev0, ev1, 2 * m * N * K))
    if m:
        _count_launch(2 if act_bits else 1)
    return out


# ---------------------------------------------------------------------------
# torch.ops.rpfq.* (CUDA only)
# ---------------------------------------------------------------------------

_LIB = torch.library.Library("rpfq", "DEF")
_LIB.define("gemm(Tensor x, Tensor w, Tensor? bias=None, Tensor? residual=None, int activation=0) -> Tensor")
_LIB.define("act_quant(Tensor x, int num_bits) -> Tensor")
_LIB.define("prepack(Tensor[] codes, Tensor[] gamma_real, Tensor[] gamma_imag, int n_c, int k_c, "
            "int code_bits=2, int rounding=0) -> Tensor")
# The packed layer as the reference stores it: codes / gammas of the U stages
# then the W stages (export_rpfq_vit_to_mlx.py:384-423 key order), exactly the
# tensors a caller of QATLinearComplexPhase's packed form holds.
_LIB.define("wide_linear(Tensor x, Tensor[] codes, Tensor[] gamma_re, Tensor[] gamma_im, Tensor? bias, int n_c, "
            "int k_c, int act_bits=0, bool gelu=False) -> Tensor")
_LIB.define("wide_linear_dense(Tensor x, Tensor dense, Tensor? bias, int n_c, int k_c, int act_bits=0, "
            "int activation=0, Tensor? residual=None) -> Tensor")


def _op_gemm(x, w, bias=None, residual=None, activation=0):
    return gemm(x, w, bias, residual, int(activation))


def _op_act_quant(x, num_bits):
    return act_quant(x, int(num_bits))


def _planes_from_lists(codes, gamma_real, gamma_imag, n_c, k_c, code_bits, bias=None):
    if len(codes) % 2 or not (len(codes) == len(gamma_real) == len(gamma_imag)) or not codes:
        raise ValueError("codes / gammas must list the U stages then the W stages")
    stages = len(codes) // 2
    planes = {}
    for i in range(stages):
        planes[f"u_s{i}"] = (codes[i], gamma_real[i], gamma_imag[i])
        planes[f"w_s{i}"] = (codes[stages + i], gamma_real[stages + i], gamma_imag[stages + i])
    return PackedLayer(int(n_c), int(k_c), stages, int(code_bits), planes, bias)


def _op_prepack(codes, gamma_real, gamma_imag, n_c, k_c, code_bits=2, rounding=0):
    layer = _planes_from_lists(codes, gamma_real, gamma_imag, n_c, k_c, code_bits)
    return prepack(layer, "rne" if int(rounding) == 0 else "ties_away")


# Decoded coefficient matrices of packed layers called through the packed op
# with more rows than the fused decode path takes: keyed by the planes'
# storage and version counters (a plane written in place decodes again). An
# entry holds its plane tensors, so their storage cannot be handed to another
# layer while the entry exists; the oldest entry goes first past the limit.
_DENSE_CACHE: dict = {}
_DENSE_CACHE_MAX = 256
dense_cache_stats = {"hits": 0, "decodes": 0}


def _cached_dense(layer: PackedLayer, tensors) -> torch.Tensor:
    key = (layer.n_c, layer.k_c, layer.stages, layer.code_bits,
           tuple((t.data_ptr(), t._version, tuple(t.shape), t.dtype) for t in tensors))
    entry = _DENSE_CACHE.get(key)
    if entry is not None:
        dense_cache_stats["hits"] += 1
        return entry[1]
    while len(_DENSE_CACHE) >= _DENSE_CACHE_MAX:
        _DENSE_CACHE.pop(next(iter(_DENSE_CACHE)))
    dense = prepack(layer)
    dense_cache_stats["decodes"] += 1
    _DENSE_CACHE[key] = (list(tensors), dense)
    return dense


def _op_wide_linear(x, codes, gamma_re, gamma_im, bias, n_c, k_c, act_bits=0, gelu=False):
    """The packed layer ``y = act(Q(W) x + b)`` straight from the reference's
    packed tensors: codes uint8 ``[n_cp, k_cp * b / 8]`` and fp16 gammas
    ``[n_cp, k_cp / 256]`` per stage (U stages, then W stages; the code width
    b follows from the codes' shape), optional fp16 bias ``[2 n_c]``, fp16
    ``x[..., 2 k_c]`` -> fp16 ``[..., 2 n_c]``. ``act_bits`` > 0 quantizes x
    first (ActivationQuantSTE); ``gelu`` applies exact GELU to the output.

    Up to ``FUSED_DECODE_MAX_ROWS`` rows (2-bit codes, ``n_c``, ``k_c``
    multiples of 8) the codes are decoded inside the GEMM and no dense matrix
    exists; otherwise the planes are decoded once into the fp16 coefficient
    matrix (kept for later calls with the same planes) and the tcgen05 GEMM
    runs over it."""
    _require(x, "x")
    from .packing import BLOCK_SIZE, round_up
    n_c, k_c = int(n_c), int(k_c)
    if n_c <= 0 or k_c <= 0:
        raise ValueError(f"n_c and k_c must be positive, got {n_c}, {k_c}")
    k_cp = round_up(k_c, BLOCK_SIZE)
    if not codes or codes[0].dim() != 2 or (codes[0].shape[1] * 8) % k_cp:
        raise ValueError("codes must be [n_cp, k_cp * code_bits / 8] uint8 tensors")
    code_bits = codes[0].shape[1] * 8 // k_cp
    if bias is not None:
        _require(bias, "bias")
        if bias.numel() != 2 * n_c:
            raise ValueError(f"bias must hold {2 * n_c} values, got {bias.numel()}")
    layer = _planes_from_lists(codes, gamma_re, gamma_im, n_c, k_c, code_bits,
                               bias if bias is not None else torch.zeros(2 * n_c, dtype=torch.float16,
                                                                          device=x.device))
    m = x.numel() // x.shape[-1] if x.dim() else 0
    act = "gelu" if gelu else "none"
    fused = m <= FUSED_DECODE_MAX_ROWS and code_bits == 2 and n_c % 8 == 0 and k_c % 8 == 0
    dense = None if fused else _cached_dense(layer, [*codes, *gamma_re, *gamma_im])
    return wide_linear(x, layer, dense, int(act_bits), activation=act)


def _op_wide_linear_dense(x, dense, bias, n_c, k_c, act_bits=0, activation=0, residual=None):
    _require(x, "x")
    if tuple(dense.shape) != (2 * int(n_c), 2 * int(k_c)):
        raise ValueError(f"dense must be [{2 * int(n_c)}, {2 * int(k_c)}], got {tuple(dense.shape)}")
    if act_bits:
        x = act_quant(x, int(act_bits))
    return gemm(x, dense, bias, residual, int(activation))


_LIB.impl("gemm", _op_gemm, "CUDA")
_LIB.impl("act_quant", _op_act_quant, "CUDA")
_LIB.impl("prepack", _op_prepack, "CUDA")
_LIB.impl("wide_linear", _op_wide_linear, "CUDA")
_LIB.impl("wide_linear_dense", _op_wide_linear_dense, "CUDA")
