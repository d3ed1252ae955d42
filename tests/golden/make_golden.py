#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference checkout is available (``--ref``, default the
``RPFQ_REFERENCE_ROOT`` environment variable, as for the build); the
fixtures it writes are committed, so the tests never need the reference at
run time. Fixtures:

* ``golden_exporter.npz`` — the reference exporter
  (RPFQ-ViTApple/scripts/export_rpfq_vit_to_mlx.py): ``save_quantized_linear``
  packed planes, ``quantized_forward_weight`` dense weight and the layer output
  ``F.linear(x, W_q, b)`` for seeded float weights (a generic case, a case
  full of |re| == |im| ties, and a 1-stage case).
* ``golden_actquant.npz`` — ``ActivationQuantSTE.forward``
  (RPFQ-ViT-main/quant_models/quant_i.py:442-455) at 2, 4 and 8 bits,
  including an all-zero row and exact .5 products.
* ``golden_qat.npz`` — ``QATLinearComplexPhase.forward`` (quant_i.py:513-554)
  with complex_phase_v2 on the same weights, act-quant on and off.
* ``golden_refcpp.npz`` — the reference's C++ runtime built from its sources
  (oracle/_ref): ``wideLinearReference`` output and the fp16 coefficient
  planes of ``buildFusedWideLinearCache`` for a seeded synthetic packed layer.
* ``golden_vision.npz`` — ``VisionAwareActivationQuantizer.forward``
  (RPFQ-ViT-main/quant_models/quant_rpfq_vit_vision.py:26-171) on seeded
  token batches: the saliency mask and the quantized Re / Im halves. The
  module imports timm at its top, which this container lacks, so the class
  definition (and ``EPS``) is taken out of the file with ``ast`` and executed
  alone, unchanged.
* ``golden_vitref.npz`` — the reference's pure-torch runtime forward,
  ``forward_runtime_path`` with ``capture_runtime_block_trace``
  (RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:588-688), on a small
  3-block ViT (so that block 0, block 1 and the later-block branch all run)
  whose quantized linears are rebuilt by the script's own
  ``reconstruct_export_weight`` (:328-383) and ``quantized_forward_weight``
  (head), as its ``build_runtime_state`` (:439-515) does. The script imports
  timm and PIL at its top, so these functions are taken out of it with
  ``ast`` and executed unchanged next to the exporter module they import.

``--only NAME`` regenerates one fixture (exporter, actquant, qat, refcpp, vision, vitref).
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("RPFQ_REFERENCE_ROOT", "/root/reference"))
    ap.add_argument("--only", default=None, choices=["exporter", "actquant", "qat", "refcpp", "vision", "vitref"])
    args = ap.parse_args()
    if args.only == "vision":
        make_vision(args.ref)
        return
    if args.only == "vitref":
        make_vitref(args.ref)
        return
    sys.path.insert(0, os.path.join(args.ref, "RPFQ-ViTApple", "scripts"))
    sys.path.insert(0, os.path.join(args.ref, "RPFQ-ViT-main", "quant_models"))
    sys.path.insert(0, REPO)
    import export_rpfq_vit_to_mlx as ex  # noqa: E402
    import quant_i  # noqa: E402

    torch.manual_seed(0)
    out: dict[str, np.ndarray] = {}

    # ---- exporter cases --------------------------------------------------
    cases = {
        "generic": (40, 72, 2, lambda g, n, k: torch.randn(n, k, generator=g) * 0.02),
        "medium": (70, 260, 2, lambda g, n, k: torch.randn(n, k, generator=g) * 0.05),
        # integer weights: many |re| == |im| ties and exact zeros
        "ties": (24, 40, 2, lambda g, n, k: torch.randint(-2, 3, (n, k), generator=g).float()),
        "onestage": (40, 72, 1, lambda g, n, k: torch.randn(n, k, generator=g) * 0.02),
    }
    for name, (n_c, k_c, stages, draw) in cases.items():
        g = torch.Generator().manual_seed(1000 + n_c + k_c + stages)
        w = draw(g, 2 * n_c, 2 * k_c)
        b = torch.randn(2 * n_c, generator=g) * 0.02
        x = torch.randn(7, 2 * k_c, generator=g)
        n_cp = ex.round_up(n_c, ex.BLOCK_SIZE)
        k_cp = ex.round_up(k_c, ex.BLOCK_SIZE)
        target: dict[str, torch.Tensor] = {}
        ex.save_quantized_linear(target, "layer", w, b, k_cp, n_cp, stages)
        dense = ex.quantized_forward_weight(w, stages)
        y = F.linear(x, dense, target["layer.bias"].float())
        out[f"{name}.weight"] = w.numpy()
        out[f"{name}.bias_f32"] = b.numpy()
        out[f"{name}.x"] = x.numpy()
        out[f"{name}.dims"] = np.array([n_c, k_c, stages], np.int64)
        for key, t in target.items():
            out[f"{name}.{key[len('layer.'):]}"] = t.numpy()
        out[f"{name}.dense"] = dense.numpy()
        out[f"{name}.y"] = y.numpy()
    np.savez_compressed(os.path.join(HERE, "golden_exporter.npz"), **out)

    # ---- activation quantization ------------------------------------------
    aq: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(7)
    x = torch.randn(9, 96, generator=g) * 3.0
    x[3] = 0.0                           # amax clamp at 1e-5
    x[4, :48] = torch.linspace(-1.0, 1.0, 48)
    x[5, :48] = torch.arange(48).float() / 47.0 * 7.0 - 3.5   # products near .5
    x = x.half().float()                  # fp16-representable, as the GPU path sees it
    aq["x"] = x.numpy()
    for bits in (2, 4, 8):
        qr, qi = quant_i.ActivationQuantSTE.forward(None, x[:, :48], x[:, 48:], bits)
        aq[f"q{bits}"] = torch.cat((qr, qi), dim=-1).numpy()
    np.savez_compressed(os.path.join(HERE, "golden_actquant.npz"), **aq)

    # ---- QAT module forward (module-interface reference) ------------------
    qat: dict[str, np.ndarray] = {}
    gen = cases["generic"]
    n_c, k_c = gen[0], gen[1]
    for act in (False, True):
        layer = quant_i.QATLinearComplexPhase(
            quant_method_u="complex_phase_v2", quant_method_w="complex_phase_v2",
            enable_act_quant=act, act_num_bits=4, in_features=2 * k_c, out_features=2 * n_c, bias=True)
        with torch.no_grad():
            layer.weight.copy_(torch.from_numpy(out["generic.weight"]))
            layer.bias.copy_(torch.from_numpy(out["generic.bias_f32"]))
            y = layer(torch.from_numpy(out["generic.x"]))
        qat[f"y_act{int(act)}"] = y.numpy()
    np.savez_compressed(os.path.join(HERE, "golden_qat.npz"), **qat)

    # ---- reference C++ runtime -------------------------------------------
    from oracle import packed_ref as pr  # noqa: E402
    from oracle import ref_lib  # noqa: E402
    if ref_lib.load() is None:
        raise SystemExit("oracle/_ref/librpfq_ref.so missing: run `make -C oracle` first")
    rc: dict[str, np.ndarray] = {}
    n_c, k_c = 100, 300
    packed = pr.random_packed_numpy(n_c, k_c, seed=11)
    xr = np.random.default_rng(12).standard_normal((5, 2 * k_c)).astype(np.float16).astype(np.float32)
    rc["dims"] = np.array([n_c, k_c], np.int64)
    rc["x"] = xr
    for key, val in packed.items():
        rc[f"packed.{key}"] = val
    rc["y_reference"] = ref_lib.wide_linear(packed, xr, n_c, k_c, mode=0)
    rc["y_fp16cache"] = ref_lib.wide_linear(packed, xr, n_c, k_c, mode=2, threads=2)
    for key, val in ref_lib.coefficient_planes(packed, n_c, k_c).items():
        rc[f"plane.{key}"] = val
    np.savez_compressed(os.path.join(HERE, "golden_refcpp.npz"), **rc)
    make_vision(args.ref)
    make_vitref(args.ref)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


def _reference_vision_quantizer(ref: str):
    """The reference's VisionAwareActivationQuantizer class, executed from its
    own source without the module's timm imports."""
    import ast
    import math
    path = os.path.join(ref, "RPFQ-ViT-main", "quant_models", "quant_rpfq_vit_vision.py")
    tree = ast.parse(open(path).read(), path)
    keep = [n for n in tree.body
            if (isinstance(n, ast.ClassDef) and n.name == "VisionAwareActivationQuantizer")
            or (isinstance(n, ast.Assign) and any(getattr(t, "id", None) == "EPS" for t in n.targets))]
    ns = {"torch": torch, "nn": torch.nn, "math": math}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns["VisionAwareActivationQuantizer"]


def make_vision(ref: str) -> None:
    VAQ = _reference_vision_quantizer(ref)
    # name: (batch, tokens, k_c, salient_ratio, clip_ratio, energy_weight, protect_cls, two_d)
    cases = {
        "vitb": (2, 197, 16, 0.25, 0.75, 0.5, True, False),
        "nocls": (2, 197, 16, 0.1, 0.5, 0.3, False, False),
        "all_salient": (1, 197, 16, 1.0, 0.75, 0.5, True, False),
        "no_salient": (1, 197, 16, 0.0, 0.75, 0.5, True, False),
        "grid4": (3, 17, 8, 0.25, 0.75, 1.0, True, False),
        "zero_token": (1, 50, 24, 0.3, 0.9, 0.0, True, False),
        "fallback_tokens": (2, 198, 16, 0.25, 0.75, 0.5, True, False),
        "fallback_2d": (1, 40, 16, 0.25, 0.75, 0.5, True, True),
    }
    out: dict[str, np.ndarray] = {}
    for i, (name, (b, t, k, ratio, clip, wgt, cls, two_d)) in enumerate(cases.items()):
        g = torch.Generator().manual_seed(5000 + i)
        # per-token magnitudes vary so that token scales and saliency differ
        mag = torch.exp(torch.randn(b, t, 1, generator=g) * 0.7)
        xr = (torch.randn(b, t, k, generator=g) * mag).half().float()
        xi = (torch.randn(b, t, k, generator=g) * mag).half().float()
        if name == "zero_token":
            xr[:, 7] = 0.0
            xi[:, 7] = 0.0
        q = VAQ(salient_token_ratio=ratio, background_clip_ratio=clip, energy_score_weight=wgt,
                protect_cls_token=cls)
        if two_d:
            xr, xi = xr.reshape(b * t, k), xi.reshape(b * t, k)
        with torch.no_grad():
            mask = q._build_saliency_mask(xr, xi)
            qr, qi = q(xr, xi)
        out[f"{name}.params"] = np.array([ratio, clip, wgt, float(cls)], np.float64)
        out[f"{name}.x_real"] = xr.numpy().astype(np.float16)
        out[f"{name}.x_imag"] = xi.numpy().astype(np.float16)
        out[f"{name}.q_real"] = qr.numpy()
        out[f"{name}.q_imag"] = qi.numpy()
        out[f"{name}.mask"] = (np.ones(xr.shape[:-1], bool) if mask is None
                               else mask.squeeze(-1).numpy()).astype(np.uint8)
    np.savez_compressed(os.path.join(HERE, "golden_vision.npz"), **out)



# Small ViT of the vitref fixture: hidden 64 (32 complex, padded to 256), 2
# heads, 3 blocks, MLP 128, 16 x 16 images of 8 x 8 patches (5 tokens), 10
# classes, LayerNorm eps 1e-6 (timm ViT).
VITREF = dict(hidden=64, heads=2, depth=3, mlp=128, img=16, patch=8, classes=10, eps=1e-6, batch=2)


def _reference_runtime_functions(ref: str):
    """forward_runtime_path and the helpers it calls, executed from the
    reference audit script's own source without its module-level imports
    (timm, PIL), next to the exporter functions that script imports."""
    import ast
    from dataclasses import dataclass
    from typing import Any
    sys.path.insert(0, os.path.join(ref, "RPFQ-ViTApple", "scripts"))
    import export_rpfq_vit_to_mlx as ex  # noqa: E402
    path = os.path.join(ref, "RPFQ-ViTApple", "scripts", "audit_rpfq_vit_ios_parity.py")
    tree = ast.parse(open(path).read(), path)
    names = {"RuntimeLayer", "patchify_tensor", "reconstruct_export_weight", "layer_norm", "linear",
             "capture_runtime_block_trace", "forward_runtime_path"}
    keep = [n for n in tree.body if isinstance(n, (ast.ClassDef, ast.FunctionDef)) and n.name in names]
    assert {n.name for n in keep} == names
    ns = {"torch": torch, "F": F, "dataclass": dataclass, "Any": Any, "__name__": "audit_extract"}
    for k in ("widely_linear_decompose", "residual_phase_quantize", "legacy_residual_phase_quantize",
              "dequantize_axis"):
        ns[k] = getattr(ex, k)
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns, ex


def make_vitref(ref: str) -> None:
    ns, ex = _reference_runtime_functions(ref)
    RL = ns["RuntimeLayer"]
    c = VITREF
    d, mlp = c["hidden"], c["mlp"]
    g = torch.Generator().manual_seed(4242)

    def rnd(*shape, std=0.05):
        return torch.randn(*shape, generator=g) * std

    state = {"patch_w": rnd(d, 3 * c["patch"] ** 2, std=0.02), "patch_b": rnd(d, std=0.02),
             "cls_token": rnd(1, 1, d, std=0.02), "pos_embed": rnd(1, 1 + (c["img"] // c["patch"]) ** 2, d, std=0.02),
             "norm_w": 1 + rnd(d, std=0.1), "norm_b": rnd(d, std=0.1),
             "head_w": rnd(c["classes"], d), "head_b": rnd(c["classes"], std=0.02)}
    pad = lambda n: -(-n // ex.BLOCK_SIZE) * ex.BLOCK_SIZE  # noqa: E731
    layers = []
    for i in range(c["depth"]):
        for name, (n_out, n_in) in (("qkv", (3 * d, d)), ("proj", (d, d)), ("fc1", (mlp, d)), ("fc2", (d, mlp))):
            state[f"blocks.{i}.{name}.w"] = rnd(n_out, n_in)
            state[f"blocks.{i}.{name}.b"] = rnd(n_out, std=0.02)
        for nm in ("norm1", "norm2"):
            state[f"blocks.{i}.{nm}.w"] = 1 + rnd(d, std=0.1)
            state[f"blocks.{i}.{nm}.b"] = rnd(d, std=0.1)
        lay = {nm: RL(state[f"blocks.{i}.{nm}.w"], state[f"blocks.{i}.{nm}.b"]) for nm in ("norm1", "norm2")}
        for name in ("qkv", "proj", "fc1", "fc2"):
            w = state[f"blocks.{i}.{name}.w"]
            wq = ns["reconstruct_export_weight"](w, pad(w.shape[1] // 2), pad(w.shape[0] // 2), 2, legacy=False)
            lay[name] = RL(wq, state[f"blocks.{i}.{name}.b"])
        layers.append(lay)
    runtime = {"patch_embed": RL(state["patch_w"], state["patch_b"]), "cls_token": state["cls_token"],
               "pos_embed": state["pos_embed"], "norm": RL(state["norm_w"], state["norm_b"]),
               "head": RL(ex.quantized_forward_weight(state["head_w"], stages=2).float(), state["head_b"]),
               "layers": layers}
    images = torch.randn(c["batch"], 3, c["img"], c["img"], generator=g)
    patches = torch.cat([ns["patchify_tensor"](im, c["patch"]) for im in images], dim=0)
    caps = ns["forward_runtime_path"](runtime, patches, c["heads"], c["eps"])
    out = {f"state.{k}": v.numpy() for k, v in state.items()}
    out["images"] = images.numpy()
    for k in ("patch_embed", "block0", "block1", "final_norm", "logits"):
        out[f"ref.{k}"] = caps[k].numpy()
    out["config"] = np.array([c[k] for k in ("hidden", "heads", "depth", "mlp", "img", "patch", "classes")], np.int64)
    np.savez_compressed(os.path.join(HERE, "golden_vitref.npz"), **out)


if __name__ == "__main__":
    main()
