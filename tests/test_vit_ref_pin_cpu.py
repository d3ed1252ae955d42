"""CPU pin of the whole-model oracle (oracle/vit_ref.py) to the reference's
own runtime forward: ``forward_runtime_path`` / ``capture_runtime_block_trace``
(RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:588-688) with weights
rebuilt by the script's ``reconstruct_export_weight``, executed by
tests/golden/make_golden.py on a 3-block ViT (golden_vitref.npz).

``vit_ref.vit_forward`` on the same float weights — its quantized linears
rebuilt by the oracle's exporter restatement (packed_ref.pack_linear ->
dense_weight_from_packed) — must give the reference's logits to 1e-6 of
max|logit| in float32, and the rebuilt dense weights must equal the
reference's bit for bit."""

import os

import numpy as np
import torch

from oracle import packed_ref as pr
from oracle import vit_ref
from rpfq_review_b200.vit import ViTConfig

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_vitref.npz")


def _weights(g, cfg):
    s = {k[len("state."):]: g[k] for k in g.files if k.startswith("state.")}
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    w = {"patch_w": t(s["patch_w"]), "patch_b": t(s["patch_b"]), "cls_tokens": t(s["cls_token"]),
         "pos_embed": t(s["pos_embed"]), "norm_w": t(s["norm_w"]), "norm_b": t(s["norm_b"])}

    def dense(weight):
        n, k = weight.shape
        return pr.dense_weight_from_packed(pr.pack_linear(weight, None, 2), n // 2, k // 2)

    for i in range(cfg.depth):
        for name in ("qkv", "proj", "fc1", "fc2"):
            w[f"blocks.{i}.{name}"] = (t(dense(s[f"blocks.{i}.{name}.w"])), t(s[f"blocks.{i}.{name}.b"]))
        for nm in ("norm1", "norm2"):
            w[f"blocks.{i}.{nm}_w"] = t(s[f"blocks.{i}.{nm}.w"])
            w[f"blocks.{i}.{nm}_b"] = t(s[f"blocks.{i}.{nm}.b"])
    w["head"] = (t(dense(s["head_w"])), t(s["head_b"]))
    return w


def test_vit_ref_matches_reference_runtime_forward():
    g = np.load(GOLD)
    hidden, heads, depth, mlp, img, patch, classes = (int(v) for v in g["config"])
    cfg = ViTConfig("vitref", dim=hidden, depth=depth, heads=heads, mlp=mlp, img=img, patch=patch, classes=classes)
    assert cfg.tokens == g["ref.block0"].shape[1]
    w = _weights(g, cfg)
    logits = vit_ref.vit_forward(w, cfg, torch.from_numpy(g["images"])).numpy()
    ref = g["ref.logits"]
    assert logits.shape == ref.shape
    assert np.abs(logits - ref).max() <= 1e-6 * np.abs(ref).max()
    assert np.array_equal(logits.argmax(-1), ref.argmax(-1))


def test_oracle_dense_reconstruction_matches_reference_bitwise():
    """The oracle's exporter restatement rebuilds the head's dense weight as
    the reference does (quantized_forward_weight): the reference logits come
    back bit for bit from its golden final norm through the oracle's weight,
    with the reference's own call, linear(x[:, :1, :], head).reshape(B, -1)."""
    g = np.load(GOLD)
    s = {k[len("state."):]: g[k] for k in g.files if k.startswith("state.")}
    n, k = s["head_w"].shape
    dense = pr.dense_weight_from_packed(pr.pack_linear(s["head_w"], None, 2), n // 2, k // 2)
    fn = torch.from_numpy(g["ref.final_norm"])
    y = torch.nn.functional.linear(fn[:, :1, :], torch.from_numpy(dense), torch.from_numpy(s["head_b"]))
    y = y.reshape(fn.shape[0], -1).numpy()
    assert np.array_equal(y, g["ref.logits"])
