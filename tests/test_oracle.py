"""CPU tests: the oracle against the golden vectors made by the reference
itself (tests/golden/make_golden.py), plus the host-side packer.

Tolerances: integer / byte / fp16-bit results are compared bit for bit;
float64 GEMM restatements within 1e-6 of max|y| (summation order only).
"""

import os

import numpy as np
import pytest
import torch

from oracle import packed_ref as pr
from tests.helpers import to_numpy_packed

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ("generic", "medium", "ties", "onestage")


@pytest.fixture(scope="module")
def exporter():
    return np.load(os.path.join(GOLD, "golden_exporter.npz"))


def _packed_keys(g, name):
    stages = int(g[f"{name}.dims"][2])
    keys = [f"{t}_s{s}.{f}" for t in "uw" for s in range(stages) for f in ("codes", "gamma_real", "gamma_imag")]
    return keys + ["bias"]


@pytest.mark.parametrize("name", CASES)
def test_oracle_packer_matches_exporter(exporter, name):
    """pack_linear restates save_quantized_linear (export…py:384-423) bit for bit."""
    g = exporter
    n_c, k_c, stages = (int(v) for v in g[f"{name}.dims"])
    p = pr.pack_linear(g[f"{name}.weight"], g[f"{name}.bias_f32"], stages)
    for key in _packed_keys(g, name):
        assert np.array_equal(p[key], g[f"{name}.{key}"]), key


@pytest.mark.parametrize("name", CASES)
def test_product_packer_matches_exporter(exporter, name):
    """The product's torch packer (rpfq_review_b200.packing.pack_linear) on CPU."""
    from rpfq_review_b200.packing import pack_linear
    g = exporter
    n_c, k_c, stages = (int(v) for v in g[f"{name}.dims"])
    layer = pack_linear(torch.from_numpy(g[f"{name}.weight"]), torch.from_numpy(g[f"{name}.bias_f32"]), stages)
    p = to_numpy_packed(layer)
    for key in _packed_keys(g, name):
        assert np.array_equal(p[key], g[f"{name}.{key}"]), key


@pytest.mark.parametrize("name", CASES)
def test_oracle_dense_and_forward(exporter, name):
    """dense_weight_from_packed == quantized_forward_weight (export…py:336-375),
    and the layer forward matches F.linear on it."""
    g = exporter
    n_c, k_c, stages = (int(v) for v in g[f"{name}.dims"])
    packed = {k: g[f"{name}.{k}"] for k in _packed_keys(g, name)}
    dense = pr.dense_weight_from_packed(packed, n_c, k_c)
    assert np.array_equal(dense, g[f"{name}.dense"])
    y = pr.wide_linear(g[f"{name}.x"], dense, packed["bias"].astype(np.float32))
    assert pr.max_rel_err(y, g[f"{name}.y"]) < 1e-6


@pytest.mark.parametrize("bits", (2, 4, 8))
def test_oracle_act_quant_bit_exact(bits):
    """act_quant == ActivationQuantSTE.forward (quant_i.py:442-455), bit for bit."""
    g = np.load(os.path.join(GOLD, "golden_actquant.npz"))
    assert np.array_equal(pr.act_quant(g["x"], bits), g[f"q{bits}"])


def test_oracle_vs_reference_cpp_golden():
    """Against the reference's C++ runtime (oracle/_ref, golden_refcpp.npz):
    fp16 planes bit-exact in ties-away mode; RNE differs only on exact ties;
    wideLinearReference output within 1e-6."""
    g = np.load(os.path.join(GOLD, "golden_refcpp.npz"))
    n_c, k_c = (int(v) for v in g["dims"])
    packed = {k[len("packed."):]: g[k] for k in g.files if k.startswith("packed.")}
    ta = pr.coefficient_planes(packed, n_c, k_c, "ties_away")
    rne = pr.coefficient_planes(packed, n_c, k_c, "rne")
    for key in ("rr", "ir", "ri", "ii"):
        ref = g[f"plane.{key}"].view(np.uint16)
        assert np.array_equal(ta[key].view(np.uint16), ref), key
        diff = rne[key].view(np.uint16) != ref
        # every RNE / ties-away difference is one ulp
        assert np.all(np.abs(rne[key].view(np.uint16)[diff].astype(np.int32) - ref[diff].astype(np.int32)) == 1)
    dense = pr.dense_weight_from_packed(packed, n_c, k_c)
    y = pr.wide_linear(g["x"], dense, packed["bias"].astype(np.float32))
    assert pr.max_rel_err(g["y_reference"], y) < 1e-6
    y16 = pr.wide_linear(g["x"], pr.dense_fp16_from_planes(ta), packed["bias"].astype(np.float32))
    assert pr.max_rel_err(g["y_fp16cache"], y16) < 1e-6


def test_exhaustive_code_decode():
    """All 256 byte values x 4 lanes: unpack matches get2BitCode
    (phase_linear.cpp:15-19, 145-153) and the codebook of dequantize_axis
    (export…py:236-247): 0:-1, 1:+1, 2:-i, 3:+i."""
    byte = np.arange(256, dtype=np.uint8).reshape(256, 1)
    codes = pr.unpack_codes(byte, 256, 4)
    for lane in range(4):
        assert np.array_equal(codes[:, lane], (np.arange(256) >> (2 * lane)) & 3)
    assert np.array_equal(pr.pack_codes(codes), byte)
    gamma = np.full((256, 1), np.float16(0.5), np.float16)
    packed = np.zeros((256, 64), np.uint8)
    packed[:, 0] = np.arange(256)
    re, im = pr.dequantize_axis(packed, gamma, gamma, 256, 256)
    want_re = {0: -2.0, 1: 2.0, 2: 0.0, 3: 0.0}
    want_im = {0: 0.0, 1: 0.0, 2: -2.0, 3: 2.0}
    for lane in range(4):
        c = codes[:, lane]
        assert np.array_equal(re[:, lane], np.vectorize(want_re.get)(c).astype(np.float32))
        assert np.array_equal(im[:, lane], np.vectorize(want_im.get)(c).astype(np.float32))


@pytest.mark.parametrize("bits", (3, 4))
def test_bitstream_pack_roundtrip(bits):
    """3/4-bit extension: product pack_bits and oracle unpack_bits are inverses."""
    from rpfq_review_b200.packing import pack_bits
    g = torch.Generator().manual_seed(bits)
    codes = torch.randint(0, 1 << bits, (7, 256), generator=g, dtype=torch.int64).to(torch.uint8)
    packed = pack_bits(codes, bits).numpy()
    assert packed.shape == (7, 256 * bits // 8)
    assert np.array_equal(pr.unpack_bits(packed, 256, bits), codes.numpy())


def test_synthetic_generator_seeded():
    """random_packed is deterministic and follows the stated distribution."""
    from rpfq_review_b200.packing import random_packed
    a = random_packed(100, 300, seed=3)
    b = random_packed(100, 300, seed=3)
    for k in a.planes:
        for x, y in zip(a.planes[k], b.planes[k]):
            assert torch.equal(x, y)
    assert a.n_cp == 256 and a.k_cp == 512
    codes = pr.unpack_codes(a.planes["u_s0"][0].numpy(), 256, 512)
    assert codes[100:].max() == 0 and codes[:, 300:].max() == 0  # padding codes 0
    hist = np.bincount(codes[:100, :300].ravel(), minlength=4) / 30000.0
    assert np.all(np.abs(hist - 0.25) < 0.02)
    g = a.planes["u_s0"][1].float().numpy()
    assert np.all(g[:, 0] == g[:, 1])  # broadcast over 256-column blocks
    s = 1.0 / g[:, 0]
    assert abs(np.log(s).mean()) < 0.1 and abs(np.log(s).std() - 0.5) < 0.1


def test_packed_state_dict_validation():
    """from_state_dict validates like loadPhaseParams (phase_linear.cpp:42-88)."""
    from rpfq_review_b200.packing import PackedLayer, random_packed
    layer = random_packed(40, 72, seed=1)
    sd = layer.state_dict("blk.")
    back = PackedLayer.from_state_dict(sd, "blk.", 144, 80)
    assert back.stages == 2 and back.n_cp == 256 and back.k_cp == 256
    bad = dict(sd)
    bad["blk.u_s1.gamma_real"] = torch.zeros_like(sd["blk.u_s1.gamma_real"])
    with pytest.raises(ValueError, match="Zero gamma"):
        PackedLayer.from_state_dict(bad, "blk.", 144, 80)
    bad = dict(sd)
    bad["blk.w_s0.codes"] = sd["blk.w_s0.codes"][:, :10]
    with pytest.raises(ValueError, match="shape mismatch"):
        PackedLayer.from_state_dict(bad, "blk.", 144, 80)
    bad = dict(sd)
    del bad["blk.w_s1.gamma_imag"]
    with pytest.raises(ValueError, match="Missing packed tensor"):
        PackedLayer.from_state_dict(bad, "blk.", 144, 80)
    with pytest.raises(ValueError, match="even"):
        PackedLayer.from_state_dict(sd, "blk.", 143, 80)


def test_drop_in_constructor_errors():
    """QATLinearComplexPhase keeps the reference constructor's error behaviour."""
    from rpfq_review_b200 import QATLinearComplexPhase
    with pytest.raises(ValueError, match="even"):
        QATLinearComplexPhase("complex_phase_v2", "complex_phase_v2", in_features=7, out_features=8)
    with pytest.raises(ValueError, match="Unsupported"):
        QATLinearComplexPhase("nope", "complex_phase_v2", in_features=8, out_features=8)
    with pytest.raises(NotImplementedError):
        QATLinearComplexPhase("complex_phase_next_v1", "complex_phase_v2", in_features=8, out_features=8)
    layer = QATLinearComplexPhase("complex_phase_v2", "complex_phase_v2", True, 4, False, 32, 16, 8)
    assert layer.in_features == 16 and layer.out_features == 8 and layer.stages == 2
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.zeros(2, 16))


VISION_CASES = ["vitb", "nocls", "all_salient", "no_salient", "grid4", "zero_token", "fallback_tokens",
                "fallback_2d"]


@pytest.mark.parametrize("name", VISION_CASES)
def test_vision_oracle_matches_reference_golden(name):
    """oracle/vision_ref.py restates VisionAwareActivationQuantizer
    (quant_rpfq_vit_vision.py:26-171): same saliency mask, quantized values
    bit for bit (golden_vision.npz, produced by the reference class)."""
    from oracle import vision_ref as vr
    g = np.load(os.path.join(GOLD, "golden_vision.npz"))
    ratio, clip, wgt, cls = (float(v) for v in g[f"{name}.params"])
    xr, xi = g[f"{name}.x_real"].astype(np.float32), g[f"{name}.x_imag"].astype(np.float32)
    qr, qi, mask = vr.vision_act_quant(xr, xi, ratio, clip, wgt, bool(cls))
    assert np.array_equal(mask.astype(np.uint8), g[f"{name}.mask"])
    assert np.array_equal(qr.view(np.uint32), g[f"{name}.q_real"].view(np.uint32))
    assert np.array_equal(qi.view(np.uint32), g[f"{name}.q_imag"].view(np.uint32))
