"""GPU parity tests of the sm_100a kernels through the C ABI (needs a B200).

Bars (stated per test):
* K1 decode (prepack): bit-exact fp16 against the oracle's restatement of
  buildFusedWideLinearCache (RNE) and against the reference C++ cache
  (ties-away mode).
* activation quantization: bit-exact fp16 against fp16(ActivationQuantSTE).
* GEMM / layer: max|y - y_ref| / max|y_ref| <= 1e-3 against the float64
  oracle; the GEMM against the fp16 coefficients
  it consumes is held to 2e-3 of the element-wise fp16 output rounding bound.
"""

import os

import numpy as np
import pytest
import torch

from oracle import packed_ref as pr
from tests.helpers import elem_rel_err, from_numpy_packed, rel_err, to_numpy_packed

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-3


def _ops():
    from rpfq_review_b200 import ops
    return ops


@pytest.mark.parametrize("n_c,k_c,stages", [(384, 384, 2), (1152, 384, 2), (40, 72, 2), (500, 384, 2),
                                            (48, 48, 2), (37, 130, 1), (64, 300, 3), (96, 260, 4)])
def test_prepack_bit_exact(cuda, n_c, k_c, stages):
    from rpfq_review_b200.packing import random_packed
    layer = random_packed(n_c, k_c, seed=n_c * 7 + k_c, stages=stages, device=cuda)
    dense = _ops().prepack(layer).cpu().numpy()
    want = pr.dense_fp16_from_planes(pr.coefficient_planes(to_numpy_packed(layer), n_c, k_c))
    assert dense.shape == (2 * n_c, 2 * k_c)
    assert np.array_equal(dense.view(np.uint16), want.view(np.uint16))


def test_prepack_ties_away_matches_reference_cpp(cuda):
    """Ties-away mode reproduces the reference's buildFusedWideLinearCache
    output (golden_refcpp.npz) bit for bit."""
    g = np.load(os.path.join(GOLD, "golden_refcpp.npz"))
    n_c, k_c = (int(v) for v in g["dims"])
    packed = {k[len("packed."):]: g[k] for k in g.files if k.startswith("packed.")}
    layer = from_numpy_packed(packed, n_c, k_c, cuda)
    dense = _ops().prepack(layer, rounding="ties_away").cpu().numpy().view(np.uint16)
    planes = {"rr": dense[:n_c, :k_c], "ir": dense[:n_c, k_c:], "ri": dense[n_c:, :k_c], "ii": dense[n_c:, k_c:]}
    for key, val in planes.items():
        assert np.array_equal(val, g[f"plane.{key}"].view(np.uint16)), key


def test_prepack_exhaustive_codes(cuda):
    """Every byte value 0..255 in every one of the 4 planes (all 4 lanes of
    each byte), against the oracle decode, bit for bit."""
    from rpfq_review_b200.packing import random_packed
    n_c, k_c = 1024, 4  # row r: plane r // 256 holds byte value r % 256
    layer = random_packed(n_c, k_c, seed=5, device="cpu")
    for p, name in enumerate(("u_s0", "u_s1", "w_s0", "w_s1")):
        codes = layer.planes[name][0].clone()
        codes[p * 256:(p + 1) * 256, 0] = torch.arange(256, dtype=torch.uint8)
        layer.planes[name] = (codes, *layer.planes[name][1:])
    np_layer = to_numpy_packed(layer)
    dense = _ops().prepack(layer.to(cuda)).cpu().numpy()
    want = pr.dense_fp16_from_planes(pr.coefficient_planes(np_layer, n_c, k_c))
    assert np.array_equal(dense.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("bits", (3, 4))
def test_prepack_wide_codes(cuda, bits):
    """3/4-bit uniform-phase extension against the oracle (bit-exact)."""
    from rpfq_review_b200.packing import random_packed
    layer = random_packed(200, 300, seed=bits, code_bits=bits, device=cuda)
    dense = _ops().prepack(layer).cpu().numpy()
    want = pr.dense_fp16_from_planes(pr.coefficient_planes(to_numpy_packed(layer), 200, 300, code_bits=bits))
    assert np.array_equal(dense.view(np.uint16), want.view(np.uint16))


GEMM_SHAPES = [
    # (m, n, k)
    (1576, 768, 768),     # cfg1: ViT-B proj at batch 8
    (1576, 2304, 768),    # ViT-B qkv
    (394, 3072, 768),     # ViT-B fc1
    (394, 768, 3072),     # ViT-B fc2
    (1, 768, 768),
    (127, 1000, 768),     # head, partial last tile
    (129, 96, 96),        # Swin-T stage-1 proj (K tail 96 = 64 + 32)
    (300, 264, 136),
    (5000, 384, 384),
]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("block_n,cta_pair", [(0, 0), (128, 0), (256, 1), (256, 2)])
def test_gemm_matches_fp64(cuda, m, n, k, block_n, cta_pair):
    g = torch.Generator().manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g).half()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, generator=g) * 0.1).half()
    y = _ops().gemm(x.to(cuda), w.to(cuda), b.to(cuda), block_n=block_n, cta_pair=cta_pair).cpu()
    ref = x.double() @ w.double().T + b.double()
    assert rel_err(y.numpy(), ref.numpy()) < TOL
    # fp32 accumulation: every element within its fp16 output rounding + accumulation slack
    err = (y.double() - ref).abs()
    assert torch.all(err <= ref.abs() * 2.0 ** -10 + 1e-3 * ref.abs().max())
    # element-wise relative error, floor 1e-3 of max|ref| (the same operands, so only
    # accumulation order and the fp16 output rounding of 2^-11 remain)
    assert elem_rel_err(y.numpy(), ref.numpy(), floor=1e-3) < 2e-3


@pytest.mark.parametrize("m,n,k", [(777, 3072, 768), (390, 768, 3072)])
@pytest.mark.parametrize("cta_pair", [1, 2])
def test_gemm_epilogue_gelu_residual(cuda, m, n, k, cta_pair):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(m, k, generator=g).half()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, generator=g) * 0.1).half()
    r = torch.randn(m, n, generator=g).half()
    y = _ops().gemm(x.to(cuda), w.to(cuda), b.to(cuda), residual=r.to(cuda), activation="gelu", block_n=256,
                    cta_pair=cta_pair).cpu()
    lin = x.double() @ w.double().T + b.double()
    ref = torch.nn.functional.gelu(lin) + r.double()
    assert rel_err(y.numpy(), ref.numpy()) < TOL


def test_gemm_strided_rows(cuda):
    """x and y as column slices of wider buffers (row strides != row length)."""
    g = torch.Generator().manual_seed(4)
    big = torch.randn(300, 1024, generator=g).half().to(cuda)
    w = (torch.randn(256, 768, generator=g) / 28.0).half().to(cuda)
    out = torch.zeros(300, 512, dtype=torch.float16, device=cuda)
    _ops().gemm(big[:, 128:896], w, out=out[:, 128:384])
    ref = big[:, 128:896].double() @ w.double().T
    assert rel_err(out[:, 128:384].cpu().numpy(), ref.cpu().numpy()) < TOL
    assert torch.all(out[:, :128] == 0) and torch.all(out[:, 384:] == 0)


@pytest.mark.parametrize("m,n,k", [(1576, 768, 768), (300, 1000, 768), (129, 96, 96), (700, 768, 3072),
                                   (257, 384, 1536)])
@pytest.mark.parametrize("cta_pair", [1, 2])
def test_gemm_fp32_output_and_residual(cuda, m, n, k, cta_pair):
    """fp32 output with an fp32 residual added in place (the model's residual stream)."""
    g = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, k, generator=g).half()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, generator=g) * 0.1).half()
    r = torch.randn(m, n, generator=g) * 3.0
    res = r.to(cuda)
    y = _ops().gemm(x.to(cuda), w.to(cuda), b.to(cuda), residual=res, out=res, block_n=256, cta_pair=cta_pair)
    assert y.data_ptr() == res.data_ptr() and y.dtype == torch.float32
    ref = x.double() @ w.double().T + b.double() + r.double()
    err = (y.cpu().double() - ref).abs()
    # fp32 output: only accumulation-order error remains
    assert float(err.max()) < 1e-5 * float(ref.abs().max()) * k ** 0.5
    y2 = _ops().gemm(x.to(cuda), w.to(cuda), b.to(cuda), residual=r.to(cuda), out_dtype=torch.float32, block_n=256,
                     cta_pair=cta_pair)
    assert torch.equal(y2, y)


SPLIT_SHAPES = [
    (198, 768, 3072),     # one image through ViT-B fc2
    (198, 2304, 768),     # one image through ViT-B qkv
    (1, 384, 1536),       # a single row
    (300, 1000, 768),     # partial last tile in m and n
    (129, 96, 96),        # two k-blocks, K tail
    (64, 256, 4096),
]


@pytest.mark.parametrize("m,n,k", SPLIT_SHAPES)
@pytest.mark.parametrize("split_k", [0, 2, 3, 8])
@pytest.mark.parametrize("block_n", [128, 256])
def test_gemm_split_k_matches_fp64(cuda, m, n, k, split_k, block_n):
    """Split-K over a cluster (forced counts and the automatic choice): bias
    + GELU into fp16, and bias + fp32 residual in place, against float64."""
    ops = _ops()
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, generator=g).half()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, generator=g) * 0.1).half()
    xc, wc, bc = x.to(cuda), w.to(cuda), b.to(cuda)
    lin = x.double() @ w.double().T + b.double()
    y = ops.gemm(xc, wc, bc, activation="gelu", block_n=block_n, cta_pair=1, split_k=split_k).cpu()
    ref = torch.nn.functional.gelu(lin)
    assert rel_err(y.numpy(), ref.numpy()) < TOL
    err = (y.double() - ref).abs()
    assert torch.all(err <= ref.abs() * 2.0 ** -10 + 1e-3 * ref.abs().max())
    r = torch.randn(m, n, generator=g) * 3.0
    res = r.to(cuda)
    y2 = ops.gemm(xc, wc, bc, residual=res, out=res, block_n=block_n, cta_pair=1, split_k=split_k)
    ref2 = lin + r.double()
    assert float((y2.cpu().double() - ref2).abs().max()) < 1e-5 * float(ref2.abs().max()) * k ** 0.5


@pytest.mark.parametrize("m,n,k", [(198, 768, 3072), (300, 1000, 768)])
def test_gemm_split_k_deterministic_and_close_to_one_pass(cuda, m, n, k):
    """Partials are summed in a fixed order: repeated calls are bit-identical;
    against the one-pass GEMM only the fp32 summation order differs."""
    ops = _ops()
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).half().to(cuda)
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half().to(cuda)
    b = (torch.randn(n, generator=g) * 0.1).to(cuda)
    outs = [ops.gemm(x, w, b, out_dtype=torch.float32, cta_pair=1, split_k=4) for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    one = ops.gemm(x, w, b, out_dtype=torch.float32, cta_pair=1, split_k=1)
    assert float((outs[0] - one).abs().max()) < 1e-5 * float(one.abs().max()) * k ** 0.5
    assert not torch.equal(outs[0], one) or k <= 256  # the split path really ran


def test_gemm_split_k_automatic_choice(cuda):
    """The automatic choice splits small-M, long-K products and leaves large
    ones alone; the workspace query bounds every automatic split and asks for
    the stream-K workspace exactly when a shape's pair tiles leave a tail."""
    from rpfq_review_b200 import _lib
    L = _lib.lib()
    full = L.rpfq_gemm_workspace_bytes(0, 0, 0)
    assert full >= 148 * 128 * 256 * 4
    small = L.rpfq_gemm_workspace_bytes(198, 768, 3072)
    assert 0 < small <= full
    assert L.rpfq_gemm_workspace_bytes(50432, 768, 768) == 0  # 591 pair tiles: last wave 99 % full
    assert L.rpfq_gemm_workspace_bytes(9728, 768, 4096) == full  # 114 pair tiles, long K: stream-K tail
    assert L.rpfq_gemm_workspace_bytes(6304, 768, 3072) == 0  # 75 pair tiles: narrow tail, no workspace
    assert L.rpfq_gemm_workspace_bytes(9728, 768, 768) == 0  # short K: whole tiles
    assert L.rpfq_gemm_workspace_bytes(198, 768, 128) == 0  # two k-blocks: nothing to split


@pytest.mark.parametrize("d", [96, 192, 384, 768, 1024, 1536, 3072])
@pytest.mark.parametrize("act_bits", [0, 4])
def test_layernorm_kernel(cuda, d, act_bits):
    """fp32 -> fp16 LayerNorm vs torch (fp16 rounding), and the fused
    act-quant equals LN followed by the act-quant kernel, bit for bit. m = 1003
    leaves the last warp of the 96- / 192-wide layouts (4 / 2 rows per warp)
    partly empty."""
    g = torch.Generator().manual_seed(d)
    m = 1003
    x = (torch.randn(m, d, generator=g) * 4 + 1).to(cuda)
    w = (torch.randn(d, generator=g) * 0.2 + 1).half().to(cuda)
    b = (torch.randn(d, generator=g) * 0.1).half().to(cuda)
    ops = _ops()
    h = ops.layernorm(x, w, b, 1e-6)
    ref = torch.nn.functional.layer_norm(x.double(), (d,), w.double(), b.double(), 1e-6)
    assert rel_err(h.cpu().numpy(), ref.cpu().numpy()) < 1e-3
    if act_bits:
        hq = ops.layernorm(x, w, b, 1e-6, act_bits=act_bits)
        want = ops.act_quant(h, act_bits)
        assert torch.equal(hq.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("bits", (2, 4, 8))
def test_act_quant_bit_exact(cuda, bits):
    g = np.load(os.path.join(GOLD, "golden_actquant.npz"))
    x = torch.from_numpy(g["x"]).half().to(cuda)
    y = _ops().act_quant(x, bits).cpu().numpy()
    want = g[f"q{bits}"].astype(np.float16)
    assert np.array_equal(y.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("m,k", [(1576, 768), (33, 3072), (5, 96), (3, 100)])
def test_act_quant_random_bit_exact(cuda, m, k):
    gen = torch.Generator().manual_seed(m * k)
    x = (torch.randn(m, k, generator=gen) * 2).half()
    y = _ops().act_quant(x.to(cuda), 4).cpu().numpy()
    want = pr.act_quant(x.float().numpy(), 4).astype(np.float16)
    assert np.array_equal(y.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("act_bits", [0, 4])
def test_layer_cfg1_vs_reference_path(cuda, act_bits):
    """cfg1 (M = 8 x 197, K = N = 768): the whole layer against the reference
    deployment path F.linear(act_quant(x), quantized_forward_weight) in float64."""
    from rpfq_review_b200 import PackedPhaseLinear
    from rpfq_review_b200.packing import random_packed
    layer = random_packed(384, 384, seed=0, device=cuda)
    mod = PackedPhaseLinear.from_packed(layer, enable_act_quant=act_bits > 0, act_num_bits=act_bits or 4)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1576, 768, generator=g).half()
    y = mod(x.to(cuda)).float().cpu().numpy()
    np_layer = to_numpy_packed(layer)
    dense = pr.dense_weight_from_packed(np_layer, 384, 384)
    ref = pr.wide_linear(x.float().numpy(), dense, np_layer["bias"].astype(np.float32),
                         act_bits=act_bits or None)
    assert rel_err(y, ref) < TOL
    # element-wise, on the operands the GEMM sees (the fp16 coefficient planes):
    # each output within 2e-3 of its own magnitude, floor 1e-3 of max|ref|; against
    # the float32 exporter weight the coefficients' own fp16 rounding (2^-12 per
    # weight) adds a cancellation term that only the normalised measure bounds
    # (and the GEMM input the quantizer writes, q / s stored as fp16)
    planes = pr.dense_fp16_from_planes(pr.coefficient_planes(np_layer, 384, 384)).astype(np.float32)
    xin = x.float().numpy()
    if act_bits:
        xin = pr.act_quant(xin, act_bits).astype(np.float16).astype(np.float32)
    ref16 = pr.wide_linear(xin, planes, np_layer["bias"].astype(np.float32))
    assert elem_rel_err(y, ref16, floor=1e-3) < 2e-3


def test_layer_against_reference_cpp_golden(cuda):
    """Against wideLinearReference of the reference's C++ runtime (golden)."""
    from rpfq_review_b200 import PackedPhaseLinear
    g = np.load(os.path.join(GOLD, "golden_refcpp.npz"))
    n_c, k_c = (int(v) for v in g["dims"])
    packed = {k[len("packed."):]: g[k] for k in g.files if k.startswith("packed.")}
    mod = PackedPhaseLinear.from_packed(from_numpy_packed(packed, n_c, k_c, cuda))
    y = mod(torch.from_numpy(g["x"]).to(cuda)).cpu().numpy()
    assert rel_err(y, g["y_reference"]) < TOL


@pytest.mark.parametrize("name", ["generic", "medium", "ties", "onestage"])
def test_drop_in_module_vs_exporter_golden(cuda, name):
    """QATLinearComplexPhase (drop-in) packs the float weight like the exporter
    and matches F.linear(x, quantized_forward_weight(W), b) from the golden."""
    from rpfq_review_b200 import QATLinearComplexPhase
    g = np.load(os.path.join(GOLD, "golden_exporter.npz"))
    n_c, k_c, stages = (int(v) for v in g[f"{name}.dims"])
    method = f"complex_phase_v{stages}"
    layer = QATLinearComplexPhase(method, method, False, 4, False, 32, 2 * k_c, 2 * n_c, bias=True).to(cuda)
    with torch.no_grad():
        layer.weight.copy_(torch.from_numpy(g[f"{name}.weight"]))
        layer.bias.copy_(torch.from_numpy(g[f"{name}.bias_f32"]))
    x = torch.from_numpy(g[f"{name}.x"]).to(cuda)
    y = layer(x).cpu().numpy()
    # the GPU path sees x in fp16; compare against the reference path on the same input
    ref = pr.wide_linear(x.half().float().cpu().numpy(), g[f"{name}.dense"], g[f"{name}.bias"].astype(np.float32))
    assert rel_err(y, ref) < TOL
    assert rel_err(y, g[f"{name}.y"]) < 2e-3  # includes fp16 rounding of x itself


@pytest.mark.parametrize("act_bits", [0, 4])
def test_drop_in_module_vs_qat_reference(cuda, act_bits):
    """The drop-in against the reference's own QAT forward
    (QATLinearComplexPhase.forward, golden_qat.npz y_act0 / y_act1, made by
    the reference class). The drop-in packs like the exporter, and the
    exporter and the QAT forward part at two second-stage axis decisions of
    this weight (tests/test_qat_gap_cpu.py): with those two codes imposed on
    the restated QAT forward (float32 scales, oracle/qat_ref.py) the drop-in
    is within the 1e-3 layer bar; against the raw golden it is within the
    reference's own exporter-vs-QAT gap, measured from the goldens here, plus
    1e-3."""
    from oracle import qat_ref
    from rpfq_review_b200 import QATLinearComplexPhase
    g = np.load(os.path.join(GOLD, "golden_exporter.npz"))
    q = np.load(os.path.join(GOLD, "golden_qat.npz"))
    n_c, k_c = 40, 72
    layer = QATLinearComplexPhase("complex_phase_v2", "complex_phase_v2", act_bits > 0, act_bits or 4, False, 32,
                                  2 * k_c, 2 * n_c, bias=True).to(cuda)
    with torch.no_grad():
        layer.weight.copy_(torch.from_numpy(g["generic.weight"]))
        layer.bias.copy_(torch.from_numpy(g["generic.bias_f32"]))
    x = torch.from_numpy(g["generic.x"]).to(cuda).half()
    y = layer(x).float().cpu().numpy()
    x16 = x.float().cpu().numpy()
    ref = pr.wide_linear(x16, g["generic.dense"], g["generic.bias"].astype(np.float32), act_bits=act_bits or None)
    assert rel_err(y, ref) < TOL
    codes = {}
    for tag in "uw":
        c = g[f"generic.{tag}_s1.codes"]
        codes[tag] = [None, pr.unpack_codes(c, c.shape[0], c.shape[1] * 4)[:n_c, :k_c]]
    forced = qat_ref.forward(g["generic.weight"], g["generic.bias_f32"], x16, act_bits, force_codes=codes)
    assert rel_err(y, forced) < TOL
    golden = q["y_act1" if act_bits else "y_act0"]
    gap = rel_err(ref, golden)  # the reference's exporter-vs-QAT gap on this weight (fp16 x)
    assert rel_err(y, golden) < gap + TOL


def test_cuda_graph_capture_replays(cuda):
    """The layer launches no host sync and captures into a CUDA graph."""
    from rpfq_review_b200 import PackedPhaseLinear
    from rpfq_review_b200.packing import random_packed
    mod = PackedPhaseLinear.from_packed(random_packed(384, 384, seed=2, device=cuda), activation="gelu")
    x = torch.randn(512, 768, device=cuda).half()
    y0 = mod(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        mod(x)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = mod(x)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y0)


def test_no_device_errors_recorded(cuda):
    from rpfq_review_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_gemm_fp32_bias_matches_fp16_bias(cuda, out_dtype):
    """RPFQ_GEMM_BIAS_F32: the same bias values widened to fp32 give
    bit-identical outputs (the epilogue adds in fp32 either way)."""
    ops = _ops()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(300, 256, generator=g).half().to(cuda)
    w = (torch.randn(512, 256, generator=g) * 0.05).half().to(cuda)
    b16 = (torch.randn(512, generator=g) * 0.1).half().to(cuda)
    for act in ("none", "gelu"):
        y16 = ops.gemm(x, w, b16, activation=act, out_dtype=out_dtype)
        y32 = ops.gemm(x, w, b16.float(), activation=act, out_dtype=out_dtype)
        assert torch.equal(y16, y32)


def test_layernorm_row_gather(cuda):
    """rpfq_layernorm_rows_sm100: output row r is LN(x[rows[r]]), bit-identical
    to the ungathered kernel's row; an index outside x is reported through the
    device error word (code 901) and its output row is left untouched."""
    from rpfq_review_b200 import _lib
    ops = _ops()
    g = torch.Generator().manual_seed(5)
    m, d = 3136, 96
    x = torch.randn(m, d, generator=g).to(cuda)
    w = (torch.randn(d, generator=g) * 0.2 + 1).half().to(cuda)
    b = (torch.randn(d, generator=g) * 0.1).half().to(cuda)
    perm = torch.randperm(m, generator=g).to(torch.int32).to(cuda)
    full = ops.layernorm(x, w, b, 1e-5, act_bits=4)
    gathered = ops.layernorm(x, w, b, 1e-5, act_bits=4, rows=perm)
    assert torch.equal(gathered, full[perm.long()])
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    bad = perm.clone()
    bad[10] = m + 5
    out = torch.zeros(m, d, dtype=torch.float16, device=cuda)
    ops.layernorm(x, w, b, 1e-5, rows=bad, out=out)
    torch.cuda.synchronize()
    assert _lib.device_error() == 901
    assert torch.count_nonzero(out[10]) == 0
    # the rows that share a warp with the bad one (four 96-wide rows per warp) are written as usual
    full0 = ops.layernorm(x, w, b, 1e-5)
    keep = torch.arange(m, device=cuda) != 10
    assert torch.equal(out[keep], full0[perm.long()][keep])


@pytest.mark.parametrize("c,side,act_bits", [(96, 56, 0), (192, 28, 4), (384, 14, 0)])
def test_layernorm_patch_merge_gather(cuda, c, side, act_bits):
    """rpfq_layernorm_ex_sm100 with merge_side: bit-identical to the plain
    kernel on torch's concatenation of the four strided slices (Swin
    PatchMerging), for the three Swin-T merges."""
    ops = _ops()
    g = torch.Generator().manual_seed(c)
    B = 3
    x = torch.randn(B, side * side, c, generator=g).to(cuda)
    w = (torch.randn(4 * c, generator=g) * 0.2 + 1).half().to(cuda)
    b = (torch.randn(4 * c, generator=g) * 0.1).half().to(cuda)
    xs = x.view(B, side, side, c)
    cat = torch.cat([xs[:, 0::2, 0::2], xs[:, 1::2, 0::2], xs[:, 0::2, 1::2], xs[:, 1::2, 1::2]], dim=-1)
    want = ops.layernorm(cat.reshape(-1, 4 * c).contiguous(), w, b, 1e-5, act_bits=act_bits)
    got, _ = ops.layernorm_ex(x, w, b, 1e-5, act_bits, merge_side=side)
    assert torch.equal(got, want)


@pytest.mark.parametrize("d", [96, 384, 768])
def test_layernorm_permuted_residual_add(cuda, d):
    """rpfq_layernorm_ex_sm100 with add / add_rows and an in-place y32: the
    residual stream becomes x + add[add_rows] (exactly: one fp32 add per
    element) and the fp16 output is the plain kernel's LayerNorm of it; an
    add index outside [0, add_bound) is reported as code 902."""
    from rpfq_review_b200 import _lib
    ops = _ops()
    g = torch.Generator().manual_seed(d)
    m = 2 * 3136
    x = torch.randn(m, d, generator=g).to(cuda)
    o = torch.randn(m, d, generator=g).to(cuda)
    w = (torch.randn(d, generator=g) * 0.2 + 1).half().to(cuda)
    b = (torch.randn(d, generator=g) * 0.1).half().to(cuda)
    inv = torch.randperm(m, generator=g).to(torch.int32).to(cuda)
    want_x = x + o[inv.long()]
    want_h = ops.layernorm(want_x, w, b, 1e-5, act_bits=4)
    xs = x.clone()
    h, z = ops.layernorm_ex(xs, w, b, 1e-5, 4, add=o, add_rows=inv, out32=xs, out32_prenorm=True)
    assert z.data_ptr() == xs.data_ptr()
    assert torch.equal(xs, want_x)
    assert torch.equal(h, want_h)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    bad = inv.clone()
    bad[7] = m
    ops.layernorm_ex(x.clone(), w, b, 1e-5, add=o, add_rows=bad, out32=torch.zeros_like(x), out32_prenorm=True)
    torch.cuda.synchronize()
    assert _lib.device_error() == 902


@pytest.mark.parametrize("d", [96, 768])
def test_layernorm_fp32_output(cuda, d):
    """fp32 output of the normalized rows (Swin's patch-embedding norm, in
    place): within fp32 rounding of torch's LayerNorm, and its fp16 rounding
    equals the kernel's own fp16 output."""
    ops = _ops()
    g = torch.Generator().manual_seed(d + 1)
    x = torch.randn(4096, d, generator=g).to(cuda) * 3 + 1
    w = (torch.randn(d, generator=g) * 0.2 + 1).half().to(cuda)
    b = (torch.randn(d, generator=g) * 0.1).half().to(cuda)
    ref = torch.nn.functional.layer_norm(x.double(), (d,), w.double(), b.double(), 1e-5)
    h16 = ops.layernorm(x, w, b, 1e-5)
    y = x.clone()
    ops.layernorm_ex(y, w, b, 1e-5, fp16_out=False, out32=y)
    assert float((y.double() - ref).abs().max()) < 1e-5
    assert torch.equal(y.half(), h16)


def test_gelu_epilogue_accuracy(cuda):
    """The epilogue's GELU (A&S 7.1.26 erf, |error| <= 1.5e-7, with the SFU
    reciprocal and exp2) against float64 exact-erf GELU, read through an
    identity GEMM with fp32 output: |err| <= 5e-7 * max(1, |x|) for |x| <= 12,
    and the far tails (x for large x, 0 for very negative x)."""
    ops = _ops()
    k = 64
    vals = torch.cat([torch.linspace(-12, 12, 64 * 1000), torch.tensor([-40.0, -20.0, 20.0, 40.0, 0.0, -0.0])])
    m = (vals.numel() + k - 1) // k
    x = torch.zeros(m * k)
    x[: vals.numel()] = vals
    x = x.half().view(m, k)  # the GEMM operand is fp16: compare on the rounded values
    eye = torch.eye(k, dtype=torch.float16)
    y = ops.gemm(x.to(cuda), eye.to(cuda), None, activation="gelu", out_dtype=torch.float32).cpu().double()
    ref = torch.nn.functional.gelu(x.double())
    err = (y - ref).abs()
    bound = 5e-7 * torch.clamp(x.double().abs(), min=1.0)
    assert bool((err <= bound).all()), float((err / bound).max())


def _patchify_ref(images: torch.Tensor, p: int) -> torch.Tensor:
    """The reference's patchify_tensor (audit_rpfq_vit_ios_parity.py:125-134),
    batched: CHW patch order."""
    B, C, H, W = images.shape
    x = images.reshape(B, C, H // p, p, W // p, p).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(B, (H // p) * (W // p), C * p * p)


@pytest.mark.parametrize("B,C,H,W,p,dtype", [(3, 3, 224, 224, 16, torch.float16), (2, 3, 224, 224, 16, torch.float32),
                                             (2, 3, 32, 48, 8, torch.float16), (1, 1, 48, 16, 16, torch.float32),
                                             (0, 3, 224, 224, 16, torch.float16), (2, 3, 224, 224, 4, torch.float16),
                                             (1, 3, 32, 24, 4, torch.float32)])
def test_patch_unfold_bit_exact(cuda, B, C, H, W, p, dtype):
    """rpfq_patch_unfold_sm100 against the reference's patch order: bit-exact
    fp16 rows (fp32 images rounded to nearest even, as .to(float16)), into a
    fresh tensor and into a strided row view of a wider buffer."""
    ops = _ops()
    g = torch.Generator().manual_seed(B * 1000 + H + p)
    images = (torch.randn(B, C, H, W, generator=g) * 3).to(dtype).to(cuda)
    want = _patchify_ref(images.to(torch.float16), p)
    got = ops.patch_unfold(images, p)
    assert got.shape == want.shape
    assert torch.equal(got.view(torch.int16), want.contiguous().view(torch.int16))
    k = C * p * p
    wide = torch.full((B * (H // p) * (W // p), k + 24), 7.0, dtype=torch.float16, device=cuda)
    ops.patch_unfold(images, p, out=wide[:, :k])
    assert torch.equal(wide[:, :k].view(torch.int16), want.reshape(-1, k).view(torch.int16))
    assert bool((wide[:, k:] == 7.0).all())


def test_patch_unfold_rejects_bad_shapes(cuda):
    from rpfq_review_b200 import _lib
    ops = _ops()
    with pytest.raises(ValueError):
        ops.patch_unfold(torch.zeros(1, 3, 30, 32, dtype=torch.float16, device=cuda), 16)  # 16 does not divide 30
    out = torch.empty(4, 108, dtype=torch.float16, device=cuda)
    rc = _lib.lib().rpfq_patch_unfold_sm100(out.data_ptr(), 0, 1, 3, 12, 12, 6, out.data_ptr(), 108, None)
    assert rc != 0 and b"multiple of 4" in _lib.lib().rpfq_last_error()


@pytest.mark.parametrize("d,ntok", [(768, 1), (384, 2), (1024, 1)])
def test_layernorm_token_assembly(cuda, d, ntok):
    """The first LayerNorm pass of PackedViT assembles the residual stream: row
    (b, t) gathers source row t (class tokens) or ntok + b * patches + t - ntok
    (patch embeddings), adds position row t, writes the fp32 stream and its
    LayerNorm; both equal the torch assembly (one fp32 add) and the plain
    kernel's LayerNorm of it, bit for bit."""
    ops = _ops()
    g = torch.Generator().manual_seed(d + ntok)
    B, n_p = 5, 196
    L = n_p + ntok
    src = torch.randn(ntok + B * n_p, d, generator=g).to(cuda)
    pos = torch.randn(L, d, generator=g).to(cuda)
    w = (torch.randn(d, generator=g) * 0.2 + 1).half().to(cuda)
    b = (torch.randn(d, generator=g) * 0.1).half().to(cuda)
    t = torch.arange(L, dtype=torch.int32).repeat(B)
    bi = torch.arange(B, dtype=torch.int32).repeat_interleave(L)
    rows = torch.where(t < ntok, t, ntok + bi * n_p + (t - ntok)).to(torch.int32)
    want_x = torch.empty(B, L, d, device=cuda)
    want_x[:, :ntok] = src[:ntok] + pos[:ntok]
    want_x[:, ntok:] = src[ntok:].view(B, n_p, d) + pos[ntok:]
    want_h = ops.layernorm(want_x, w, b, 1e-6, act_bits=4)
    x = torch.empty(B, L, d, device=cuda)
    h, _ = ops.layernorm_ex(src, w, b, 1e-6, 4, rows=rows.to(cuda), add=pos, add_rows=t.to(cuda), out32=x,
                            out32_prenorm=True)
    assert torch.equal(x, want_x)
    assert torch.equal(h.view(B, L, d), want_h)
