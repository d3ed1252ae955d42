"""CPU tests of the C-ABI library: it loads, exports every symbol that
include/rpfq_b200.h declares, and its host-side validation rejects bad
descriptors before anything touches a GPU (no compute call is made here)."""

import ctypes
import os
import re

import pytest

from rpfq_review_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(REPO, "include", "rpfq_b200.h")).read()
    return sorted(set(re.findall(r"\b(rpfq_[a-z0-9_]+)\s*\(", src)))


def test_header_matches_binding():
    assert _declared_symbols() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in _declared_symbols():
        assert hasattr(L, name), name
    assert L.rpfq_version() >= 100


def test_struct_layouts_match_header():
    """ctypes mirrors of the header structs have the C sizes."""
    assert ctypes.sizeof(_lib.RpfqPhasePlane) == 24
    assert ctypes.sizeof(_lib.RpfqPackedLinear) == 6 * 4 + 8 * 24
    assert ctypes.sizeof(_lib.RpfqGemmArgs) == 8 * 9 + 4 * 6 + 4 * 2 + 8 * 2
    assert ctypes.sizeof(_lib.RpfqWideLinearArgs) == 8 * 10 + 4 * 2 + 8 + 4 * 2 + 8 * 2


@pytest.mark.parametrize("bad", ["null", "k", "n", "ldx", "act", "block_n", "split_k", "split_no_ws",
                                 "ws_align", "split_pair"])
def test_gemm_validation_rejects_before_launch(bad):
    L = _lib.lib()
    a = _lib.RpfqGemmArgs(x=16, ldx=64, w=32, y=48, ldy=64, m=4, n=64, k=64)
    if bad == "null":
        a.x = None
    elif bad == "k":
        a.k = 60
    elif bad == "n":
        a.n = 12
    elif bad == "ldx":
        a.ldx = 32
    elif bad == "act":
        a.activation = 7
    elif bad == "block_n":
        a.block_n = 96
    elif bad == "split_k":
        a.split_k = 9
        a.workspace, a.workspace_bytes = 4096, 1 << 20
    elif bad == "split_no_ws":
        a.split_k = 4
    elif bad == "ws_align":
        a.workspace, a.workspace_bytes = 4100, 1 << 20
    elif bad == "split_pair":
        a.split_k, a.cta_pair = 2, 2
        a.workspace, a.workspace_bytes = 4096, 1 << 20
    rc = L.rpfq_gemm_sm100(ctypes.byref(a), None)
    if bad == "block_n":
        # block_n is checked after the device set-up, which needs a GPU
        assert rc != _lib.RPFQ_OK
        return
    assert rc == _lib.RPFQ_ERR_INVALID
    assert L.rpfq_last_error().decode()


def test_prepack_validation():
    L = _lib.lib()
    s = _lib.RpfqPackedLinear(n_c=10, k_c=10, n_cp=250, k_cp=256, stages=2, code_bits=2)
    assert L.rpfq_prepack_sm100(ctypes.byref(s), 16, 0, None) == _lib.RPFQ_ERR_INVALID
    assert b"multiples of 256" in L.rpfq_last_error()
    s.n_cp = 256
    s.stages = 5
    assert L.rpfq_prepack_sm100(ctypes.byref(s), 16, 0, None) == _lib.RPFQ_ERR_INVALID
    s.stages = 2
    assert L.rpfq_prepack_sm100(ctypes.byref(s), 16, 0, None) == _lib.RPFQ_ERR_INVALID  # null planes
    assert b"null" in L.rpfq_last_error()


def test_act_quant_validation():
    L = _lib.lib()
    assert L.rpfq_act_quant_sm100(16, 8, 16, 8, 4, 7, 4, None) == _lib.RPFQ_ERR_INVALID
    assert L.rpfq_act_quant_sm100(16, 8, 16, 8, 4, 8, 9, None) == _lib.RPFQ_ERR_INVALID
    assert L.rpfq_act_quant_sm100(None, 8, 16, 8, 4, 8, 4, None) == _lib.RPFQ_ERR_INVALID


def test_torch_ops_registered():
    import torch
    import rpfq_review_b200.ops  # noqa: F401
    for name in ("gemm", "act_quant", "prepack", "wide_linear", "wide_linear_dense"):
        assert hasattr(torch.ops.rpfq, name)
    # CUDA-only: a CPU call fails in the dispatcher instead of falling back
    with pytest.raises(Exception):
        torch.ops.rpfq.act_quant(torch.zeros(2, 8, dtype=torch.float16), 4)
    # the packed-layer op takes the reference's packed tensors (codes, gammas, bias, n_c, k_c, act_bits, gelu)
    schema = str(torch.ops.rpfq.wide_linear.default._schema)
    assert ("wide_linear(Tensor x, Tensor[] codes, Tensor[] gamma_re, Tensor[] gamma_im, Tensor? bias, int n_c, "
            "int k_c, int act_bits=0, bool gelu=False) -> Tensor") in schema
    with pytest.raises(Exception):
        torch.ops.rpfq.wide_linear(torch.zeros(2, 8, dtype=torch.float16), [torch.zeros(256, 64, dtype=torch.uint8)] * 2,
                                   [torch.zeros(256, 1, dtype=torch.float16)] * 2,
                                   [torch.zeros(256, 1, dtype=torch.float16)] * 2, None, 4, 4)


def test_pack_linear_validation():
    """rpfq_pack_linear_sm100 / rpfq_pack_workspace_bytes reject bad shapes,
    stage counts, strides and workspaces before any device work."""
    L = _lib.lib()
    assert L.rpfq_pack_workspace_bytes(0, 8) == 0
    ws = L.rpfq_pack_workspace_bytes(48, 40)
    assert ws >= 16 * 48 * 40
    outs = (_lib.RpfqPhasePlaneOut * 2)()
    for o in outs:
        o.codes, o.gamma_real, o.gamma_imag = 64, 128, 256
    args = dict(weight=16, ldw=80, n_c=48, k_c=40, stages=2, ws=4096, ws_bytes=ws)

    def call(**kw):
        a = {**args, **kw}
        return L.rpfq_pack_linear_sm100(a["weight"], a["ldw"], a["n_c"], a["k_c"], a["stages"], outs, outs,
                                        a["ws"], a["ws_bytes"], None)

    assert call(weight=None) == _lib.RPFQ_ERR_INVALID
    assert call(n_c=0) == _lib.RPFQ_ERR_INVALID
    assert call(stages=5) == _lib.RPFQ_ERR_INVALID and b"stages" in L.rpfq_last_error()
    assert call(ldw=60) == _lib.RPFQ_ERR_INVALID and b"ldw" in L.rpfq_last_error()
    assert call(ws=4100) == _lib.RPFQ_ERR_INVALID  # not 16-byte aligned
    assert call(ws_bytes=ws - 1) == _lib.RPFQ_ERR_INVALID and b"workspace" in L.rpfq_last_error()


def test_vision_attention_layernorm_validation():
    L = _lib.lib()
    # vision-aware quantizer: the reference's ValueError messages
    assert L.rpfq_vision_act_quant_sm100(16, 64, 16, 64, 2, 197, 64, 1.5, 0.75, 0.5, 1, None, None, 0,
                                         None) == _lib.RPFQ_ERR_INVALID
    assert b"salient_token_ratio must be in [0, 1]." in L.rpfq_last_error()
    assert L.rpfq_vision_act_quant_sm100(16, 64, 16, 64, 2, 197, 64, 0.25, 0.0, 0.5, 1, None, None, 0,
                                         None) == _lib.RPFQ_ERR_INVALID
    assert L.rpfq_vision_act_quant_sm100(16, 64, 16, 64, 2, 197, 60, 0.25, 0.75, 0.5, 1, None, None, 0,
                                         None) == _lib.RPFQ_ERR_INVALID  # k % 16
    assert L.rpfq_vision_workspace_bytes(2, 197) == 24 * 2 * 197
    # attention: head dim 64 and <= 256 tokens only
    assert L.rpfq_attention_sm100(16, 2, 197, 12, 80, 32, 768, None) == _lib.RPFQ_ERR_UNSUPPORTED
    assert L.rpfq_attention_sm100(16, 2, 300, 12, 64, 32, 768, None) == _lib.RPFQ_ERR_UNSUPPORTED
    assert L.rpfq_attention_sm100(None, 2, 197, 12, 64, 32, 768, None) == _lib.RPFQ_ERR_INVALID
    # LayerNorm gather: misaligned index array
    assert L.rpfq_layernorm_rows_sm100(16, 96, 10, 18, 16, 16, 16, 96, 10, 96, ctypes.c_float(1e-5), 0,
                                       None) == _lib.RPFQ_ERR_INVALID


def test_patch_unfold_validation():
    """rpfq_patch_unfold_sm100 rejects bad shapes, strides and alignment on the
    host, before any device work (no GPU needed)."""
    L = _lib.lib()
    # images pointer, f32, batch, channels, height, width, patch, out pointer, ldp, stream
    assert L.rpfq_patch_unfold_sm100(None, 0, 1, 3, 224, 224, 16, 16, 768, None) == _lib.RPFQ_ERR_INVALID
    assert L.rpfq_patch_unfold_sm100(16, 0, 1, 3, 224, 224, 6, 16, 768, None) == _lib.RPFQ_ERR_INVALID  # patch % 4
    assert b"multiple of 4" in L.rpfq_last_error()
    assert L.rpfq_patch_unfold_sm100(16, 0, 1, 3, 224, 200, 16, 16, 768, None) == _lib.RPFQ_ERR_INVALID  # 16 ∤ 200
    assert L.rpfq_patch_unfold_sm100(16, 0, 1, 3, 224, 224, 16, 16, 700, None) == _lib.RPFQ_ERR_INVALID  # ldp < 768
    assert L.rpfq_patch_unfold_sm100(16, 0, 1, 3, 224, 224, 16, 16, 772, None) == _lib.RPFQ_ERR_INVALID  # ldp % 8
    assert L.rpfq_patch_unfold_sm100(16, 0, 1, 3, 224, 224, 4, 16, 50, None) == _lib.RPFQ_ERR_INVALID  # ldp % 4
    assert L.rpfq_patch_unfold_sm100(8, 0, 1, 3, 224, 224, 16, 16, 768, None) == _lib.RPFQ_ERR_INVALID  # alignment
    assert b"16-byte aligned" in L.rpfq_last_error()
    assert L.rpfq_patch_unfold_sm100(16, 0, 0, 3, 224, 224, 16, 16, 768, None) == _lib.RPFQ_OK  # no images


def test_patch_unfold_wrapper_rejects_cpu_tensors():
    import torch
    from rpfq_review_b200 import ops
    with pytest.raises(ValueError):
        ops.patch_unfold(torch.zeros(1, 3, 32, 32), 16)


def test_noalloc_size_guard_on_host():
    """rpfq_wide_linear_noalloc_sm100 refuses, before any device work, an m
    whose quantized activations exceed its built-in scratch — including an m
    so large that m * 2 k_c * 2 bytes would wrap a 64-bit product."""
    L = _lib.lib()
    s = _lib.RpfqPackedLinear(n_c=384, k_c=384, n_cp=512, k_cp=512, stages=2, code_bits=2)
    for arr in (s.u, s.w):
        for i in range(2):
            arr[i].codes, arr[i].gamma_real, arr[i].gamma_imag = 4096, 8192, 12288
    a = _lib.RpfqWideLinearArgs(layer=ctypes.pointer(s), dense=16, x=32, ldx=768, y=48, ldy=768, act_bits=4)
    for m in ((8 << 20) // (768 * 2) + 1, (1 << 64) // (768 * 2) + 1):
        a.m = m
        assert L.rpfq_wide_linear_noalloc_sm100(ctypes.byref(a), None) == _lib.RPFQ_ERR_INVALID
        assert b"scratch" in L.rpfq_last_error()
