"""GPU test of rpfq_wide_linear_noalloc_sm100, the allocation-free variant of
the whole-layer entry point (for callers that cannot allocate device memory
while they run a layer, e.g. a server request path that must not call the
synchronising cudaMalloc / cudaFree, or a plugin host with no allocator).

Called through the C ABI with ctypes, it must give the same output as the
allocating entry point rpfq_wide_linear_sm100 (given a caller scratch
buffer) bit for bit — both run the same kernels on the same inputs, only the
scratch address differs — on two calls in a row, and reject an m whose
quantized activations exceed its built-in scratch (also one whose byte count
would wrap a 64-bit product). This file sorts last so that a run stopping at
the first failure has already run every other test."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _args(layer_struct, dense, x, y, bias, act_bits, scratch=None):
    from rpfq_review_b200 import _lib
    return _lib.RpfqWideLinearArgs(layer=ctypes.pointer(layer_struct), dense=dense.data_ptr(), x=x.data_ptr(),
                                   ldx=x.shape[1], bias=bias.data_ptr(), residual=None, ldr=0, y=y.data_ptr(),
                                   ldy=y.shape[1], m=x.shape[0], act_bits=act_bits, activation=0,
                                   scratch=None if scratch is None else scratch.data_ptr(), flags=0)


def test_no_alloc_entry_matches_allocating_entry(cuda):
    from rpfq_review_b200 import _lib, ops
    from rpfq_review_b200.packing import random_packed

    lib = _lib.lib()
    layer = random_packed(384, 384, seed=21, device=cuda)
    dense = ops.prepack(layer)
    s = ops.layer_struct(layer)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call, m in enumerate((1576, 777)):  # two calls in a row, different inputs
        g = torch.Generator(device=cuda).manual_seed(100 + call)
        x = (torch.randn(m, 768, device=cuda, generator=g) * (1 + call)).half()
        y_ref = torch.empty(m, 768, dtype=torch.float16, device=cuda)
        scratch = torch.empty(m, 768, dtype=torch.float16, device=cuda)
        a_ref = _args(s, dense, x, y_ref, layer.bias, 4, scratch)
        _lib.check(lib.rpfq_wide_linear_sm100(ctypes.byref(a_ref), stream), "rpfq_wide_linear_sm100")
        y = torch.full((m, 768), float("nan"), dtype=torch.float16, device=cuda)
        a = _args(s, dense, x, y, layer.bias, 4)
        _lib.check(lib.rpfq_wide_linear_noalloc_sm100(ctypes.byref(a), stream), "rpfq_wide_linear_noalloc_sm100")
        torch.cuda.synchronize(cuda)
        assert torch.isfinite(y).all()  # the NaN fill shows any row left unwritten
        assert torch.equal(y, y_ref)
    # quantized activations larger than the built-in 8 MiB are refused, not overrun
    m_big = (8 << 20) // (768 * 2) + 1
    xb = torch.zeros(m_big, 768, dtype=torch.float16, device=cuda)
    yb = torch.empty(m_big, 768, dtype=torch.float16, device=cuda)
    rc = lib.rpfq_wide_linear_noalloc_sm100(ctypes.byref(_args(s, dense, xb, yb, layer.bias, 4)), stream)
    assert rc == _lib.RPFQ_ERR_INVALID
    assert b"scratch" in lib.rpfq_last_error()
    # an m so large that m * 2 k_c * 2 bytes wraps around 2^64 is refused the same way
    a_wrap = _args(s, dense, xb, yb, layer.bias, 4)
    a_wrap.m = (1 << 64) // (768 * 2) + 1
    assert lib.rpfq_wide_linear_noalloc_sm100(ctypes.byref(a_wrap), stream) == _lib.RPFQ_ERR_INVALID
    assert b"scratch" in lib.rpfq_last_error()
    assert _lib.device_error() == 0
