"""GPU tests of the GEMM's stream-K tail (CTA pairs whose 256 x 256 tiles do
not fill whole waves: the last one to two waves are shared out by k-blocks;
a tile cut between two pairs continues, in the second pair's TMEM, from the
first pair's fp32 accumulator).

Each case checks that the plan really takes the tail (rpfq_gemm_plan_sm100),
compares the result with float64, checks that it is bit-identical to the
data-parallel schedule of the same tiles (no workspace) — a cut tile runs the
same operations as an uncut one — and that the flag words at the end of the
workspace are back to zero."""

import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3

# (m, n, k, epilogue): shapes whose last wave of pair tiles is more than half
# full (the narrow tail takes the emptier ones) and idles long enough for the
# tail (rpfq_b200.cu plan_gemm): 114 pair tiles on 74 pairs with K = 4096
# (idle 0.46 of a 64-k-block wave), ragged m, GELU, and fp32 output over 416
# tiles.
CASES = [
    (9728, 768, 4096, "residual_f32"),
    (9700, 768, 4096, "none"),
    (4864, 1536, 4096, "gelu"),
    (13312, 2048, 4096, "f32"),
]


def _inputs(m, n, k, epi, dev):
    g = torch.Generator().manual_seed(m * 7 + n * 3 + k)
    x = torch.randn(m, k, generator=g).half()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, generator=g) * 0.1).half()
    r = torch.randn(m, n, generator=g) if epi == "residual_f32" else None
    return x.to(dev), w.to(dev), b.to(dev), (r.to(dev) if r is not None else None)


def _run(ops, x, w, b, r, epi, split_k):
    out_dtype = torch.float32 if epi in ("residual_f32", "f32") else torch.float16
    out = r.clone() if r is not None else torch.empty(x.shape[0], w.shape[0], dtype=out_dtype, device=x.device)
    return ops.gemm(x, w, b, residual=out if r is not None else None, out=out,
                    activation="gelu" if epi == "gelu" else "none", split_k=split_k)


@pytest.mark.parametrize("m,n,k,epi", CASES)
def test_stream_k_tail(cuda, m, n, k, epi):
    from rpfq_review_b200 import _lib, ops
    out_dtype = torch.float32 if epi in ("residual_f32", "f32") else torch.float16
    plan = ops.gemm_plan(m, n, k, out_dtype=out_dtype, residual=epi == "residual_f32", device=cuda)
    assert plan["cta_pair"] == 2 and plan["stream_k_tiles"] > 0, plan
    assert plan["units"] <= plan["stream_k_tiles"] < 2 * plan["units"]
    dp = ops.gemm_plan(m, n, k, out_dtype=out_dtype, residual=epi == "residual_f32", split_k=1, cta_pair=2,
                       device=cuda)
    assert dp["stream_k_tiles"] == 0

    x, w, b, r = _inputs(m, n, k, epi, cuda)
    y_sk = _run(ops, x, w, b, r, epi, 0)
    y_sk2 = _run(ops, x, w, b, r, epi, 0)
    y_dp = ops.gemm(x, w, b, residual=(r.clone() if r is not None else None),
                    out=(r.clone() if r is not None else None), out_dtype=out_dtype,
                    activation="gelu" if epi == "gelu" else "none", split_k=1, cta_pair=2)
    torch.cuda.synchronize(cuda)
    assert torch.equal(y_sk, y_sk2), "stream-K results differ between two calls"
    lin = x.double() @ w.double().T + b.double()
    ref = torch.nn.functional.gelu(lin) if epi == "gelu" else lin
    if r is not None:
        ref = ref + r.double()
    assert rel_err(y_sk.cpu().numpy(), ref.cpu().numpy()) < TOL
    assert torch.equal(y_sk, y_dp), "stream-K and data-parallel schedules differ"
    ws = ops._workspaces[(cuda.index, torch.cuda.current_stream(cuda).cuda_stream)]
    assert int(ws[-8192:].count_nonzero()) == 0, "stream-K flags left set"
    assert _lib.device_error() == 0


def test_stream_k_only_where_it_pays(cuda):
    """A last wave at most half full takes the narrow tail instead; a short K
    keeps whole tiles (the tail's fixup costs more than its short wave);
    without a workspace nothing takes the tail."""
    from rpfq_review_b200 import ops
    for n in (768, 2304, 3072):
        plan = ops.gemm_plan(6304, n, 768, device=cuda)
        assert plan["stream_k_tiles"] == 0 and plan["pieces"] > 0
    assert ops.gemm_plan(9728, 768, 768, device=cuda)["stream_k_tiles"] == 0  # K = 768
    assert ops.gemm_plan(9728, 768, 4096, split_k=1, device=cuda)["stream_k_tiles"] == 0
    assert ops.gemm_plan(50432, 768, 3072, device=cuda)["stream_k_tiles"] == 0  # 591 tiles: last wave 99 % full


def test_stream_k_in_cuda_graph(cuda):
    """The tail replays from a CUDA graph: the flags are cleared inside every
    replay, so consecutive replays stay bit-identical."""
    from rpfq_review_b200 import ops
    x, w, b, r = _inputs(9728, 768, 4096, "none", cuda)
    assert ops.gemm_plan(9728, 768, 4096, device=cuda)["stream_k_tiles"] > 0
    out = torch.empty(9728, 768, dtype=torch.float16, device=cuda)
    ref = ops.gemm(x, w, b).clone()
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(side):
        ops.gemm(x, w, b, out=out)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            ops.gemm(x, w, b, out=out)
        for _ in range(3):
            out.zero_()
            g.replay()
    torch.cuda.current_stream(cuda).wait_stream(side)
    torch.cuda.synchronize(cuda)
    assert torch.equal(out, ref)
