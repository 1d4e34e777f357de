"""Concurrent calls on two CUDA streams: each (device, stream) has its own scratch workspace
(activation split, fp16 activation and row scales, split-K partial planes), so GEMV and GEMM calls running at the same
time on different streams give the same bits as the same calls on one stream."""

import pytest
import torch

from tests.helpers import rel_err
from xanosmerks_b200.ops import GGUFTensor, qlinear
from xanosmerks_b200.synth import make_weight

pytestmark = pytest.mark.gpu


def test_qlinear_two_streams_match_one_stream():
    n, k = 4096, 4096
    w1 = GGUFTensor(make_weight("Q4_K", n, k, seed=201), "Q4_K", (n, k))
    w2 = GGUFTensor(make_weight("Q6_K", n, k, seed=202), "Q6_K", (n, k))
    g = torch.Generator().manual_seed(203)
    xs = [torch.randn(m, k, generator=g).to(torch.bfloat16).cuda() for m in (1, 4, 96, 300)]
    # one stream
    ref = [(qlinear(w1, x).clone(), qlinear(w2, x).clone()) for x in xs]
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    s1.wait_stream(torch.cuda.current_stream())
    s2.wait_stream(torch.cuda.current_stream())
    outs = []
    for _ in range(3):                        # the second and third rounds reuse the per-stream buffers
        for x in xs:
            with torch.cuda.stream(s1):
                a = qlinear(w1, x)
            with torch.cuda.stream(s2):
                b = qlinear(w2, x)
            outs.append((a, b))
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(outs):
        ra, rb = ref[i % len(xs)]
        assert torch.equal(a, ra), i
        assert torch.equal(b, rb), i
    # the larger request on a stream grows that stream's buffer only
    big = torch.randn(2048, k, generator=g).to(torch.bfloat16).cuda()
    s1.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s1):
        yb = qlinear(w1, big)
    with torch.cuda.stream(s2):
        y4 = qlinear(w2, xs[1])
    torch.cuda.synchronize()
    assert torch.equal(y4, ref[1][1])
    # 300 rows of 4096 x 4096 take the split-K path, 2048 rows do not: only the summation order differs
    assert rel_err(yb[:300].cpu().numpy(), qlinear(w1, big[:300]).cpu().numpy()) < 1e-5
