"""The adaptive forward (analyzer + attention core) launches only
stream-ordered work, so a serving loop can capture it in a CUDA graph once
and replay it: the replay must reproduce the eager result bit for bit."""

import math

import pytest
import torch

from adaattn_b200 import PrecisionMode, analyze, attention_forward
from adaattn_b200.core import possible_precisions
from adaattn_b200.workloads import WORKLOADS, make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["adaptive_mix", "precision_mix"])
def test_adaptive_forward_replays_from_a_cuda_graph(name, cuda_device):
    w = WORKLOADS[name]
    q, k, v = make_qkv(w, seed=0, device=cuda_device)
    d = w.head_dim
    scale = 1.0 / math.sqrt(d)
    g = torch.Generator().manual_seed(1)
    wd = torch.empty(max(1, d // 2), d)
    torch.nn.init.orthogonal_(wd, generator=g)
    wd = wd.to(w.dtype).to(cuda_device)
    pm = possible_precisions(True, PrecisionMode.FP16, False)
    out = torch.empty_like(q)

    def step():
        t = analyze(q, k, scale=scale)
        attention_forward(q, k, v, scale=scale, causal=w.causal, table=t, w_down=wd,
                          possible_mask=pm, low_rank_possible=True, out=out)

    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    torch.cuda.synchronize()
    eager = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(2):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
