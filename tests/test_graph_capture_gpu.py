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


def test_decoder_forward_replays_from_a_cuda_graph(cuda_device):
    """The whole host decoder (ada_linear projections and feed-forward,
    ada_layer_norm, the adaptive attention, the statistics update on the
    device) captured once and replayed: the logits equal the eager forward's
    bit for bit, and the running statistics advance once per replay. The
    module's NaN check (a host-side test of the output, on by default) is
    skipped while a capture is in progress, so the default configuration
    captures."""
    from adaattn_b200.host_model import AdaptiveTransformer
    torch.manual_seed(0)
    m = AdaptiveTransformer(vocab_size=1000, embed_dim=256, num_heads=4, num_layers=2, ff_dim=1024,
                            max_seq_len=256, dropout=0.0)
    m.init_gpt2_weights()
    assert m.blocks[0].attention.config.enable_nan_check
    m = m.to(cuda_device).bfloat16().eval()
    ids = torch.randint(0, 1000, (2, 256), device=cuda_device)
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.no_grad(), torch.cuda.stream(side):
        for _ in range(2):
            eager = m(ids).clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            out = m(ids)
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    torch.cuda.synchronize()
    calls = m.blocks[0].attention.get_statistics()["call_count"]
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    assert m.blocks[0].attention.get_statistics()["call_count"] == calls + 2
    del graph
