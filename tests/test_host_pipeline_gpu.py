"""Host-resident operands through ada_attn_fwd_host: chunks of (b, h) slices copied
in, computed and copied out on overlapping streams. Every (b, h) slice is
computed by the same kernels as the device-resident call, so the results are
bit-identical to it."""

import math

import pytest
import torch

from adaattn_b200 import PrecisionMode, attention_forward, attention_forward_host

pytestmark = pytest.mark.gpu


def _host(b, h, n, d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(b, h, n, d, generator=g)).to(dtype).pin_memory() for _ in range(3)]


@pytest.mark.parametrize("chunk_slices", [0, 1, 4])  # 4: chunks across batch rows, ragged last
@pytest.mark.parametrize("prec,low", [(PrecisionMode.BF16, False), (PrecisionMode.FP16, True),
                                      (PrecisionMode.FP32, False)])
@pytest.mark.parametrize("causal", [False, True])
def test_host_pipeline_matches_device_call(chunk_slices, prec, low, causal, cuda_device):
    b, h, n, d = 5, 3, 200, 128
    q, k, v = _host(b, h, n, d, torch.bfloat16, seed=31)
    w = None
    if low:
        g = torch.Generator().manual_seed(32)
        w = torch.empty(64, d)
        torch.nn.init.orthogonal_(w, generator=g)
        w = w.bfloat16().to(cuda_device)
    scale = 1.0 / math.sqrt(d)
    got = attention_forward_host(q, k, v, scale=scale, causal=causal, static_precision=prec,
                                 static_low_rank=low, w_down=w, device=cuda_device,
                                 chunk_slices=chunk_slices)
    torch.cuda.synchronize()
    want = attention_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), scale=scale,
                             causal=causal, static_precision=prec, static_low_rank=low, w_down=w)
    assert torch.equal(got, want.cpu().contiguous())


def test_host_pipeline_refuses_device_and_strided_tensors(cuda_device):
    q, k, v = _host(2, 2, 64, 64, torch.float16, seed=33)
    with pytest.raises(TypeError):
        attention_forward_host(q.to(cuda_device), k, v, scale=0.125, device=cuda_device)
    with pytest.raises(Exception):
        attention_forward_host(q.transpose(1, 2), k, v, scale=0.125, device=cuda_device)
