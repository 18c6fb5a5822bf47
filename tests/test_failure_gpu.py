"""Failure detection without faulting the GPU.

A device-side wait that nothing will satisfy gives up after its time limit,
records ADA_ERR_TIMEOUT in the library's status word and returns; the host
reads the status and raises, and the CUDA context stays usable.
"""

import pytest
import torch

from adaattn_b200 import KernelError, PrecisionMode, ShapeError, attention_forward
from adaattn_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda_device):
    lib = _lib.load()
    _lib.poll_device_status(cuda_device)  # start clean
    with torch.cuda.device(cuda_device):
        rc = lib.ada_debug_bounded_wait(2_000_000, _lib.stream_ptr(cuda_device))  # 2 ms
    assert rc == 0
    with pytest.raises(KernelError) as e:
        _lib.poll_device_status(cuda_device)
    assert e.value.code == -7
    # the status word was cleared and the context still runs kernels
    _lib.poll_device_status(cuda_device)
    q = torch.randn(1, 2, 128, 64, device=cuda_device, dtype=torch.bfloat16)
    out = attention_forward(q, q, q, scale=0.125, static_precision=PrecisionMode.BF16)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    _lib.poll_device_status(cuda_device)


def test_host_side_argument_errors(cuda_device):
    q = torch.randn(1, 2, 64, 64, device=cuda_device)
    k = torch.randn(1, 3, 64, 64, device=cuda_device)
    with pytest.raises(ShapeError):
        attention_forward(q, k, k, scale=0.125, static_precision=PrecisionMode.FP32)
    with pytest.raises(KernelError):
        attention_forward(q, q, q, scale=0.125, static_precision=PrecisionMode.FP16,
                          static_low_rank=True)  # low rank without rank_proj_down
    big = torch.randn(1, 1, 16, 160, device=cuda_device)
    with pytest.raises(KernelError):
        attention_forward(big, big, big, scale=0.1, static_precision=PrecisionMode.FP32)
