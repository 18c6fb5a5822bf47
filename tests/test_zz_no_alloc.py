"""The analyzer entry point that allocates nothing (ada_analyze_noalloc).

Some callers cannot call cudaMalloc: code that must stay inside a device-memory
budget fixed at start-up, or code that runs the analyzer from a place where
its memory allocator is not reachable. ada_analyze_noalloc serves them by
keeping the per-head scratch that ada_analyze takes from a workspace in a
fixed array inside the library.

The test calls it through the C ABI twice in a row, the second time on other
inputs with fewer heads (it reuses the array the first call left behind), and
checks each result against the workspace entry point, ada_analyze, on the same
inputs: decisions identical, statistics identical (the same kernels run on the
same data). It also checks that the size limit is refused with a clear error
and that bad arguments give the same error codes as ada_analyze. This file is
collected last so that a run stopping at the first failure has run every other
test first.
"""

import ctypes
import math

import pytest
import torch

from adaattn_b200 import PrecisionMode
from adaattn_b200 import _lib
from adaattn_b200.workloads import WORKLOADS, make_qkv

pytestmark = pytest.mark.gpu

LIMIT = 65536  # batch * heads the fixed scratch covers


def _params(scale, granularity):
    p = _lib.AdaAnalyzeParams()
    p.rank_threshold = 0.95
    p.scale = scale
    p.eps = 1e-6
    p.enable_adaptive_rank = 1
    p.enable_adaptive_precision = 1
    p.default_precision = PrecisionMode.FP16.code
    p.allow_fp8 = 0
    p.granularity = granularity
    p.sample_stride = 1
    return p


def _outputs(b, h, dev):
    return (torch.empty(b, h, 2, dtype=torch.int32, device=dev),
            torch.empty(b, h, 4, dtype=torch.float32, device=dev),
            torch.empty(_lib.SUMMARY_LEN, dtype=torch.float32, device=dev))


def _with_workspace(lib, q, k, p, dev):
    dec, st, sm = _outputs(q.shape[0], q.shape[1], dev)
    ws = torch.empty(lib.ada_analyze_workspace_bytes(q.shape[0], q.shape[1]), dtype=torch.uint8,
                     device=dev)
    rc = lib.ada_analyze(_lib.tensor(q), _lib.tensor(k), p, dec.data_ptr(), st.data_ptr(),
                         sm.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "ada_analyze")
    return dec, st, sm


def _no_alloc(lib, q, k, p, dev):
    dec, st, sm = _outputs(q.shape[0], q.shape[1], dev)
    rc = lib.ada_analyze_noalloc(_lib.tensor(q), _lib.tensor(k), p, dec.data_ptr(), st.data_ptr(),
                                 sm.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "ada_analyze_noalloc")
    return dec, st, sm


@pytest.mark.parametrize("granularity", [0, 1])
@pytest.mark.parametrize("workload,b,h,n", [("adaptive_mix", 2, 8, 512),
                                            ("precision_mix", 4, 32, 256)])
def test_no_alloc_matches_workspace_entry_point(workload, b, h, n, granularity, cuda_device):
    lib = _lib.load()
    w = WORKLOADS[workload].scaled(batch=b, heads=h, seq=n)
    q, k, _ = make_qkv(w, seed=0, device=str(cuda_device))
    # The second call gets other inputs and fewer heads, so an entry the first
    # call left behind in the shared array would change its result.
    w2 = WORKLOADS[workload].scaled(batch=max(1, b // 2), heads=max(1, h // 2), seq=n)
    q2, k2, _ = make_qkv(w2, seed=7, device=str(cuda_device))
    p = _params(1.0 / math.sqrt(w.head_dim), granularity)
    with torch.cuda.device(cuda_device):
        want = _with_workspace(lib, q, k, p, cuda_device)
        want2 = _with_workspace(lib, q2, k2, p, cuda_device)
        first = _no_alloc(lib, q, k, p, cuda_device)
        second = _no_alloc(lib, q2, k2, p, cuda_device)
    torch.cuda.synchronize()
    n_summary = 10  # entries ADA_SUM_NE .. ADA_SUM_N_TOTAL; the rest are reserved
    for got, ref in ((first, want), (second, want2)):
        assert torch.equal(got[0], ref[0])
        torch.testing.assert_close(got[1], ref[1], rtol=0, atol=0, equal_nan=True)
        torch.testing.assert_close(got[2][:n_summary], ref[2][:n_summary], rtol=0, atol=0,
                                   equal_nan=True)


def test_no_alloc_reports_the_same_errors_as_the_workspace_entry_point(cuda_device):
    lib = _lib.load()
    good = torch.zeros(1, 2, 8, 64, device=cuda_device, dtype=torch.bfloat16)
    p = _params(0.125, 0)
    dec, st, sm = _outputs(1, 2, cuda_device)
    ws = torch.empty(lib.ada_analyze_workspace_bytes(1, 2), dtype=torch.uint8, device=cuda_device)
    bad_rank = _lib.tensor(good)
    bad_rank.ndim = 3
    bad_dtype = _lib.tensor(good)
    bad_dtype.dtype = 5  # ADA_I32
    other_k = torch.zeros(1, 3, 8, 64, device=cuda_device, dtype=torch.bfloat16)
    cases = [(bad_rank, _lib.tensor(good), -2),         # ADA_ERR_SHAPE
             (bad_dtype, _lib.tensor(good), -3),        # ADA_ERR_DTYPE
             (_lib.tensor(good), _lib.tensor(other_k), -2)]
    with torch.cuda.device(cuda_device):
        for qa, ka, code in cases:
            rc_ws = lib.ada_analyze(qa, ka, p, dec.data_ptr(), st.data_ptr(), sm.data_ptr(),
                                    ws.data_ptr(), ws.numel(), _lib.stream_ptr(cuda_device))
            rc_na = lib.ada_analyze_noalloc(qa, ka, p, dec.data_ptr(), st.data_ptr(),
                                            sm.data_ptr(), _lib.stream_ptr(cuda_device))
            assert rc_ws == rc_na == code


def test_no_alloc_refuses_more_heads_than_its_scratch(cuda_device):
    lib = _lib.load()
    base = torch.zeros(1, 1, 8, 64, device=cuda_device)
    big = base.expand(1, LIMIT + 1, 8, 64)  # stride 0 over heads: no memory behind it
    p = _params(0.125, 0)
    dec = torch.empty(2, dtype=torch.int32, device=cuda_device)
    st = torch.empty(4, dtype=torch.float32, device=cuda_device)
    sm = torch.empty(_lib.SUMMARY_LEN, dtype=torch.float32, device=cuda_device)
    with torch.cuda.device(cuda_device):
        rc = lib.ada_analyze_noalloc(_lib.tensor(big), _lib.tensor(big), p, dec.data_ptr(),
                                     st.data_ptr(), sm.data_ptr(), _lib.stream_ptr(cuda_device))
    assert rc == -9  # ADA_ERR_UNSUPPORTED
    assert "65536" in _lib.last_error()
