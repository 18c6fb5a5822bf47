"""The C-ABI library without a GPU: it loads, exports every entry point the
header declares, reports its ABI version, and rejects bad calls with status
codes instead of crashing. No compute is launched."""

import ctypes
import os
import subprocess

import pytest

from adaattn_b200 import _lib

pytestmark = pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH),
                                reason="library not built (run __graft_entry__.build())")


def test_library_loads_and_version():
    lib = _lib.load()
    assert lib.ada_abi_version() == 1


def test_every_header_function_is_exported():
    names = _lib.header_functions()
    assert len(names) >= 12
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported
    assert set(_lib._SIGNATURES) == set(names)


def test_struct_layouts_match_header():
    assert ctypes.sizeof(_lib.AdaTensor) == 8 + 4 + 4 + 8 * 4 + 8 * 4
    assert ctypes.sizeof(_lib.AdaAnalyzeParams) == 8 + 4 + 4 + 4 * 6 + 4 * 2
    assert ctypes.sizeof(_lib.AdaFwdParams) == 4 * 8


def test_bad_arguments_return_codes():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(64)
    assert lib.ada_get_last_error(buf, 64) == 0
    assert lib.ada_get_last_error(None, 0) == -1
    # Null tensors: rejected before any device work (no GPU needed to answer).
    rc = lib.ada_analyze(None, None, None, None, None, None, None, 0, None)
    assert rc < 0
    rc = lib.ada_attn_fwd(None, None, None, None, None, None, None, 0, 0, None, None, 0, None)
    assert rc < 0
    assert lib.ada_analyze_workspace_bytes(8, 32) == 1024
    assert lib.ada_analyze_workspace_bytes(0, 32) == 0


def test_workspace_query_is_host_only():
    """The workspace size is computed from shapes alone (no device calls)."""
    import torch
    lib = _lib.load()
    q = torch.empty(2, 4, 256, 128, dtype=torch.bfloat16)
    p = _lib.AdaFwdParams()
    p.scale = 128 ** -0.5
    p.causal = 1
    counters = 256  # work-item counters of the dynamically scheduled launches
    p.static_precision = 2  # BF16, bf16 inputs: read in place, only the counters
    t = _lib.tensor(q)
    assert lib.ada_attn_fwd_workspace_bytes(t, t, t, None, None, p, 0, 0) == counters
    p.static_precision = 1  # FP16 on bf16 inputs: a cast copy of q, k, v
    n = lib.ada_attn_fwd_workspace_bytes(t, t, t, None, None, p, 0, 0)
    assert n == 3 * 2 * 4 * 256 * 128 * 2 + counters
    p.static_precision = 3  # FP8 E4M3: 8-bit copies plus scales
    n8 = lib.ada_attn_fwd_workspace_bytes(t, t, t, None, None, p, 0, 0)
    assert n8 >= 3 * 2 * 4 * 256 * 128


def test_host_pipeline_checks_layout_before_any_device_work():
    import torch
    from adaattn_b200 import ShapeError, attention_forward_host
    q = torch.zeros(2, 4, 8, 16, dtype=torch.float16)
    with pytest.raises(ShapeError):
        attention_forward_host(q.transpose(1, 2), q, q, scale=0.25, device="cuda:0")


def test_workspace_queries_without_a_gpu():
    """Plan-only queries need no device: the forward workspace grows with the
    FP32 tensor-core operands when FP32 heads of 16-bit inputs are possible,
    and the host pipeline's staging buffer holds two chunks of slices plus a workspace."""
    import torch
    lib = _lib.load()
    q = torch.zeros(4, 2, 256, 128, dtype=torch.bfloat16)
    tq = _lib.tensor(q)
    p = _lib.AdaFwdParams()
    p.scale = 0.125
    p.static_precision = 2  # BF16
    dense_bf16 = lib.ada_attn_fwd_workspace_bytes(tq, tq, tq, None, None, p, 0, 0)
    p.static_precision = 0  # FP32: dense heads read q, k in place; v goes to a scaled fp16 copy
    dense_fp32 = lib.ada_attn_fwd_workspace_bytes(tq, tq, tq, None, None, p, 0, 0)
    assert dense_fp32 >= dense_bf16 + 4 * 2 * 256 * 128 * 2
    p.static_precision = 2
    one = lib.ada_attn_fwd_host_buffer_bytes(tq, tq, tq, None, p, 1)
    two = lib.ada_attn_fwd_host_buffer_bytes(tq, tq, tq, None, p, 2)
    slice_bytes = 256 * 128 * 2  # one (b, h) slice of q
    assert one >= 2 * 4 * slice_bytes and two >= 2 * 4 * 2 * slice_bytes and two > one
    bad = _lib.tensor(q.transpose(2, 3))
    assert lib.ada_attn_fwd_host_buffer_bytes(bad, tq, tq, None, p, 1) == 0
