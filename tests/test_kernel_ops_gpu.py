"""The kernel-level ops of the reference's native module (_adaattn_cuda,
src/adaattn/kernels/bindings.cpp:21-135) through this library's C ABI.

  ada_flash_attention_forward   [B, N, H, D] attention, scale and causal knobs
  adaptive_attention_forward    the same at a requested precision (runs on
                                ada_attn_fwd with a static decision)
  ada_compute_entropy           -sum w log(w + 1e-10) per row
  ada_estimate_effective_rank   exp(mean row entropy)
  ada_determine_target_ranks    clamp(1.5 * rank) below the threshold, else max

Attention outputs are checked against the reference's own results (the
golden fixture made from adaattn.kernels, the Python path its callers run)
and against the oracle with the per-precision bars of tests/parity.py; the
entropy helpers against the oracle's restatement and the reference's known
answers (tests/unit/test_entropy.py:21-48).
"""

import math

import pytest
import torch

import oracle as O
from adaattn_b200 import kernels
from golden_util import kernel_op_inputs, load
from parity import half_spacing, record

pytestmark = pytest.mark.gpu

_PREC_OF_DTYPE = {torch.float32: O.FP32, torch.float16: O.FP16, torch.bfloat16: O.BF16}


def _bar(dtype, ref32, got, own=0.0):
    """parity.py's bar for a head computed in ``dtype``: FP32 1e-5, FP16 2e-3,
    BF16 max(2e-3, 1.5 x the reference's own error), plus the final cast."""
    mag = max(ref32.abs().max().item(), got.abs().max().item())
    m = max(1.0, mag)
    if dtype == torch.float32:
        return 1e-5 * m + half_spacing(got.dtype, mag)
    if dtype == torch.float16:
        return 2e-3 * m + half_spacing(got.dtype, mag) + half_spacing(torch.float16, mag)
    return max(2e-3 * m, 1.5 * own) + half_spacing(got.dtype, mag)


def _fp32_reference(q, k, v, scale, causal):
    return O.kernel_flash_attention_forward(q.float(), k.float(), v.float(), scale, causal)


@pytest.mark.parametrize("name", ["float32", "float16", "bfloat16"])
def test_flash_attention_forward(name, cuda_device):
    q, k, v = kernel_op_inputs()[name]
    rec = load("kernel_ops")[f"flash_{name}"]
    for scale, causal, key in ((None, False, "out"), (0.2, True, "out_causal")):
        got = kernels.flash_attention_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                              scale, causal)
        torch.cuda.synchronize()
        assert got.shape == q.shape and got.dtype == q.dtype
        got = got.cpu()
        s = scale if scale is not None else q.shape[-1] ** -0.5
        ref32 = _fp32_reference(q, k, v, s, causal)
        reference = rec[key]                         # the reference's own output
        own = (reference.float() - ref32).abs().max().item()
        err = (got.float() - ref32).abs().max().item()
        bar = _bar(q.dtype, ref32, got, own)
        record(f"flash/{name}/{key}", O.PREC_NAMES[_PREC_OF_DTYPE[q.dtype]], err, bar)
        assert err <= bar, f"{name} {key}: {err:.3e} > {bar:.3e} (reference's own {own:.3e})"
        # and the oracle restates the reference exactly
        torch.testing.assert_close(O.kernel_flash_attention_forward(q, k, v, scale, causal), reference,
                                   rtol=0, atol=0)


@pytest.mark.parametrize("name", ["float32", "float16", "bfloat16"])
def test_adaptive_attention_forward(name, cuda_device):
    q, k, v = kernel_op_inputs()[name]
    rec = load("kernel_ops")[f"adaptive_{name}"]
    cases = (("fp16", None, True), ("bf16", None, False), ("fp32", 0.15, True))
    for precision, scale, causal in cases:
        got = kernels.adaptive_attention_forward(q.to(cuda_device), k.to(cuda_device),
                                                 v.to(cuda_device), precision=precision,
                                                 softmax_scale=scale, causal=causal)
        torch.cuda.synchronize()
        assert got.shape == q.shape and got.dtype == q.dtype
        got = got.cpu()
        s = scale if scale is not None else q.shape[-1] ** -0.5
        ref32 = _fp32_reference(q, k, v, s, causal)
        reference = rec[precision]
        own = (reference.float() - ref32).abs().max().item()
        cdt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[precision]
        err = (got.float() - ref32).abs().max().item()
        # the reference computes in `precision` and casts to the inputs' dtype:
        # its own error bounds how close a result in that precision can be
        bar = max(_bar(cdt, ref32, got, own), 1.5 * own + half_spacing(got.dtype, ref32.abs().max().item()))
        record(f"adaptive/{name}/{precision}", O.PREC_NAMES[_PREC_OF_DTYPE[cdt]], err, bar)
        assert err <= bar, f"{name} {precision}: {err:.3e} > {bar:.3e} (reference's own {own:.3e})"
        torch.testing.assert_close(
            O.kernel_adaptive_attention_forward(q, k, v, precision, scale, causal), reference,
            rtol=0, atol=0)


def _probs(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.softmax(torch.randn(*shape, generator=g) * 3.0, dim=-1).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_compute_entropy_and_effective_rank(dtype, cuda_device):
    w = _probs((2, 3, 40, 77), dtype, 31)
    ent = kernels.compute_entropy(w.to(cuda_device)).cpu()
    rank = kernels.estimate_effective_rank(w.to(cuda_device)).cpu()
    assert ent.shape == (2, 3, 40) and ent.dtype == dtype
    assert rank.shape == (2, 3) and rank.dtype == dtype
    want_e = O.compute_entropy(w)
    want_r = O.estimate_effective_rank(w)
    # same expression, each step rounded to the dtype; only the order of the
    # row sum differs (a few units in the last place of the dtype). In fp16,
    # w + 1e-10 rounds to 0 where w is 0, so log gives -inf and 0 * -inf NaN:
    # the reference's rows with a zero weight are NaN, and so are these.
    tol = {torch.float32: 1e-5, torch.float16: 4e-3, torch.bfloat16: 3e-2}[dtype]
    torch.testing.assert_close(ent.float(), want_e.float(), rtol=tol, atol=tol, equal_nan=True)
    torch.testing.assert_close(rank.float(), want_r.float(), rtol=2 * tol, atol=2 * tol,
                               equal_nan=True)


def test_entropy_known_answers(cuda_device):
    # tests/unit/test_entropy.py:21-48: uniform over n gives log(n), one-hot ~0.
    uniform = torch.full((4, 8, 10), 0.1, device=cuda_device)
    ent = kernels.compute_entropy(uniform).cpu()
    torch.testing.assert_close(ent, torch.full((4, 8), math.log(10)), rtol=1e-5, atol=0)
    peaked = torch.zeros(3, 10, device=cuda_device)
    peaked[:, 0] = 1.0
    assert (kernels.compute_entropy(peaked).cpu() < 0.01).all()
    rank = kernels.estimate_effective_rank(uniform).cpu()
    torch.testing.assert_close(rank, torch.full((4,), 10.0), rtol=1e-5, atol=0)


def test_determine_target_ranks(cuda_device):
    eff = torch.tensor([0.5, 4.0, 7.9, 10.0, 21.3, 31.99, 32.0, 100.0, 85.0, 5.33])
    for kw in ({}, {"min_rank": 4, "max_rank": 64, "threshold": 50.0}):
        got = kernels.determine_target_ranks(eff.to(cuda_device), **kw).cpu()
        want = O.determine_target_ranks(eff, **kw)
        assert got.dtype == torch.int64
        assert torch.equal(got, want), (kw, got, want)
