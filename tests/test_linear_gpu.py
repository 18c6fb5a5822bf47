"""The dense layers on either side of the path on the tensor cores (ada_linear):
y = act(x Wᵀ + b) + r with the bias, GELU and residual sum fused.

Checked element by element against the oracle's float64 restatement with
PyTorch's rounding points (oracle.linear_layer). Bar per element:

    c * (spacing(|h|) + K * 2^-24 * (|x| |W|ᵀ))  +  [gelu] spacing(|gelu(h)|)
                                               +  [residual] spacing(|y|)

with h = x Wᵀ + b and c = 1.13 with GELU (the largest slope of GELU), else 1:
the worst-case fp32 summation error of K products and one unit in the last
place of h (a rounding that the accumulation error tips across a boundary),
carried through the later steps, plus one unit for each later rounding that
this can tip in turn. Spacings are taken one part in 64 above each magnitude
(a value can round up into the next binade). At least 95 % of the elements must equal the oracle exactly (a
wrong bias, activation or sum would change nearly all of them; fp32
accumulation order alone tips 1-2 % of fp16 results at K = 3072).
The same bar holds against PyTorch's own ops on the device (cuBLAS).
"""

import math

import pytest
import torch
import torch.nn.functional as F

import oracle as O
from adaattn_b200 import core
from parity import record

pytestmark = pytest.mark.gpu


def _spacing(t: torch.Tensor, dtype) -> torch.Tensor:
    mant = {torch.bfloat16: 7, torch.float16: 10}[dtype]
    tiny = {torch.bfloat16: 2.0 ** -133, torch.float16: 2.0 ** -24}[dtype]
    e = torch.floor(torch.log2(t.abs().clamp_min(1e-30)))
    return torch.maximum(torch.exp2(e - mant), torch.full_like(t, tiny))


def _inputs(m, n, k, dtype, seed, bias=True, resid=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w = (torch.randn(n, k, generator=g) / math.sqrt(k)).to(dtype)
    b = (torch.randn(n, generator=g) * 0.1).to(dtype) if bias else None
    r = torch.randn(m, n, generator=g).to(dtype) if resid else None
    return x, w, b, r


def _bar(x, w, h64, y_a, y_b, act, resid, scale=1.0):
    """The per-element bar above for two results y_a, y_b of the same layer."""
    dt = x.dtype
    up = 1.0 + 2.0 ** -6
    acc = scale * x.shape[-1] * 2.0 ** -24 * (x.double().abs() @ w.double().abs().t())
    c = 1.13 if act == "gelu" else 1.0
    bar = c * (scale * _spacing(h64.abs() * up + acc, dt).double() + acc)
    if act == "gelu":
        g = F.gelu(h64.to(dt).float()).double()
        bar = bar + scale * _spacing(g.abs() * up + bar, dt).double()
    if resid:
        mag = torch.maximum(y_a.double().abs(), y_b.double().abs())
        bar = bar + scale * _spacing(mag * up, dt).double()
    return bar


def _check(name, got, x, w, b, r, act):
    got = got.cpu()
    want, h64 = O.linear_layer(x, w, b, act, r)
    dt = x.dtype
    bar = _bar(x, w, h64, want, got, act, r is not None)
    diff = (got.double() - want.double()).abs()
    worst = (diff - bar).max().item()
    exact = (got == want).double().mean().item()
    record(f"linear/{name}", str(dt).split(".")[-1], diff.max().item(), (bar.max()).item())
    assert worst <= 0, f"{name}: {(diff > bar).sum().item()} elements above the bar (worst excess {worst:.3e})"
    assert exact >= 0.95, f"{name}: only {exact:.4f} of the elements match the oracle exactly"
    return want


SHAPES = [
    # (M, N, K)
    (1, 8, 8),
    (100, 200, 72),
    (128, 256, 64),
    (300, 768, 768),
    (1024, 2304, 768),
    (257, 1000, 3072),
    (64, 50257, 768),   # a vocabulary head: N not a multiple of 8
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_linear_bias(shape, dtype, cuda_device):
    m, n, k = shape
    x, w, b, _ = _inputs(m, n, k, dtype, seed=m + n + k)
    got = core.linear(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    assert got.shape == (m, n) and got.dtype == dtype
    _check(f"bias/{m}x{n}x{k}", got, x, w, b, None, None)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_gelu_and_residual(dtype, cuda_device):
    dev = cuda_device
    for (m, n, k), act, resid in (((513, 3072, 768), "gelu", False), ((513, 768, 3072), None, True),
                                  ((200, 264, 136), "gelu", True), ((70, 24, 16), None, False)):
        x, w, b, r = _inputs(m, n, k, dtype, seed=7 * m + n, resid=resid)
        got = core.linear(x.to(dev), w.to(dev), b.to(dev), residual=r.to(dev) if r is not None else None,
                          activation=act)
        torch.cuda.synchronize()
        _check(f"{act}/{'r' if resid else 'nr'}/{m}x{n}x{k}", got, x, w, b, r, act)
        # and against PyTorch's own ops on the device (cuBLAS GEMM)
        ref = F.linear(x.to(dev), w.to(dev), b.to(dev))
        if act == "gelu":
            ref = F.gelu(ref)
        if r is not None:
            ref = ref + r.to(dev)
        torch.cuda.synchronize()
        _, h64 = O.linear_layer(x, w, b, act, r)
        # two independent fp32 accumulations: twice the bar
        bar = _bar(x, w, h64, ref.cpu(), got.cpu(), act, resid, scale=2.0)
        assert ((got.cpu().double() - ref.cpu().double()).abs() <= bar).all()


def test_linear_no_bias_and_strided_views(cuda_device):
    dev = cuda_device
    x, w, _, _ = _inputs(333, 640, 256, torch.bfloat16, seed=3, bias=False)
    # x as a column slice of a wider buffer (row stride 384), 3-D leading dims
    wide = torch.zeros(333, 384, dtype=torch.bfloat16)
    wide[:, 64:320] = x
    xd = wide.to(dev)[:, 64:320]
    got = core.linear(xd.view(9, 37, 256), w.to(dev))
    torch.cuda.synchronize()
    assert got.shape == (9, 37, 640)
    _check("nobias/strided", got.reshape(333, 640), x, w, None, None, None)


def test_linear_empty_and_errors(cuda_device):
    dev = cuda_device
    w = torch.randn(16, 32, device=dev, dtype=torch.bfloat16)
    y = core.linear(torch.empty(0, 32, device=dev, dtype=torch.bfloat16), w)
    assert y.shape == (0, 16)
    with pytest.raises(TypeError):
        core.linear(torch.randn(4, 32, device=dev), w)          # fp32 x
    with pytest.raises(TypeError):
        core.linear(torch.randn(4, 32, device=dev, dtype=torch.float16), w)  # mixed dtypes
    with pytest.raises(Exception):
        core.linear(torch.randn(4, 31, device=dev, dtype=torch.bfloat16),
                    torch.randn(16, 31, device=dev, dtype=torch.bfloat16))  # K not a multiple of 8
    with pytest.raises(ValueError):
        core.linear(torch.randn(4, 32, device=dev, dtype=torch.bfloat16), w, activation="relu")


def test_linear_gradients(cuda_device):
    """Autograd through the fused layer matches float64 autograd of the
    same function (bf16 gradients: 2 % of the largest entry)."""
    dev = cuda_device
    x, w, b, r = _inputs(96, 136, 64, torch.bfloat16, seed=9, resid=True)
    xs = [t.to(dev).requires_grad_(True) for t in (x, w, b, r)]
    y = core.linear(xs[0], xs[1], xs[2], residual=xs[3], activation="gelu")
    g = torch.Generator().manual_seed(10)
    dy = torch.randn(96, 136, generator=g).to(torch.bfloat16)
    y.backward(dy.to(dev))
    ref = [t.double().requires_grad_(True) for t in (x, w, b, r)]
    F.gelu(F.linear(ref[0], ref[1], ref[2])).add(ref[3]).backward(dy.double())
    for name, got, want in zip(("dx", "dw", "db", "dr"), xs, ref):
        err = (got.grad.double().cpu() - want.grad).abs().max().item()
        bar = 2e-2 * max(1.0, want.grad.abs().max().item())
        record(f"linear/grad/{name}", "bf16", err, bar)
        assert err <= bar, f"{name}: {err:.3e} > {bar:.3e}"
