"""Attention backward (ada_attn_bwd) and the module's autograd.

The kernels compute the gradients of softmax(q kᵀ·scale + mask) v in fp32 at
the operands' values, taking the row term Delta = sum(dO * out) from the
forward's output in the inputs' dtype. The functional entry point is checked
against the same formulas in float64 with the same forward output
(oracle.attention_grads_from_out): max|got - ref| <= 2e-5 * max(1, max|ref|),
fp32 accumulation error. The module, in fp32 with FP32 decisions, is checked
against float64 autograd of the whole module: 1e-4 relative.
"""

import math

import pytest
import torch

import oracle as O
from adaattn_b200 import AdaAttention, PrecisionMode, analyze
from adaattn_b200.core import attention_backward, attention_forward
from parity import record

pytestmark = pytest.mark.gpu


def _inputs(b, h, nq, nk, d, dtype, seed, dv=None):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(b, h, nq, d, generator=g) * 0.7).to(dtype)
    k = (torch.randn(b, h, nk, d, generator=g) * 0.7).to(dtype)
    v = torch.randn(b, h, nk, dv or d, generator=g).to(dtype)
    dout = torch.randn(b, h, nq, dv or d, generator=g).to(dtype)
    return q, k, v, dout


def _check(name, got, ref, bar_rel=2e-5):
    got = got.double().cpu()
    m = max(1.0, ref.abs().max().item())
    err = (got - ref).abs().max().item()
    bar = bar_rel * m
    record(f"bwd/{name}", "FP32", err, bar)
    assert err <= bar, f"{name}: {err:.3e} > {bar:.3e}"


CASES = [
    # (dtype, d, nq, nk, causal, mask)
    (torch.float32, 64, 128, 128, False, None),
    (torch.float32, 64, 100, 170, True, None),
    (torch.bfloat16, 128, 256, 256, True, None),
    (torch.float16, 128, 130, 70, False, "bool"),
    (torch.bfloat16, 96, 90, 200, False, "float"),
    (torch.float32, 32, 64, 64, True, "float"),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-d{c[1]}-{c[2]}x{c[3]}-c{int(c[4])}-{c[5]}")
def test_dense_gradients(case, cuda_device):
    dtype, d, nq, nk, causal, mask_kind = case
    q, k, v, dout = _inputs(2, 3, nq, nk, d, dtype, seed=11)
    mask = None
    if mask_kind == "bool":
        g = torch.Generator().manual_seed(12)
        mask = torch.rand(2, nk, generator=g) > 0.3
        mask[:, 0] = True
    elif mask_kind == "float":
        g = torch.Generator().manual_seed(13)
        mask = torch.randn(2, nq, nk, generator=g)
    scale = 1.0 / math.sqrt(d)
    dev = cuda_device
    qd, kd, vd, dod = (t.to(dev) for t in (q, k, v, dout))
    md = mask.to(dev) if mask is not None else None
    out = attention_forward(qd, kd, vd, scale=scale, causal=causal, static_precision=PrecisionMode.FP32,
                            attention_mask=md)
    dq, dk, dv = attention_backward(qd, kd, vd, out, dod, scale=scale, causal=causal, attention_mask=md)
    torch.cuda.synchronize()
    rq, rk, rv, _ = O.attention_grads_from_out(q, k, v, out.cpu(), dout, scale, causal, mask)
    _check("dq", dq, rq)
    _check("dk", dk, rk)
    _check("dv", dv, rv)
    if dtype == torch.float32:  # and the true gradients of the exact function
        tq, tk, tv, _ = O.attention_grads(q, k, v, dout, scale, causal, mask)
        _check("exact/dq", dq, tq, 1e-4)
        _check("exact/dk", dk, tk, 1e-4)
        _check("exact/dv", dv, tv, 1e-4)


@pytest.mark.parametrize("causal", [False, True])
def test_low_rank_gradients(causal, cuda_device):
    b, h, n, d, r = 1, 2, 150, 128, 64
    q, k, v, dout = _inputs(b, h, n, n, d, torch.bfloat16, seed=21)
    g = torch.Generator().manual_seed(22)
    w = torch.empty(r, d)
    torch.nn.init.orthogonal_(w, generator=g)
    w = w.to(torch.bfloat16)
    scale = 1.0 / math.sqrt(d)
    dev = cuda_device
    qd, kd, vd, dod, wd = (t.to(dev) for t in (q, k, v, dout, w))
    q_low = torch.nn.functional.linear(qd, wd)
    k_low = torch.nn.functional.linear(kd, wd)
    out = attention_forward(qd, kd, vd, scale=scale, causal=causal, static_precision=PrecisionMode.FP32,
                            static_low_rank=True, w_down=wd)
    dql, dkl, dv = attention_backward(q_low, k_low, vd, out, dod, scale=scale, causal=causal)
    torch.cuda.synchronize()
    wf = wd.float()
    dq = torch.matmul(dql, wf)
    dk = torch.matmul(dkl, wf)
    dw = torch.einsum("bhnr,bhnd->rd", dql, qd.float()) + torch.einsum("bhnr,bhnd->rd", dkl, kd.float())
    rq, rk, rv, rw = O.attention_grads_from_out(q, k, v, out.cpu(), dout, scale, causal, w_down=w)
    _check("low/dq", dq, rq)
    _check("low/dk", dk, rk)
    _check("low/dv", dv, rv)
    _check("low/dw", dw, rw)


def test_per_head_decisions_route_each_head(cuda_device):
    """A decision table with dense and low-rank heads: each head's gradients
    follow its own branch (the kernel serves the heads whose flag matches)."""
    b, h, n, d, r = 2, 4, 128, 64, 32
    q, k, v, dout = _inputs(b, h, n, n, d, torch.float32, seed=31)
    g = torch.Generator().manual_seed(32)
    w = torch.empty(r, d)
    torch.nn.init.orthogonal_(w, generator=g)
    dev = cuda_device
    qd, kd, vd, dod, wd = (t.to(dev) for t in (q, k, v, dout, w))
    table = analyze(qd, kd, scale=d ** -0.5)
    # heads alternate dense / low rank
    low = torch.tensor([[i % 2 for i in range(h)] for _ in range(b)], dtype=torch.int32, device=dev)
    table.decisions[..., 1] = low
    table.decisions[..., 0] = PrecisionMode.FP32.code
    scale = d ** -0.5
    out = attention_forward(qd, kd, vd, scale=scale, table=table, w_down=wd, low_rank_possible=True)
    dq, dk, dv = attention_backward(qd, kd, vd, out, dod, scale=scale, table=table, low_rank=False)
    ql, kl = torch.nn.functional.linear(qd, wd), torch.nn.functional.linear(kd, wd)
    dql, dkl, dvl = attention_backward(ql, kl, vd, out, dod, scale=scale, table=table, low_rank=True)
    dq = dq + torch.matmul(dql, wd)
    dk = dk + torch.matmul(dkl, wd)
    dv = dv + dvl
    torch.cuda.synchronize()
    for bb in range(b):
        for hh in range(h):
            sl = (slice(bb, bb + 1), slice(hh, hh + 1))
            rq, rk, rv, _ = O.attention_grads_from_out(q[sl], k[sl], v[sl], out[sl].cpu(), dout[sl], scale,
                                                       False, w_down=w if hh % 2 else None)
            _check(f"route/b{bb}h{hh}/dq", dq[sl], rq)
            _check(f"route/b{bb}h{hh}/dk", dk[sl], rk)
            _check(f"route/b{bb}h{hh}/dv", dv[sl], rv)


def test_module_gradient_flow(cuda_device):
    """The reference's gradient-flow test (test_adaattn_unified.py:146-159),
    in eval mode (attention-probability dropout is forward-only here), plus
    a check of every gradient against float64 autograd of the same module
    with FP32 decisions."""
    torch.manual_seed(5)
    m = AdaAttention(embed_dim=256, num_heads=4, enable_adaptive_precision=False,
                     default_precision=PrecisionMode.FP32, decision_granularity="global").to(cuda_device).eval()
    g = torch.Generator().manual_seed(6)
    xs = [torch.randn(2, 64, 256, generator=g) for _ in range(3)]
    q, k, v = (x.to(cuda_device).requires_grad_(True) for x in xs)
    out, _ = m(q, k, v)
    loss = (out * torch.linspace(-1, 1, 256, device=cuda_device)).sum()
    loss.backward()
    assert q.grad is not None and k.grad is not None and v.grad is not None
    for t in (q.grad, k.grad, v.grad):
        assert torch.isfinite(t).all()
    # float64 reference of the same module (the decision the module took)
    low = bool(m.last_decisions.low_rank.flatten()[0])
    sd = {kk: vv.detach().double().cpu() for kk, vv in m.state_dict().items()
          if vv.is_floating_point() and not kk.startswith("_")}
    xd = [x.double().requires_grad_(True) for x in xs]
    b_, n_, e_ = xd[0].shape
    hh, dd = 4, 64

    def proj(x, name):
        return torch.nn.functional.linear(x, sd[f"{name}.weight"], sd[f"{name}.bias"])

    qh = proj(xd[0], "q_proj").view(b_, n_, hh, dd).transpose(1, 2)
    kh = proj(xd[1], "k_proj").view(b_, n_, hh, dd).transpose(1, 2)
    vh = proj(xd[2], "v_proj").view(b_, n_, hh, dd).transpose(1, 2)
    if low:
        wdn = sd["rank_proj_down.weight"]
        qh, kh = torch.nn.functional.linear(qh, wdn), torch.nn.functional.linear(kh, wdn)
    p = torch.softmax(torch.matmul(qh, kh.transpose(-2, -1)) * dd ** -0.5, dim=-1)
    o = torch.matmul(p, vh).transpose(1, 2).reshape(b_, n_, e_)
    ref = proj(o, "out_proj")
    (ref * torch.linspace(-1, 1, 256, dtype=torch.float64)).sum().backward()
    for name, got, want in (("dq", q.grad, xd[0].grad), ("dk", k.grad, xd[1].grad), ("dv", v.grad, xd[2].grad)):
        _check(f"module/{name}", got, want, 1e-4)
