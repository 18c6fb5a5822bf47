"""The host block's LayerNorm (ada_layer_norm) and the module's running
statistics update (ada_record_statistics) on the device.

LayerNorm: against a float64 evaluation of nn.LayerNorm on the same 16-bit
inputs and parameters, every element within one unit in the last place of the
result's dtype plus 2^-20 of the largest output (the kernel computes in fp32
and rounds once; a sum order other than PyTorch's can tip a rounding by one
unit, and the fp32 mean's rounding shows in outputs near zero), and at least 97 % of the
elements equal to PyTorch's own 16-bit LayerNorm on the device.

Statistics: bit-equal to the PyTorch updates they replace
(src/adaattn/attention/adaattn.py:486-498) for fp32, fp64 and bf16 buffers.
"""

import pytest
import torch
import torch.nn.functional as F

from adaattn_b200 import core
from parity import record

pytestmark = pytest.mark.gpu


def _spacing(t: torch.Tensor, dtype) -> torch.Tensor:
    mant = {torch.bfloat16: 7, torch.float16: 10}[dtype]
    tiny = {torch.bfloat16: 2.0 ** -133, torch.float16: 2.0 ** -24}[dtype]
    e = torch.floor(torch.log2(t.abs().clamp_min(1e-30)))
    return torch.maximum(torch.exp2(e - mant), torch.full_like(t, tiny))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,e,affine", [(1, 64, True), (37, 768, True), (300, 1000, False),
                                        (1024, 768, True), (5, 2048, True), (9, 136, "weight")])
def test_layer_norm_matches_torch(m, e, affine, dtype, cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(m * 7 + e)
    x = (torch.randn(m, e, generator=g) * 3 + 0.5).to(dtype)
    w = b = None
    if affine:
        w = (1 + 0.2 * torch.randn(e, generator=g)).to(dtype)
        if affine is True:
            b = (0.1 * torch.randn(e, generator=g)).to(dtype)
    got = core.layer_norm(x.to(dev), w.to(dev) if w is not None else None,
                          b.to(dev) if b is not None else None, 1e-5)
    want_dev = F.layer_norm(x.to(dev), (e,), w.to(dev) if w is not None else None,
                            b.to(dev) if b is not None else None, 1e-5)
    torch.cuda.synchronize()
    ref = F.layer_norm(x.double(), (e,), w.double() if w is not None else None,
                       b.double() if b is not None else None, 1e-5)
    err = (got.cpu().double() - ref).abs()
    # one unit in the last place, plus the fp32 mean's own rounding for
    # outputs near zero (where the bf16/fp16 spacing is finer than it)
    bar = _spacing(ref.abs() * (1 + 2.0 ** -6), dtype).double() + 2.0 ** -20 * ref.abs().max().item()
    record(f"layer_norm/{m}x{e}", str(dtype).split(".")[-1], err.max().item(), bar.max().item())
    assert (err <= bar).all(), f"{(err > bar).sum().item()} elements beyond one unit"
    same = (got == want_dev).float().mean().item()
    assert same >= 0.97, f"only {same:.3f} of the elements equal PyTorch's LayerNorm"


def test_layer_norm_views_and_errors(cuda_device):
    dev = cuda_device
    wide = torch.randn(64, 512, device=dev, dtype=torch.bfloat16)
    x = wide[:, 128:384].view(8, 8, 256)   # row stride 512, 3-D
    w = torch.randn(256, device=dev, dtype=torch.bfloat16)
    b = torch.randn(256, device=dev, dtype=torch.bfloat16)
    got = core.layer_norm(x, w, b)
    want = F.layer_norm(x, (256,), w, b)
    assert got.shape == x.shape
    assert (got.float() - want.float()).abs().max().item() <= 2.0 ** -6 * want.float().abs().max().item()
    assert core.layer_norm(torch.empty(0, 64, device=dev, dtype=torch.bfloat16), None, None).shape == (0, 64)
    with pytest.raises(TypeError):
        core.layer_norm(torch.randn(4, 64, device=dev), None, None)
    with pytest.raises(Exception):
        core.layer_norm(torch.randn(4, 60, device=dev, dtype=torch.bfloat16), None, None)  # E % 8
    with pytest.raises(Exception):
        core.layer_norm(torch.randn(4, 4096, device=dev, dtype=torch.bfloat16), None, None)  # E > 2048


@pytest.mark.parametrize("lr_dtype,pd_dtype", [(torch.float64, torch.float32),
                                               (torch.float32, torch.float32),
                                               (torch.bfloat16, torch.float16)])
def test_record_statistics_matches_torch_updates(lr_dtype, pd_dtype, cuda_device):
    dev = cuda_device
    calls = [torch.tensor([0.5, 3.0, 0.9, 0.7, 3, 1, 2, 0, 4, 7, 0, 0], dtype=torch.float32),
             torch.tensor([0.6, 9.0, 0.99, 0.2, 5, 3, 1, 1, 0, 5, 0, 0], dtype=torch.float32),
             torch.tensor([0.1, 1.0, 0.3, 0.9, 0, 0, 0, 3, 0, 3, 0, 0], dtype=torch.float32)]
    cc = torch.tensor(0, device=dev)
    lr = torch.tensor(0.25, dtype=lr_dtype, device=dev)
    pd = torch.full((4,), 0.125, dtype=pd_dtype, device=dev)
    cc_ref, lr_ref, pd_ref = cc.clone(), lr.clone(), pd.clone()
    for s in calls:
        s = s.to(dev)
        core.record_statistics(s, cc, lr, pd)
        total = s[9]
        cc_ref += 1
        lr_ref += (s[4] / total).to(lr_dtype)
        pd_ref += (s[5:9] / total).to(pd_dtype)
    torch.cuda.synchronize()
    assert int(cc) == 3 == int(cc_ref)
    assert torch.equal(lr, lr_ref)
    assert torch.equal(pd, pd_ref)


def test_module_statistics_after_forwards(cuda_device):
    """get_statistics after a few adaptive forwards: the device-side update
    gives the ratios the decisions imply."""
    from adaattn_b200 import AdaAttention
    torch.manual_seed(3)
    m = AdaAttention(embed_dim=256, num_heads=4).to(cuda_device).eval()
    x = torch.randn(2, 128, 256, device=cuda_device)
    with torch.no_grad():
        lr_sum, prec_sum = 0.0, torch.zeros(4)
        for _ in range(3):
            m(x, x, x)
            s = m.last_decisions.summary.cpu()
            lr_sum += float(s[4] / s[9])
            prec_sum += s[5:9] / s[9]
    st = m.get_statistics()
    assert st["call_count"] == 3
    assert abs(st["low_rank_ratio"] - lr_sum / 3) <= 1e-6
