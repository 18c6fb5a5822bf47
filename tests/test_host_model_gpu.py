"""The decoder hosting AdaAttention in the GPT-2-small workload: its tied
head (padded weight, logits as a view) against the plain Linear."""

import pytest
import torch

from adaattn_b200.host_model import AdaptiveTransformer

pytestmark = pytest.mark.gpu


def test_tied_head_logits_match_linear(cuda_device):
    torch.manual_seed(0)
    m = AdaptiveTransformer(vocab_size=1000, embed_dim=128, num_heads=2, num_layers=2, ff_dim=256,
                            max_seq_len=64)
    m.init_gpt2_weights()
    m = m.to(cuda_device).bfloat16().eval()
    ids = torch.randint(0, 1000, (2, 64), device=cuda_device)
    h = torch.randn(2, 64, 128, device=cuda_device).bfloat16()
    with torch.no_grad():
        got = m._logits(h)
        want = torch.nn.functional.linear(h.float(), m.head.weight.float())
        assert got.shape == (2, 64, 1000)
        err = (got.float() - want).abs().max().item()
        assert err <= 2.0 ** -7 * want.abs().max().item() + 1e-3
        flat = got.reshape(-1, 1000)  # row-wise use of the view
        assert torch.equal(flat.argmax(-1), got.argmax(-1).reshape(-1))
        logits = m(ids)
        assert logits.shape == (2, 64, 1000) and torch.isfinite(logits.float()).all()
        # a changed weight is picked up (the padded copy is rebuilt)
        m.head.weight.mul_(2.0)
        assert torch.allclose(m._logits(h).float(), 2.0 * got.float(), rtol=0, atol=1e-2 * got.float().abs().max().item())


def test_self_attention_stacked_projection_matches_separate(cuda_device):
    """Self-attention (query is key is value) projects through one GEMM with
    the stacked q/k/v weights; the result equals the three-Linear path."""
    from adaattn_b200 import AdaAttention
    torch.manual_seed(1)
    m = AdaAttention(embed_dim=256, num_heads=4).to(cuda_device).bfloat16().eval()
    x = (torch.randn(2, 200, 256, device=cuda_device) * 0.5).bfloat16()
    with torch.no_grad():
        fused, _ = m(x, x, x)
        sep, _ = m(x, x.clone(), x.clone())
        err = (fused.float() - sep.float()).abs().max().item()
        assert err <= 2.0 ** -7 * max(1.0, sep.float().abs().max().item())
        # a parameter update reaches the stacked copy
        m.k_proj.weight.mul_(0.5)
        fused2, _ = m(x, x, x)
        sep2, _ = m(x, x.clone(), x.clone())
        err2 = (fused2.float() - sep2.float()).abs().max().item()
        assert err2 <= 2.0 ** -7 * max(1.0, sep2.float().abs().max().item())


def test_small_transformer_matches_reference(cuda_device):
    """The reference's examples/transformer_integration.py decoder at a small
    size (fixture made by running the reference, tests/golden/make_golden.py)
    with this package's AdaAttention in every block, global decisions as the
    reference makes them, fp32.

    Each block is fed the reference's own input to that block, so the check
    isolates one block at a time; then the whole model's logits. Bar: twice
    what replacing the reference's attention precision by FP32 moves the same
    output (its own precision noise), plus 2e-5 relative for the fp32 GEMMs,
    LayerNorms and GELU on the GPU against the CPU."""
    from golden_util import TRANSFORMER, load, transformer_ids, transformer_state
    rec = load("transformer_small")
    m = AdaptiveTransformer(**TRANSFORMER, decision_granularity="global")
    m.load_state_dict(transformer_state(m.state_dict()), strict=False)
    m = m.to(cuda_device).eval()
    ids = transformer_ids().to(cuda_device)
    prec_code = {"FP32": 0, "FP16": 1, "BF16": 2, "FP8": 3, "AUTO": 4}
    with torch.no_grad():
        pos = torch.arange(ids.shape[1], device=cuda_device).unsqueeze(0)
        x = m.token_embedding(ids) + m.position_embedding(pos)
        for i, (blk, ref) in enumerate(zip(m.blocks, rec["blocks"])):
            y = blk(x)
            dec = blk.attention.last_decisions
            assert int(dec.precision.flatten()[0]) == prec_code[ref["precision"]]
            assert bool(dec.low_rank.flatten()[0]) == ref["low_rank"]
            want = ref["y"].to(cuda_device)
            err = (y - want).abs().max().item()
            bar = 2 * ref["fp32_attention_diff"] + 2e-5 * want.abs().max().item()
            print(f"block {i}: {ref['precision']} low_rank={ref['low_rank']} err {err:.3e} bar {bar:.3e}")
            assert err <= bar, f"block {i}: {err:.3e} > {bar:.3e}"
            x = want  # the next block gets the reference's input
        logits = m(ids)
        want = rec["logits"].to(cuda_device)
        err = (logits.float() - want).abs().max().item()
        bar = 2 * rec["fp32_attention_diff"] + 2e-5 * want.abs().max().item()
        print(f"logits: err {err:.3e} bar {bar:.3e}")
        assert err <= bar, f"logits: {err:.3e} > {bar:.3e}"
