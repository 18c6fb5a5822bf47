"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures were produced by running the AdaAttn reference on seeded inputs
(tests/golden/make_golden.py). The oracle uses the same PyTorch CPU operations
in the same dtypes, so decisions must agree exactly and outputs bit for bit.
"""

import math

import pytest
import torch

import oracle as O
from golden_util import CASE_NAMES, PREC_CODE, inputs, load, oracle_config


@pytest.mark.parametrize("name", CASE_NAMES)
def test_decisions_match_reference(name):
    rec = load(name)
    q, k, v = inputs(rec)
    cfg = oracle_config(rec)
    scale = rec["scale"]
    g = O.analyze(q, k, cfg, scale)
    assert g["low_rank"] == rec["global"]["low_rank"]
    assert g["precision"] == PREC_CODE[rec["global"]["precision"]]
    assert g["effective_rank"] == rec["global"]["effective_rank"]
    ph = O.analyze_per_head(q, k, cfg, scale)
    ref = rec["per_head"]
    assert torch.equal(ph["low_rank"], ref["low_rank"])
    want = torch.tensor([[PREC_CODE[p] for p in row] for row in ref["precision"]],
                        dtype=torch.int32)
    assert torch.equal(ph["precision"], want)
    eff = ph["ne"] * min(q.shape[2], k.shape[2])
    assert torch.equal(eff, ref["effective_rank"])


@pytest.mark.parametrize("name", CASE_NAMES)
def test_outputs_match_reference(name):
    rec = load(name)
    q, k, v = inputs(rec)
    cfg = oracle_config(rec)
    rows = rec["rows"]
    masks = {"none": None, **rec["masks"]}
    for mname, mask in masks.items():
        for gran in ("global", "per_head"):
            out, _ = O.adaptive_forward(
                q, k, v, cfg, rec["scale"], rec["w_down"],
                "global" if gran == "global" else "head", mask)
            want = rec["outputs"][mname][gran]
            got = out[:, :, rows]
            assert got.dtype == want.dtype
            torch.testing.assert_close(got, want, rtol=0, atol=0,
                                       equal_nan=True,
                                       msg=f"{name}/{mname}/{gran}")


def test_module_forward_matches_reference():
    rec = load("module_forward")
    cfg = O.OracleConfig()
    y, _ = O.module_forward(rec["x"], rec["x"], rec["x"], rec["state_dict"],
                            rec["num_heads"], cfg, "global")
    torch.testing.assert_close(y, rec["y"], rtol=1e-6, atol=1e-6)


def test_uniform_attention_kat():
    rec = load("kat")["uniform"]
    cfg = O.OracleConfig()
    z = torch.zeros(1, 2, 64, 64)
    g = torch.Generator().manual_seed(3)
    kk = torch.randn(1, 2, 64, 64, generator=g)
    d = O.analyze(z, kk, cfg, 1.0 / 8.0)
    assert d["low_rank"] == rec["low_rank"]
    assert d["precision"] == PREC_CODE[rec["precision"]]
    assert d["effective_rank"] == pytest.approx(rec["effective_rank"], rel=0,
                                                abs=0)
    # Uniform rows: entropy log(S) up to the eps term, so ne is ~1.
    assert d["ne"] == pytest.approx(1.0, abs=1e-4)


@pytest.mark.parametrize("case", ["rsvd_rank2", "rsvd_batch"])
def test_randomized_svd_matches_reference(case):
    rec = load("kat")[case]
    a = rec["A"]
    m, n = a.shape[-2], a.shape[-1]
    omega = O.rsvd_sketch(a.shape[:-2], n, rec["rank"], m, rec["seed"],
                          oversample=rec["oversample"])
    u, s, vh = O.randomized_svd(a, rec["rank"], omega, n_power=2)
    torch.testing.assert_close(s, rec["S"], rtol=1e-5, atol=1e-5)
    recon = u @ torch.diag_embed(s) @ vh
    recon_ref = rec["U"] @ torch.diag_embed(rec["S"]) @ rec["Vh"]
    torch.testing.assert_close(recon, recon_ref, rtol=1e-4, atol=1e-4)
    if case == "rsvd_rank2":
        # The reference's own acceptance bar (test_low_rank.py:58-59).
        assert torch.allclose(a, recon, rtol=0.05)


def test_cholesky_qr_variant_agrees():
    rec = load("kat")["rsvd_batch"]
    a = rec["A"].double()
    omega = O.rsvd_sketch(a.shape[:-2], a.shape[-1], rec["rank"], a.shape[-2],
                          rec["seed"], oversample=rec["oversample"]).double()
    _, s_h, _ = O.randomized_svd(a, rec["rank"], omega, 2, "householder")
    _, s_c, _ = O.randomized_svd(a, rec["rank"], omega, 2, "cholesky")
    torch.testing.assert_close(s_c, s_h, rtol=1e-8, atol=1e-8)


def test_fp8_oracle_error_is_bounded():
    """The E4M3 restatement stays near fp32 on uniform-ish heads."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 2, 256, 64, generator=g) * 0.5
    k = torch.randn(1, 2, 256, 64, generator=g) * 0.5
    v = torch.randn(1, 2, 256, 64, generator=g)
    ref = O.dense_attention(q, k, v, O.FP32, 0.125, True)
    got = O.fp8_dense_attention(q, k, v, 0.125, True)
    err = (got - ref).abs().max().item()
    assert 0 < err < 0.1


# --------------------------------------------------------------------------
# Kernel-level ops (adaattn.kernels / _adaattn_cuda) and the small
# AdaptiveTransformer of examples/transformer_integration.py.
# --------------------------------------------------------------------------

def test_kernel_ops_match_reference():
    from golden_util import kernel_op_inputs
    rec = load("kernel_ops")
    for name, (q, k, v) in kernel_op_inputs().items():
        f = rec[f"flash_{name}"]
        torch.testing.assert_close(O.kernel_flash_attention_forward(q, k, v), f["out"], rtol=0, atol=0)
        torch.testing.assert_close(O.kernel_flash_attention_forward(q, k, v, 0.2, True), f["out_causal"],
                                   rtol=0, atol=0)
        a = rec[f"adaptive_{name}"]
        torch.testing.assert_close(O.kernel_adaptive_attention_forward(q, k, v, "fp16", None, True),
                                   a["fp16"], rtol=0, atol=0)
        torch.testing.assert_close(O.kernel_adaptive_attention_forward(q, k, v, "bf16", None, False),
                                   a["bf16"], rtol=0, atol=0)
        torch.testing.assert_close(O.kernel_adaptive_attention_forward(q, k, v, "fp32", 0.15, True),
                                   a["fp32"], rtol=0, atol=0)


def test_entropy_helpers_known_answers():
    # tests/unit/test_entropy.py:21-48 (uniform -> log n, one-hot -> ~0)
    uniform = torch.ones(4, 8, 10) / 10
    torch.testing.assert_close(O.compute_entropy(uniform), torch.full((4, 8), math.log(10)),
                               rtol=1e-5, atol=0)
    peaked = torch.zeros(10)
    peaked[0] = 1.0
    assert O.compute_entropy(peaked) < 0.01
    torch.testing.assert_close(O.estimate_effective_rank(uniform), torch.full((4,), 10.0),
                               rtol=1e-5, atol=0)
    eff = torch.tensor([4.0, 10.0, 31.0, 32.0, 100.0])
    assert O.determine_target_ranks(eff).tolist() == [8, 15, 46, 128, 128]


def _transformer_oracle(state, ids, cfg_heads):
    """The example's forward (examples/transformer_integration.py:47-58,
    :117-132) with the oracle's AdaAttention in each block (global decisions,
    as the reference makes them); returns (logits, per-block outputs)."""
    import torch.nn.functional as F
    e = state["token_embedding.weight"].shape[1]
    pos = torch.arange(ids.shape[1])
    x = F.embedding(ids, state["token_embedding.weight"]) + F.embedding(pos, state["position_embedding.weight"])
    ys = []
    i = 0
    while f"blocks.{i}.norm1.weight" in state:
        p = f"blocks.{i}."
        att = {k[len(p) + len("attention."):]: v for k, v in state.items() if k.startswith(p + "attention.")}
        a, _ = O.module_forward(x, x, x, att, cfg_heads, O.OracleConfig(), "global")
        x = F.layer_norm(x + a, (e,), state[p + "norm1.weight"], state[p + "norm1.bias"])
        h = F.linear(x, state[p + "ff.0.weight"], state[p + "ff.0.bias"])
        h = F.linear(F.gelu(h), state[p + "ff.3.weight"], state[p + "ff.3.bias"])
        x = F.layer_norm(x + h, (e,), state[p + "norm2.weight"], state[p + "norm2.bias"])
        ys.append(x)
        i += 1
    x = F.layer_norm(x, (e,), state["norm.weight"], state["norm.bias"])
    return F.linear(x, state["token_embedding.weight"]), ys


def test_transformer_oracle_matches_reference():
    """Pins the oracle's module restatement inside the example decoder."""
    from golden_util import TRANSFORMER, transformer_ids, transformer_state
    from adaattn_b200.host_model import AdaptiveTransformer
    rec = load("transformer_small")
    template = AdaptiveTransformer(**TRANSFORMER).state_dict()
    state = transformer_state(template)
    logits, ys = _transformer_oracle(state, transformer_ids(), TRANSFORMER["num_heads"])
    for got, blk in zip(ys, rec["blocks"]):
        torch.testing.assert_close(got, blk["y"], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(logits, rec["logits"], rtol=1e-6, atol=1e-6)
