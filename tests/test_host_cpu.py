"""Host-side logic of the module and the functional API (no GPU needed)."""

import pytest
import torch

import oracle as O
from adaattn_b200 import (AdaAttention, AttentionConfig, MemoryError, NumericalError,
                          PrecisionMode, ShapeError, analyze, attention_forward)
from adaattn_b200.core import expand_mask, possible_precisions
from golden_util import load


def test_precision_codes_follow_reference_order():
    # adaattn.py:480-485 order; AUTO = 4
    assert [m.code for m in PrecisionMode] == [0, 1, 2, 3, 4]
    assert PrecisionMode.FP8.to_dtype() == torch.float16
    assert PrecisionMode.AUTO.to_dtype() == torch.float16
    assert PrecisionMode.from_dtype(torch.bfloat16) is PrecisionMode.BF16
    assert PrecisionMode.coerce("bf16") is PrecisionMode.BF16
    for m in PrecisionMode:
        assert PrecisionMode.from_code(m.code) is m


def test_config_validation_matches_reference():
    AttentionConfig().validate()
    for bad in (dict(embed_dim=0), dict(num_heads=0), dict(embed_dim=10, num_heads=3),
                dict(dropout=1.0), dict(min_rank_ratio=0.0), dict(max_memory_fraction=0.0)):
        with pytest.raises(ValueError):
            AttentionConfig(**bad).validate()
    assert AttentionConfig(embed_dim=768, num_heads=12).head_dim == 64


def test_error_types():
    e = ShapeError("bad", expected_shape=(1, 2), actual_shape=(3,))
    assert "Expected shape" in str(e)
    assert issubclass(NumericalError, Exception)
    assert "Required" in str(MemoryError("oom", required_memory=2e9, available_memory=1e9))


def test_possible_precision_sets():
    fp16 = PrecisionMode.FP16
    m = possible_precisions(True, fp16, False)
    assert m == (1 << 0) | (1 << 1) | (1 << 2)
    m8 = possible_precisions(True, fp16, True)
    assert m8 & (1 << 3) and m8 & (1 << 1)  # default FP16 still reachable
    assert possible_precisions(False, PrecisionMode.BF16, True) == 1 << 2


def test_expand_mask_shapes():
    m2 = torch.ones(2, 7, dtype=torch.bool)
    e = expand_mask(m2, 2, 3, 5, 7)
    assert e.shape == (2, 3, 5, 7) and e.dtype == torch.uint8 and e.stride(1) == 0
    m3 = torch.randn(2, 5, 7)
    e = expand_mask(m3, 2, 3, 5, 7)
    assert e.shape == (2, 3, 5, 7) and e.stride(1) == 0
    with pytest.raises(ShapeError):
        expand_mask(torch.ones(7), 2, 3, 5, 7)


def test_module_construction_and_names():
    m = AdaAttention(embed_dim=256, num_heads=4)
    assert m.config.embed_dim == 256 and m.config.num_heads == 4
    assert m.enable_adaptive_rank and m.enable_adaptive_precision
    assert m.rank_proj_down.weight.shape == (32, 64)
    r = repr(m)
    assert "AdaAttention" in r and "adaptive_rank" in r and "adaptive_precision" in r
    s = m.get_statistics()
    assert s["call_count"] == 0 and s["low_rank_ratio"] == 0.0
    m2 = AdaAttention(embed_dim=256, num_heads=4, enable_adaptive_rank=False)
    assert m2.rank_proj_down is None


def test_reference_state_dict_loads():
    rec = load("module_forward")
    m = AdaAttention(embed_dim=rec["embed_dim"], num_heads=rec["num_heads"])
    missing, unexpected = m.load_state_dict(rec["state_dict"], strict=True)
    assert not missing and not unexpected
    assert int(m._call_count) == rec["stats"]["call_count"]
    assert torch.equal(m.q_proj.weight, rec["state_dict"]["q_proj.weight"])


def test_input_validation_like_reference():
    m = AdaAttention(embed_dim=64, num_heads=2)
    x = torch.randn(2, 8, 64)
    with pytest.raises(ShapeError):
        m(torch.randn(2, 8), x, x)
    with pytest.raises(ShapeError):
        m(x, torch.randn(3, 8, 64), x)
    with pytest.raises(ShapeError):
        m(x, torch.randn(2, 9, 64), x)
    with pytest.raises(ShapeError):
        m(torch.randn(2, 8, 32), x, x)
    with pytest.raises(TypeError):
        m(x.numpy(), x, x)


def test_cpu_tensors_are_refused():
    """There is no CPU path: the hot path fails loudly off the GPU."""
    q = torch.randn(1, 2, 16, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        analyze(q, q, scale=0.125)
    with pytest.raises(RuntimeError, match="CUDA"):
        attention_forward(q, q, q, scale=0.125)
    m = AdaAttention(embed_dim=128, num_heads=2).eval()
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 16, 128), torch.randn(1, 16, 128), torch.randn(1, 16, 128))


def test_oracle_config_defaults_match_module():
    cfg = O.OracleConfig()
    m = AdaAttention()
    assert cfg.rank_threshold == m.rank_threshold
    assert cfg.default_precision == m.default_precision.code
    assert cfg.allow_fp8 == m.allow_fp8 and cfg.eps == m.config.eps
