"""The CPU oracle against the golden vectors the reference itself produced.

``tests/golden/*.pt`` were written by ``tests/golden/make_golden.py`` from the
reference's own ``BaselineTransformer`` / ``generate_random_case`` /
``compare_outputs``. These tests pin the oracle restatement to them: same
seeded weights (state_dict hash), same inputs (hash), same outputs, same
accuracy-rule verdicts.
"""

from __future__ import annotations

import pytest
import torch

from conftest import golden_cases, load_golden
from oracle import baseline as ob


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_reference_golden(name):
    rec = load_golden(name)
    cfg = ob.TransformerConfig(**rec["config"])
    model = ob.make_baseline(cfg, rec["model_seed"])
    assert ob.state_dict_checksum(model) == rec["state_sha256"]
    x, mask = ob.generate_random_case(cfg, rec["input_seed"], rec["padding_ratio"])
    assert torch.equal(mask, rec["mask"])
    import hashlib

    assert hashlib.sha256(x.float().numpy().tobytes()).hexdigest() == rec["input_sha256"]
    with torch.inference_mode():
        y = model(x, mask)
    # Same op sequence on the same CPU build: agreement to float32 rounding.
    assert torch.allclose(y, rec["output"], rtol=0, atol=2e-5), (
        (y - rec["output"]).abs().max()
    )
    res = ob.compare_outputs(rec["output"], y)
    assert res.passed and res.failed_elements == 0


@pytest.mark.parametrize("name", golden_cases())
def test_compare_rule_matches_reference_verdict(name):
    rec = load_golden(name)
    y = rec["output"]
    pert = y.clone()
    flat = pert.view(-1)
    idx = rec["perturb_index"]
    flat[idx] += torch.linspace(-0.01, 0.01, idx.numel())
    res = ob.compare_outputs(y, pert)
    assert res.failed_elements == rec["perturb_failed"]
    assert abs(res.max_abs_error - rec["perturb_max_abs"]) < 1e-9
    assert tuple(res.worst_index) == tuple(rec["perturb_worst_index"])


def test_compare_rule_is_or_not_isclose():
    ref = torch.tensor([1.0, 1.0, 0.0, 10.0])
    # 0.0025 > atol but <= 2% of 1.0 -> passes; 0.003 at ref 0 -> fails;
    # 0.19 at ref 10 -> passes (rel); torch.isclose would also accept 0.0219.
    opt = torch.tensor([1.0025, 1.0219, 0.003, 10.19])
    res = ob.compare_outputs(ref, opt)
    assert res.failed_elements == 2
    assert not res.passed


def test_causal_prefix_property():
    """Rows [:, :S'] of a causal model depend only on inputs [:, :S'] -- the
    basis of the long-sequence (S=100000) prefix parity check."""
    cfg = ob.TransformerConfig(1, 96, 64, 4, 64, 2, True)
    model = ob.make_baseline(cfg, 3)
    x, _ = ob.generate_random_case(cfg, 4)
    with torch.inference_mode():
        full = model(x)
        pre = model(x[:, :40])
    assert torch.allclose(full[:, :40], pre, atol=1e-5, rtol=0)


def test_blockwise_attention_matches_explicit():
    torch.manual_seed(0)
    q, k, v = (torch.randn(300, 16) for _ in range(3))
    out = ob.blockwise_causal_attention_fp64(q, k, v, 0.25, block=64)
    sc = (q.double() @ k.double().T) * 0.25
    sc = sc.masked_fill(torch.ones(300, 300, dtype=torch.bool).triu(1), float("-inf"))
    ref = torch.softmax(sc, -1) @ v.double()
    assert torch.allclose(out, ref, atol=1e-12)


def test_rows_attention_oracle_equals_blockwise():
    """causal_attention_rows_fp64 (late-row spot checks) agrees with the
    blockwise float64 attention on every row it is asked for."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(300, 16, generator=g) for _ in range(3))
    full = ob.blockwise_causal_attention_fp64(q, k, v, 0.25, block=64)
    rows = torch.tensor([0, 5, 150, 299])
    assert torch.allclose(ob.causal_attention_rows_fp64(q, k, v, rows, 0.25), full[rows],
                          atol=1e-12, rtol=0)
