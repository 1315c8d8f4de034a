"""The reference's validation scenarios (validate_transformer.py:43-104), as
tests: its default CLI model (torch_transformer_benchmark.py:1567-1572:
B=8, S=128, D=512, H=8, F=2048, 6 layers, non-causal), the same model causal,
a fixed padding mask replayed through a CUDA graph, the module with its fused
kernel switched off (the reference's "native fallbacks" run), each over
several accuracy trials with seed + trial (torch_transformer_benchmark.py
:1331-1338) against the FP32 oracle with the reference's rule. The CPU
scenario is in test_host.py (the package's eager BaselineTransformer)."""

from __future__ import annotations

import pytest
import torch

from oracle import baseline as ob

pytestmark = pytest.mark.gpu

RTOL, ATOL = 0.02, 0.002
SEED = 1234
DEFAULT_CLI = dict(batch_size=8, seq_len=128, d_model=512, num_heads=8, ffn_dim=2048,
                   num_layers=6, causal=False)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _pair(pkg, cfg, dev):
    oracle_model = ob.make_baseline(ob.TransformerConfig(**cfg), SEED)
    cand = pkg.UserOptimizedTransformer(pkg.TransformerConfig(**cfg))
    cand.load_state_dict(oracle_model.state_dict(), strict=True)
    return oracle_model, cand.to(dev).eval()


def _trials(oracle_model, cand, cfg, dev, trials=3, padding=0.0):
    for t in range(trials):
        x, mask = ob.generate_random_case(ob.TransformerConfig(**cfg), SEED + t, padding)
        with torch.inference_mode():
            ref = oracle_model(x, mask)
            y = cand(x.to(dev), mask.to(dev)).cpu()
        res = ob.compare_outputs(ref, y, RTOL, ATOL)
        assert res.failed_elements == 0, (t, res.failed_elements, res.max_abs_error)


@pytest.mark.parametrize("causal", [False, True])
def test_default_cli_model(pkg, dev, causal):
    cfg = {**DEFAULT_CLI, "causal": causal}
    oracle_model, cand = _pair(pkg, cfg, dev)
    _trials(oracle_model, cand, cfg, dev)


def test_fixed_padding_mask_cuda_graph(pkg, dev):
    """padding_ratio 0.25 through maybe_cuda_graph: replay equals eager bit for
    bit and passes the rule."""
    cfg = DEFAULT_CLI
    oracle_model, cand = _pair(pkg, cfg, dev)
    x, mask = ob.generate_random_case(ob.TransformerConfig(**cfg), SEED, 0.25)
    assert not bool(mask.all())
    xd, md = x.to(dev), mask.to(dev)
    graphed, ok, reason = pkg.maybe_cuda_graph(cand, xd, md, enabled=True)
    assert ok, reason
    with torch.inference_mode():
        eager = cand(xd, md)
        replay = graphed(xd, md)
        ref = oracle_model(x, mask)
    assert torch.equal(eager, replay)
    res = ob.compare_outputs(ref, replay.cpu(), RTOL, ATOL)
    assert res.failed_elements == 0, (res.failed_elements, res.max_abs_error)


def test_fused_kernel_switched_off(pkg, dev):
    """A config the fused kernel serves (c1), with the module's fused path
    off: the per-op kernel chain runs and passes the rule."""
    cfg = dict(batch_size=4, seq_len=128, d_model=128, num_heads=4, ffn_dim=128, num_layers=4,
               causal=True)
    oracle_model, cand = _pair(pkg, cfg, dev)
    cand.enable_fused_forward(False)
    import ctypes

    mdl = cand._prepare(dev)[3]
    assert pkg._lib.load().tfx_forward_workspace_bytes(ctypes.byref(mdl), 4, 128) > 0
    _trials(oracle_model, cand, cfg, dev, padding=0.25)
