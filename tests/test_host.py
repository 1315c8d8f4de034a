"""Host-side logic of the drop-in module, on the CPU (no GPU, no kernels):
config validation, parameter names and seeded initialisation identical to
the reference model, weight packing layout, mask handling, and the
no-fallback rule."""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden
from oracle import baseline as ob


def test_config_validation_matches_reference(pkg):
    pkg.TransformerConfig(4, 128, 128, 4, 128, 4, True).validate()
    bad = [
        dict(batch_size=0), dict(seq_len=0), dict(d_model=0), dict(num_heads=0),
        dict(num_heads=3), dict(ffn_dim=0), dict(num_layers=0),
    ]
    base = dict(batch_size=4, seq_len=128, d_model=128, num_heads=4, ffn_dim=128,
                num_layers=4, causal=True)
    for b in bad:
        kw = {**base, **b}
        with pytest.raises(ValueError):
            pkg.TransformerConfig(**kw).validate()
        with pytest.raises(ValueError):
            ob.TransformerConfig(**kw).validate()


def test_official_shapes_contain_the_benchmark_configs(pkg):
    shapes = pkg.OFFICIAL_BENCHMARK_SHAPES
    assert shapes[3] == pkg.TransformerConfig(4, 128, 128, 4, 128, 4, True)
    assert shapes[6] == pkg.TransformerConfig(10000, 128, 128, 4, 128, 4, True)
    assert shapes[8] == pkg.TransformerConfig(64, 128, 1024, 4, 1024, 4, True)
    assert shapes[11] == pkg.TransformerConfig(64, 128, 128, 16, 128, 4, True)
    assert shapes[14] == pkg.TransformerConfig(32, 100000, 1024, 16, 1024, 2, True)
    assert "official-6" in pkg.UserOptimizedTransformer(shapes[6]).shape_execution_plan.describe()


@pytest.mark.parametrize("name", ["c1", "c3_b1", "c5_s256"])
def test_seeded_init_and_state_dict_match_reference(pkg, name):
    """torch.manual_seed(s) + construction draws the reference's weights, and
    the state_dict keys are the reference's (golden state hash)."""
    rec = load_golden(name)
    torch.manual_seed(rec["model_seed"])
    cand = pkg.UserOptimizedTransformer(pkg.TransformerConfig(**rec["config"]))
    assert ob.state_dict_checksum(cand) == rec["state_sha256"]
    oracle_model = ob.make_baseline(ob.TransformerConfig(**rec["config"]), rec["model_seed"])
    assert list(cand.state_dict().keys()) == list(oracle_model.state_dict().keys())
    cand.load_state_dict(oracle_model.state_dict(), strict=True)


def test_weight_packing_layout(pkg):
    cfg = pkg.TransformerConfig(2, 16, 64, 4, 96, 2, True)
    torch.manual_seed(0)
    m = pkg.UserOptimizedTransformer(cfg)
    key, keep, layers, model = m._prepare(torch.device("cpu"))
    assert model.d_model == 64 and model.num_heads == 4 and model.ffn_dim == 96
    assert model.num_layers == 2 and model.causal == 1
    ptrs = {t.data_ptr(): t for t in keep}
    att = m.layers[1].attention
    qkv = ptrs[layers[1].qkv_weight]
    assert qkv.dtype == torch.float16 and qkv.shape == (192, 64)
    ref = torch.cat((att.q_proj.weight, att.k_proj.weight, att.v_proj.weight)).half()
    assert torch.equal(qkv, ref)
    bias = ptrs[layers[1].qkv_bias]
    assert bias.dtype == torch.float32 and torch.equal(
        bias, torch.cat((att.q_proj.bias, att.k_proj.bias, att.v_proj.bias)))
    w1 = ptrs[layers[0].ffn_in_weight]
    assert w1.shape == (96, 64) and w1.dtype == torch.float16
    # cache hit on an unchanged model, repack after an in-place update
    assert m._prepare(torch.device("cpu"))[0] == key
    with torch.no_grad():
        m.layers[0].ffn_in.weight.add_(1.0)
    assert m._prepare(torch.device("cpu"))[0] != key


def test_mask_handling(pkg):
    cfg = pkg.TransformerConfig(3, 8, 64, 4, 64, 1, True)
    m = pkg.UserOptimizedTransformer(cfg)
    x = torch.zeros(3, 8, 64)
    assert m._valid_lengths(x, None) is None
    assert m._valid_lengths(x, torch.ones(3, 8, dtype=torch.bool)) is None
    mask = torch.arange(8)[None, :] < torch.tensor([8, 5, 1])[:, None]
    lengths = m._valid_lengths(x, mask)
    assert lengths.dtype == torch.int32 and lengths.tolist() == [8, 5, 1]
    holes = mask.clone()
    holes[0, 3] = False
    bits = m._valid_lengths(x, holes)
    assert bits.dtype == torch.int32 and bits.shape == (3, 1)
    assert bits[:, 0].tolist() == [0b11110111, 0b11111, 0b1]
    with pytest.raises(ValueError):
        m._valid_lengths(x, torch.ones(3, 7, dtype=torch.bool))


def test_key_bitmask_layout(pkg):
    """Bit k of word w of row b is mask[b, 32w + k], including bit 31 (sign)
    and a ragged last word."""
    from importlib import import_module

    model = import_module(pkg.__name__ + ".model")
    g = torch.Generator().manual_seed(0)
    mask = torch.rand(4, 70, generator=g) > 0.5
    mask[0, 31] = True
    words = model.key_bitmask(mask)
    assert words.shape == (4, 3) and words.dtype == torch.int32
    u = words.to(torch.int64) & 0xFFFFFFFF
    for b in range(4):
        for t in range(70):
            assert bool((u[b, t // 32] >> (t % 32)) & 1) == bool(mask[b, t])
        assert int(u[b, 2]) >> 6 == 0  # bits past S are zero


def test_no_cpu_fallback(pkg):
    m = pkg.UserOptimizedTransformer(pkg.TransformerConfig(1, 8, 128, 4, 128, 1, True))
    with pytest.raises(RuntimeError):
        m(torch.zeros(1, 8, 128))


@pytest.mark.parametrize("name", ["c1", "padded_c1", "ragged_s37", "noncausal_small", "c4_b2"])
def test_package_baseline_forward_matches_golden(pkg, name):
    """The package's own BaselineTransformer (eager FP32, no oracle import)
    reproduces the reference's recorded outputs, masks included."""
    rec = load_golden(name)
    cfg = pkg.TransformerConfig(**rec["config"])
    torch.manual_seed(rec["model_seed"])
    model = pkg.BaselineTransformer(cfg).eval()
    assert ob.state_dict_checksum(model) == rec["state_sha256"]
    x, mask = ob.generate_random_case(ob.TransformerConfig(**rec["config"]), rec["input_seed"],
                                      rec["padding_ratio"])
    with torch.inference_mode():
        y = model(x, mask)
    assert torch.allclose(y, rec["output"], atol=2e-5, rtol=0), (y - rec["output"]).abs().max()


def test_package_baseline_forward_equals_oracle_on_holes(pkg):
    """Arbitrary (non-prefix) masks: the package baseline and the oracle agree."""
    cfg = dict(batch_size=3, seq_len=20, d_model=64, num_heads=4, ffn_dim=96, num_layers=2,
               causal=True)
    oracle_model = ob.make_baseline(ob.TransformerConfig(**cfg), 3)
    torch.manual_seed(3)
    model = pkg.BaselineTransformer(pkg.TransformerConfig(**cfg)).eval()
    x = torch.randn(3, 20, 64, generator=torch.Generator().manual_seed(4))
    mask = torch.rand(3, 20, generator=torch.Generator().manual_seed(5)) > 0.3
    mask[:, 0] = True
    with torch.inference_mode():
        assert torch.allclose(model(x, mask), oracle_model(x, mask), atol=1e-6, rtol=0)


def test_cpu_scenario_of_the_reference_validation(pkg):
    """validate_transformer.py:77-104's CPU run (B=2, S=16, D=128, H=4,
    F=512, 2 layers, FP32): the package's eager BaselineTransformer against
    the oracle on two seeded trials."""
    cfg = dict(batch_size=2, seq_len=16, d_model=128, num_heads=4, ffn_dim=512, num_layers=2,
               causal=False)
    oracle_model = ob.make_baseline(ob.TransformerConfig(**cfg), 1234)
    torch.manual_seed(1234)
    model = pkg.BaselineTransformer(pkg.TransformerConfig(**cfg)).eval()
    for t in range(2):
        x, mask = ob.generate_random_case(ob.TransformerConfig(**cfg), 1234 + t)
        with torch.inference_mode():
            res = ob.compare_outputs(oracle_model(x, mask), model(x, mask), 0.02, 0.002)
        assert res.failed_elements == 0 and res.max_abs_error < 1e-5


def test_fused_toggle_is_per_module(pkg):
    cfg = pkg.TransformerConfig(2, 16, 64, 4, 96, 1, True)
    a = pkg.UserOptimizedTransformer(cfg)
    b = pkg.UserOptimizedTransformer(cfg)
    a.enable_fused_forward(False)
    assert a._prepare(torch.device("cpu"))[3].path == pkg._lib.TFX_PATH_CHAIN
    assert b._prepare(torch.device("cpu"))[3].path == pkg._lib.TFX_PATH_AUTO
    a.enable_fused_forward(True)
    assert a._prepare(torch.device("cpu"))[3].path == pkg._lib.TFX_PATH_AUTO


def test_inference_tensor_parameters_pack_once_and_repack_on_change(pkg):
    """Parameters created under inference_mode have no version counter: the
    packed weights are reused while their contents are unchanged and rebuilt
    after an in-place update."""
    cfg = pkg.TransformerConfig(2, 16, 64, 4, 96, 1, True)
    with torch.inference_mode():
        m = pkg.UserOptimizedTransformer(cfg)
        first = m._prepare(torch.device("cpu"))
        assert m._prepare(torch.device("cpu")) is first
        m.layers[0].ffn_out.weight.mul_(2.0)
        assert m._prepare(torch.device("cpu")) is not first


def test_toggles_keep_reference_contract(pkg):
    m = pkg.UserOptimizedTransformer(pkg.TransformerConfig(1, 8, 128, 4, 128, 1, True))
    m.enable_mixed_precision(torch.float16)
    with pytest.warns(UserWarning):
        m.enable_mixed_precision(torch.bfloat16)
    with pytest.raises(ValueError):
        m.enable_mixed_precision(torch.float64)
    with pytest.raises(ValueError):
        m.enable_attention_fp16_accumulation(True)
    m.enable_attention_fp16_accumulation(False)
    m.enable_triton_fused_norm(True)
    m.enable_triton_fused_ffn(True)


def test_kv_cache_contract(pkg):
    """torch_transformer_benchmark.py:409-424, 1000-1003: causal models only,
    eval mode only, reset clears the length, CPU inputs are refused."""
    cfg = pkg.TransformerConfig(1, 8, 128, 4, 128, 1, False)
    with pytest.raises(ValueError, match="causal"):
        pkg.UserOptimizedTransformer(cfg).enable_kv_cache(True)
    m = pkg.UserOptimizedTransformer(pkg.TransformerConfig(1, 8, 128, 4, 128, 1, True))
    with pytest.raises(RuntimeError, match="eval"):
        m.enable_kv_cache(True)
    m.eval()
    m.enable_kv_cache(True)
    assert m.kv_cache_length == 0
    with pytest.raises(RuntimeError, match="CUDA inference"):
        m(torch.zeros(1, 2, 128))
    m._kv_cache_length = 3  # as after a decoded chunk
    with pytest.raises(RuntimeError, match="reset the KV cache"):
        m.enable_mixed_precision(torch.float16)
    m.reset_kv_cache()
    assert m.kv_cache_length == 0
    m.enable_mixed_precision(torch.float16)
    m.enable_kv_cache(False)
    assert not m._kv_cache_enabled


def test_ops_reject_cpu_tensors(pkg):
    x = torch.zeros(4, 128)
    with pytest.raises(ValueError):
        pkg.ops.layer_norm(x, torch.ones(128), torch.zeros(128), 1e-5, torch.float16)
    with pytest.raises(ValueError):
        pkg.ops.linear(x.half(), torch.zeros(32, 128).half(), torch.zeros(32))
