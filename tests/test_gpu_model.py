"""Whole-forward parity on a B200 against the FP32 oracle and the golden
vectors, with the reference's elementwise rule
(|opt-ref| <= 0.002 OR |opt-ref| <= 0.02*|ref|, failed_elements == 0;
torch_transformer_benchmark.py:1260-1264)."""

from __future__ import annotations

import pytest
import torch

from conftest import golden_cases, load_golden
from oracle import baseline as ob

pytestmark = pytest.mark.gpu

RTOL, ATOL = 0.02, 0.002


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _pair(pkg, cfg_kwargs, model_seed, dev):
    ocfg = ob.TransformerConfig(**cfg_kwargs)
    oracle_model = ob.make_baseline(ocfg, model_seed)
    cand = pkg.UserOptimizedTransformer(pkg.TransformerConfig(**cfg_kwargs))
    cand.load_state_dict(oracle_model.state_dict(), strict=True)
    return oracle_model, cand.to(dev).eval()


@pytest.mark.parametrize("name", golden_cases())
def test_forward_matches_golden(pkg, dev, name):
    rec = load_golden(name)
    cfg = rec["config"]
    _, cand = _pair(pkg, cfg, rec["model_seed"], dev)
    x, mask = ob.generate_random_case(ob.TransformerConfig(**cfg), rec["input_seed"],
                                      rec["padding_ratio"])
    with torch.inference_mode():
        y = cand(x.to(dev), mask.to(dev)).cpu()
    res = ob.compare_outputs(rec["output"], y, RTOL, ATOL)
    assert res.failed_elements == 0, (
        f"{name}: failed {res.failed_elements}/{res.total_elements} max_abs={res.max_abs_error}"
    )


def _check_config(pkg, dev, cfg_kwargs, trials=1, seed=1234):
    oracle_model, cand = _pair(pkg, cfg_kwargs, seed, dev)
    ocfg = ob.TransformerConfig(**cfg_kwargs)
    worst = 0.0
    for t in range(trials):
        x, mask = ob.generate_random_case(ocfg, seed + t)
        with torch.inference_mode():
            ref = oracle_model(x, mask)
            y = cand(x.to(dev), mask.to(dev)).cpu()
        res = ob.compare_outputs(ref, y, RTOL, ATOL)
        assert res.failed_elements == 0, (cfg_kwargs, res.failed_elements, res.max_abs_error)
        worst = max(worst, res.max_abs_error)
    return worst


def test_c1_full(pkg, dev):
    _check_config(pkg, dev, dict(batch_size=4, seq_len=128, d_model=128, num_heads=4,
                                 ffn_dim=128, num_layers=4, causal=True), trials=3)


def test_c2_geometry_b256(pkg, dev):
    _check_config(pkg, dev, dict(batch_size=256, seq_len=128, d_model=128, num_heads=4,
                                 ffn_dim=128, num_layers=4, causal=True))


def test_c3_full(pkg, dev):
    _check_config(pkg, dev, dict(batch_size=64, seq_len=128, d_model=1024, num_heads=4,
                                 ffn_dim=1024, num_layers=4, causal=True))


def test_c4_full(pkg, dev):
    _check_config(pkg, dev, dict(batch_size=64, seq_len=128, d_model=128, num_heads=16,
                                 ffn_dim=128, num_layers=4, causal=True))


@pytest.mark.parametrize("cfg", [
    # head_dim 128, ragged length, causal, padded batch
    dict(batch_size=3, seq_len=300, d_model=256, num_heads=2, ffn_dim=512, num_layers=2,
         causal=True),
    # head_dim 64, non-causal, length not a multiple of 8 (V^T row padding)
    dict(batch_size=2, seq_len=261, d_model=256, num_heads=4, ffn_dim=256, num_layers=2,
         causal=False),
])
def test_tcgen05_attention_head_dims_padded(pkg, dev, cfg):
    """head_dim 64/128 run the tcgen05 attention on a transposed V; padding
    masks keys past each sequence's length."""
    oracle_model, cand = _pair(pkg, cfg, 4321, dev)
    x, mask = ob.generate_random_case(ob.TransformerConfig(**cfg), 99, 0.3)
    with torch.inference_mode():
        ref = oracle_model(x, mask)
        y = cand(x.to(dev), mask.to(dev)).cpu()
    res = ob.compare_outputs(ref, y, RTOL, ATOL)
    assert res.failed_elements == 0, (res.failed_elements, res.max_abs_error)


def test_graph_replay_matches_eager(pkg, dev):
    cfg = dict(batch_size=4, seq_len=128, d_model=128, num_heads=4, ffn_dim=128,
               num_layers=4, causal=True)
    _, cand = _pair(pkg, cfg, 1234, dev)
    x, mask = ob.generate_random_case(ob.TransformerConfig(**cfg), 77)
    x, mask = x.to(dev), mask.to(dev)
    graphed, ok, reason = pkg.maybe_cuda_graph(cand, x, mask, enabled=True)
    assert ok, reason
    with torch.inference_mode():
        eager = cand(x, mask)
        replay = graphed(x, mask)
    assert torch.equal(eager, replay)


def test_no_device_timeout_recorded(pkg, dev):
    torch.cuda.synchronize()
    assert pkg._lib.read_device_error() == 0


FUSED_CASES = [
    # (batch, seq, d_model, heads, ffn, layers, causal[, padding_ratio])
    (4, 128, 128, 4, 128, 4, True),     # c1
    (300, 128, 128, 4, 128, 4, True),   # c2 geometry, several tiles per CTA
    (3, 128, 128, 16, 128, 2, True),    # head_dim 8 (c4 geometry): zero-padded K copies
    (5, 32, 128, 16, 128, 2, False),    # head_dim 8, 4 sequences per tile, non-causal
    (9, 128, 128, 16, 128, 2, True, 0.5),  # head_dim 8, prefix padding
    (3, 128, 128, 8, 128, 2, True),     # head_dim 16
    (3, 128, 128, 2, 128, 2, True),     # head_dim 64
    (2, 128, 128, 1, 128, 2, True),     # head_dim 128
    (5, 32, 128, 4, 128, 2, True),      # 4 sequences per tile, partial last tile
    (1203, 32, 128, 4, 128, 2, True),   # one CTA per tile (301 tiles), partial last tile
    # One CTA per tile (more tiles than half the SMs): the Q, K, V^T product order
    (160, 128, 128, 8, 128, 2, True),   # head_dim 16
    (160, 128, 128, 2, 128, 2, True),   # head_dim 64
    (160, 128, 128, 4, 128, 2, True, 0.5),  # head_dim 32, prefix padding (general instantiation)
    (7, 1, 128, 4, 128, 2, True),       # one token per sequence
    (6, 64, 128, 4, 128, 2, False),     # non-causal, block-diagonal tiles
    (2, 16, 128, 4, 128, 3, True),
    (9, 128, 128, 4, 128, 2, True, 0.5),   # prefix padding masks
    (9, 32, 128, 4, 128, 2, False, 0.6),
]


@pytest.mark.parametrize("case", FUSED_CASES)
def test_fused_forward_and_op_chain_match_oracle(pkg, dev, case):
    """The fused whole-forward kernel and the per-op kernel chain both pass
    the rule against the oracle on the same weights and inputs."""
    import ctypes

    b, s, d, h, f, l, causal = case[:7]
    pad = case[7] if len(case) > 7 else 0.0
    kw = dict(batch_size=b, seq_len=s, d_model=d, num_heads=h, ffn_dim=f, num_layers=l,
              causal=causal)
    oracle_model, cand = _pair(pkg, kw, 99, dev)
    x, mask = ob.generate_random_case(ob.TransformerConfig(**kw), 5, pad)
    lib = pkg._lib.load()
    _, _, _, mdl = cand._prepare(dev)
    outs = {}
    for policy in (1, 0):
        cand.enable_fused_forward(bool(policy))
        need = lib.tfx_forward_workspace_bytes(ctypes.byref(mdl), b, s)
        assert (need == 0) == (policy == 1), need
        with torch.inference_mode():
            outs[policy] = cand(x.to(dev), mask.to(dev)).cpu()
    with torch.inference_mode():
        ref = oracle_model(x, mask)
    for policy, y in outs.items():
        res = ob.compare_outputs(ref, y, RTOL, ATOL)
        assert res.failed_elements == 0, (case, policy, res.failed_elements, res.max_abs_error)
    assert (outs[0] - outs[1]).abs().max() < 2e-3


def test_no_device_timeout_after_fused(pkg, dev):
    torch.cuda.synchronize()
    assert pkg._lib.read_device_error() == 0


@pytest.mark.parametrize("cfg", [
    dict(batch_size=4, seq_len=128, d_model=128, num_heads=4, ffn_dim=128, num_layers=2,
         causal=True),   # fused whole-forward kernel
    dict(batch_size=2, seq_len=96, d_model=256, num_heads=4, ffn_dim=256, num_layers=2,
         causal=True),   # per-op chain (workspace shared across steps)
])
def test_streaming_forward_matches_model(pkg, dev, cfg):
    """Pipelined host-to-host forward of 5 different batches (slots reused)
    equals model(x) batch by batch, bit for bit."""
    _, cand = _pair(pkg, cfg, 1234, dev)
    b, s, d = cfg["batch_size"], cfg["seq_len"], cfg["d_model"]
    xs = [torch.randn(b, s, d, generator=torch.Generator().manual_seed(40 + i)).pin_memory()
          for i in range(5)]
    ys = [torch.full((b, s, d), float("nan")).pin_memory() for _ in range(5)]
    sf = pkg.StreamingForward(cand, dev, b, s)
    with torch.inference_mode():
        done = sf.run(xs, ys)
        done.synchronize()
        for x, y in zip(xs, ys):
            assert torch.equal(y, cand(x.to(dev)).cpu())


@pytest.mark.parametrize("cfg", [
    dict(batch_size=4, seq_len=128, d_model=128, num_heads=4, ffn_dim=128, num_layers=2,
         causal=True),   # fused whole-forward kernel
    dict(batch_size=2, seq_len=96, d_model=256, num_heads=4, ffn_dim=256, num_layers=2,
         causal=True),   # per-op chain
])
def test_streaming_capture_replays_match_model(pkg, dev, cfg):
    """StreamingForward.capture: the whole pipeline as one CUDA Graph over
    fixed pinned buffers; each replay (after refilling the inputs in place)
    equals model(x) batch by batch, bit for bit."""
    _, cand = _pair(pkg, cfg, 1234, dev)
    b, s, d = cfg["batch_size"], cfg["seq_len"], cfg["d_model"]
    xs = [torch.empty(b, s, d).pin_memory() for _ in range(3)]
    ys = [torch.full((b, s, d), float("nan")).pin_memory() for _ in range(3)]
    sf = pkg.StreamingForward(cand, dev, b, s)
    with torch.inference_mode():
        graph = sf.capture(xs, ys)
        for rep in range(2):
            for i, x in enumerate(xs):
                x.copy_(torch.randn(b, s, d, generator=torch.Generator().manual_seed(70 + 10 * rep + i)))
            graph.replay()
            torch.cuda.synchronize()
            for x, y in zip(xs, ys):
                assert torch.equal(y, cand(x.to(dev)).cpu())


@pytest.mark.parametrize("shape_id", list(range(1, 14)))
def test_official_shapes_match_oracle(pkg, dev, shape_id):
    """Every shape of the reference's official table (torch_transformer_benchmark.py:80-95)
    except 14 (c5: the prefix test above) on the GPU, full batch, against the FP32
    oracle on the first sequences (batch items are independent)."""
    import dataclasses

    cfg = dataclasses.asdict(pkg.OFFICIAL_BENCHMARK_SHAPES[shape_id])
    oracle_model, cand = _pair(pkg, cfg, 1234, dev)
    x, mask = ob.generate_random_case(ob.TransformerConfig(**cfg), 4321 + shape_id)
    n = min(cfg["batch_size"], 64)
    with torch.inference_mode():
        y = cand(x.to(dev), mask.to(dev)).cpu()
        ref = oracle_model(x[:n].contiguous(), mask[:n].contiguous())
    res = ob.compare_outputs(ref, y[:n], RTOL, ATOL)
    assert res.failed_elements == 0, (shape_id, res.failed_elements, res.max_abs_error)
    assert bool(torch.isfinite(y).all())


HOLE_CASES = [
    # (batch, seq, d_model, heads, ffn, layers, causal): fused kernel and chain
    (9, 128, 128, 4, 128, 2, True),    # fused, one sequence per tile
    (9, 32, 128, 4, 128, 2, False),    # fused, 4 sequences per tile
    (40, 8, 128, 8, 128, 2, True),     # fused, 16 sequences per tile (seq < 32)
    (9, 64, 128, 16, 128, 2, True),    # fused, head_dim 8
    (3, 200, 128, 4, 128, 2, True),    # chain, head_dim 32 attention
    (2, 261, 256, 4, 256, 2, False),   # chain, head_dim 64 (tcgen05, V transposed)
    (2, 150, 256, 2, 256, 2, True),    # chain, head_dim 128
    (4, 100, 128, 16, 128, 2, True),   # chain, head_dim 8
]


@pytest.mark.parametrize("case", HOLE_CASES)
def test_arbitrary_padding_masks_match_oracle(pkg, dev, case):
    """Padding masks with holes anywhere (not a prefix): the reference masks
    those keys in every layer and zeroes their output rows
    (torch_transformer_benchmark.py:237-253, 288-289, 314-316). Padded tokens
    carry random inputs, so any leak into a valid row would show."""
    b, s, d, h, f, l, causal = case
    kw = dict(batch_size=b, seq_len=s, d_model=d, num_heads=h, ffn_dim=f, num_layers=l,
              causal=causal)
    oracle_model, cand = _pair(pkg, kw, 31, dev)
    x = torch.randn(b, s, d, generator=torch.Generator().manual_seed(s))
    mask = torch.rand(b, s, generator=torch.Generator().manual_seed(s + 1)) > 0.35
    mask[0, 0] = False  # a causal query with no visible key
    mask[-1] = True     # and one unpadded sequence
    outs = []
    for fused in (True, False):
        cand.enable_fused_forward(fused)
        with torch.inference_mode():
            outs.append(cand(x.to(dev), mask.to(dev)).cpu())
    with torch.inference_mode():
        ref = oracle_model(x, mask)
    for y in outs:
        assert bool(torch.isfinite(y).all())
        assert bool((y[~mask] == 0).all())
        res = ob.compare_outputs(ref, y, RTOL, ATOL)
        assert res.failed_elements == 0, (case, res.failed_elements, res.max_abs_error)


@pytest.mark.parametrize("heads,seq", [(4, 128), (16, 128), (8, 32), (2, 128)])
def test_cta_pair_mode_equals_single_cta_mode(pkg, dev, heads, seq):
    """A batch of few tiles runs each tile on a CTA pair (heads split, ctx
    exchanged through distributed shared memory); a large batch runs one CTA
    per tile. The per-tile arithmetic is the same, so the same sequences give
    bit-identical outputs in both modes."""
    kw = dict(batch_size=256, seq_len=seq, d_model=128, num_heads=heads, ffn_dim=128,
              num_layers=2, causal=True)
    _, cand = _pair(pkg, kw, 17, dev)
    per_tile = 128 // seq
    small_b = 8 * per_tile                    # 8 tiles: CTA pairs
    big_b = 200 * per_tile                    # 200 tiles: more than half the SMs, one CTA each
    x = torch.randn(big_b, seq, 128, generator=torch.Generator().manual_seed(heads + seq))
    with torch.inference_mode():
        y_big = cand(x.to(dev))
        y_small = cand(x[:small_b].contiguous().to(dev))
    assert torch.equal(y_small, y_big[:small_b])


@pytest.mark.parametrize("heads,batch", [(4, 8), (4, 400), (16, 64), (16, 400), (1, 300)])
def test_plain_instantiation_equals_general_path(pkg, dev, heads, batch):
    """Causal 128-token sequences without a mask run the fused kernel's PLAIN
    instantiation (mask bookkeeping compiled out). The same input with an
    all-ones key bitmask runs the general instantiation; both must give
    bit-identical outputs, in CTA-pair mode (few tiles) and one-CTA mode."""
    import ctypes
    kw = dict(batch_size=batch, seq_len=128, d_model=128, num_heads=heads, ffn_dim=128,
              num_layers=2, causal=True)
    _, cand = _pair(pkg, kw, 29, dev)
    mdl = cand._prepare(dev)[3]
    lib = pkg._lib.load()
    x = torch.randn(batch, 128, 128, generator=torch.Generator().manual_seed(heads * batch)).to(dev)
    bits = pkg.model.key_bitmask(torch.ones(batch, 128, dtype=torch.bool, device=dev))
    y_plain = torch.empty_like(x)
    y_general = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    pkg._lib.check(lib.tfx_forward(ctypes.byref(mdl), x.data_ptr(), y_plain.data_ptr(), batch,
                                   128, None, None, 0, stream), "tfx_forward")
    pkg._lib.check(lib.tfx_forward_masked(ctypes.byref(mdl), x.data_ptr(), y_general.data_ptr(),
                                          batch, 128, bits.data_ptr(), None, 0, stream),
                   "tfx_forward_masked")
    torch.cuda.synchronize()
    assert torch.equal(y_plain, y_general)
