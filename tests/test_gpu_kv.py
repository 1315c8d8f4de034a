"""KV-cached incremental decoding on a B200 (tfx_forward_kv through the
module API), against the FP32 oracle.

The reference's KV path (torch_transformer_benchmark.py:409-462, 747-765,
1085-1086) feeds a sequence in chunks; chunk tokens attend every cached key
at or before their position. For a causal model that is exactly the full
forward's rows for those positions, so the oracle is the FP32 baseline on
the concatenated prefix, compared with the reference's elementwise rule
(|opt-ref| <= 0.002 OR <= 0.02*|ref|, no failed element).
"""

from __future__ import annotations

import pytest
import torch

from oracle import baseline as ob

pytestmark = pytest.mark.gpu

RTOL, ATOL = 0.02, 0.002


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


KV_CASES = [
    # (batch, capacity, d_model, heads, ffn, layers, chunk sizes)
    (2, 48, 128, 4, 128, 2, [20, 1, 1, 7, 1, 10]),      # hd 32: mma kernel
    (2, 16, 128, 16, 128, 2, [5, 1, 3, 1]),             # hd 8
    (2, 12, 128, 8, 128, 1, [3, 1, 1, 1, 2]),           # hd 16
    (2, 300, 256, 4, 512, 2, [130, 1, 1, 140, 1]),      # hd 64: tcgen05, chunk crosses a tile
    (3, 200, 256, 2, 256, 1, [64, 1, 70, 2]),           # hd 128
    (1, 160, 512, 2, 512, 1, [40, 1, 1, 90]),           # hd 256
    (1, 260, 128, 4, 128, 1, [1] + [1] * 6 + [250]),    # decode from one token, then a long chunk
    # 16 new tokens: the last split-KV decode step; 17: the offset path. Long
    # caches with few (batch, head) pairs split the keys over several CTAs.
    (1, 2100, 128, 2, 128, 1, [2000, 1, 16, 17, 1]),     # hd 64, up to 8 splits
    (2, 700, 128, 4, 128, 1, [600, 16, 3, 17, 2]),       # hd 32
    (1, 1100, 512, 2, 512, 1, [1000, 1, 5, 16]),         # hd 256, several splits
    (1, 600, 128, 16, 128, 1, [520, 1, 16, 9]),          # hd 8
]


def _models(pkg, dev, b, cap, d, h, f, layers, seed=77):
    kw = dict(batch_size=b, seq_len=cap, d_model=d, num_heads=h, ffn_dim=f, num_layers=layers,
              causal=True)
    ocfg = ob.TransformerConfig(**kw)
    oracle_model = ob.make_baseline(ocfg, seed)
    cand = pkg.UserOptimizedTransformer(pkg.TransformerConfig(**kw))
    cand.load_state_dict(oracle_model.state_dict(), strict=True)
    x, _ = ob.generate_random_case(ocfg, seed + 1)
    return oracle_model, cand.to(dev).eval(), x


def _decode(cand, x, chunks, dev):
    outs, start = [], 0
    with torch.inference_mode():
        for n in chunks:
            outs.append(cand(x[:, start:start + n].to(dev)).cpu())
            start += n
            assert cand.kv_cache_length == start
    return torch.cat(outs, dim=1)


@pytest.mark.parametrize("b,cap,d,h,f,layers,chunks", KV_CASES)
def test_incremental_decode_matches_full_forward_oracle(pkg, dev, b, cap, d, h, f, layers,
                                                        chunks):
    oracle_model, cand, x = _models(pkg, dev, b, cap, d, h, f, layers)
    total = sum(chunks)
    with torch.inference_mode():
        ref = oracle_model(x[:, :total].contiguous(), None)
    cand.enable_kv_cache(True)
    got = _decode(cand, x, chunks, dev)
    res = ob.compare_outputs(ref, got, RTOL, ATOL)
    assert res.failed_elements == 0, (chunks, res.failed_elements, res.max_abs_error)
    # After a reset the same sequence decodes again, in another chunking.
    cand.reset_kv_cache()
    again = _decode(cand, x, [total - 1, 1], dev)
    res = ob.compare_outputs(ref, again, RTOL, ATOL)
    assert res.failed_elements == 0, ("rechunked", res.failed_elements, res.max_abs_error)


def test_kv_cache_rules_on_device(pkg, dev):
    """Capacity, padding and shape rules (torch_transformer_benchmark.py:
    431-458, 1057-1063), raised before anything is enqueued."""
    _, cand, x = _models(pkg, dev, 2, 16, 128, 4, 128, 1)
    cand.enable_kv_cache(True)
    with torch.inference_mode():
        cand(x[:, :10].to(dev))
        with pytest.raises(ValueError, match="capacity exceeded"):
            cand(torch.randn(2, 7, 128, device=dev))  # 10 + 7 > 16
        assert cand.kv_cache_length == 10
        mask = torch.ones(2, 2, dtype=torch.bool, device=dev)
        mask[1, 1] = False
        with pytest.raises(ValueError, match="padding"):
            cand(x[:, 10:12].to(dev), mask)
        cand(x[:, 10:12].to(dev), torch.ones(2, 2, dtype=torch.bool, device=dev))
        assert cand.kv_cache_length == 12
        with pytest.raises(RuntimeError, match="does not match"):
            cand(x[:1, 12:13].to(dev))


def test_graph_helper_keeps_kv_decoding_eager(pkg, dev):
    _, cand, x = _models(pkg, dev, 1, 16, 128, 4, 128, 1)
    cand.enable_kv_cache(True)
    wrapped, graphed, reason = pkg.maybe_cuda_graph(cand, x[:, :4].to(dev), None, True)
    assert wrapped is cand and not graphed and "KV-cache" in reason
    assert cand.kv_cache_length == 0


def test_no_device_timeout_after_kv(pkg, dev):
    torch.cuda.synchronize()
    assert pkg._lib.read_device_error() == 0
