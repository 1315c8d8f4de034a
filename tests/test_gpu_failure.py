"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every pipelined kernel of the library waits on mbarriers for a bounded time
and, on timeout, records a code in the per-device error word and unwinds
(drains its own copies, frees TMEM) instead of hanging. Here a wait that
cannot complete (an mbarrier no thread arrives on) runs out after a short
limit; the test checks the recorded code, that the kernel returned (the
stream synchronises within seconds), that the word is cleared by the read,
and that an ordinary forward afterwards still passes the accuracy rule.
"""

from __future__ import annotations

import time

import pytest
import torch

from oracle import baseline as ob

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def test_bounded_wait_runs_out_and_the_context_survives(pkg, dev):
    lib = pkg._lib.load()
    torch.cuda.synchronize()
    assert pkg._lib.read_device_error() == 0
    stream = torch.cuda.current_stream(dev).cuda_stream
    t0 = time.perf_counter()
    # ~10 ms at the B200's 1.9 GHz SM clock
    pkg._lib.check(lib.tfx_selftest_bounded_wait(20_000_000, stream), "tfx_selftest_bounded_wait")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 5.0, elapsed
    assert pkg._lib.read_device_error() == pkg._lib.TFX_DEV_TIMEOUT_ACCUM
    assert pkg._lib.read_device_error() == 0  # the read cleared it

    kw = dict(batch_size=4, seq_len=128, d_model=128, num_heads=4, ffn_dim=128, num_layers=2,
              causal=True)
    ref_model = ob.make_baseline(ob.TransformerConfig(**kw), 8)
    model = pkg.UserOptimizedTransformer(pkg.TransformerConfig(**kw))
    model.load_state_dict(ref_model.state_dict(), strict=True)
    model = model.to(dev).eval()
    x, _ = ob.generate_random_case(ob.TransformerConfig(**kw), 9)
    with torch.inference_mode():
        y = model(x.to(dev)).cpu()
        ref = ref_model(x)
    res = ob.compare_outputs(ref, y, 0.02, 0.002)
    assert res.failed_elements == 0, (res.failed_elements, res.max_abs_error)
    assert pkg._lib.read_device_error() == 0
