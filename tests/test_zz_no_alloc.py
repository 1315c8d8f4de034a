"""The allocation-free forward entry point, tfx_forward_static.

It exists for callers that cannot allocate device memory themselves (a
plugin inside a runtime that owns all GPU memory, an FFI binding that can
only pass the input and output buffers, a serving loop that must not
allocate after start-up): it runs the same per-op kernel chain as
tfx_forward, but keeps the intermediates in a fixed 32 MiB device array
inside the library instead of a caller workspace.

Checked through the C ABI: two calls in a row (the second on different
inputs, with a padding mask, over the leftovers of the first) must match
tfx_forward with a caller workspace on the same inputs, within the
element tolerance the other tests use (|diff| <= 0.002); requests needing
more than the array are rejected on the host. This file is collected last
on purpose and is self-contained, so it also passes in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL = 0.002
CFG = dict(batch_size=3, seq_len=40, d_model=256, num_heads=4, ffn_dim=512, num_layers=2,
           causal=True)  # d_model != 128: tfx_forward runs the per-op chain, which uses scratch


@pytest.fixture(scope="module")
def setup(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda:0")
    torch.manual_seed(21)
    model = pkg.UserOptimizedTransformer(pkg.TransformerConfig(**CFG)).to(dev).eval()
    _, _, _, mdl = model._prepare(dev)
    return pkg, dev, model, mdl


def test_static_scratch_forward_matches_workspace_forward(setup):
    pkg, dev, _, mdl = setup
    lib = pkg._lib.load()
    b, s, d = CFG["batch_size"], CFG["seq_len"], CFG["d_model"]
    need = lib.tfx_forward_workspace_bytes(ctypes.byref(mdl), b, s)
    assert need > 0, "this config must take the scratch-using per-op chain"
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    lengths = torch.tensor([40, 23, 1], dtype=torch.int32, device=dev)
    for call, (seed, valid) in enumerate(((1, None), (2, lengths))):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(b, s, d, generator=g).to(dev)
        y_ws = torch.full_like(x, float("nan"))
        y_static = torch.full_like(x, float("nan"))
        vl = valid.data_ptr() if valid is not None else None
        pkg._lib.check(lib.tfx_forward(ctypes.byref(mdl), x.data_ptr(), y_ws.data_ptr(), b, s,
                                       vl, ws.data_ptr(), need, stream), "tfx_forward")
        pkg._lib.check(lib.tfx_forward_static(ctypes.byref(mdl), x.data_ptr(),
                                              y_static.data_ptr(), b, s, vl, stream),
                       "tfx_forward_static")
        torch.cuda.synchronize(dev)
        assert torch.isfinite(y_static).all(), f"call {call}: non-finite output"
        err = (y_static - y_ws).abs().max().item()
        assert err <= ATOL, f"call {call}: max |static - workspace| = {err}"
    assert pkg._lib.read_device_error() == 0


def test_static_scratch_rejects_oversized_requests(setup):
    pkg, dev, _, mdl = setup
    lib = pkg._lib.load()
    x = torch.zeros(1, 8, CFG["d_model"], device=dev)
    y = torch.empty_like(x)
    # 10000 x 128 tokens at d_model 256 need ~5.9 GB of scratch, far above 32 MiB.
    st = lib.tfx_forward_static(ctypes.byref(mdl), x.data_ptr(), y.data_ptr(), 10000, 128,
                                None, torch.cuda.current_stream(dev).cuda_stream)
    assert st == pkg._lib.TFX_ERR_WORKSPACE
    assert b"32" in lib.tfx_last_error_message() or b"scratch" in lib.tfx_last_error_message()
