"""The allocation-free forward entry point, tfx_forward_static.

It exists for callers that cannot allocate device memory themselves (a
plugin inside a runtime that owns all GPU memory, an FFI binding that can
only pass the input and output buffers, a serving loop that must not
allocate after start-up): it runs the same kernels as tfx_forward, but keeps
the per-op chain's intermediates in a fixed 32 MiB device array inside the
library instead of a caller workspace.

Checked through the C ABI. Two calls in a row must give exactly what
tfx_forward with a caller workspace gives on the same inputs (the kernels are
deterministic and only the scratch address differs, so any dependence on
stale scratch contents would show as a difference): the first call uses a
longer sequence than the second, so the second runs over leftovers laid out
differently, and the array is first filled with NaN intermediates by a call
on a NaN input. Requests needing more than the array are rejected on the
host, and a config served by the fused whole-forward kernel (no scratch)
goes through the same entry point. This file is collected last on purpose
and is self-contained, so it also passes in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(batch_size=3, seq_len=40, d_model=256, num_heads=4, ffn_dim=512, num_layers=2,
           causal=True)  # d_model != 128: tfx_forward runs the per-op chain, which uses scratch


def _model(pkg, dev, cfg, seed):
    torch.manual_seed(seed)
    model = pkg.UserOptimizedTransformer(pkg.TransformerConfig(**cfg)).to(dev).eval()
    _, _, _, mdl = model._prepare(dev)
    return model, mdl


@pytest.fixture(scope="module")
def setup(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda:0")
    model, mdl = _model(pkg, dev, CFG, 21)
    return pkg, dev, model, mdl


def _both(pkg, lib, mdl, x, vl, dev):
    """(tfx_forward with a caller workspace, tfx_forward_static) on x."""
    b, s, _ = x.shape
    stream = torch.cuda.current_stream(dev).cuda_stream
    need = lib.tfx_forward_workspace_bytes(ctypes.byref(mdl), b, s)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    y_ws = torch.full_like(x, float("nan"))
    y_static = torch.full_like(x, float("nan"))
    vptr = vl.data_ptr() if vl is not None else None
    pkg._lib.check(lib.tfx_forward(ctypes.byref(mdl), x.data_ptr(), y_ws.data_ptr(), b, s, vptr,
                                   ws.data_ptr(), need, stream), "tfx_forward")
    pkg._lib.check(lib.tfx_forward_static(ctypes.byref(mdl), x.data_ptr(), y_static.data_ptr(),
                                          b, s, vptr, stream), "tfx_forward_static")
    torch.cuda.synchronize(dev)
    return y_ws, y_static, need


def test_static_scratch_forward_matches_workspace_forward(setup):
    pkg, dev, _, mdl = setup
    lib = pkg._lib.load()
    b, d = CFG["batch_size"], CFG["d_model"]
    # Leave NaN intermediates everywhere the chain writes at the longest shape.
    x_nan = torch.full((b, 64, d), float("nan"), device=dev)
    y_nan = torch.empty_like(x_nan)
    pkg._lib.check(lib.tfx_forward_static(ctypes.byref(mdl), x_nan.data_ptr(), y_nan.data_ptr(),
                                          b, 64, None, torch.cuda.current_stream(dev).cuda_stream),
                   "tfx_forward_static (NaN fill)")
    torch.cuda.synchronize(dev)
    # Then two calls in a row, the first longer than the second.
    for call, (seed, s, lengths) in enumerate(((1, 64, None), (2, 40, [40, 23, 1]))):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(b, s, d, generator=g).to(dev)
        vl = torch.tensor(lengths, dtype=torch.int32, device=dev) if lengths else None
        y_ws, y_static, need = _both(pkg, lib, mdl, x, vl, dev)
        assert need > 0, "this config must take the scratch-using per-op chain"
        assert torch.isfinite(y_static).all(), f"call {call}: non-finite output"
        assert torch.equal(y_static, y_ws), (
            f"call {call}: max |static - workspace| = {(y_static - y_ws).abs().max().item()}")
    assert pkg._lib.read_device_error() == 0


def test_static_entry_serves_the_fused_kernel_without_scratch(pkg):
    """d_model = ffn_dim = 128: the fused kernel needs no scratch at all, and
    the static entry point gives the same output as tfx_forward."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda:0")
    cfg = dict(batch_size=5, seq_len=128, d_model=128, num_heads=4, ffn_dim=128, num_layers=2,
               causal=True)
    _, mdl = _model(pkg, dev, cfg, 5)
    lib = pkg._lib.load()
    x = torch.randn(5, 128, 128, generator=torch.Generator().manual_seed(3)).to(dev)
    y_ws, y_static, need = _both(pkg, lib, mdl, x, None, dev)
    assert need == 0
    assert torch.equal(y_static, y_ws)
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
    msg = lib.tfx_last_error_message().decode()
    assert "more than the library's fixed 33554432-byte array" in msg, msg
