"""The C-ABI library: it loads without a GPU, exports every symbol that
include/tfx.h declares, and rejects bad arguments on the host (no kernel is
launched, no CUDA call made) with the documented status codes."""

from __future__ import annotations

import ctypes
import pathlib
import re

import pytest

from conftest import ROOT, load_package

HEADER = ROOT / "include" / "tfx.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(tfx_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    pkg = load_package()
    build = __import__("importlib").import_module(pkg.__name__ + ".build")
    build.build()
    return pkg._lib.load()


def test_header_declares_the_expected_api():
    syms = declared_symbols()
    for name in ("tfx_layer_norm", "tfx_residual_layer_norm", "tfx_linear", "tfx_attention",
                 "tfx_forward", "tfx_forward_workspace_bytes", "tfx_version"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_python_binding_covers_the_header():
    pkg = load_package()
    assert set(declared_symbols()) == set(pkg._lib.SIGNATURES)


def test_version_and_status_strings(lib):
    assert lib.tfx_version() >= 100
    assert lib.tfx_status_string(0) == b"ok"
    assert b"alignment" in lib.tfx_status_string(-3) or b"misaligned" in lib.tfx_status_string(-3)


def test_host_side_argument_errors(lib):
    pkg = load_package()
    L = pkg._lib
    # null tensors
    assert lib.tfx_linear(None, None, None, None, None, 4, 32, 8, 0, None) == L.TFX_ERR_INVALID_ARGUMENT
    assert b"null" in lib.tfx_last_error_message()
    # unsupported shapes are rejected before any device work
    fake = ctypes.c_void_p(256)
    assert lib.tfx_linear(fake, fake, fake, None, fake, 4, 33, 8, 0, None) == L.TFX_ERR_UNSUPPORTED
    assert lib.tfx_linear(fake, fake, fake, None, fake, 4, 32, 8, 2, None) == L.TFX_ERR_INVALID_ARGUMENT
    assert lib.tfx_linear(fake, fake, fake, None, fake, 4, 32, 8, 9, None) in (
        L.TFX_ERR_INVALID_ARGUMENT,)
    odd = ctypes.c_void_p(258)
    assert lib.tfx_linear(odd, fake, fake, None, fake, 4, 32, 8, 0, None) == L.TFX_ERR_MISALIGNED
    assert lib.tfx_layer_norm(fake, fake, fake, fake, 0, 4, 30, 1e-5, 1, None) == L.TFX_ERR_UNSUPPORTED
    assert lib.tfx_layer_norm(fake, fake, fake, fake, 7, 4, 32, 1e-5, 1, None) == L.TFX_ERR_INVALID_ARGUMENT
    assert lib.tfx_attention(fake, fake, fake, 96, fake, 96, 1, 4, 16, 24, 0.2, 1, None, None) == \
        L.TFX_ERR_UNSUPPORTED
    assert lib.tfx_attention(fake, fake, fake, 64, fake, 96, 1, 4, 16, 24, 0.2, 1, None, None) == \
        L.TFX_ERR_INVALID_ARGUMENT


def test_forward_rejects_bad_models(lib):
    pkg = load_package()
    L = pkg._lib
    m = L.TfxModel()
    m.d_model, m.num_heads, m.ffn_dim, m.num_layers = 128, 5, 128, 1
    assert lib.tfx_forward_workspace_bytes(ctypes.byref(m), 1, 1) == -1
    layers = (L.TfxLayer * 1)()
    m.layers = ctypes.cast(layers, ctypes.POINTER(L.TfxLayer))
    m.num_heads = 4
    # every pointer null -> invalid argument, nothing launched
    assert lib.tfx_forward(ctypes.byref(m), ctypes.c_void_p(256), ctypes.c_void_p(512), 1, 1,
                           None, ctypes.c_void_p(1024), 1 << 20, None) == L.TFX_ERR_INVALID_ARGUMENT
    m.num_heads = 3  # head_dim not integral
    assert lib.tfx_forward_workspace_bytes(ctypes.byref(m), 1, 1) == -1


def test_forward_rejects_overlap_and_bad_path(lib):
    """x and y ranges must be disjoint (not only different pointers), and the
    model's path must be a tfx_path; both checked on the host."""
    pkg = load_package()
    L = pkg._lib
    m = L.TfxModel()
    m.d_model, m.num_heads, m.ffn_dim, m.num_layers, m.causal, m.eps = 128, 4, 128, 1, 1, 1e-5
    layers = (L.TfxLayer * 1)()
    for f, _ in L.TfxLayer._fields_:
        setattr(layers[0], f, 256)
    m.layers = ctypes.cast(layers, ctypes.POINTER(L.TfxLayer))
    m.final_norm_weight = m.final_norm_bias = 256
    x = 1 << 20
    # y starts half-way into x's 2 x 8 x 128 floats
    st = lib.tfx_forward(ctypes.byref(m), ctypes.c_void_p(x), ctypes.c_void_p(x + 4096), 2, 8,
                         None, None, 0, None)
    assert st == L.TFX_ERR_INVALID_ARGUMENT
    assert b"overlap" in lib.tfx_last_error_message()
    m.path = 7
    assert lib.tfx_forward_workspace_bytes(ctypes.byref(m), 2, 8) == -1
    st = lib.tfx_forward(ctypes.byref(m), ctypes.c_void_p(x), ctypes.c_void_p(x + 8192), 2, 8,
                         None, None, 0, None)
    assert st == L.TFX_ERR_INVALID_ARGUMENT
    assert b"path" in lib.tfx_last_error_message()


def test_workspace_size_formula(lib):
    pkg = load_package()
    L = pkg._lib
    m = L.TfxModel()
    m.d_model, m.num_heads, m.ffn_dim, m.num_layers = 128, 4, 128, 1
    layers = (L.TfxLayer * 1)()
    for f, _ in L.TfxLayer._fields_:
        setattr(layers[0], f, 256)
    m.layers = ctypes.cast(layers, ctypes.POINTER(L.TfxLayer))
    m.final_norm_weight = m.final_norm_bias = 256
    rows = 10 * 128
    per_row = 2 * 128 + 2 * 384 + 2 * 128 + 4 * 128 + 2 * 128
    # D = F = 128, seq | 128: the fused whole-forward kernel needs no workspace
    assert lib.tfx_forward_workspace_bytes(ctypes.byref(m), 10, 128) == 0
    m.path = L.TFX_PATH_CHAIN
    need = lib.tfx_forward_workspace_bytes(ctypes.byref(m), 10, 128)
    m.path = L.TFX_PATH_AUTO
    # h, qkv, ctx (fp16, D, 3D, D) + residual (fp32, D) + ffn hidden (fp16, F)
    assert need == rows * per_row
    # seq not dividing 128: the per-op chain and its workspace
    assert lib.tfx_forward_workspace_bytes(ctypes.byref(m), 10, 100) == 1000 * per_row


def test_workspace_holds_transposed_v_for_tcgen05_attention(lib):
    """head_dim 64: the h buffer also holds V^T [B][D][S rounded up to 8]."""
    pkg = load_package()
    L = pkg._lib
    m = L.TfxModel()
    m.d_model, m.num_heads, m.ffn_dim, m.num_layers = 256, 4, 512, 1
    layers = (L.TfxLayer * 1)()
    for f, _ in L.TfxLayer._fields_:
        setattr(layers[0], f, 256)
    m.layers = ctypes.cast(layers, ctypes.POINTER(L.TfxLayer))
    m.final_norm_weight = m.final_norm_bias = 256

    def up(n):
        return (n + 255) // 256 * 256

    b, s, d, f = 3, 261, 256, 512
    rows = b * s
    vt = 2 * b * d * ((s + 7) // 8 * 8)
    expect = up(max(2 * rows * d, vt)) + up(2 * rows * 3 * d) + up(2 * rows * d) + \
        up(4 * rows * d) + up(2 * rows * f)
    assert lib.tfx_forward_workspace_bytes(ctypes.byref(m), b, s) == expect


def test_transposed_v_entry_points_validate_on_the_host(lib):
    pkg = load_package()
    L = pkg._lib
    assert lib.tfx_attention_vt_ld(261) == 264
    assert lib.tfx_attention_vt_ld(0) == -1
    assert lib.tfx_transpose_v(None, 64, None, 1, 1, 64, None) == L.TFX_ERR_INVALID_ARGUMENT
    assert lib.tfx_transpose_v(256, 96, 512, 1, 8, 96, None) == L.TFX_ERR_UNSUPPORTED  # cols % 64
    assert lib.tfx_transpose_v(264, 64, 512, 1, 8, 64, None) == L.TFX_ERR_MISALIGNED
    # head_dim 32 has no tcgen05 attention kernel
    assert lib.tfx_attention_vt(256, 512, 768, 96, 1024, 32, 1, 1, 8, 32, 0.17, 1, None,
                                None) == L.TFX_ERR_UNSUPPORTED
    assert lib.tfx_attention_vt(256, 512, 768, 192, 1024, 64, 1, 1, 8, 64, -1.0, 1, None,
                                None) == L.TFX_ERR_UNSUPPORTED
    assert lib.tfx_attention_vt(None, 512, 768, 192, 1024, 64, 1, 1, 8, 64, 0.125, 1, None,
                                None) == L.TFX_ERR_INVALID_ARGUMENT


def _fake_model(L, d=128, h=4, f=128, layers=1, causal=1):
    m = L.TfxModel()
    m.d_model, m.num_heads, m.ffn_dim, m.num_layers = d, h, f, layers
    arr = (L.TfxLayer * layers)()
    for i in range(layers):
        for name, _ in L.TfxLayer._fields_:
            setattr(arr[i], name, 256)
    m.layers = ctypes.cast(arr, ctypes.POINTER(L.TfxLayer))
    m.final_norm_weight = m.final_norm_bias = 256
    m.causal = causal
    m.eps = 1e-5
    return m, arr


def test_kv_forward_validates_on_the_host(lib):
    """tfx_forward_kv: the reference's KV-cache rules (causal only, capacity,
    torch_transformer_benchmark.py:409-440) and the ABI's pointer rules,
    all checked before anything is enqueued."""
    pkg = load_package()
    L = pkg._lib
    m, keep = _fake_model(L)
    x, y, kc, vc, ws = (ctypes.c_void_p(v) for v in (4096, 8192, 12288, 16384, 1 << 20))
    need = lib.tfx_forward_kv_workspace_bytes(ctypes.byref(m), 2, 3)
    # the KV path is always the per-op chain: the chain's workspace for 2 x 3 rows, plus
    # (new_tokens <= 16: decode steps) split-KV partials for up to 4096 (batch, head,
    # split) rows: fp32 O [rows][3][head_dim 32] and (max, sum) pairs
    per_row = 2 * 128 + 2 * 384 + 2 * 128 + 4 * 128 + 2 * 128
    part = 4096 * 3 * 32 * 4 + 4096 * 3 * 8
    assert need == 6 * per_row + (part + 255) // 256 * 256
    big = lib.tfx_forward_kv_workspace_bytes(ctypes.byref(m), 2, 17)  # no decode scratch
    assert big == 34 * per_row
    call = lambda **kw: lib.tfx_forward_kv(  # noqa: E731
        ctypes.byref(kw.get("model", m)), kw.get("x", x), kw.get("y", y), kw.get("batch", 2),
        kw.get("new", 3), kw.get("start", 5), kw.get("cap", 8), kw.get("kc", kc),
        kw.get("vc", vc), kw.get("ws", ws), kw.get("ws_bytes", need), None)
    assert call(start=6) == L.TFX_ERR_INVALID_ARGUMENT  # 6 + 3 > 8
    assert b"capacity exceeded" in lib.tfx_last_error_message()
    assert call(start=-1) == L.TFX_ERR_INVALID_ARGUMENT
    assert call(new=0) == L.TFX_ERR_INVALID_ARGUMENT
    assert call(kc=None) == L.TFX_ERR_INVALID_ARGUMENT
    assert call(vc=ctypes.c_void_p(16386)) == L.TFX_ERR_MISALIGNED
    assert call(ws=ctypes.c_void_p((1 << 20) + 16)) == L.TFX_ERR_MISALIGNED
    assert call(ws_bytes=need - 1) == L.TFX_ERR_WORKSPACE
    assert call(y=x) == L.TFX_ERR_INVALID_ARGUMENT
    nc, keep2 = _fake_model(L, causal=0)
    assert call(model=nc) == L.TFX_ERR_UNSUPPORTED
    assert b"causal" in lib.tfx_last_error_message()
    assert lib.tfx_forward_kv_workspace_bytes(ctypes.byref(m), 0, 3) == -1


def test_selftest_limit_is_checked_on_the_host(lib):
    pkg = load_package()
    L = pkg._lib
    assert lib.tfx_selftest_bounded_wait(0, None) == L.TFX_ERR_INVALID_ARGUMENT
    assert lib.tfx_selftest_bounded_wait(3_000_000_000, None) == L.TFX_ERR_INVALID_ARGUMENT
    assert b"limit_cycles" in lib.tfx_last_error_message()
